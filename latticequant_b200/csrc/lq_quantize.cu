// lq_quantize.cu -- E8 quantisation, symbolisation, coset packing, histograms.
//
// Reference: llm/compressed_kv_cache.py:198-253
//   x_scaled = t_heads / scale; all_q = encode_e8(x_scaled)       (core/e8_quantizer.py:61-83)
//   decompressed_out = (all_q * scale).to(orig_dtype)
//   coset, free, c8h = e8_to_symbols(all_q)                       (core/entropy_coder.py:46-68)
//   per (coset, coord) stream: counts over the chunk -> build_rans_table
//   coset_packed = pack_coset_bits(coset)                         (:46-54)
//
// One warp walks one tile of TB blocks, 32 blocks per step, one block per
// lane: a 16-byte (or 2x16-byte for fp32) load of the block, the E8 search
// in registers, and per step one ballot that is directly the 32-bit word of
// the packed coset bitmap.  The ballot also ranks each block inside its
// coset, which places its 8 symbols in the tile's 8 coordinate columns:
// coset-0 blocks from the front in block order, coset-1 blocks from the back
// -- so each rANS lane later reads its symbols contiguously, 8 at a time.
// The columns are int8: a block whose symbols all lie in [-127, 127] (one
// test per block) stores them directly; a symbol outside is stored as -128
// with its full value at the same index of an int16 plane, and the tile is
// flagged so that the encoder looks there.  Symbol counts go to a
// shared-memory histogram per CTA (values in [-127, 127], the same test),
// falling back to global atomics outside that window, and are flushed once
// per CTA.
#include "lq_common.cuh"

namespace lq {
namespace {

constexpr int kQWarps = 8;          // tiles per CTA
constexpr int kSmemHalf = 127;      // shared histogram window [-127, 127]: the int8 column range
constexpr int kSmemBins = 2 * kSmemHalf + 1;

__device__ __forceinline__ void red_shared_add1(uint32_t addr) {
    asm volatile("red.shared.add.u32 [%0], 1;" ::"r"(addr) : "memory");
}

// Outlier side channel (off when limit == 0): a token (bpt consecutive
// blocks) with a symbol outside [-limit, limit] goes whole to a record list
// (block index, coset, 8 symbols per block) and is coded as zero blocks, so
// every stream's alphabet stays within 2*limit + 5 values.  The reference has
// no such path: its table build never ends for alphabets over L.
struct OutlierArgs {
    int limit;           // 0 = off
    uint32_t bpt;        // blocks per token (1, 2, 4, 8, 16 or 32)
    uint32_t *words;     // [n_chunks][ceil(N/32)] bitmap of extracted blocks (may be NULL)
    int32_t *rec;        // [n_chunks][cap][10]
    uint32_t *count;     // [n_chunks]
    uint32_t cap;
};

// TBC: the tile size as a compile-time constant (0 = take TB), so that the
// eight column stores of a block address with immediate offsets.
template <int DT, int DQ, bool QO, uint32_t TBC>
__global__ void __launch_bounds__(32 * kQWarps, 3) quantize_kernel(
    const void *__restrict__ x, uint32_t n_heads, uint32_t bph, FastDiv bph_div, const float *__restrict__ scale_f32,
    uint32_t TB, uint32_t n_tiles, SymCols sc8, uint32_t *__restrict__ coset_words,
    uint32_t *__restrict__ tile_n0, uint32_t *__restrict__ hist, void *__restrict__ deq, float *__restrict__ q_out,
    OutlierArgs oa, uint32_t *__restrict__ err) {
    __shared__ uint32_t sh_hist[LQ_NSTREAMS * kSmemBins];
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t chunk = blockIdx.y;
    const uint32_t N = n_heads * bph;
    const uint32_t words_per_chunk = (N + 31) / 32;

    for (int i = threadIdx.x; i < LQ_NSTREAMS * kSmemBins; i += blockDim.x) sh_hist[i] = 0;
    __syncthreads();
    const uint32_t hist_base = static_cast<uint32_t>(__cvta_generic_to_shared(sh_hist));

    if constexpr (TBC != 0) TB = TBC;
    const uint32_t tile = blockIdx.x * kQWarps + warp;
    uint32_t flags = 0;
    if (tile < n_tiles) {
        const uint32_t b0 = tile * TB;
        const uint32_t tb = (b0 + TB <= N) ? TB : N - b0;
        const int64_t cblk0 = (int64_t)chunk * N;  // first block of the chunk
        const int64_t col0 = ((int64_t)chunk * n_tiles + tile) * TB * 8;  // [8][TB] coordinate columns
        int8_t *cols = sc8.cols + col0;
        int16_t *wide = sc8.wide + col0;
        bool esc = false;
        const float *sc_chunk = scale_f32 + (int64_t)chunk * n_heads;
        uint32_t *cw = coset_words + (int64_t)chunk * words_per_chunk + b0 / 32;
        // per-thread position: block b = b0 + off + lane lives in head `head`, at `rem` within it
        uint32_t head = bph_div.div(b0 + lane);
        uint32_t rem = b0 + lane - head * bph;
        uint32_t cur_head = 0xffffffffu;
        float sc = 1.0f, rcp = 1.0f;
        bool fast = false;
        uint32_t n0 = 0, n1 = 0;  // running coset counts
        // one block in flight ahead of the one being searched
        RawBlock8 cur = {};
        if (lane < tb) cur = load_raw8<DT>(x, cblk0 + b0 + lane);
        for (uint32_t off = 0; off < tb; off += 32) {
            const bool active = (off + lane) < tb;
            RawBlock8 nxt = {};
            if (off + 32 + lane < tb) nxt = load_raw8<DT>(x, cblk0 + b0 + off + 32 + lane);
            int sym[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int coset = 0;
            if (active) {
                if (head != cur_head) {
                    cur_head = head;
                    sc = sc_chunk[head];
                    rcp = __frcp_rn(sc);
                    fast = scale_ok_for_fast_div(sc);
                }
                const int64_t blk = cblk0 + b0 + off + lane;
                float v[8], xs[8], q[8];
                raw8_to_float<DT>(cur, v);
                div_block_by_scale<(DQ >= 0) || QO>(v, sc, rcp, fast, xs);
                bool finite;
                coset = e8_nearest_symbols<(DQ >= 0) || QO>(xs, q, sym, &finite);
                if (!finite) flags |= LQ_EF_NONFINITE;
                if constexpr (DQ >= 0) {
                    float o[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(q[i], sc);
                    store_block8<DQ>(deq, blk, o);
                }
                if constexpr (QO) {
                    float4 *qp = reinterpret_cast<float4 *>(q_out) + 2 * blk;
                    qp[0] = make_float4(q[0], q[1], q[2], q[3]);
                    qp[1] = make_float4(q[4], q[5], q[6], q[7]);
                }
            }
            if (oa.limit > 0) {  // uniform
                bool out = false;
                if (active) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) out |= (sym[i] > oa.limit) || (sym[i] < -oa.limit);
                }
                const uint32_t ob = __ballot_sync(0xffffffffu, out);
                if (ob) {
                    const uint32_t tm = (oa.bpt >= 32 ? 0xffffffffu : ((1u << oa.bpt) - 1u)) << ((lane / oa.bpt) * oa.bpt);
                    out = active && (ob & tm) != 0u;  // the whole token
                    if (out) {
                        const uint32_t idx = atomicAdd(&oa.count[chunk], 1u);
                        if (idx < oa.cap) {
                            int32_t *r = oa.rec + ((size_t)chunk * oa.cap + idx) * 10;
                            r[0] = (int32_t)(b0 + off + lane);
                            r[1] = coset;
#pragma unroll
                            for (int i = 0; i < 8; ++i) r[2 + i] = sym[i];
                        } else {
                            flags |= LQ_EF_CAPACITY;
                        }
                        coset = 0;
#pragma unroll
                        for (int i = 0; i < 8; ++i) sym[i] = 0;
                    }
                }
                const uint32_t ow = __ballot_sync(0xffffffffu, out);
                if (oa.words && lane == 0) oa.words[(int64_t)chunk * words_per_chunk + (b0 + off) / 32] = ow;
            }
            const uint32_t ball = __ballot_sync(0xffffffffu, active && coset);
            const uint32_t act = __ballot_sync(0xffffffffu, active);
            if (lane == 0) cw[off / 32] = ball;
            const uint32_t lt = (1u << lane) - 1u;
            if (active) {
                const uint32_t row = coset ? tb - 1 - (n1 + __popc(ball & lt)) : n0 + __popc(act & ~ball & lt);
                const uint32_t sh = hist_base + (uint32_t)coset * (8 * kSmemBins * 4);
                // one test for the whole block: every (sym + half) at most 2 * half as unsigned
                uint32_t top = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) top = max(top, (uint32_t)(sym[i] + kSmemHalf));
                if (top < (uint32_t)kSmemBins) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        cols[i * TB + row] = (int8_t)sym[i];
                        red_shared_add1(sh + (uint32_t)(i * kSmemBins + sym[i] + kSmemHalf) * 4u);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int v = sym[i];
                        const bool in8 = (uint32_t)(v + kSmemHalf) < (uint32_t)kSmemBins;
                        cols[i * TB + row] = in8 ? (int8_t)v : (int8_t)-128;
                        if (!in8) {
                            wide[i * TB + row] = (int16_t)v;
                            esc = true;
                        }
                        if ((uint32_t)(v + kSmemHalf) < (uint32_t)kSmemBins) {
                            red_shared_add1(sh + (uint32_t)(i * kSmemBins + v + kSmemHalf) * 4u);
                        } else if ((uint32_t)(v + LQ_SYM_LIMIT) < (uint32_t)(2 * LQ_SYM_LIMIT)) {
                            uint32_t *gh = hist + ((int64_t)chunk * LQ_NSTREAMS + coset * 8 + i) * LQ_HIST_BINS;
                            atomicAdd(&gh[v + LQ_SYM_LIMIT], 1u);
                        } else {
                            // outside the histogram window (float->int saturates, so huge values land here)
                            flags |= LQ_EF_SYMRANGE;
                        }
                    }
                }
            }
            const uint32_t c1 = __popc(ball);
            n1 += c1;
            n0 += __popc(act) - c1;
            cur = nxt;
            rem += 32;
            while (rem >= bph) {
                rem -= bph;
                ++head;
            }
        }
        const bool tesc = __any_sync(0xffffffffu, esc);
        if (lane == 0) {
            tile_n0[(int64_t)chunk * n_tiles + tile] = n0;
            sc8.esc[(int64_t)chunk * n_tiles + tile] = tesc ? 1u : 0u;
        }
    }
    if (flags) raise_flag(err, flags);
    __syncthreads();
    uint32_t *gh = hist + (int64_t)chunk * LQ_NSTREAMS * LQ_HIST_BINS;
    for (int i = threadIdx.x; i < LQ_NSTREAMS * kSmemBins; i += blockDim.x) {
        const uint32_t c = sh_hist[i];
        if (c) {
            const int s = i / kSmemBins, v = i % kSmemBins - kSmemHalf;
            atomicAdd(&gh[s * LQ_HIST_BINS + v + LQ_SYM_LIMIT], c);
        }
    }
}

template <int DT, int DQ, bool QO>
int launch_quantize(const void *x, int64_t n_chunks, int64_t n_heads, int64_t bph, const float *scale_f32, int64_t TB,
                    SymCols sym_rows, uint32_t *coset_words, uint32_t *tile_n0, uint32_t *hist, void *deq,
                    float *q_out, const OutlierArgs &oa, uint32_t *err, cudaStream_t st) {
    const int64_t N = n_heads * bph;
    const int64_t n_tiles = ceil_div(N, TB);
    dim3 grid((unsigned)ceil_div(n_tiles, kQWarps), (unsigned)n_chunks);
    if constexpr (DQ < 0 && !QO) {
        if (TB == 1024) {
            quantize_kernel<DT, DQ, QO, 1024><<<grid, 32 * kQWarps, 0, st>>>(
                x, (uint32_t)n_heads, (uint32_t)bph, FastDiv((uint32_t)bph), scale_f32, (uint32_t)TB,
                (uint32_t)n_tiles, sym_rows, coset_words, tile_n0, hist, deq, q_out, oa, err);
            return check_launch();
        }
    }
    quantize_kernel<DT, DQ, QO, 0><<<grid, 32 * kQWarps, 0, st>>>(x, (uint32_t)n_heads, (uint32_t)bph, FastDiv((uint32_t)bph),
                                                               scale_f32, (uint32_t)TB, (uint32_t)n_tiles, sym_rows,
                                                               coset_words, tile_n0, hist, deq, q_out, oa, err);
    return check_launch();
}

template <int DT, bool QO>
int dispatch_deq(int deq_dtype, const void *x, int64_t n_chunks, int64_t n_heads, int64_t bph, const float *sc,
                 int64_t TB, SymCols sym_rows, uint32_t *cw, uint32_t *tn0, uint32_t *hist, void *deq, float *q_out,
                 const OutlierArgs &oa, uint32_t *err, cudaStream_t st) {
    if (deq == nullptr)
        return launch_quantize<DT, -1, QO>(x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq, q_out,
                                           oa, err, st);
    switch (deq_dtype) {
        case LQ_F32:
            return launch_quantize<DT, LQ_F32, QO>(x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq,
                                                   q_out, oa, err, st);
        case LQ_F16:
            return launch_quantize<DT, LQ_F16, QO>(x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq,
                                                   q_out, oa, err, st);
        case LQ_BF16:
            return launch_quantize<DT, LQ_BF16, QO>(x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq,
                                                    q_out, oa, err, st);
        default:
            return LQ_ERR_INVALID;
    }
}

template <int DT>
int dispatch_q(int deq_dtype, const void *x, int64_t n_chunks, int64_t n_heads, int64_t bph, const float *sc,
               int64_t TB, SymCols sym_rows, uint32_t *cw, uint32_t *tn0, uint32_t *hist, void *deq, float *q_out,
               const OutlierArgs &oa, uint32_t *err, cudaStream_t st) {
    return q_out ? dispatch_deq<DT, true>(deq_dtype, x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq,
                                          q_out, oa, err, st)
                 : dispatch_deq<DT, false>(deq_dtype, x, n_chunks, n_heads, bph, sc, TB, sym_rows, cw, tn0, hist, deq,
                                           q_out, oa, err, st);
}

__global__ void encode_e8_kernel(const float *__restrict__ x, int64_t n, float *__restrict__ out, int d8_only) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    float v[8], q[8], res[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[8 * b + i];
    if (d8_only) d8_nearest(v, q, res);
    else e8_nearest(v, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[8 * b + i] = q[i];
}

}  // namespace
}  // namespace lq

namespace lq {
namespace {
int quantize_entry(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph, const float *scale_f32,
                   int64_t tile_blocks, void *sym_cols, uint32_t *coset_words, uint32_t *tile_n0, uint32_t *hist,
                   void *deq, int deq_dtype, float *q_out, const OutlierArgs &oa, uint32_t *err, void *stream) {
    if (n_chunks < 0 || n_heads < 0 || bph < 0) return LQ_ERR_INVALID;
    if (tile_blocks <= 0 || (tile_blocks % 32) != 0) return LQ_ERR_INVALID;
    if (n_chunks == 0 || n_heads * bph == 0) return LQ_OK;
    if (!x || !scale_f32 || !sym_cols || !coset_words || !tile_n0 || !hist) return LQ_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (deq && (reinterpret_cast<uintptr_t>(deq) & 15)) ||
        (reinterpret_cast<uintptr_t>(sym_cols) & 15) || (q_out && (reinterpret_cast<uintptr_t>(q_out) & 15)))
        return LQ_ERR_INVALID;
    const SymCols sym_rows = sym_cols_view(sym_cols, n_chunks * ceil_div(n_heads * bph, tile_blocks), tile_blocks);
    if (n_chunks > 65535) return LQ_ERR_INVALID;
    if (n_heads * bph >= (int64_t)1 << 31) return LQ_ERR_INVALID;  // blocks per chunk are indexed in 32 bits
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(hist, 0, sizeof(uint32_t) * (size_t)n_chunks * LQ_NSTREAMS * LQ_HIST_BINS, st) != cudaSuccess)
        return LQ_ERR_CUDA;
    switch (dtype) {
        case LQ_F32:
            return dispatch_q<LQ_F32>(deq_dtype, x, n_chunks, n_heads, bph, scale_f32, tile_blocks, sym_rows,
                                      coset_words, tile_n0, hist, deq, q_out, oa, err, st);
        case LQ_F16:
            return dispatch_q<LQ_F16>(deq_dtype, x, n_chunks, n_heads, bph, scale_f32, tile_blocks, sym_rows,
                                      coset_words, tile_n0, hist, deq, q_out, oa, err, st);
        case LQ_BF16:
            return dispatch_q<LQ_BF16>(deq_dtype, x, n_chunks, n_heads, bph, scale_f32, tile_blocks, sym_rows,
                                       coset_words, tile_n0, hist, deq, q_out, oa, err, st);
        default:
            return LQ_ERR_INVALID;
    }
}

// One thread per record: the extracted block's point (symbols_to_e8) times
// its head's fp16 scale, into the decoded output (and its symbols into sym_out).
template <int DO>
__global__ void patch_outliers_kernel(const int32_t *__restrict__ rec, const uint32_t *__restrict__ count,
                                      uint32_t cap, uint32_t n_heads, uint32_t bph, const uint16_t *__restrict__ scale,
                                      void *__restrict__ out, int32_t *__restrict__ sym_out, uint32_t *err) {
    const uint32_t chunk = blockIdx.y;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t n = min(count[chunk], cap);
    if (i >= n) return;
    const int32_t *r = rec + ((size_t)chunk * cap + i) * 10;
    const uint32_t blk = (uint32_t)r[0];
    const uint32_t N = n_heads * bph;
    if (blk >= N) {
        raise_flag(err, LQ_EF_BITSTREAM);
        return;
    }
    int sym[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) sym[k] = r[2 + k];
    const size_t gb = (size_t)chunk * N + blk;
    if (sym_out) {
#pragma unroll
        for (int k = 0; k < 8; ++k) sym_out[8 * gb + k] = sym[k];
    }
    if constexpr (DO >= 0) {
        float q[8];
        e8_from_symbols(r[1], sym, q);
        const float sc = __half2float(__ushort_as_half(scale[(size_t)chunk * n_heads + blk / bph]));
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = __fmul_rn(q[k], sc);
        store_block8<DO>(out, gb, q);
    }
}
}  // namespace
}  // namespace lq

extern "C" int lq_e8_quantize(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph,
                              const float *scale_f32, int64_t tile_blocks, void *sym_cols, uint32_t *coset_words,
                              uint32_t *tile_n0, uint32_t *hist, void *deq, int deq_dtype, float *q_out,
                              uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    const lq::OutlierArgs off{0, 1, nullptr, nullptr, nullptr, 0};
    return lq::quantize_entry(x, dtype, n_chunks, n_heads, bph, scale_f32, tile_blocks, sym_cols, coset_words, tile_n0,
                              hist, deq, deq_dtype, q_out, off, err, stream);
}

extern "C" int lq_e8_quantize_outliers(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph,
                                       const float *scale_f32, int64_t tile_blocks, void *sym_cols,
                                       uint32_t *coset_words, uint32_t *tile_n0, uint32_t *hist, void *deq,
                                       int deq_dtype, float *q_out, int limit, int blocks_per_token,
                                       uint32_t *outlier_words, int32_t *outlier_rec, uint32_t *outlier_count,
                                       int64_t outlier_cap, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (limit <= 0 || limit > 0x3fffffff || blocks_per_token <= 0 || blocks_per_token > 32 ||
        (blocks_per_token & (blocks_per_token - 1)) || (tile_blocks % blocks_per_token) || (bph % blocks_per_token) ||
        !outlier_rec || !outlier_count || outlier_cap < 0 || outlier_cap > 0x7fffffff)
        return LQ_ERR_INVALID;
    if (n_chunks > 0 &&
        cudaMemsetAsync(outlier_count, 0, sizeof(uint32_t) * (size_t)n_chunks, lq::as_stream(stream)) != cudaSuccess)
        return LQ_ERR_CUDA;
    const lq::OutlierArgs oa{limit, (uint32_t)blocks_per_token, outlier_words, outlier_rec, outlier_count,
                             (uint32_t)outlier_cap};
    return lq::quantize_entry(x, dtype, n_chunks, n_heads, bph, scale_f32, tile_blocks, sym_cols, coset_words, tile_n0,
                              hist, deq, deq_dtype, q_out, oa, err, stream);
}

extern "C" int lq_patch_outliers(const int32_t *outlier_rec, const uint32_t *outlier_count, int64_t n_chunks,
                                 int64_t outlier_cap, int64_t n_heads, int64_t bph, const uint16_t *scale_f16,
                                 void *out, int out_dtype, int32_t *sym_out, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_chunks < 0 || outlier_cap < 0 || n_heads < 0 || bph <= 0 || outlier_cap > 0x7fffffff) return LQ_ERR_INVALID;
    if (n_chunks == 0 || outlier_cap == 0 || n_heads == 0) return LQ_OK;
    if (!outlier_rec || !outlier_count || (!out && !sym_out) || (out && !scale_f16) || n_chunks > 65535 ||
        n_heads * bph >= ((int64_t)1 << 31))
        return LQ_ERR_INVALID;
    if (out && (reinterpret_cast<uintptr_t>(out) & 15)) return LQ_ERR_INVALID;
    dim3 grid((unsigned)lq::ceil_div(outlier_cap, 128), (unsigned)n_chunks);
    cudaStream_t st = lq::as_stream(stream);
    const uint32_t cap = (uint32_t)outlier_cap, nh = (uint32_t)n_heads, b = (uint32_t)bph;
    if (!out) lq::patch_outliers_kernel<-1><<<grid, 128, 0, st>>>(outlier_rec, outlier_count, cap, nh, b, scale_f16,
                                                                   out, sym_out, err);
    else if (out_dtype == LQ_F32)
        lq::patch_outliers_kernel<LQ_F32><<<grid, 128, 0, st>>>(outlier_rec, outlier_count, cap, nh, b, scale_f16, out,
                                                                sym_out, err);
    else if (out_dtype == LQ_F16)
        lq::patch_outliers_kernel<LQ_F16><<<grid, 128, 0, st>>>(outlier_rec, outlier_count, cap, nh, b, scale_f16, out,
                                                                sym_out, err);
    else if (out_dtype == LQ_BF16)
        lq::patch_outliers_kernel<LQ_BF16><<<grid, 128, 0, st>>>(outlier_rec, outlier_count, cap, nh, b, scale_f16,
                                                                 out, sym_out, err);
    else
        return LQ_ERR_INVALID;
    return lq::check_launch();
}

extern "C" int lq_encode_e8(const float *x, int64_t n, float *out, int d8_only, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!x || !out) return LQ_ERR_INVALID;
    lq::encode_e8_kernel<<<(unsigned)lq::ceil_div(n, 256), 256, 0, lq::as_stream(stream)>>>(x, n, out, d8_only);
    return lq::check_launch();
}

extern "C" size_t lq_sym_cols_bytes(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks) {
    if (n_chunks <= 0 || n_vectors <= 0 || tile_blocks <= 0 || (tile_blocks % 32) != 0) return 0;
    return lq::sym_cols_bytes(n_chunks * lq::ceil_div(n_vectors, tile_blocks), tile_blocks);
}
