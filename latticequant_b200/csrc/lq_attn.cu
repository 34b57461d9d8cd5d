// lq_attn.cu -- fused dequant + decode attention over compressed K/V chunks.
//
// The reference serves attention from a decompressed bf16 buffer: update()
// (llm/compressed_kv_cache.py:342-395) returns the dequantised K/V and
// transformers runs SDPA over it with repeat_kv; its fused analogue
// (llm/fused_triton_merge.py) only merges the compact 4-bit layout into that
// buffer.  Here one kernel streams the entropy-coded K and V tiles straight
// from HBM, rebuilds each E8 block in registers (symbols_to_e8,
// core/entropy_coder.py:71-89, times the fp16 head scale of
// llm/compressed_kv_cache.py:330) and folds it into the attention of the
// GQA query group that reads that KV head, so no dequantised tensor exists.
//
// Work split: a CTA owns a range of tile pairs of one (batch, kv-head) head;
// a warp owns one tile pair (tokens of two consecutive tiles).
//   phase K  the chunk's K tables in shared memory; the warp decodes its K
//            tiles in position order (lq_tiledec.cuh) and each lane, which
//            always holds the same 8 channels of a token, multiplies them
//            with the same 8 channels of the G query heads; a butterfly over
//            the token's lanes gives the G scores of the token (shared memory)
//   softmax  per warp: m = max score, p = 2^(s - m), l = sum p (base 2)
//   phase V  V tables replace the K tables; the warp decodes its V tiles
//            and each lane accumulates p * v for its 8 channels in registers
//   merge    warps merge (m, l, o) in a fixed order -> one partial per CTA;
//            a second kernel merges a head's partials into o and lse.
// Every sum runs in a fixed order, so results are deterministic.
#include <algorithm>

#include "lq_attn_common.cuh"

namespace lq {
namespace {

constexpr int kAttnRing = 48;  // ring rows: rounds take 3-6 token groups of 16 blocks

struct AttnArgs {
    ChunkDev k, v;
    const void *q;        // [B][Hkv*G][D] in q dtype
    uint32_t n_kv_heads;  // attention heads = B * n_kv_heads
    uint32_t seq;         // tokens per attention head
    uint32_t scale_tok;   // 0: one scale per head (scale[head]); 1: one per token (scale[head * seq + t])
    uint32_t tph;         // tiles per head
    uint32_t n_pairs;     // tile pairs per head
    uint32_t nct;         // CTAs per head
    uint32_t tpt;         // tokens per tile
    uint32_t region0;     // bytes of the table / merge region
    uint32_t warp_bytes;  // bytes of per-warp shared memory
    float qk_log2;        // sm_scale * log2(e)
    float *part;          // [heads][nct][G][D + 2]: o (unnormalised), m, l
    const uint32_t *tok_mask;  // optional [heads][ceil(seq/32)] tokens to leave out
    uint32_t *redo;            // [heads][nct]: 1 where a lane of the CTA read past its bits
    uint32_t *err;
};

template <int G, int BPT>
__host__ __device__ constexpr int attn_threads() {
    return G <= 2 ? 768 : G <= 4 ? 640 : 512;
}

// The 16 tables of a chunk in their shared-memory form (smem_entry), so a
// CTA can fill its table region with one bulk copy.
__global__ void staged_tables_kernel(const uint32_t *__restrict__ dec_tab, const int32_t *__restrict__ tab_lo,
                                     uint32_t n_tables, uint32_t *__restrict__ out) {
    const uint32_t t = blockIdx.x;  // table
    if (t >= n_tables) return;
    const int s = (int)(t % LQ_NSTREAMS);
    const int lo = tab_lo[t], c = s >> 3, mul = (s & 7) == 7 ? 4 : 2;
    for (uint32_t i = threadIdx.x; i < LQ_L; i += blockDim.x)
        out[(size_t)t * LQ_L + i] = smem_entry(dec_tab[(size_t)t * LQ_L + i], lo, c, mul);
}

// Per-head sums of the G partial dots a token's BPT lanes hold, transposed
// on the way: with H (G rounded up to a power of two, H <= BPT) values per
// lane, each of the first log2(H) butterfly steps keeps half of the heads
// the lane carries and sends its partner the other half, so those steps
// move H/2, H/4, ..., 1 values instead of G each; the rest is a plain
// butterfly.  Lane jc ends with head jc / (BPT / H) summed over all BPT
// lanes (heads G..H-1 are zero padding).
template <int G>
__host__ __device__ constexpr int pow2_heads() {
    return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
}

template <int G, int BPT>
__device__ __forceinline__ float head_sums_transposed(const float (&dot)[G], uint32_t jc) {
    constexpr int H = pow2_heads<G>();
    static_assert(H <= BPT, "one lane per head at least");
    float a[H];
#pragma unroll
    for (int i = 0; i < H; ++i) a[i] = i < G ? dot[i < G ? i : 0] : 0.0f;
#pragma unroll
    for (int n = H, o = BPT / 2; n > 1; n >>= 1, o >>= 1) {
        const bool up = (jc & (uint32_t)o) != 0u;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = up ? a[n / 2 + i] : a[i];
            const float send = up ? a[i] : a[n / 2 + i];
            a[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float s = a[0];
#pragma unroll
    for (int o = BPT / (2 * H); o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// Fused attention partial of CTA `cx` of head `head`.  BPT = blocks per
// token = head_dim / 8.  CHECKED = false decodes optimistically and records
// in a.redo whether a lane read past its bits (only a malformed stream
// does); attn_redo_kernel then recomputes those CTAs with CHECKED = true.
// Keeping the exact decode out of the main kernel keeps that kernel to one
// copy of the decoder and within its registers.
template <int G, int BPT, int QDT, bool CHECKED>
__device__ __forceinline__ void attn_partial_cta(const AttnArgs &a, uint32_t cx, uint32_t head) {
    static_assert(BPT == 8 || BPT == 16, "head_dim 64 or 128");
    static_assert(G >= 1 && G <= 8, "query group 1..8");
    constexpr int D = 8 * BPT, GP = padded_g<G>(), TPG = 16 / BPT;
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t *dtab = reinterpret_cast<uint32_t *>(smem);
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const uint32_t lane = threadIdx.x & 31, dc = lane % BPT;
    unsigned char *wb = smem + a.region0 + (size_t)warp * a.warp_bytes;
    const uint32_t ring = smem_addr(wb);
    const uint32_t dta = smem_addr(dtab);
    float *sc = reinterpret_cast<float *>(wb + (kAttnRing + 2) * kRingStride * 2);

    const uint32_t pb = (uint32_t)(((uint64_t)cx * a.n_pairs) / a.nct);
    const uint32_t pe = (uint32_t)(((uint64_t)(cx + 1) * a.n_pairs) / a.nct);
    const uint32_t pair = pb + (uint32_t)warp;
    const bool wact = pair < pe;
    const bool act0 = wact, act1 = wact && 2 * pair + 1 < a.tph;
    const uint32_t tile0 = head * a.tph + 2 * pair;

    // query channels 8*dc .. 8*dc+7 of the G heads reading this kv head, as
    // packed channel pairs (2c, 2c+1) for fma.rn.f32x2 against the block's pairs
    const uint32_t b = head / a.n_kv_heads, kvh = head % a.n_kv_heads;
    unsigned long long q2[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int64_t row = (int64_t)b * a.n_kv_heads * G + (int64_t)kvh * G + g;
        float x0[8];
        load_block8<QDT>(a.q, row * BPT + dc, x0);
#pragma unroll
        for (int c = 0; c < 4; ++c) q2[g][c] = f2_pack(x0[2 * c], x0[2 * c + 1]);
    }

    // ---- phase K: scores
    // set when a lane of the CTA read past its bits (optimistic decode only)
    __shared__ uint32_t s_overrun;
    __shared__ __align__(8) uint64_t s_tab_bar;  // completion of the bulk table copies (K: phase 0, V: phase 1)
    const uint32_t tbar = smem_addr(&s_tab_bar);
    const bool bulk = a.k.staged_tab != nullptr && a.v.staged_tab != nullptr;
    if (threadIdx.x == 0) {
        s_overrun = 0u;
        if (bulk) {
            mbar_init(tbar, 1);
            bulk_load(dta, a.k.staged_tab, (uint32_t)kTablesSmem, tbar);
        }
    }
    if (!bulk) stage_tables(a.k, 0, dtab);
    __syncthreads();
    // a copy that never completes leaves the flag raised and stale tables:
    // every table index is masked, so stale entries give wrong values only
    if (bulk) mbar_wait(tbar, 0, a.err);
    if (wact) {
        auto epi_k = [&](bool ok, int t, uint32_t grp, uint32_t j, uint32_t cc, const uint4 blk) {
            unsigned long long k2[4];
            ring_point2(blk, k2);
            // per-lane partial dots over its 8 channels: the even and the odd
            // channels as the two halves of fma.rn.f32x2, then their sum
            float dot[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                unsigned long long s2 = f2_mul(q2[g][0], k2[0]);
#pragma unroll
                for (int c = 1; c < 4; ++c) s2 = f2_fma(q2[g][c], k2[c], s2);
                float lo, hi;
                f2_unpack(s2, lo, hi);
                dot[g] = lo + hi;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) dot[g] = ok ? dot[g] : 0.f;
            const uint32_t jc = j % BPT;
            const uint32_t tok = grp * TPG + j / BPT;
            float *row = sc + ((uint32_t)t * a.tpt + tok) * GP;
            constexpr uint32_t LPH = BPT / pow2_heads<G>();  // lanes per head after the transposing steps
            const float hs = head_sums_transposed<G, BPT>(dot, jc);
            if (ok && jc % LPH == 0u && jc / LPH < (uint32_t)G) row[jc / LPH] = hs;
        };
        if (decode_two_tiles_ordered<kAttnRing, CHECKED>(a.k, 0, tile0, act0, act1, dta, ring, epi_k, a.err))
            s_overrun = 1u;
    }
    __syncwarp();

    // ---- softmax statistics of this warp's tokens (base 2)
    const float ck = a.scale_tok ? a.qk_log2 : __half2float(__ushort_as_half(a.k.scale_f16[head])) * a.qk_log2;
    const uint32_t ntok = 2 * a.tpt;
    // token i of the warp is token (2*pair + i/tpt)*tpt + i%tpt of the head
    auto tok_of = [&](uint32_t i) {
        const uint32_t t = i < a.tpt ? 0u : 1u;
        return (2 * pair + t) * a.tpt + (i - t * a.tpt);
    };
    auto tok_scale = [&](const uint16_t *sc16, uint32_t i) {
        return __half2float(__ushort_as_half(sc16[(size_t)head * a.seq + tok_of(i)]));
    };
    const uint32_t mwords = (a.seq + 31) >> 5;
    auto masked = [&](uint32_t i) {
        if (!a.tok_mask) return false;
        const uint32_t tok = tok_of(i);
        return ((a.tok_mask[(size_t)head * mwords + (tok >> 5)] >> (tok & 31)) & 1u) != 0u;
    };
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
    }
    for (uint32_t i = lane; i < ntok; i += 32) {
        const bool v = i < a.tpt ? act0 : act1;
        if (!v || masked(i)) continue;
        const float cki = a.scale_tok ? ck * tok_scale(a.k.scale_f16, i) : ck;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            sc[i * GP + g] *= cki;
            m[g] = fmaxf(m[g], sc[i * GP + g]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], off));
    }
    for (uint32_t i = lane; i < ntok; i += 32) {
        const bool v = i < a.tpt ? act0 : act1;
        if (!v) continue;
        if (masked(i)) {  // left out: zero weight
#pragma unroll
            for (int g = 0; g < G; ++g) sc[i * GP + g] = 0.f;
            continue;
        }
        // with per-token V scales the token's scale rides on its weight p
        const float cvi = a.scale_tok ? tok_scale(a.v.scale_f16, i) : 1.0f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float p = exp2f(sc[i * GP + g] - m[g]);
            sc[i * GP + g] = p * cvi;
            l[g] += p;
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
    }
    __syncwarp();

    // ---- phase V: p * v accumulated per lane over its 8 channels
    __syncthreads();  // every warp is done with the K tables
    if (bulk) {
        if (threadIdx.x == 0) bulk_load(dta, a.v.staged_tab, (uint32_t)kTablesSmem, tbar);
        mbar_wait(tbar, 1, a.err);
    } else {
        stage_tables(a.v, 0, dtab);
        __syncthreads();
    }
    // p * v accumulated as packed channel pairs (i, i+1) per head
    unsigned long long acc2[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2[g][i] = 0ull;
    if (wact) {
        auto epi_v = [&](bool ok, int t, uint32_t grp, uint32_t j, uint32_t cc, const uint4 blk) {
            if (!ok) return;
            unsigned long long v2[4];
            ring_point2(blk, v2);
            const uint32_t tok = grp * TPG + j / BPT;
            const float *pp = sc + ((uint32_t)t * a.tpt + tok) * GP;
            float p[GP];
#pragma unroll
            for (int g4 = 0; g4 < GP; g4 += 4) {
                const float4 f = *reinterpret_cast<const float4 *>(pp + g4);
                p[g4] = f.x;
                p[g4 + 1] = f.y;
                p[g4 + 2] = f.z;
                p[g4 + 3] = f.w;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const unsigned long long pg = f2_pack(p[g], p[g]);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc2[g][i] = f2_fma(pg, v2[i], acc2[g][i]);
            }
        };
        if (decode_two_tiles_ordered<kAttnRing, CHECKED>(a.v, 0, tile0, act0, act1, dta, ring, epi_v, a.err))
            s_overrun = 1u;
    }
    float acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) f2_unpack(acc2[g][i], acc[g][2 * i], acc[g][2 * i + 1]);
    // lanes holding the same channels: the two tiles (xor 16), two tokens per group for BPT 8 (xor 8)
#pragma unroll
    for (int off = 16; off >= BPT; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[g][i] += __shfl_xor_sync(0xffffffffu, acc[g][i], off);
    }

    // ---- merge the warps in a fixed order
    __syncthreads();  // every warp is done with the V tables: the region holds the merge buffer
    if (!CHECKED && threadIdx.x == 0) a.redo[head * a.nct + cx] = s_overrun;
    float *mrg = reinterpret_cast<float *>(smem);
    const int rs = D + 2;
    if (lane < (uint32_t)BPT) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 8; ++i) mrg[(warp * G + g) * rs + 8 * (int)lane + i] = acc[g][i];
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            mrg[(warp * G + g) * rs + D] = m[g];
            mrg[(warp * G + g) * rs + D + 1] = l[g];
        }
    }
    __syncthreads();
    const float cv = a.scale_tok ? 1.0f : __half2float(__ushort_as_half(a.v.scale_f16[head]));
    float *out = a.part + ((size_t)head * a.nct + cx) * G * rs;
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int g = e / D, dd = e % D;
        float mx = -INFINITY;
        for (int w = 0; w < nwarps; ++w) mx = fmaxf(mx, mrg[(w * G + g) * rs + D]);
        float o = 0.f, ls = 0.f;
        for (int w = 0; w < nwarps; ++w) {
            const float mw = mrg[(w * G + g) * rs + D];
            if (mw == -INFINITY) continue;
            const float f = exp2f(mw - mx);
            o = fmaf(mrg[(w * G + g) * rs + dd], f, o);
            ls = fmaf(mrg[(w * G + g) * rs + D + 1], f, ls);
        }
        out[g * rs + dd] = o * cv;
        if (dd == 0) {
            out[g * rs + D] = mx;
            out[g * rs + D + 1] = ls;
        }
    }
}

template <int G, int BPT, int QDT>
__global__ void __launch_bounds__(attn_threads<G, BPT>(), 1) attn_partial_kernel(AttnArgs a) {
    attn_partial_cta<G, BPT, QDT, false>(a, blockIdx.x, blockIdx.y);
}

// The CTAs the optimistic pass flagged, again with the exact decode (their
// partials are overwritten); a grid of at most one CTA per SM walks them.
template <int G, int BPT, int QDT>
__global__ void __launch_bounds__(attn_threads<G, BPT>(), 1) attn_redo_kernel(AttnArgs a, uint32_t n_cta) {
    for (uint32_t c = blockIdx.x; c < n_cta; c += gridDim.x) {
        if (a.redo[c] == 0u) continue;  // the same for every thread of the CTA
        __syncthreads();                // the previous CTA's merge buffer is read out
        attn_partial_cta<G, BPT, QDT, true>(a, c % a.nct, c / a.nct);
    }
}

struct AttnPlan {
    int nwarps;
    uint32_t nct, n_pairs, tph, tpt, region0, warp_bytes;
    size_t smem, part_floats;
    size_t redo_off, ws_bytes;  // workspace: partials, then the redo flags
};

size_t attn_warp_bytes(int G, uint32_t tpt) {
    return (size_t)(kAttnRing + 2) * kRingStride * 2 + (size_t)2 * tpt * ((G + 3) & ~3) * 4;
}

int attn_plan(int64_t n_heads, int64_t bph, int64_t tile_blocks, int G, int D, AttnPlan *p) {
    if (n_heads <= 0 || bph <= 0 || tile_blocks <= 0 || G < 1 || G > 8 || (D != 64 && D != 128)) return LQ_ERR_INVALID;
    const int bpt = D / 8;
    if (tile_blocks % 32 != 0 || bph % tile_blocks != 0 || bph % bpt != 0) return LQ_ERR_INVALID;
    if (n_heads > 65535 || n_heads * bph >= ((int64_t)1 << 31)) return LQ_ERR_INVALID;
    p->tph = (uint32_t)(bph / tile_blocks);
    p->tpt = (uint32_t)(tile_blocks / bpt);
    p->n_pairs = (p->tph + 1) / 2;
    const size_t wb = attn_warp_bytes(G, p->tpt);
    int nw = G <= 2 ? 24 : G <= 4 ? 20 : 16;
    for (;; --nw) {
        if (nw < 4) return LQ_ERR_INVALID;  // tiles too long for shared memory
        const size_t r0 = (std::max<size_t>(kTablesSmem, (size_t)nw * G * (D + 2) * 4) + 127) & ~(size_t)127;
        if (r0 + (size_t)nw * wb <= 227 * 1024) {
            p->region0 = (uint32_t)r0;
            break;
        }
    }
    p->nwarps = nw;
    p->warp_bytes = (uint32_t)wb;
    p->smem = p->region0 + (size_t)nw * wb;
    p->nct = (uint32_t)ceil_div(p->n_pairs, nw);
    p->part_floats = (size_t)n_heads * p->nct * G * (D + 2);
    p->redo_off = (p->part_floats * 4 + 255) & ~(size_t)255;
    p->ws_bytes = p->redo_off + (((size_t)n_heads * p->nct * 4 + 255) & ~(size_t)255);
    return LQ_OK;
}

template <int G, int BPT, int QDT>
int launch_partial(const AttnArgs &a, const AttnPlan &p, uint32_t n_heads, cudaStream_t st) {
    auto kern = attn_partial_kernel<G, BPT, QDT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem) != cudaSuccess)
        return LQ_ERR_CUDA;
    kern<<<dim3(p.nct, n_heads), 32 * p.nwarps, p.smem, st>>>(a);
    int rc = check_launch();
    if (rc != LQ_OK) return rc;
    auto redo = attn_redo_kernel<G, BPT, QDT>;
    if (cudaFuncSetAttribute(redo, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem) != cudaSuccess)
        return LQ_ERR_CUDA;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return LQ_ERR_CUDA;
    const uint32_t n_cta = p.nct * n_heads;
    redo<<<std::min<uint32_t>(n_cta, (uint32_t)std::max(sms, 1)), 32 * p.nwarps, p.smem, st>>>(a, n_cta);
    return check_launch();
}

template <int G, int BPT>
int launch_partial_q(const AttnArgs &a, const AttnPlan &p, uint32_t n_heads, int q_dtype, cudaStream_t st) {
    switch (q_dtype) {
        case LQ_F32: return launch_partial<G, BPT, LQ_F32>(a, p, n_heads, st);
        case LQ_F16: return launch_partial<G, BPT, LQ_F16>(a, p, n_heads, st);
        case LQ_BF16: return launch_partial<G, BPT, LQ_BF16>(a, p, n_heads, st);
        default: return LQ_ERR_INVALID;
    }
}

template <int G>
int launch_partial_g(const AttnArgs &a, const AttnPlan &p, uint32_t n_heads, int q_dtype, int D, cudaStream_t st) {
    return D == 128 ? launch_partial_q<G, 16>(a, p, n_heads, q_dtype, st)
                    : launch_partial_q<G, 8>(a, p, n_heads, q_dtype, st);
}

bool view_ok(const lq_chunk_view *c) {
    return c && c->lane_off && c->lane_nbits && c->lane_state && c->coset_words && c->tile_n0 && c->tab_lo &&
           c->tab_nsym && c->tab_freq && c->dec_tab && c->scale_f16 && c->n_words >= 0 &&
           (c->n_words == 0 || c->words) && (reinterpret_cast<uintptr_t>(c->staged_tab) & 15) == 0;
}

ChunkDev to_dev(const lq_chunk_view *c) {
    const int64_t N = c->n_heads * c->bph;
    return ChunkDev{c->words,        (uint32_t)c->n_words, c->lane_off,          c->lane_nbits,
                    c->lane_state,   c->coset_words,       c->tile_n0,           (uint32_t)c->n_heads,
                    (uint32_t)c->bph, (uint32_t)c->tile_blocks, (uint32_t)ceil_div(N, c->tile_blocks), c->tab_lo,
                    c->tab_nsym,     c->tab_freq,          c->dec_tab,           c->scale_f16,
                    c->staged_tab};
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" size_t lq_attn_decode_workspace(int64_t n_heads, int64_t bph, int64_t tile_blocks, int group,
                                           int head_dim) {
    AttnPlan p;
    if (attn_plan(n_heads, bph, tile_blocks, group, head_dim, &p) != LQ_OK) return 0;
    return p.ws_bytes;
}

extern "C" int lq_attn_decode(const lq_chunk_view *k, const lq_chunk_view *v, const void *q, int q_dtype,
                              int64_t batch, int64_t n_kv_heads, int64_t seq_len, int scale_per_token, int group,
                              int head_dim, float sm_scale, void *out, int out_dtype, float *lse,
                              const uint32_t *tok_mask, void *workspace, size_t workspace_bytes, uint32_t *err,
                              void *stream) {
    LQ_NVTX_RANGE();
    if (!view_ok(k) || !view_ok(v) || !q || !out || !workspace || batch <= 0 || n_kv_heads <= 0 || seq_len <= 0)
        return LQ_ERR_INVALID;
    if (k->n_heads != v->n_heads || k->bph != v->bph || k->tile_blocks != v->tile_blocks) return LQ_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128) return LQ_ERR_INVALID;
    const int64_t heads = batch * n_kv_heads, bph = seq_len * (head_dim / 8);
    if (scale_per_token ? (k->n_heads != heads * seq_len || k->bph != head_dim / 8)
                        : (k->n_heads != heads || k->bph != bph))
        return LQ_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15)) return LQ_ERR_INVALID;
    if (!(sm_scale > 0.f) || !isfinite(sm_scale)) return LQ_ERR_INVALID;
    AttnPlan p;
    const int rc = attn_plan(heads, bph, k->tile_blocks, group, head_dim, &p);
    if (rc != LQ_OK) return rc;
    if (workspace_bytes < p.ws_bytes) return LQ_ERR_CAPACITY;
    if (out_dtype != LQ_F32 && out_dtype != LQ_F16 && out_dtype != LQ_BF16) return LQ_ERR_INVALID;
    cudaStream_t st = as_stream(stream);
    AttnArgs a;
    a.k = to_dev(k);
    a.v = to_dev(v);
    a.q = q;
    a.n_kv_heads = (uint32_t)n_kv_heads;
    a.seq = (uint32_t)seq_len;
    a.scale_tok = scale_per_token ? 1u : 0u;
    a.tph = p.tph;
    a.n_pairs = p.n_pairs;
    a.nct = p.nct;
    a.tpt = p.tpt;
    a.region0 = p.region0;
    a.warp_bytes = p.warp_bytes;
    a.qk_log2 = sm_scale * kLog2e;
    a.part = static_cast<float *>(workspace);
    a.tok_mask = tok_mask;
    a.redo = reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(workspace) + p.redo_off);
    a.err = err;
    const uint32_t nh = (uint32_t)heads;
    int r;
    switch (group) {
        case 1: r = launch_partial_g<1>(a, p, nh, q_dtype, head_dim, st); break;
        case 2: r = launch_partial_g<2>(a, p, nh, q_dtype, head_dim, st); break;
        case 3: r = launch_partial_g<3>(a, p, nh, q_dtype, head_dim, st); break;
        case 4: r = launch_partial_g<4>(a, p, nh, q_dtype, head_dim, st); break;
        case 5: r = launch_partial_g<5>(a, p, nh, q_dtype, head_dim, st); break;
        case 6: r = launch_partial_g<6>(a, p, nh, q_dtype, head_dim, st); break;
        case 7: r = launch_partial_g<7>(a, p, nh, q_dtype, head_dim, st); break;
        case 8: r = launch_partial_g<8>(a, p, nh, q_dtype, head_dim, st); break;
        default: return LQ_ERR_INVALID;
    }
    if (r != LQ_OK) return r;
    const unsigned rows = (unsigned)(heads * group);
    const float *part = a.part;
    const uint32_t hkv = (uint32_t)n_kv_heads, G = (uint32_t)group, D = (uint32_t)head_dim;
    return launch_attn_combine(part, rows, hkv, G, D, p.nct, out, out_dtype, lse, st);
}


extern "C" int lq_stage_tables(const uint32_t *dec_tab, const int32_t *tab_lo, int64_t n_tables, uint32_t *staged,
                               void *stream) {
    LQ_NVTX_RANGE();
    if (n_tables < 0 || n_tables > 0x7fffffff) return LQ_ERR_INVALID;
    if (n_tables == 0) return LQ_OK;
    if (!dec_tab || !tab_lo || !staged || (reinterpret_cast<uintptr_t>(staged) & 15)) return LQ_ERR_INVALID;
    staged_tables_kernel<<<(unsigned)n_tables, 256, 0, as_stream(stream)>>>(dec_tab, tab_lo, (uint32_t)n_tables, staged);
    return check_launch();
}
