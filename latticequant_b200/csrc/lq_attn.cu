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

#include "lq_tiledec.cuh"

namespace lq {
namespace {

constexpr int kAttnRing = 48;  // ring rows: rounds take 3-6 token groups of 16 blocks
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

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

template <int G>
__host__ __device__ constexpr int padded_g() {
    return (G + 3) & ~3;
}

template <int G, int BPT>
__host__ __device__ constexpr int attn_threads() {
    return G <= 2 ? 768 : G <= 4 ? 640 : 512;
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

    // query channels 8*dc .. 8*dc+7 of the G heads reading this kv head
    const uint32_t b = head / a.n_kv_heads, kvh = head % a.n_kv_heads;
    // as packed pairs of heads (g, g+1) for fma.rn.f32x2; an odd last head alone
    constexpr int GH = G / 2;
    unsigned long long q2[GH > 0 ? GH : 1][8];
    float qlast[8];
#pragma unroll
    for (int g = 0; g < G; g += 2) {
        const int64_t row = (int64_t)b * a.n_kv_heads * G + (int64_t)kvh * G + g;
        float x0[8], x1[8];
        load_block8<QDT>(a.q, row * BPT + dc, x0);
        if (g + 1 < G) {
            load_block8<QDT>(a.q, (row + 1) * BPT + dc, x1);
#pragma unroll
            for (int i = 0; i < 8; ++i) q2[g / 2][i] = f2_pack(x0[i], x1[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) qlast[i] = x0[i];
        }
    }

    // ---- phase K: scores
    // set when a lane of the CTA read past its bits (optimistic decode only)
    __shared__ uint32_t s_overrun;
    if (threadIdx.x == 0) s_overrun = 0u;
    stage_tables(a.k, 0, dtab);
    __syncthreads();
    if (wact) {
        auto epi_k = [&](bool ok, int t, uint32_t grp, uint32_t j, uint32_t cc, const uint4 blk) {
            float kq[8];
            ring_point(blk, kq);
            // per-lane partial dots over its 8 channels, i in order, two heads per fma.rn.f32x2
            float dot[G];
#pragma unroll
            for (int g = 0; g + 1 < G; g += 2) {
                unsigned long long s2 = f2_mul(q2[g / 2][0], f2_pack(kq[0], kq[0]));
#pragma unroll
                for (int i = 1; i < 8; ++i) s2 = f2_fma(q2[g / 2][i], f2_pack(kq[i], kq[i]), s2);
                f2_unpack(s2, dot[g], dot[g + 1]);
            }
            if constexpr (G % 2) {
                float s = __fmul_rn(qlast[0], kq[0]);
#pragma unroll
                for (int i = 1; i < 8; ++i) s = __fmaf_rn(qlast[i], kq[i], s);
                dot[G - 1] = s;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) dot[g] = ok ? dot[g] : 0.f;
            const uint32_t jc = j % BPT;
            const uint32_t tok = grp * TPG + j / BPT;
            float *row = sc + ((uint32_t)t * a.tpt + tok) * GP;
            if constexpr (G == 4 && BPT == 16) {
                // transposing reduction over the token's 16 lanes: halve the
                // heads a lane carries at each of the first two steps
                const bool h8 = (jc & 8u) != 0, h4 = (jc & 4u) != 0;
                float a0 = h8 ? dot[2] : dot[0], a1 = h8 ? dot[3] : dot[1];
                const float s0 = h8 ? dot[0] : dot[2], s1 = h8 ? dot[1] : dot[3];
                a0 += __shfl_xor_sync(0xffffffffu, s0, 8);
                a1 += __shfl_xor_sync(0xffffffffu, s1, 8);
                float bsum = h4 ? a1 : a0;
                bsum += __shfl_xor_sync(0xffffffffu, h4 ? a0 : a1, 4);
                bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
                bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
                // lane jc holds head (jc >> 2) & 3 (bit 3 picked heads 2-3, bit 2 the odd one)
                if (ok && (jc & 3u) == 0) row[jc >> 2] = bsum;
            } else {
#pragma unroll
                for (int off = BPT / 2; off >= 1; off >>= 1) {
#pragma unroll
                    for (int g = 0; g < G; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], off);
                }
                if (ok && jc < (uint32_t)G) {
                    float v = dot[0];
#pragma unroll
                    for (int g = 1; g < G; ++g) v = (jc == (uint32_t)g) ? dot[g] : v;
                    row[jc] = v;
                }
            }
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
    stage_tables(a.v, 0, dtab);
    __syncthreads();
    // p * v accumulated as packed channel pairs (i, i+1) per head
    unsigned long long acc2[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2[g][i] = 0ull;
    if (wact) {
        auto epi_v = [&](bool ok, int t, uint32_t grp, uint32_t j, uint32_t cc, const uint4 blk) {
            if (!ok) return;
            float vq[8];
            ring_point(blk, vq);
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
            unsigned long long v2[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v2[i] = f2_pack(vq[2 * i], vq[2 * i + 1]);
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

// ---------------------------------------------------------------- compact layout
// Decode attention straight from the compact fixed-rate layout
// (core/compact_storage.py:87-222; the reference merges it into an fp16
// buffer for SDPA, llm/fused_triton_merge.py:33-177).  A block is either
// representable -- `bits` bytes big-endian [coset | u0..u6 | u7 >> 1] -- or
// an fp16 fallback row (already scaled).  Its place in either array follows
// from a bit per block and the count of representable blocks before each
// 32-block word, so a warp step covering 32 consecutive blocks (2 tokens of
// head_dim 128, 4 of 64) finds every lane's block with one popcount.
// Nothing is serial per block, so the kernel streams HBM.
struct CompactDev {
    const uint8_t *packed;
    const uint4 *fallback;
    const uint32_t *mask_words;
    const int32_t *word_rank;
    const float *scales;
    uint32_t n_repr, n_fallback, n_words;
    int bits;
};

struct CompactArgs {
    CompactDev k, v;
    const void *q;
    uint32_t n_kv_heads, seq, bph;
    uint32_t nct, tok_per_cta;
    float qk_log2;
    float *part;
    uint32_t *err;
};

constexpr int kCompactThreads = 512;
constexpr int kCompactWarps = kCompactThreads / 32;
constexpr int kCStageTok = 128;     // tokens per shared-memory stage (two CTAs fit an SM)
constexpr int kCTokPerCta = 1024;   // tokens per CTA (4 stages)

// Shared-memory stage of one chunk's blocks of kCStageTok tokens: mask words,
// their ranks, the representable codes (from a 16-byte-aligned start) and the
// fallback rows, copied in with cp.async.
template <int BPT>
struct CStage {
    static constexpr int kBlocks = kCStageTok * BPT, kWords = kBlocks / 32;
    static constexpr int kPackedBytes = (kBlocks * 5 + 16 + 15) & ~15;  // bits <= 5, + alignment slack
    static constexpr int kWordsOff = 0, kRanksOff = kWords * 4, kPackedOff = kWords * 8;
    static constexpr int kFallbackOff = kPackedOff + kPackedBytes;
    static constexpr int kBytes = kFallbackOff + kBlocks * 16;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Where a stage's data starts in the chunk's arrays.
struct CStageSpan {
    uint32_t w0, nw;       // first mask word, words
    uint32_t r0, r1;       // representable blocks before the stage / after it
    uint32_t a0;           // byte of the packed array the staged copy starts at (16-byte aligned)
    bool bad;              // ranks inconsistent with the arrays: nothing is copied, blocks read as zeros
};

__device__ __forceinline__ CStageSpan cstage_span(const CompactDev &c, uint32_t b0, uint32_t b1) {
    CStageSpan s;
    s.w0 = b0 >> 5;
    s.nw = (b1 - b0) >> 5;
    s.r0 = (uint32_t)__ldg(c.word_rank + s.w0);
    s.r1 = s.w0 + s.nw < c.n_words ? (uint32_t)__ldg(c.word_rank + s.w0 + s.nw) : c.n_repr;
    s.a0 = (s.r0 * (uint32_t)c.bits) & ~15u;
    s.bad = !(s.r0 <= s.r1 && s.r1 - s.r0 <= 32u * s.nw && s.r1 <= c.n_repr && b0 >= s.r0 &&
              b0 + 32u * s.nw - s.r1 <= c.n_fallback);
    return s;
}

// All threads: copy one stage into shared memory at `buf` (and commit).
template <int BPT>
__device__ __forceinline__ void cstage_issue(const CompactDev &c, const CStageSpan &s, uint32_t b0, uint32_t buf) {
    using S = CStage<BPT>;
    if (s.bad) {  // the blocks raise the flag when read
        cp_async_commit();
        return;
    }
    for (uint32_t i = threadIdx.x; i < s.nw; i += blockDim.x) {
        cp_async4(buf + S::kWordsOff + 4 * i, c.mask_words + s.w0 + i);
        cp_async4(buf + S::kRanksOff + 4 * i, c.word_rank + s.w0 + i);
    }
    const uint32_t total = c.n_repr * (uint32_t)c.bits, a1 = s.r1 * (uint32_t)c.bits;
    for (uint32_t off = s.a0 + 16u * threadIdx.x; off < a1; off += 16u * blockDim.x)
        cp_async16(buf + S::kPackedOff + (off - s.a0), c.packed + off, min(16u, total - off));
    const uint32_t f0 = b0 - s.r0, f1 = b0 + 32u * s.nw - s.r1;
    for (uint32_t r = f0 + threadIdx.x; r < f1; r += blockDim.x)
        cp_async16(buf + S::kFallbackOff + 16u * (r - f0), c.fallback + r, 16u);
    cp_async_commit();
}

// The lane's block of a warp step from a stage: 32 consecutive blocks =
// mask word `wi` of the stage.  For a representable block the scale-free E8
// point (u - R + coset/2, coordinate 7 with the parity bit of the other
// seven) and sc = the head scale; for a fallback row its fp16 values, sc = 1.
template <int BPT, bool B4>
__device__ __forceinline__ void cstage_block(const CompactDev &c, const CStageSpan &s, uint32_t buf, uint32_t wi,
                                             uint32_t lane, float head_scale, float x[8], float &sc, uint32_t *err) {
    using S = CStage<BPT>;
    // The stage's index was validated when it arrived (a mismatch raised the
    // flag); here every index is only clamped into the staged arrays, so a
    // damaged chunk reads garbage values but never outside shared memory.
    (void)err;
    const uint32_t w = lds_u32(buf + S::kWordsOff + 4 * wi);
    const uint32_t r0 = lds_u32(buf + S::kRanksOff + 4 * wi);
    const uint32_t below = __popc(w & ((1u << lane) - 1u));
    if ((w >> lane) & 1u) {
        // stage-relative rank, compared unsigned: a rank below the stage's wraps
        uint32_t pr = r0 + below - s.r0;
        pr = pr < (s.bad ? 0u : s.r1 - s.r0) ? pr : 0u;
        const int b = B4 ? 4 : c.bits, R = 1 << (b - 1);
        uint32_t u[7], c7u, coset, par;
        const uint32_t pbyte = s.bad ? 0u : pr * (uint32_t)b + (s.r0 * (uint32_t)b - s.a0);  // byte in the staged codes
        if constexpr (B4) {
            const uint32_t v = __byte_perm(lds_u32(buf + S::kPackedOff + pbyte), 0u, 0x0123u);
            coset = v >> 31;
#pragma unroll
            for (int i = 0; i < 7; ++i) u[i] = (v >> (27 - 4 * i)) & 15u;
            c7u = v & 7u;
            par = __popc(v & 0x08888888u) & 1u;  // low bits of u0..u6
        } else {
            const uint32_t o = buf + S::kPackedOff + pbyte;
            uint64_t acc = 0;
            for (int i = 0; i < b; ++i) acc = (acc << 8) | (lds_u32((o + i) & ~3u) >> (8 * ((o + i) & 3u)) & 0xffu);
            c7u = (uint32_t)(acc & ((1ull << (b - 1)) - 1));
            acc >>= (b - 1);
            par = 0;
#pragma unroll
            for (int i = 6; i >= 0; --i) {
                u[i] = (uint32_t)(acc & ((1ull << b) - 1));
                par ^= u[i];
                acc >>= b;
            }
            par &= 1u;
            coset = (uint32_t)(acc & 1u);
        }
        // u - R + coset/2 exactly: 2u + coset in the mantissa of 2^22 (spacing
        // 1/2) reads 2^22 + u + coset/2; 2^22 + R is exact, so is the difference
        const uint32_t base = 0x4A800000u | coset;
        const float bias = 4194304.0f + (float)R;
#pragma unroll
        for (int i = 0; i < 7; ++i) x[i] = __int_as_float((u[i] << 1) | base) - bias;
        // coordinate 7 = 2*c7u + parity(sum of the signed others) - R; R is even, so that parity is par
        x[7] = __int_as_float(((2u * c7u + par) << 1) | base) - bias;
        sc = head_scale;
    } else {
        // fallback rows before this block: the stage's first row is b0 - r0 of the chunk
        uint32_t f = 32u * wi + lane - below - (r0 - s.r0);
        f = f < (s.bad ? 0u : 32u * s.nw - (s.r1 - s.r0)) ? f : 0u;
        const uint4 h = lds_v4(buf + S::kFallbackOff + 16u * f);
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&hw[i]));
            x[2 * i] = f2.x;
            x[2 * i + 1] = f2.y;
        }
        sc = 1.f;
    }
}

template <int G, int BPT, int QDT, bool B4>
__global__ void __launch_bounds__(kCompactThreads, G <= 4 ? 2 : 1) attn_compact_kernel(CompactArgs a) {
    static_assert(BPT == 8 || BPT == 16, "head_dim 64 or 128");
    using S = CStage<BPT>;
    constexpr int D = 8 * BPT, GP = padded_g<G>(), TPS = 32 / BPT;  // tokens per warp step
    constexpr int kWarpTok = kCStageTok / kCompactWarps;           // tokens of a warp per stage
    constexpr int kSteps = kWarpTok / TPS;
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31, dc = lane % BPT, tl = lane / BPT;
    const uint32_t head = blockIdx.y;
    const uint32_t T0 = blockIdx.x * a.tok_per_cta, T1 = min(T0 + a.tok_per_cta, a.seq);
    const uint32_t nst = (T1 - T0 + kCStageTok - 1) / kCStageTok;
    float *sc = reinterpret_cast<float *>(smem);  // [tok_per_cta][GP]
    const uint32_t bufs = smem_addr(smem + (size_t)kCTokPerCta * GP * 4);
    const uint32_t b = head / a.n_kv_heads, kvh = head % a.n_kv_heads;
    const float sk = a.k.scales[head], sv = a.v.scales[head];
    const uint32_t hb0 = head * a.bph;
    auto stage_blocks = [&](uint32_t st, uint32_t &b0, uint32_t &b1) {
        const uint32_t t0 = T0 + st * kCStageTok, t1 = min(t0 + kCStageTok, T1);
        b0 = hb0 + t0 * BPT;
        b1 = hb0 + t1 * BPT;
    };

    constexpr int GH = G / 2;
    unsigned long long q2[GH > 0 ? GH : 1][8];
    float qlast[8];
#pragma unroll
    for (int g = 0; g < G; g += 2) {
        const int64_t row = (int64_t)b * a.n_kv_heads * G + (int64_t)kvh * G + g;
        float x0[8], x1[8];
        load_block8<QDT>(a.q, row * BPT + dc, x0);
        if (g + 1 < G) {
            load_block8<QDT>(a.q, (row + 1) * BPT + dc, x1);
#pragma unroll
            for (int i = 0; i < 8; ++i) q2[g / 2][i] = f2_pack(x0[i], x1[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) qlast[i] = x0[i];
        }
    }

    // where every stage of both phases starts in the chunks' arrays, read
    // once (8 threads in parallel) so no copy waits for a rank load
    constexpr int kMaxStages = kCTokPerCta / kCStageTok;
    __shared__ CStageSpan spans[2][kMaxStages];
    if (threadIdx.x < 2 * kMaxStages) {
        const uint32_t ph = threadIdx.x / kMaxStages, st = threadIdx.x % kMaxStages;
        if (st < nst) {
            uint32_t b0, b1;
            stage_blocks(st, b0, b1);
            spans[ph][st] = cstage_span(ph ? a.v : a.k, b0, b1);
        }
    }
    __syncthreads();

    // one phase (K or V) over the CTA's stages, double-buffered
    auto phase = [&](const CompactDev &c, const CStageSpan *sp, auto &&body) {
        uint32_t b0, b1;
        stage_blocks(0, b0, b1);
        cstage_issue<BPT>(c, sp[0], b0, bufs);
        if (nst > 1) {
            stage_blocks(1, b0, b1);
            cstage_issue<BPT>(c, sp[1], b0, bufs + S::kBytes);
        }
        for (uint32_t st = 0; st < nst; ++st) {
            if (st + 1 < nst) cp_async_wait<1>();
            else cp_async_wait<0>();
            __syncthreads();
            const uint32_t buf = bufs + (st & 1u) * S::kBytes;
            const CStageSpan s = sp[st];
            // the stage's index must chain: rank(w+1) - rank(w) = popcount(word w),
            // from the stage's first rank to its last
            if (s.bad && threadIdx.x == 0) raise_flag(a.err, LQ_EF_BITSTREAM);
            for (uint32_t i = threadIdx.x; i < s.nw && !s.bad; i += blockDim.x) {
                const uint32_t ri = lds_u32(buf + S::kRanksOff + 4 * i);
                const uint32_t rn = i + 1 < s.nw ? lds_u32(buf + S::kRanksOff + 4 * (i + 1)) : s.r1;
                if (rn - ri != (uint32_t)__popc(lds_u32(buf + S::kWordsOff + 4 * i)) || (i == 0 && ri != s.r0))
                    raise_flag(a.err, LQ_EF_BITSTREAM);
            }
            const uint32_t t0 = T0 + st * kCStageTok;
            // the warp's steps in this stage (sequence lengths are whole steps,
            // so every token of a step taken is in range)
            const uint32_t tw = t0 + (uint32_t)(warp * kWarpTok);
            const int nsteps = tw >= T1 ? 0 : (int)min((uint32_t)kSteps, (T1 - tw) / TPS);
#pragma unroll 2
            for (int j = 0; j < nsteps; ++j) {
                const uint32_t tb = tw + (uint32_t)(j * TPS);  // step's first token
                const uint32_t wi = (uint32_t)(warp * kWarpTok + j * TPS) * BPT / 32u;
                body(s, buf, wi, tb + tl, true);
            }
            __syncthreads();
            if (st + 2 < nst) {
                stage_blocks(st + 2, b0, b1);
                cstage_issue<BPT>(c, sp[st + 2], b0, buf);
            }
        }
    };

    // ---- phase K: scores (base 2) of the CTA's tokens into shared memory
    phase(a.k, spans[0], [&](const CStageSpan &s, uint32_t buf, uint32_t wi, uint32_t tok, bool ok) {
        float kx[8], scl;
        cstage_block<BPT, B4>(a.k, s, buf, wi, lane, sk, kx, scl, a.err);
        float dot[G];
#pragma unroll
        for (int g = 0; g + 1 < G; g += 2) {
            unsigned long long s2 = f2_mul(q2[g / 2][0], f2_pack(kx[0], kx[0]));
#pragma unroll
            for (int i = 1; i < 8; ++i) s2 = f2_fma(q2[g / 2][i], f2_pack(kx[i], kx[i]), s2);
            f2_unpack(s2, dot[g], dot[g + 1]);
        }
        if constexpr (G % 2) {
            float d = __fmul_rn(qlast[0], kx[0]);
#pragma unroll
            for (int i = 1; i < 8; ++i) d = __fmaf_rn(qlast[i], kx[i], d);
            dot[G - 1] = d;
        }
        const float f = ok ? scl * a.qk_log2 : 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) dot[g] *= f;
        float *row = sc + (tok - T0) * GP;
        if constexpr (G == 4 && BPT == 16) {
            // transposing reduction over the token's 16 lanes (as in the rANS kernel)
            const bool h8 = (dc & 8u) != 0, h4 = (dc & 4u) != 0;
            float a0 = h8 ? dot[2] : dot[0], a1 = h8 ? dot[3] : dot[1];
            const float s0 = h8 ? dot[0] : dot[2], s1 = h8 ? dot[1] : dot[3];
            a0 += __shfl_xor_sync(0xffffffffu, s0, 8);
            a1 += __shfl_xor_sync(0xffffffffu, s1, 8);
            float bsum = h4 ? a1 : a0;
            bsum += __shfl_xor_sync(0xffffffffu, h4 ? a0 : a1, 4);
            bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
            bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
            if (ok && (dc & 3u) == 0) row[dc >> 2] = bsum;
        } else {
#pragma unroll
            for (int off = BPT / 2; off >= 1; off >>= 1) {
#pragma unroll
                for (int g = 0; g < G; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], off);
            }
            if (ok && dc < (uint32_t)G) {
                float v = dot[0];
#pragma unroll
                for (int g = 1; g < G; ++g) v = (dc == (uint32_t)g) ? dot[g] : v;
                row[dc] = v;
            }
        }
    });

    // ---- softmax statistics of the warp's tokens (its kWarpTok of each stage)
    __syncwarp();
    auto tok_rel = [&](uint32_t i) {  // i-th token of this warp, relative to T0
        return (i / kWarpTok) * kCStageTok + (uint32_t)warp * kWarpTok + i % kWarpTok;
    };
    const uint32_t nmine = nst * kWarpTok;
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
    }
    for (uint32_t i = lane; i < nmine; i += 32) {
        const uint32_t t = tok_rel(i);
        if (T0 + t >= T1) continue;
#pragma unroll
        for (int g = 0; g < G; ++g) m[g] = fmaxf(m[g], sc[t * GP + g]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], off));
    }
    for (uint32_t i = lane; i < nmine; i += 32) {
        const uint32_t t = tok_rel(i);
        if (T0 + t >= T1) continue;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float p = exp2f(sc[t * GP + g] - m[g]);
            sc[t * GP + g] = p;
            l[g] += p;
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
    }
    __syncwarp();

    // ---- phase V: p * v per lane over its 8 channels
    unsigned long long acc2[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2[g][i] = 0ull;
    phase(a.v, spans[1], [&](const CStageSpan &s, uint32_t buf, uint32_t wi, uint32_t tok, bool ok) {
        float vx[8], scl;
        cstage_block<BPT, B4>(a.v, s, buf, wi, lane, sv, vx, scl, a.err);
        if (!ok) return;
        const float *pp = sc + (tok - T0) * GP;
        unsigned long long v2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v2[i] = f2_pack(vx[2 * i], vx[2 * i + 1]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float pg = pp[g] * scl;
            const unsigned long long p2 = f2_pack(pg, pg);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc2[g][i] = f2_fma(p2, v2[i], acc2[g][i]);
        }
    });
    float acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) f2_unpack(acc2[g][i], acc[g][2 * i], acc[g][2 * i + 1]);
    // lanes holding the same channels: the other tokens of a step
#pragma unroll
    for (int off = 16; off >= BPT; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[g][i] += __shfl_xor_sync(0xffffffffu, acc[g][i], off);
    }

    // ---- merge the warps in a fixed order (the stage buffers are done with)
    float *mrg = reinterpret_cast<float *>(smem + (size_t)kCTokPerCta * GP * 4);
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
    float *out = a.part + ((size_t)head * a.nct + blockIdx.x) * G * rs;
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int g = e / D, dd = e % D;
        float mx = -INFINITY;
        for (int w = 0; w < kCompactWarps; ++w) mx = fmaxf(mx, mrg[(w * G + g) * rs + D]);
        float o = 0.f, ls = 0.f;
        for (int w = 0; w < kCompactWarps; ++w) {
            const float mw = mrg[(w * G + g) * rs + D];
            if (mw == -INFINITY) continue;
            const float f = exp2f(mw - mx);
            o = fmaf(mrg[(w * G + g) * rs + dd], f, o);
            ls = fmaf(mrg[(w * G + g) * rs + D + 1], f, ls);
        }
        out[g * rs + dd] = o;
        if (dd == 0) {
            out[g * rs + D] = mx;
            out[g * rs + D + 1] = ls;
        }
    }
}

// One block per query row: merge the head's CTA partials into o = O / L and
// lse = ln(sum exp(s)) (natural log of the unnormalised softmax mass).
template <int ODT>
__global__ void attn_combine_kernel(const float *__restrict__ part, uint32_t n_kv_heads, uint32_t G, uint32_t D,
                                    uint32_t nct, void *__restrict__ out, float *__restrict__ lse) {
    const uint32_t row = blockIdx.x;  // head * G + g
    const uint32_t head = row / G, g = row % G;
    const uint32_t b = head / n_kv_heads, kvh = head % n_kv_heads;
    const uint32_t orow = (b * n_kv_heads + kvh) * G + g;  // (b, q-head) with q-head = kvh * G + g
    const size_t rs = D + 2;
    const float *p = part + (size_t)head * nct * G * rs + (size_t)g * rs;
    float mx = -INFINITY;
    for (uint32_t c = 0; c < nct; ++c) mx = fmaxf(mx, p[(size_t)c * G * rs + D]);
    float ls = 0.f;
    for (uint32_t c = 0; c < nct; ++c) {
        const float mc = p[(size_t)c * G * rs + D];
        if (mc != -INFINITY) ls = fmaf(p[(size_t)c * G * rs + D + 1], exp2f(mc - mx), ls);
    }
    const float inv = 1.f / ls;
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
        for (uint32_t c = 0; c < nct; ++c) {
            const float mc = p[(size_t)c * G * rs + D];
            if (mc != -INFINITY) o = fmaf(p[(size_t)c * G * rs + d], exp2f(mc - mx), o);
        }
        Elem<ODT>::store(out, (int64_t)orow * D + d, o * inv);
    }
    if (lse && threadIdx.x == 0) lse[orow] = (mx + log2f(ls)) * kLn2;
}

// Merge of attention parts over disjoint key sets (sequence shards, chunks):
// o = sum_i o_i exp(lse_i - lse), lse = log sum_i exp(lse_i).
template <int ODT>
__global__ void attn_merge_kernel(const float *__restrict__ o_parts, const float *__restrict__ lse_parts,
                                  int64_t n_parts, int64_t rows, uint32_t D, void *__restrict__ out,
                                  float *__restrict__ lse) {
    const int64_t row = blockIdx.x;
    float mx = -INFINITY;
    for (int64_t i = 0; i < n_parts; ++i) mx = fmaxf(mx, lse_parts[i * rows + row]);
    float ls = 0.f;
    for (int64_t i = 0; i < n_parts; ++i) {
        const float li = lse_parts[i * rows + row];
        if (li != -INFINITY) ls += exp2f((li - mx) * kLog2e);
    }
    const float inv = 1.f / ls;
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
        for (int64_t i = 0; i < n_parts; ++i) {
            const float li = lse_parts[i * rows + row];
            if (li != -INFINITY) o = fmaf(o_parts[(i * rows + row) * D + d], exp2f((li - mx) * kLog2e), o);
        }
        Elem<ODT>::store(out, row * D + d, o * inv);
    }
    if (lse && threadIdx.x == 0) lse[row] = mx + log2f(ls) * kLn2;
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

// ---- compact-layout attention: plan and launch
struct CompactPlan {
    uint32_t nct, tok_per_cta;
    size_t smem, part_floats;
};

int compact_plan(int64_t n_heads, int64_t seq, int G, int D, CompactPlan *p) {
    if (n_heads <= 0 || seq <= 0 || G < 1 || G > 8 || (D != 64 && D != 128)) return LQ_ERR_INVALID;
    const int bpt = D / 8;
    if ((seq * bpt) % 32 != 0 || n_heads > 65535 || n_heads * seq * bpt >= ((int64_t)1 << 31)) return LQ_ERR_INVALID;
    p->tok_per_cta = kCTokPerCta;
    p->nct = (uint32_t)ceil_div(seq, p->tok_per_cta);
    const size_t gp = (size_t)((G + 3) & ~3);
    const size_t stages = 2 * (size_t)(bpt == 16 ? CStage<16>::kBytes : CStage<8>::kBytes);
    const size_t merge = (size_t)kCompactWarps * G * (D + 2) * 4;
    p->smem = (size_t)kCTokPerCta * gp * 4 + std::max(stages, merge);
    p->part_floats = (size_t)n_heads * p->nct * G * (D + 2);
    return LQ_OK;
}

template <int G, int BPT, int QDT, bool B4>
int launch_compact(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, cudaStream_t st) {
    auto kern = attn_compact_kernel<G, BPT, QDT, B4>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem) != cudaSuccess)
        return LQ_ERR_CUDA;
    kern<<<dim3(p.nct, n_heads), kCompactThreads, p.smem, st>>>(a);
    return check_launch();
}

template <int G, int BPT>
int launch_compact_q(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, int q_dtype, cudaStream_t st) {
    const bool b4 = a.k.bits == 4 && a.v.bits == 4;
    switch (q_dtype) {
        case LQ_F32:
            return b4 ? launch_compact<G, BPT, LQ_F32, true>(a, p, n_heads, st)
                      : launch_compact<G, BPT, LQ_F32, false>(a, p, n_heads, st);
        case LQ_F16:
            return b4 ? launch_compact<G, BPT, LQ_F16, true>(a, p, n_heads, st)
                      : launch_compact<G, BPT, LQ_F16, false>(a, p, n_heads, st);
        case LQ_BF16:
            return b4 ? launch_compact<G, BPT, LQ_BF16, true>(a, p, n_heads, st)
                      : launch_compact<G, BPT, LQ_BF16, false>(a, p, n_heads, st);
        default: return LQ_ERR_INVALID;
    }
}

template <int G>
int launch_compact_g(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, int q_dtype, int D, cudaStream_t st) {
    return D == 128 ? launch_compact_q<G, 16>(a, p, n_heads, q_dtype, st)
                    : launch_compact_q<G, 8>(a, p, n_heads, q_dtype, st);
}

bool compact_ok(const lq_compact_view *c, int64_t n_heads, int64_t bph) {
    if (!c || !c->mask_words || !c->word_rank || !c->scales || c->n_heads != n_heads || c->bph != bph) return false;
    if (c->bits < 3 || c->bits > 5 || c->n_repr < 0 || c->n_fallback < 0) return false;
    if (c->n_repr + c->n_fallback != n_heads * bph) return false;
    if (c->n_repr > 0 && (!c->packed || (reinterpret_cast<uintptr_t>(c->packed) & 15))) return false;
    if (c->n_fallback > 0 && (!c->fallback || (reinterpret_cast<uintptr_t>(c->fallback) & 15))) return false;
    if ((reinterpret_cast<uintptr_t>(c->mask_words) & 3) || (reinterpret_cast<uintptr_t>(c->word_rank) & 3))
        return false;
    return c->n_repr * c->bits < 0xffffffffLL;
}

CompactDev to_compact(const lq_compact_view *c) {
    return CompactDev{c->packed,
                      reinterpret_cast<const uint4 *>(c->fallback),
                      c->mask_words,
                      c->word_rank,
                      c->scales,
                      (uint32_t)c->n_repr,
                      (uint32_t)c->n_fallback,
                      (uint32_t)ceil_div(c->n_heads * c->bph, 32),
                      c->bits};
}

bool view_ok(const lq_chunk_view *c) {
    return c && c->lane_off && c->lane_nbits && c->lane_state && c->coset_words && c->tile_n0 && c->tab_lo &&
           c->tab_nsym && c->tab_freq && c->dec_tab && c->scale_f16 && c->n_words >= 0 && (c->n_words == 0 || c->words);
}

ChunkDev to_dev(const lq_chunk_view *c) {
    const int64_t N = c->n_heads * c->bph;
    return ChunkDev{c->words,        (uint32_t)c->n_words, c->lane_off,          c->lane_nbits,
                    c->lane_state,   c->coset_words,       c->tile_n0,           (uint32_t)c->n_heads,
                    (uint32_t)c->bph, (uint32_t)c->tile_blocks, (uint32_t)ceil_div(N, c->tile_blocks), c->tab_lo,
                    c->tab_nsym,     c->tab_freq,          c->dec_tab,           c->scale_f16};
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
    if (out_dtype == LQ_F32) attn_combine_kernel<LQ_F32><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    else if (out_dtype == LQ_F16) attn_combine_kernel<LQ_F16><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    else attn_combine_kernel<LQ_BF16><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    return check_launch();
}

extern "C" size_t lq_attn_compact_workspace(int64_t n_heads, int64_t seq_len, int group, int head_dim) {
    CompactPlan p;
    if (compact_plan(n_heads, seq_len, group, head_dim, &p) != LQ_OK) return 0;
    return (p.part_floats * 4 + 255) & ~(size_t)255;
}

extern "C" int lq_attn_decode_compact(const lq_compact_view *k, const lq_compact_view *v, const void *q, int q_dtype,
                                      int64_t batch, int64_t n_kv_heads, int64_t seq_len, int group, int head_dim,
                                      float sm_scale, void *out, int out_dtype, float *lse, void *workspace,
                                      size_t workspace_bytes, uint32_t *err, void *stream) {
    if (!q || !out || !workspace || batch <= 0 || n_kv_heads <= 0 || seq_len <= 0) return LQ_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128) return LQ_ERR_INVALID;
    const int64_t heads = batch * n_kv_heads, bph = seq_len * (head_dim / 8);
    if (!compact_ok(k, heads, bph) || !compact_ok(v, heads, bph)) return LQ_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15)) return LQ_ERR_INVALID;
    if (!(sm_scale > 0.f) || !isfinite(sm_scale)) return LQ_ERR_INVALID;
    if (out_dtype != LQ_F32 && out_dtype != LQ_F16 && out_dtype != LQ_BF16) return LQ_ERR_INVALID;
    CompactPlan p;
    const int rc = compact_plan(heads, seq_len, group, head_dim, &p);
    if (rc != LQ_OK) return rc;
    if (workspace_bytes < p.part_floats * 4) return LQ_ERR_CAPACITY;
    cudaStream_t st = as_stream(stream);
    CompactArgs a;
    a.k = to_compact(k);
    a.v = to_compact(v);
    a.q = q;
    a.n_kv_heads = (uint32_t)n_kv_heads;
    a.seq = (uint32_t)seq_len;
    a.bph = (uint32_t)bph;
    a.nct = p.nct;
    a.tok_per_cta = p.tok_per_cta;
    a.qk_log2 = sm_scale * kLog2e;
    a.part = static_cast<float *>(workspace);
    a.err = err;
    const uint32_t nh = (uint32_t)heads;
    int r;
    switch (group) {
        case 1: r = launch_compact_g<1>(a, p, nh, q_dtype, head_dim, st); break;
        case 2: r = launch_compact_g<2>(a, p, nh, q_dtype, head_dim, st); break;
        case 3: r = launch_compact_g<3>(a, p, nh, q_dtype, head_dim, st); break;
        case 4: r = launch_compact_g<4>(a, p, nh, q_dtype, head_dim, st); break;
        case 5: r = launch_compact_g<5>(a, p, nh, q_dtype, head_dim, st); break;
        case 6: r = launch_compact_g<6>(a, p, nh, q_dtype, head_dim, st); break;
        case 7: r = launch_compact_g<7>(a, p, nh, q_dtype, head_dim, st); break;
        case 8: r = launch_compact_g<8>(a, p, nh, q_dtype, head_dim, st); break;
        default: return LQ_ERR_INVALID;
    }
    if (r != LQ_OK) return r;
    const unsigned rows = (unsigned)(heads * group);
    const float *part = a.part;
    const uint32_t hkv = (uint32_t)n_kv_heads, G = (uint32_t)group, D = (uint32_t)head_dim;
    if (out_dtype == LQ_F32) attn_combine_kernel<LQ_F32><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    else if (out_dtype == LQ_F16) attn_combine_kernel<LQ_F16><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    else attn_combine_kernel<LQ_BF16><<<rows, D, 0, st>>>(part, hkv, G, D, p.nct, out, lse);
    return check_launch();
}

extern "C" int lq_attn_merge(const float *o_parts, const float *lse_parts, int64_t n_parts, int64_t rows,
                             int head_dim, void *out, int out_dtype, float *lse, void *stream) {
    if (n_parts < 0 || rows < 0 || head_dim <= 0 || head_dim > 1024) return LQ_ERR_INVALID;
    if (n_parts == 0 || rows == 0) return n_parts == 0 && rows > 0 ? LQ_ERR_INVALID : LQ_OK;
    if (!o_parts || !lse_parts || !out || rows > 0x7fffffff) return LQ_ERR_INVALID;
    cudaStream_t st = as_stream(stream);
    const unsigned tb = head_dim < 128 ? (unsigned)head_dim : 128u;
    if (out_dtype == LQ_F32)
        attn_merge_kernel<LQ_F32><<<(unsigned)rows, tb, 0, st>>>(o_parts, lse_parts, n_parts, rows, head_dim, out, lse);
    else if (out_dtype == LQ_F16)
        attn_merge_kernel<LQ_F16><<<(unsigned)rows, tb, 0, st>>>(o_parts, lse_parts, n_parts, rows, head_dim, out, lse);
    else if (out_dtype == LQ_BF16)
        attn_merge_kernel<LQ_BF16><<<(unsigned)rows, tb, 0, st>>>(o_parts, lse_parts, n_parts, rows, head_dim, out,
                                                                  lse);
    else
        return LQ_ERR_INVALID;
    return check_launch();
}
