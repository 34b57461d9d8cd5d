// lq_attn_compact.cu -- decode attention over the compact fixed-rate layout.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "lq_attn_common.cuh"

namespace lq {
namespace {

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

// ------------------------------------------------------ tensor-core path
// The same attention for head_dim 128 and query groups of at most 4 heads,
// with q.k and p.v on the tensor cores: mma.sync m16n8k16 with fp16 operands
// and fp32 accumulation, fed straight from the registers the blocks are
// decoded into (the decoded values never go through shared memory).
//
// Operand values.  A head's representable blocks are q * s (q the E8 point,
// s the fp32 head scale), its fallback rows fp16 values.  One MMA needs one
// common unit, u = s * 2^k (k = max(0, 1 - exponent of s), so u >= 1 when
// s < 1): the representable blocks enter as q / 2^k -- half-integers of at
// most 6 significant bits, exact in fp16 -- and the staged fallback rows are
// multiplied by 1/u in fp32 once per stage and rounded to fp16 (one rounding,
// at most 2^-11 relative, on the blocks that are fp16 already); scores and
// outputs are multiplied by u afterwards.  q (bf16/fp16/fp32 query) enters
// as fp16, p = 2^(s - m) in [0, 1] as fp16; l sums the fp32 p.
//
// 4-bit codes decode without floating-point conversions: w = (v << 1) |
// parity puts u0..u6 and 2*c7u + parity in the eight nibbles of a word, a
// byte permute + mask places two nibbles (times 16) in the mantissas of the
// fp16 pair (1024, 1024), and one fp16x2 FMA, (1024 + 16 n) * 2^-(4+k) +
// (-72 + c/2) * 2^-k, gives (n - 8 + c/2) * 2^-k exactly.
//
// Fragments.  Phase K, per group of 8 tokens: A rows are (token, half) and
// columns channels, so lane (g, t) = (lane / 4, lane % 4) holds exactly one
// block -- token g, block 4 ks + t of k-step ks -- as its four A registers
// (channels 0-3 in the row of half 0, 4-7 in the row of half 1); B columns
// are (query head h, half j) holding q[h] at the matching channels, and the
// score of (g, h) is D[(g,0)][h] + D[(g,1)][4 + h] (one shuffle).  Phase V,
// per group of 16 tokens: A = V^T (rows channels, columns tokens); lane
// (g, t) decodes blocks 2g and 2g+1 of tokens 2t, 2t+1, 2t+8, 2t+9 and pairs
// their channels across tokens with byte permutes; B = p^T.
// Four CTAs of 4 warps per SM (128 registers a thread, 47 KB of shared memory
// a CTA): a stage barrier holds 4 warps, not 8.  Against two CTAs of 8 warps
// with 128-token stages and three stages in flight, config 3 went from 0.557
// to 0.510 ms; 2-warp CTAs with 32-token stages (eight per SM) and 4-warp
// CTAs over 512 tokens with three 64-token stages in flight were no faster.
constexpr int kMThreads = 128;
constexpr int kMWarps = kMThreads / 32;  // 4 warps: 16 tokens each per stage
constexpr int kMStageTok = 64;           // tokens per stage
constexpr int kMRing = 3;                // stage buffers: two in flight while one is read
constexpr int kMFbCap = 384;             // fallback rows a stage buffer holds (3/8 of its blocks)
constexpr int kMTokPerCta = 1024;

template <bool B4>
struct MStage {
    static constexpr int kBlocks = kMStageTok * 16, kWords = kBlocks / 32;
    static constexpr int kPacked = (kBlocks * (B4 ? 4 : 5) + 16 + 15) & ~15;
    static constexpr int kWordsOff = 0, kRanksOff = kWords * 4, kPackedOff = kWords * 8;
    static constexpr int kFbOff = kPackedOff + kPacked;
    static constexpr int kZeroOff = kFbOff + kMFbCap * 16;  // a zero row read by representable blocks
    static constexpr int kBytes = kZeroOff + 16;
};

__device__ __forceinline__ void sts_v4(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ void mma_16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The unit of a head's fp16 operands and the decode constants that go with it.
struct MUnit {
    float u, inv_u, fk;         // u = s * 2^k, 1/u, 2^-k
    uint32_t hmul, hadd0, hadd1;  // fp16x2: 2^-(4+k); (-72 + c/2) * 2^-k for coset c = 0 / 1
};

__device__ __forceinline__ MUnit make_unit(float s) {
    int e = 0;
    frexpf(s, &e);
    const int k = (s > 0.f && s < 1.f) ? min(1 - e, 20) : 0;  // 2^-(4+k) stays a (subnormal) fp16 number
    MUnit m;
    m.fk = ldexpf(1.f, -k);
    m.u = s / m.fk;
    m.inv_u = 1.f / m.u;
    m.hmul = pack_half2(ldexpf(1.f, -4 - k), ldexpf(1.f, -4 - k));
    m.hadd0 = pack_half2(-72.f * m.fk, -72.f * m.fk);
    m.hadd1 = pack_half2(-71.5f * m.fk, -71.5f * m.fk);
    return m;
}

// All threads: copy one stage (mask words, ranks, codes, at most kMFbCap
// fallback rows) into shared memory at `buf` and commit the group.  Every
// copy loop has a fixed trip count (predicated copies, no divergent loops).
template <bool B4>
__device__ __forceinline__ void mstage_issue(const CompactDev &c, const CStageSpan &s, uint32_t b0, uint32_t buf) {
    using S = MStage<B4>;
    static_assert(S::kWords <= kMThreads, "one mask word per thread");
    if (!s.bad) {
        const uint32_t tid = threadIdx.x;
        if (tid < s.nw) {
            cp_async4(buf + S::kWordsOff + 4 * tid, c.mask_words + s.w0 + tid);
            cp_async4(buf + S::kRanksOff + 4 * tid, c.word_rank + s.w0 + tid);
        }
        const uint32_t bits = B4 ? 4u : (uint32_t)c.bits;
        const uint32_t total = c.n_repr * bits, a1 = s.r1 * bits;
        constexpr int kCodeIters = (S::kPacked / 16 + kMThreads - 1) / kMThreads;
#pragma unroll
        for (int it = 0; it < kCodeIters; ++it) {
            const uint32_t off = s.a0 + 16u * (tid + (uint32_t)it * kMThreads);
            if (off < a1) cp_async16(buf + S::kPackedOff + (off - s.a0), c.packed + off, min(16u, total - off));
        }
        const uint32_t f0 = b0 - s.r0, nf = min(32u * s.nw - (s.r1 - s.r0), (uint32_t)kMFbCap);
        constexpr int kFbIters = (kMFbCap + kMThreads - 1) / kMThreads;
#pragma unroll
        for (int it = 0; it < kFbIters; ++it) {
            const uint32_t r = tid + (uint32_t)it * kMThreads;
            if (r < nf) cp_async16(buf + S::kFbOff + 16u * r, c.fallback + f0 + r, 16u);
        }
    }
    cp_async_commit();
}

// Whether a stage can come in as bulk copies (the TMA engine moves each of
// its four contiguous pieces -- mask words, ranks, codes, fallback rows --
// in one request): every piece must start and end on a 16-byte boundary
// inside its array.  Other stages (a chunk's last codes, heads whose word
// index is not a multiple of 4) take the per-thread cp.async path.
template <bool B4>
__device__ __forceinline__ bool mstage_bulk_ok(const CompactDev &c, const CStageSpan &s) {
    if (s.bad) return false;
    const uint32_t bits = B4 ? 4u : (uint32_t)c.bits;
    const uint32_t a1r = (s.r1 * bits + 15u) & ~15u, total16 = (c.n_repr * bits) & ~15u;
    const uintptr_t al = reinterpret_cast<uintptr_t>(c.mask_words + s.w0) | reinterpret_cast<uintptr_t>(c.word_rank + s.w0);
    return (s.nw & 3u) == 0 && (al & 15u) == 0 && a1r <= total16;
}

// One thread: a bulk-eligible stage as up to four bulk copies completed on
// the slot's barrier.
template <bool B4>
__device__ __forceinline__ void mstage_bulk(const CompactDev &c, const CStageSpan &s, uint32_t b0, uint32_t buf,
                                            uint32_t bar) {
    using S = MStage<B4>;
    const uint32_t bits = B4 ? 4u : (uint32_t)c.bits;
    const uint32_t wbytes = 4u * s.nw;
    const uint32_t cbytes = ((s.r1 * bits + 15u) & ~15u) - s.a0;
    const uint32_t nf = min(32u * s.nw - (s.r1 - s.r0), (uint32_t)kMFbCap);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's earlier generic reads first
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2u * wbytes + cbytes + 16u * nf)
                 : "memory");
    auto copy = [&](uint32_t dst, const void *src, uint32_t bytes) {
        if (bytes)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             dst),
                         "l"(src), "r"(bytes), "r"(bar)
                         : "memory");
    };
    copy(buf + S::kWordsOff, c.mask_words + s.w0, wbytes);
    copy(buf + S::kRanksOff, c.word_rank + s.w0, wbytes);
    copy(buf + S::kPackedOff, c.packed + s.a0, cbytes);
    copy(buf + S::kFbOff, c.fallback + (b0 - s.r0), 16u * nf);
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// A block's eight values travel as four fp16x2 registers whose (low, high)
// halves are the channels (6, 2), (5, 1), (4, 0), (7, 3): the order in which
// two-nibble groups of a 4-bit code reach the fp16 mantissas with one mask
// each (mblock).  The MMA fragments are laid out to match (q's channels in
// phase K, the output rows in phase V), so the order costs nothing.
__device__ __forceinline__ constexpr int blk_ch(int r, int hi) {
    return (r == 0 ? (hi ? 2 : 6) : r == 1 ? (hi ? 1 : 5) : r == 2 ? (hi ? 0 : 4) : (hi ? 3 : 7));
}

// An fp16 row of 8 values (natural order), times m, in the register order above.
__device__ __forceinline__ uint4 row_to_regs(uint4 v, float m) {
    float f[8];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        f[2 * i] = t.x * m;
        f[2 * i + 1] = t.y * m;
    }
    return make_uint4(pack_half2(f[blk_ch(0, 0)], f[blk_ch(0, 1)]), pack_half2(f[blk_ch(1, 0)], f[blk_ch(1, 1)]),
                      pack_half2(f[blk_ch(2, 0)], f[blk_ch(2, 1)]), pack_half2(f[blk_ch(3, 0)], f[blk_ch(3, 1)]));
}

// All threads: the staged fallback rows in units of u, in register order.
template <bool B4>
__device__ __forceinline__ void mstage_rescale(const CStageSpan &s, uint32_t buf, float inv_u) {
    using S = MStage<B4>;
    if (s.bad) return;
    const uint32_t nf = min(32u * s.nw - (s.r1 - s.r0), (uint32_t)kMFbCap);
    constexpr int kIters = (kMFbCap + kMThreads - 1) / kMThreads;
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
        const uint32_t r = threadIdx.x + (uint32_t)it * kMThreads;
        if (r < nf) sts_v4(buf + S::kFbOff + 16u * r, row_to_regs(lds_v4(buf + S::kFbOff + 16u * r), inv_u));
    }
}

// A 4-bit code as the four registers: v = the big-endian code word,
// w = (v << 1) | parity holds u0..u6 and 2*c7u + parity in nibbles 7..0
// (channel i in nibble 7 - i); each mask leaves two nibbles times 16 in the
// mantissas of the fp16 pair (1024, 1024).
__device__ __forceinline__ void decode4(uint32_t v, const MUnit &m, uint32_t h[4]) {
    const uint32_t par = __popc(v & 0x08888888u) & 1u;
    const uint32_t w = (v << 1) | par;
    const uint32_t add = (v >> 31) ? m.hadd1 : m.hadd0;
    h[0] = hfma2_u32((w & 0x00F000F0u) | 0x64006400u, m.hmul, add);          // nibbles 1, 5: channels 6, 2
    h[1] = hfma2_u32(((w >> 4) & 0x00F000F0u) | 0x64006400u, m.hmul, add);   // nibbles 2, 6: channels 5, 1
    h[2] = hfma2_u32(((w >> 8) & 0x00F000F0u) | 0x64006400u, m.hmul, add);   // nibbles 3, 7: channels 4, 0
    h[3] = hfma2_u32(((w << 4) & 0x00F000F0u) | 0x64006400u, m.hmul, add);   // nibbles 0, 4: channels 7, 3
}

// One block of a stage as four fp16x2 registers (channels 0-1, 2-3, 4-5, 6-7)
// in units of u.  wd / rk: the mask word holding the block and the
// representable blocks before that word (stage-relative); bit: the block's
// bit in the word; wi: the word's index in the stage; live: the block
// belongs to a token in range (else it reads as zeros).
template <bool B4>
__device__ __forceinline__ void mblock(const CompactDev &c, const CStageSpan &s, uint32_t buf, uint32_t b0,
                                       uint32_t wd, uint32_t rk, uint32_t wi, uint32_t bit, bool live,
                                       const MUnit &m, uint32_t h[4]) {
    using S = MStage<B4>;
    const uint32_t below = __popc(wd & ((1u << bit) - 1u));
    const bool good = live && !s.bad;
    const bool rep = good && ((wd >> bit) & 1u);
    const uint32_t nrep = s.r1 - s.r0, nf = 32u * s.nw - nrep;
    uint32_t pr = rk + below;  // representable blocks of the stage before this one
    pr = pr < nrep ? pr : 0u;  // a damaged index stays inside the staged codes (flagged on arrival)
    const uint32_t f = 32u * wi + bit - rk - below;  // fallback rows of the stage before this one
    const bool fb = good && !rep && f < nf;
    uint4 fv;
    if (fb && f >= (uint32_t)kMFbCap) {  // past the staged rows (a stage more than 3/8 fallback): from HBM
        fv = row_to_regs(__ldg(c.fallback + (b0 - s.r0) + f), m.inv_u);
    } else {
        fv = lds_v4(buf + (fb ? S::kFbOff + 16u * f : S::kZeroOff));
    }
    if constexpr (B4) {
        const uint32_t raw = lds_u32(buf + S::kPackedOff + (s.r0 * 4u - s.a0) + 4u * pr);
        // a block that is not representable decodes the code of zeros: nibbles 8, coset 0
        decode4(rep ? __byte_perm(raw, 0u, 0x0123u) : 0x44444444u, m, h);
        h[0] |= fv.x;
        h[1] |= fv.y;
        h[2] |= fv.z;
        h[3] |= fv.w;
    } else {
        float x[8];
        if (rep) {
            const int b = c.bits, R = 1 << (b - 1);
            const uint32_t o = buf + S::kPackedOff + pr * (uint32_t)b + (s.r0 * (uint32_t)b - s.a0);
            uint64_t acc = 0;
            for (int i = 0; i < b; ++i)
                acc = (acc << 8) | (lds_u32((o + i) & ~3u) >> (8 * ((o + i) & 3u)) & 0xffu);
            const uint32_t c7u = (uint32_t)(acc & ((1ull << (b - 1)) - 1));
            acc >>= (b - 1);
            uint32_t u[7], par = 0;
#pragma unroll
            for (int i = 6; i >= 0; --i) {
                u[i] = (uint32_t)(acc & ((1ull << b) - 1));
                par ^= u[i];
                acc >>= b;
            }
            const uint32_t coset = (uint32_t)(acc & 1u);
            const uint32_t base = 0x4A800000u | coset;
            const float bias = 4194304.0f + (float)R;
#pragma unroll
            for (int i = 0; i < 7; ++i) x[i] = (__int_as_float((u[i] << 1) | base) - bias) * m.fk;
            x[7] = (__int_as_float(((2u * c7u + (par & 1u)) << 1) | base) - bias) * m.fk;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = 0.f;
        }
        h[0] = pack_half2(x[blk_ch(0, 0)], x[blk_ch(0, 1)]) | fv.x;
        h[1] = pack_half2(x[blk_ch(1, 0)], x[blk_ch(1, 1)]) | fv.y;
        h[2] = pack_half2(x[blk_ch(2, 0)], x[blk_ch(2, 1)]) | fv.z;
        h[3] = pack_half2(x[blk_ch(3, 0)], x[blk_ch(3, 1)]) | fv.w;
    }
}

// mblock for a stage that is full (every token in range), whose index
// chained on arrival and whose fallback rows are all staged: no range
// checks.  cw: shared address of the first code of the block's word; fw:
// of the fallback row the block would have if no block before it in its
// word were representable; lowmask: the word's bits below the block's.
template <bool B4>
__device__ __forceinline__ void mblock_fast(int bits, uint32_t cw, uint32_t fw, uint32_t zero, uint32_t wd,
                                            uint32_t lowmask, const MUnit &m, uint32_t h[4]) {
    const uint32_t below = __popc(wd & lowmask);
    const bool rep = (wd & (lowmask + 1u)) != 0u;
    const uint4 fv = lds_v4(rep ? zero : fw - 16u * below);
    if constexpr (B4) {
        const uint32_t raw = lds_u32(cw + 4u * below);
        decode4(rep ? __byte_perm(raw, 0u, 0x0123u) : 0x44444444u, m, h);
    } else {
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.f;
        if (rep) {
            const int b = bits, R = 1 << (b - 1);
            const uint32_t o = cw + (uint32_t)b * below;
            uint64_t acc = 0;
            for (int i = 0; i < b; ++i)
                acc = (acc << 8) | (lds_u32((o + i) & ~3u) >> (8 * ((o + i) & 3u)) & 0xffu);
            const uint32_t c7u = (uint32_t)(acc & ((1ull << (b - 1)) - 1));
            acc >>= (b - 1);
            uint32_t u[7], par = 0;
#pragma unroll
            for (int i = 6; i >= 0; --i) {
                u[i] = (uint32_t)(acc & ((1ull << b) - 1));
                par ^= u[i];
                acc >>= b;
            }
            const uint32_t base = 0x4A800000u | (uint32_t)(acc & 1u);
            const float bias = 4194304.0f + (float)R;
#pragma unroll
            for (int i = 0; i < 7; ++i) x[i] = (__int_as_float((u[i] << 1) | base) - bias) * m.fk;
            x[7] = (__int_as_float(((2u * c7u + (par & 1u)) << 1) | base) - bias) * m.fk;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) h[r] = pack_half2(x[blk_ch(r, 0)], x[blk_ch(r, 1)]);
    }
    h[0] |= fv.x;
    h[1] |= fv.y;
    h[2] |= fv.z;
    h[3] |= fv.w;
}

template <int G, int QDT, bool B4>
__global__ void __launch_bounds__(kMThreads, 4) attn_compact_mma_kernel(CompactArgs a) {
    static_assert(G >= 1 && G <= 4, "query groups of up to 4 heads");
    using S = MStage<B4>;
    constexpr int D = 128, GP = 4;
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t head = blockIdx.y;
    const uint32_t T0 = blockIdx.x * a.tok_per_cta, T1 = min(T0 + a.tok_per_cta, a.seq);
    const uint32_t nst = (T1 - T0 + kMStageTok - 1) / kMStageTok;
    float *sc = reinterpret_cast<float *>(smem);  // [kMTokPerCta][GP] scores, then p
    const uint32_t bufs = smem_addr(smem + (size_t)kMTokPerCta * GP * 4);
    const uint32_t b = head / a.n_kv_heads, kvh = head % a.n_kv_heads;
    const uint32_t hb0 = head * a.bph;
    const MUnit mk = make_unit(a.k.scales[head]), mv = make_unit(a.v.scales[head]);

    // q as the B operand of phase K.  A k-step's A registers (a0..a3) are the
    // four registers of block 4 ks + t, so A column pair (2t, 2t+1) of row
    // half j holds register j's channels, pair (2t+8, 2t+9) register 2 + j's;
    // lane (g, t) of B (column g = head h + 4 j) holds q[h] at those channels.
    uint32_t qb[4][2];
    {
        const uint32_t h = g & 3u, j = g >> 2;
        const int64_t row = ((int64_t)b * a.n_kv_heads + kvh) * G + h;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            float qv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                qv[i] = h < (uint32_t)G ? Elem<QDT>::load(a.q, row * D + 8 * (4 * ks + t) + i) : 0.f;
            qb[ks][0] = j ? pack_half2(qv[blk_ch(1, 0)], qv[blk_ch(1, 1)]) : pack_half2(qv[blk_ch(0, 0)], qv[blk_ch(0, 1)]);
            qb[ks][1] = j ? pack_half2(qv[blk_ch(3, 0)], qv[blk_ch(3, 1)]) : pack_half2(qv[blk_ch(2, 0)], qv[blk_ch(2, 1)]);
        }
    }

    constexpr int kMaxStages = kMTokPerCta / kMStageTok;
    __shared__ CStageSpan spans[2][kMaxStages];
    auto stage_b0 = [&](uint32_t st) { return hb0 + (T0 + st * kMStageTok) * 16u; };
    if (threadIdx.x < 2 * kMaxStages) {
        const uint32_t ph = threadIdx.x / kMaxStages, st = threadIdx.x % kMaxStages;
        if (st < nst) {
            const uint32_t t1 = min(T0 + (st + 1) * kMStageTok, T1);
            spans[ph][st] = cstage_span(ph ? a.v : a.k, stage_b0(st), hb0 + t1 * 16u);
        }
    }
    if (threadIdx.x < kMRing) sts_v4(bufs + threadIdx.x * S::kBytes + S::kZeroOff, make_uint4(0, 0, 0, 0));
    __shared__ uint32_t s_dirty[kMRing];  // per ring slot: the stage's index did not chain
    // per ring slot: completion of the stage copied into it, one phase per
    // stage (bulk copies, or a plain arrival for a cp.async stage)
    __shared__ __align__(8) uint64_t s_bar[kMRing];
    if (threadIdx.x == 0)
        for (int i = 0; i < kMRing; ++i) mbar_init(smem_addr(&s_bar[i]), 1);
    __syncthreads();

    // the stages of both phases stream through a ring of kMRing buffers: K
    // stages 0..nst-1, then V stages, two ahead of the one being read
    const uint32_t n_seq = 2 * nst;
    auto issue = [&](uint32_t q) {
        if (q < n_seq) {
            const uint32_t ph = q >= nst, st = q - ph * nst;
            const CompactDev &cq = ph ? a.v : a.k;
            const CStageSpan &sq = spans[ph][st];
            const uint32_t slot = q % kMRing, bar = smem_addr(&s_bar[slot]), dst = bufs + slot * S::kBytes;
            if (mstage_bulk_ok<B4>(cq, sq)) {
                if (threadIdx.x == 0) {
                    s_dirty[slot] = 0u;
                    mstage_bulk<B4>(cq, sq, stage_b0(st), dst, bar);
                }
                cp_async_commit();  // an empty group keeps the group count one per stage
            } else {
                if (threadIdx.x == 0) s_dirty[slot] = 0u;
                mstage_issue<B4>(cq, sq, stage_b0(st), dst);
                if (threadIdx.x == 0) mbar_arrive(bar);
            }
        } else {
            cp_async_commit();
        }
    };
    issue(0);
    issue(1);

    const float fk_score = mk.u * a.qk_log2;
    float m_[G], l_[G];
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
        m_[gg] = -INFINITY;
        l_[gg] = 0.f;
    }
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;

    for (uint32_t q = 0; q < n_seq; ++q) {
        const uint32_t ph = q >= nst, st = q - ph * nst;
        const CStageSpan s = spans[ph][st];
        const CompactDev &c = ph ? a.v : a.k;
        const uint32_t buf = bufs + (q % kMRing) * S::kBytes;
        cp_async_wait<1>();
        // a copy that never completes leaves the flag raised and stale data,
        // which every index below stays inside
        mbar_wait(smem_addr(&s_bar[q % kMRing]), (q / kMRing) & 1u, a.err);
        __syncthreads();
        if (s.bad && threadIdx.x == 0) raise_flag(a.err, LQ_EF_BITSTREAM);
        // the stage's index must chain: rank(w+1) - rank(w) = popcount(word w)
        for (uint32_t i = threadIdx.x; i < s.nw && !s.bad; i += blockDim.x) {
            const uint32_t ri = lds_u32(buf + S::kRanksOff + 4 * i);
            const uint32_t rn = i + 1 < s.nw ? lds_u32(buf + S::kRanksOff + 4 * (i + 1)) : s.r1;
            if (rn - ri != (uint32_t)__popc(lds_u32(buf + S::kWordsOff + 4 * i)) || (i == 0 && ri != s.r0)) {
                raise_flag(a.err, LQ_EF_BITSTREAM);
                s_dirty[q % kMRing] = 1u;
            }
        }
        mstage_rescale<B4>(s, buf, ph ? mv.inv_u : mk.inv_u);
        if (ph == 1 && st == 0) {
            // softmax statistics over this warp's tokens (its 16 of every stage)
            const uint32_t nmine = nst * 16;
#pragma unroll
            for (int gg = 0; gg < G; ++gg) {
                m_[gg] = -INFINITY;
                l_[gg] = 0.f;
            }
            for (uint32_t i = lane; i < nmine; i += 32) {
                const uint32_t tr = (i >> 4) * kMStageTok + (uint32_t)warp * 16 + (i & 15);
                if (T0 + tr >= T1) continue;
#pragma unroll
                for (int gg = 0; gg < G; ++gg) m_[gg] = fmaxf(m_[gg], sc[tr * GP + gg]);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int gg = 0; gg < G; ++gg) m_[gg] = fmaxf(m_[gg], __shfl_xor_sync(0xffffffffu, m_[gg], off));
            for (uint32_t i = lane; i < nmine; i += 32) {
                const uint32_t tr = (i >> 4) * kMStageTok + (uint32_t)warp * 16 + (i & 15);
                if (T0 + tr >= T1) continue;
#pragma unroll
                for (int gg = 0; gg < G; ++gg) {
                    const float p = exp2f(sc[tr * GP + gg] - m_[gg]);
                    sc[tr * GP + gg] = p;
                    l_[gg] += p;
                }
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int gg = 0; gg < G; ++gg) l_[gg] += __shfl_xor_sync(0xffffffffu, l_[gg], off);
            __syncwarp();
        }
        __syncthreads();
        issue(q + 2);  // into the buffer read in the previous iteration

        const uint32_t tw = st * kMStageTok + (uint32_t)warp * 16;  // the warp's first token, CTA-relative
        const uint32_t b0 = stage_b0(st);
        const uint32_t nrep = s.r1 - s.r0;
        // a full stage whose index chained and whose fallback rows all fit the
        // buffer takes the unchecked block decode
        const bool fast = !s.bad && s_dirty[q % kMRing] == 0u && s.nw == (uint32_t)MStage<B4>::kWords &&
                          32u * s.nw - nrep <= (uint32_t)kMFbCap;
        const int bits = c.bits;
        const uint32_t code_base = buf + S::kPackedOff + (s.r0 * (B4 ? 4u : (uint32_t)bits) - s.a0);
        const uint32_t zero = buf + S::kZeroOff;
        // word wi of the stage: its mask word and its representable blocks before it
        auto word = [&](uint32_t wi, bool live, uint32_t &wd, uint32_t &rk) {
            wd = live ? lds_u32(buf + S::kWordsOff + 4 * wi) : 0u;
            rk = live ? lds_u32(buf + S::kRanksOff + 4 * wi) - s.r0 : 0u;
        };
        const uint32_t cbits = B4 ? 4u : (uint32_t)bits;
        auto blockv = [&](auto fast_tag, uint32_t wd, uint32_t rk, uint32_t wi, uint32_t bit, bool live,
                          const MUnit &m, uint32_t h[4]) {
            if constexpr (decltype(fast_tag)::value)
                // the word's code and fallback bases (the same for its blocks, hoisted by the compiler)
                mblock_fast<B4>(bits, code_base + cbits * rk, buf + S::kFbOff + 16u * (32u * wi - rk) + 16u * bit,
                                zero, wd, (1u << bit) - 1u, m, h);
            else
                mblock<B4>(c, s, buf, b0, wd, rk, wi, bit, live, m, h);
        };
        auto phase_k = [&](auto fast_tag) {
            constexpr bool kFull = decltype(fast_tag)::value;  // every token of the stage in range
            // two groups of 8 tokens, four k-steps of 4 blocks each
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
                const uint32_t tok = tw + 8u * grp + g;  // this lane's token
                const bool live = kFull || T0 + tok < T1;
                const uint32_t wi = (tok - st * kMStageTok) >> 1;  // its word in the stage
                uint32_t wd, rk;
                word(wi, live, wd, rk);
                float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t h[4];
                    blockv(fast_tag, wd, rk, wi, 16u * (g & 1u) + 4u * ks + t, live, mk, h);
                    mma_16816(d, h[0], h[1], h[2], h[3], qb[ks][0], qb[ks][1]);
                }
                float v0 = t < 2 ? d[0] : d[2], v1 = t < 2 ? d[1] : d[3];
                v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
                v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
                if (t < 2 && live) {
                    float *row = sc + tok * GP + 2 * t;
                    row[0] = v0 * fk_score;
                    row[1] = v1 * fk_score;
                }
            }
        };
        auto phase_v = [&](auto fast_tag) {
            constexpr bool kFull = decltype(fast_tag)::value;
            // one group of 16 tokens; lane (g, t) holds blocks 2g, 2g+1 of tokens
            // 2t, 2t+1 (word t of the group) and 2t+8, 2t+9 (word 4 + t)
            uint32_t R[8][4];
#pragma unroll
            for (int hw = 0; hw < 2; ++hw) {
                const uint32_t tok = tw + 8u * hw + 2u * t;  // first of the word's two tokens
                const bool live = kFull || T0 + tok < T1;
                const uint32_t wi = (tok - st * kMStageTok) >> 1;
                uint32_t wd, rk;
                word(wi, live, wd, rk);
                blockv(fast_tag, wd, rk, wi, 2u * g, live, mv, R[4 * hw + 0]);
                blockv(fast_tag, wd, rk, wi, 2u * g + 1u, live, mv, R[4 * hw + 1]);
                blockv(fast_tag, wd, rk, wi, 16u + 2u * g, live, mv, R[4 * hw + 2]);
                blockv(fast_tag, wd, rk, wi, 17u + 2u * g, live, mv, R[4 * hw + 3]);
            }
            // p^T as the B operand: (p[g][2t], p[g][2t+1]) and (p[g][2t+8], p[g][2t+9])
            uint32_t pb0 = 0u, pb1 = 0u;
            if (g < (uint32_t)G) {
                const uint32_t ta = tw + 2u * t, tc = ta + 8u;
                const bool la = kFull || T0 + ta < T1, lc = kFull || T0 + tc < T1;
                const float pa = la ? sc[ta * GP + g] : 0.f;
                const float pbv = la ? sc[(ta + 1) * GP + g] : 0.f;
                const float pc = lc ? sc[tc * GP + g] : 0.f;
                const float pd = lc ? sc[(tc + 1) * GP + g] : 0.f;
                pb0 = pack_half2(pa, pbv);
                pb1 = pack_half2(pc, pd);
            }
            // m-tile j: output rows 16g + ch and 16g + 8 + ch, ch = blk_ch(j / 2, j % 2)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u, i = j >> 1;
                mma_16816(acc[j], __byte_perm(R[0][i], R[2][i], sel), __byte_perm(R[1][i], R[3][i], sel),
                          __byte_perm(R[4][i], R[6][i], sel), __byte_perm(R[5][i], R[7][i], sel), pb0, pb1);
            }
        };
        if (ph == 0) {
            if (fast) phase_k(std::true_type{});
            else phase_k(std::false_type{});
        } else {
            if (fast) phase_v(std::true_type{});
            else phase_v(std::false_type{});
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // the stage buffers become the merge buffer

    // ---- merge the warps in a fixed order
    float *mrg = reinterpret_cast<float *>(smem + (size_t)kMTokPerCta * GP * 4);
    constexpr int rs = D + 2;
    if (t < 2) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t hh = 2 * t + e;
            if (hh < (uint32_t)G) {
                float *o = mrg + (warp * G + hh) * rs;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int ch = blk_ch(j >> 1, j & 1);
                    o[16 * g + ch] = acc[j][e] * mv.u;
                    o[16 * g + 8 + ch] = acc[j][2 + e] * mv.u;
                }
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
            mrg[(warp * G + gg) * rs + D] = m_[gg];
            mrg[(warp * G + gg) * rs + D + 1] = l_[gg];
        }
    }
    __syncthreads();
    float *out = a.part + ((size_t)head * a.nct + blockIdx.x) * G * rs;
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int gg = e / D, dd = e % D;
        float mx = -INFINITY;
        for (int w = 0; w < kMWarps; ++w) mx = fmaxf(mx, mrg[(w * G + gg) * rs + D]);
        float o = 0.f, ls = 0.f;
        for (int w = 0; w < kMWarps; ++w) {
            const float mw = mrg[(w * G + gg) * rs + D];
            if (mw == -INFINITY) continue;
            const float f = exp2f(mw - mx);
            o = fmaf(mrg[(w * G + gg) * rs + dd], f, o);
            ls = fmaf(mrg[(w * G + gg) * rs + D + 1], f, ls);
        }
        out[gg * rs + dd] = o;
        if (dd == 0) {
            out[gg * rs + D] = mx;
            out[gg * rs + D + 1] = ls;
        }
    }
}

// ---- compact-layout attention: plan and launch
struct CompactPlan {
    uint32_t nct, tok_per_cta;
    size_t smem, part_floats;
    bool cuda_cores;  // force the CUDA-core kernel (LQ_ATTN_CUDA_CORES set)
    bool mma;         // the tensor-core kernel runs (head_dim 128, up to 4 query heads per KV head)
};

int compact_plan(int64_t n_heads, int64_t seq, int G, int D, CompactPlan *p) {
    if (n_heads <= 0 || seq <= 0 || G < 1 || G > 8 || (D != 64 && D != 128)) return LQ_ERR_INVALID;
    const int bpt = D / 8;
    if ((seq * bpt) % 32 != 0 || n_heads > 65535 || n_heads * seq * bpt >= ((int64_t)1 << 31)) return LQ_ERR_INVALID;
    p->cuda_cores = getenv("LQ_ATTN_CUDA_CORES") != nullptr;
    p->mma = D == 128 && G <= 4 && !p->cuda_cores;
    p->tok_per_cta = p->mma ? kMTokPerCta : kCTokPerCta;
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

template <int G, int QDT, bool B4>
int launch_mma(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, cudaStream_t st) {
    auto kern = attn_compact_mma_kernel<G, QDT, B4>;
    const size_t merge = (size_t)kMWarps * G * (128 + 2) * 4;
    const size_t smem = (size_t)kMTokPerCta * 4 * 4 + std::max((size_t)kMRing * MStage<B4>::kBytes, merge);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return LQ_ERR_CUDA;
    kern<<<dim3(p.nct, n_heads), kMThreads, smem, st>>>(a);
    return check_launch();
}

template <int G>
int launch_mma_q(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, int q_dtype, cudaStream_t st) {
    const bool b4 = a.k.bits == 4 && a.v.bits == 4;
    switch (q_dtype) {
        case LQ_F32:
            return b4 ? launch_mma<G, LQ_F32, true>(a, p, n_heads, st) : launch_mma<G, LQ_F32, false>(a, p, n_heads, st);
        case LQ_F16:
            return b4 ? launch_mma<G, LQ_F16, true>(a, p, n_heads, st) : launch_mma<G, LQ_F16, false>(a, p, n_heads, st);
        case LQ_BF16:
            return b4 ? launch_mma<G, LQ_BF16, true>(a, p, n_heads, st)
                      : launch_mma<G, LQ_BF16, false>(a, p, n_heads, st);
        default: return LQ_ERR_INVALID;
    }
}

// head_dim 128 with up to 4 query heads per KV head takes the tensor-core
// kernel; other shapes the CUDA-core kernel.  Both write partials in the same
// layout, [heads][tok_per_cta slices][G][D + 2], each with its own tok_per_cta.
template <int G>
int launch_compact_g(const CompactArgs &a, const CompactPlan &p, uint32_t n_heads, int q_dtype, int D, cudaStream_t st) {
    if constexpr (G <= 4) {
        if (p.mma) return launch_mma_q<G>(a, p, n_heads, q_dtype, st);
    }
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

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" size_t lq_attn_compact_workspace(int64_t n_heads, int64_t seq_len, int group, int head_dim) {
    CompactPlan p;
    if (compact_plan(n_heads, seq_len, group, head_dim, &p) != LQ_OK) return 0;
    return (p.part_floats * 4 + 255) & ~(size_t)255;
}

extern "C" int lq_attn_decode_compact(const lq_compact_view *k, const lq_compact_view *v, const void *q, int q_dtype,
                                      int64_t batch, int64_t n_kv_heads, int64_t seq_len, int group, int head_dim,
                                      float sm_scale, void *out, int out_dtype, float *lse, void *workspace,
                                      size_t workspace_bytes, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
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
    return launch_attn_combine(part, rows, hkv, G, D, p.nct, out, out_dtype, lse, st);
}
