// lq_attn_dense.cu -- decode attention over the dense end of a layer's cache,
// merged with the attention results of its compressed parts, in one launch.
//
// The reference serves decode attention from one dequantised buffer:
// update() (llm/compressed_kv_cache.py:342-395) returns the whole K/V and
// transformers' SDPA reads it with repeat_kv.  Here the compressed parts are
// attended by the fused kernels (lq_attn.cu, lq_attn_compact.cu), which leave
// one normalised o and a log-sum-exp per part and query row; the tokens kept
// dense (the open tail of the decode steps, and tails kept dequantised) are
// attended here, and everything is merged by log-sum-exp:
//   per (batch, kv head) CTA, each warp walks every 4th token of the dense
//   segments with an online softmax (base 2) for the G query heads reading
//   that kv head, lanes holding D/32 channels; the warps' (m, l, o) merge in
//   warp order, then the parts' (o, lse) join in part order.
// Every sum runs in a fixed order, so results are deterministic.
#include "lq_attn_common.cuh"

namespace lq {
namespace {

constexpr int kDenseWarps = 4;
constexpr int kDenseMaxG = 8;

struct DenseArgs {
    const void *q;  // [heads * G][D] query rows, row order (batch, kv head, g)
    const void *k[LQ_DENSE_MAX_SEGMENTS], *v[LQ_DENSE_MAX_SEGMENTS];  // [heads][cap][D]
    int64_t cap[LQ_DENSE_MAX_SEGMENTS], len[LQ_DENSE_MAX_SEGMENTS];
    const int64_t *last[LQ_DENSE_MAX_SEGMENTS];  // non-NULL: the segment holds last[0] + 1 tokens
    int n_seg, G;
    const float *o_parts, *lse_parts;  // [n_parts][rows][D], [n_parts][rows]
    int64_t n_parts, rows;
    float qk_log2;  // sm_scale * log2(e)
    void *out;      // [rows][D], query dtype
    float *lse;     // [rows] natural log, may be NULL
};

// C consecutive elements from x[i..i+C) as floats (i a multiple of C)
template <int DT, int C>
__device__ __forceinline__ void load_run(const void *x, int64_t i, float v[C]) {
    if constexpr (DT == LQ_F32) {
        if constexpr (C == 4) {
            const float4 f = __ldg(reinterpret_cast<const float4 *>(x) + i / 4);
            v[0] = f.x;
            v[1] = f.y;
            v[2] = f.z;
            v[3] = f.w;
        } else {
            const float2 f = __ldg(reinterpret_cast<const float2 *>(x) + i / 2);
            v[0] = f.x;
            v[1] = f.y;
        }
    } else {
        uint32_t w[C / 2];
        if constexpr (C == 4) {
            const uint2 u = __ldg(reinterpret_cast<const uint2 *>(x) + i / 4);
            w[0] = u.x;
            w[1] = u.y;
        } else {
            w[0] = __ldg(reinterpret_cast<const uint32_t *>(x) + i / 2);
        }
#pragma unroll
        for (int j = 0; j < C / 2; ++j) {
            float2 f;
            if constexpr (DT == LQ_F16) f = __half22float2(*reinterpret_cast<const __half2 *>(&w[j]));
            else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[j]));
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
        }
    }
}

template <int QDT, int KDT, int D>
__global__ void __launch_bounds__(32 * kDenseWarps) attn_dense_merge_kernel(DenseArgs a) {
    constexpr int C = D / 32;
    extern __shared__ __align__(16) float dsm[];  // [warps][G][D + 2]: o, m, l
    const uint32_t head = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const int G = a.G;

    float qv[kDenseMaxG][C], m[kDenseMaxG], l[kDenseMaxG], o[kDenseMaxG][C];
#pragma unroll
    for (int g = 0; g < kDenseMaxG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            o[g][c] = 0.f;
            qv[g][c] = 0.f;
        }
        if (g < G) load_run<QDT, C>(a.q, ((int64_t)head * G + g) * D + lane * C, qv[g]);
    }

    for (int s = 0; s < a.n_seg; ++s) {
        int64_t len = a.last[s] ? *a.last[s] + 1 : a.len[s];
        len = len < 0 ? 0 : (len > a.cap[s] ? a.cap[s] : len);
        const int64_t base = (int64_t)head * a.cap[s] * D + lane * C;
        for (int64_t t = warp; t < len; t += kDenseWarps) {
            float kx[C], vx[C];
            load_run<KDT, C>(a.k[s], base + t * D, kx);
            load_run<KDT, C>(a.v[s], base + t * D, vx);
            float sg[kDenseMaxG];
#pragma unroll
            for (int g = 0; g < kDenseMaxG; ++g) {
                float d = 0.f;
#pragma unroll
                for (int c = 0; c < C; ++c) d = fmaf(qv[g][c], kx[c], d);
                sg[g] = d;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int g = 0; g < kDenseMaxG; ++g)
                    if (g < G) sg[g] += __shfl_xor_sync(0xffffffffu, sg[g], off);
#pragma unroll
            for (int g = 0; g < kDenseMaxG; ++g) {
                if (g >= G) continue;
                const float sv = sg[g] * a.qk_log2;
                const float mn = fmaxf(m[g], sv);
                const float f = exp2f(m[g] - mn);  // 0 while m is -inf
                const float p = exp2f(sv - mn);
                l[g] = fmaf(l[g], f, p);
#pragma unroll
                for (int c = 0; c < C; ++c) o[g][c] = fmaf(o[g][c], f, p * vx[c]);
                m[g] = mn;
            }
        }
    }

    // the warps' partial results, merged in warp order
    constexpr int rs = D + 2;
#pragma unroll
    for (int g = 0; g < kDenseMaxG; ++g) {
        if (g >= G) continue;
        float *row = dsm + (warp * G + g) * rs;
#pragma unroll
        for (int c = 0; c < C; ++c) row[lane * C + c] = o[g][c];
        if (lane == 0) {
            row[D] = m[g];
            row[D + 1] = l[g];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int g = e / D, d = e % D;
        const int64_t r = (int64_t)head * G + g;
        // dense keys: base-2 max and mass over the warps
        float mx = -INFINITY;
        for (int w = 0; w < kDenseWarps; ++w) mx = fmaxf(mx, dsm[(w * G + g) * rs + D]);
        float od = 0.f, ld = 0.f;
        for (int w = 0; w < kDenseWarps; ++w) {
            const float mw = dsm[(w * G + g) * rs + D];
            if (mw == -INFINITY) continue;
            const float f = exp2f(mw - mx);
            od = fmaf(dsm[(w * G + g) * rs + d], f, od);
            ld = fmaf(dsm[(w * G + g) * rs + D + 1], f, ld);
        }
        // natural log-sum-exp of the dense keys (-inf without any)
        const float lse_d = ld > 0.f ? (mx + log2f(ld)) * kLn2 : -INFINITY;
        float top = lse_d;
        for (int64_t i = 0; i < a.n_parts; ++i) top = fmaxf(top, a.lse_parts[i * a.rows + r]);
        float num = 0.f, den = 0.f;
        if (lse_d != -INFINITY) {
            const float w = exp2f((lse_d - top) * kLog2e);
            num = (od / ld) * w;
            den = w;
        }
        for (int64_t i = 0; i < a.n_parts; ++i) {
            const float li = a.lse_parts[i * a.rows + r];
            if (li == -INFINITY) continue;
            const float w = exp2f((li - top) * kLog2e);
            num = fmaf(a.o_parts[(i * a.rows + r) * D + d], w, num);
            den += w;
        }
        Elem<QDT>::store(a.out, r * D + d, den > 0.f ? num / den : 0.f);
        if (a.lse && d == 0) a.lse[r] = den > 0.f ? top + logf(den) : -INFINITY;
    }
}

template <int QDT, int KDT>
int launch_dense(const DenseArgs &a, int D, uint32_t heads, cudaStream_t st) {
    const size_t smem = (size_t)kDenseWarps * a.G * (D + 2) * 4;
    if (D == 128)
        attn_dense_merge_kernel<QDT, KDT, 128><<<heads, 32 * kDenseWarps, smem, st>>>(a);
    else
        attn_dense_merge_kernel<QDT, KDT, 64><<<heads, 32 * kDenseWarps, smem, st>>>(a);
    return check_launch();
}

template <int QDT>
int launch_dense_q(const DenseArgs &a, int kv_dtype, int D, uint32_t heads, cudaStream_t st) {
    if (kv_dtype == LQ_BF16) return launch_dense<QDT, LQ_BF16>(a, D, heads, st);
    if (kv_dtype == LQ_F16) return launch_dense<QDT, LQ_F16>(a, D, heads, st);
    if (kv_dtype == LQ_F32) return launch_dense<QDT, LQ_F32>(a, D, heads, st);
    return LQ_ERR_INVALID;
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" int lq_attn_dense_merge(const void *q, int q_dtype, int n_seg, const void *const *k_seg,
                                   const void *const *v_seg, const int64_t *cap_seg, const int64_t *len_seg,
                                   const int64_t *const *last_seg, int kv_dtype, const float *o_parts,
                                   const float *lse_parts, int64_t n_parts, int64_t batch, int64_t n_kv_heads,
                                   int group, int head_dim, float sm_scale, void *out, float *lse, void *stream) {
    LQ_NVTX_RANGE();
    if (n_seg < 0 || n_seg > LQ_DENSE_MAX_SEGMENTS || n_parts < 0 || batch <= 0 || n_kv_heads <= 0 || group < 1 ||
        group > kDenseMaxG || (head_dim != 64 && head_dim != 128))
        return LQ_ERR_INVALID;
    const int64_t heads = batch * n_kv_heads;
    if (heads > 0x7fffffff || !q || !out || (n_parts > 0 && (!o_parts || !lse_parts)) ||
        (n_seg > 0 && (!k_seg || !v_seg || !cap_seg || !len_seg)))
        return LQ_ERR_INVALID;
    DenseArgs a{};
    a.q = q;
    a.n_seg = n_seg;
    a.G = group;
    for (int s = 0; s < n_seg; ++s) {
        if (!k_seg[s] || !v_seg[s] || cap_seg[s] <= 0 || len_seg[s] < 0 || len_seg[s] > cap_seg[s]) return LQ_ERR_INVALID;
        // vector loads of D/32 elements at every row start
        if (((reinterpret_cast<uintptr_t>(k_seg[s]) | reinterpret_cast<uintptr_t>(v_seg[s])) & 15) != 0)
            return LQ_ERR_INVALID;
        a.k[s] = k_seg[s];
        a.v[s] = v_seg[s];
        a.cap[s] = cap_seg[s];
        a.len[s] = len_seg[s];
        a.last[s] = last_seg ? last_seg[s] : nullptr;
    }
    if ((reinterpret_cast<uintptr_t>(q) & 15) != 0) return LQ_ERR_INVALID;
    a.o_parts = o_parts;
    a.lse_parts = lse_parts;
    a.n_parts = n_parts;
    a.rows = heads * group;
    a.qk_log2 = sm_scale * kLog2e;
    a.out = out;
    a.lse = lse;
    cudaStream_t st = as_stream(stream);
    if (q_dtype == LQ_BF16) return launch_dense_q<LQ_BF16>(a, kv_dtype, head_dim, (uint32_t)heads, st);
    if (q_dtype == LQ_F16) return launch_dense_q<LQ_F16>(a, kv_dtype, head_dim, (uint32_t)heads, st);
    if (q_dtype == LQ_F32) return launch_dense_q<LQ_F32>(a, kv_dtype, head_dim, (uint32_t)heads, st);
    return LQ_ERR_INVALID;
}
