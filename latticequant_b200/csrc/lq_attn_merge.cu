// lq_attn_merge.cu -- merging attention partials.
//
// attn_combine_kernel folds the per-CTA partials of the fused decode
// attention kernels (lq_attn.cu, lq_attn_compact.cu) into o and lse;
// attn_merge_kernel combines finished attention results over disjoint key
// sets (the sequence shards of several GPUs, or several chunks of one layer)
// from their log-sum-exp: o = sum_i o_i exp(lse_i - lse), lse = ln sum_i
// exp(lse_i).  The reference has no counterpart: it attends over one
// decompressed buffer on one GPU.
#include "lq_attn_common.cuh"

namespace lq {
namespace {

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
// o = sum_i o_i exp(lse_i - lse), lse = log sum_i exp(lse_i).  Part i's o
// rows start at o_parts + i * part_stride, its lse values at lse_parts +
// i * part_stride (strides in floats).
template <int ODT>
__global__ void attn_merge_kernel(const float *__restrict__ o_parts, const float *__restrict__ lse_parts,
                                  int64_t n_parts, int64_t o_stride, int64_t l_stride, int64_t rows, uint32_t D,
                                  void *__restrict__ out, float *__restrict__ lse) {
    const int64_t row = blockIdx.x;
    float mx = -INFINITY;
    for (int64_t i = 0; i < n_parts; ++i) mx = fmaxf(mx, lse_parts[i * l_stride + row]);
    float ls = 0.f;
    for (int64_t i = 0; i < n_parts; ++i) {
        const float li = lse_parts[i * l_stride + row];
        if (li != -INFINITY) ls += exp2f((li - mx) * kLog2e);
    }
    const float inv = 1.f / ls;
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
        for (int64_t i = 0; i < n_parts; ++i) {
            const float li = lse_parts[i * l_stride + row];
            if (li != -INFINITY) o = fmaf(o_parts[i * o_stride + row * D + d], exp2f((li - mx) * kLog2e), o);
        }
        Elem<ODT>::store(out, row * D + d, o * inv);
    }
    if (lse && threadIdx.x == 0) lse[row] = mx + log2f(ls) * kLn2;
}

int launch_merge(const float *o_parts, const float *lse_parts, int64_t n_parts, int64_t o_stride, int64_t l_stride,
                 int64_t rows, int head_dim, void *out, int out_dtype, float *lse, cudaStream_t st) {
    const unsigned tb = head_dim < 128 ? (unsigned)head_dim : 128u;
    const unsigned grid = (unsigned)rows;
    const uint32_t D = (uint32_t)head_dim;
    if (out_dtype == LQ_F32)
        attn_merge_kernel<LQ_F32><<<grid, tb, 0, st>>>(o_parts, lse_parts, n_parts, o_stride, l_stride, rows, D, out,
                                                       lse);
    else if (out_dtype == LQ_F16)
        attn_merge_kernel<LQ_F16><<<grid, tb, 0, st>>>(o_parts, lse_parts, n_parts, o_stride, l_stride, rows, D, out,
                                                       lse);
    else if (out_dtype == LQ_BF16)
        attn_merge_kernel<LQ_BF16><<<grid, tb, 0, st>>>(o_parts, lse_parts, n_parts, o_stride, l_stride, rows, D,
                                                        out, lse);
    else
        return LQ_ERR_INVALID;
    return check_launch();
}

}  // namespace

int launch_attn_combine(const float *part, uint32_t rows, uint32_t n_kv_heads, uint32_t G, uint32_t D, uint32_t nct,
                        void *out, int out_dtype, float *lse, cudaStream_t st) {
    if (out_dtype == LQ_F32) attn_combine_kernel<LQ_F32><<<rows, D, 0, st>>>(part, n_kv_heads, G, D, nct, out, lse);
    else if (out_dtype == LQ_F16) attn_combine_kernel<LQ_F16><<<rows, D, 0, st>>>(part, n_kv_heads, G, D, nct, out, lse);
    else attn_combine_kernel<LQ_BF16><<<rows, D, 0, st>>>(part, n_kv_heads, G, D, nct, out, lse);
    return check_launch();
}

}  // namespace lq

using namespace lq;

extern "C" int lq_attn_merge(const float *o_parts, const float *lse_parts, int64_t n_parts, int64_t rows,
                             int head_dim, void *out, int out_dtype, float *lse, void *stream) {
    LQ_NVTX_RANGE();
    if (n_parts < 0 || rows < 0 || head_dim <= 0 || head_dim > 1024) return LQ_ERR_INVALID;
    if (n_parts == 0 || rows == 0) return n_parts == 0 && rows > 0 ? LQ_ERR_INVALID : LQ_OK;
    if (!o_parts || !lse_parts || !out || rows > 0x7fffffff) return LQ_ERR_INVALID;
    return launch_merge(o_parts, lse_parts, n_parts, rows * head_dim, rows, rows, head_dim, out, out_dtype, lse,
                        as_stream(stream));
}

extern "C" int lq_attn_merge_packed(const float *parts, int64_t n_parts, int64_t rows, int head_dim, void *out,
                                    int out_dtype, float *lse, void *stream) {
    LQ_NVTX_RANGE();
    if (n_parts < 0 || rows < 0 || head_dim <= 0 || head_dim > 1024) return LQ_ERR_INVALID;
    if (n_parts == 0 || rows == 0) return n_parts == 0 && rows > 0 ? LQ_ERR_INVALID : LQ_OK;
    if (!parts || !out || rows > 0x7fffffff) return LQ_ERR_INVALID;
    const int64_t stride = rows * (head_dim + 1);
    return launch_merge(parts, parts + rows * head_dim, n_parts, stride, stride, rows, head_dim, out, out_dtype, lse,
                        as_stream(stream));
}
