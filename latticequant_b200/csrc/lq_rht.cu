// lq_rht.cu -- randomized Hadamard transform (core/pipeline.py:33-122).
//
// fast_hadamard_transform (:49-69) runs the butterflies r[i] = a + b,
// r[i+h] = a - b for h = 1, 2, 4, ... < d and divides by sqrt(d); every level
// is a set of independent binary32 additions, so any evaluation order gives
// torch's bits, and the final division is IEEE division by fp32(sqrt(d)), as
// torch divides a float32 tensor by a Python scalar.  RHT.forward (:103-111)
// multiplies by the sign vector first, RHT.inverse (:113-122) after.
// One CTA per vector, the vector in shared memory.
#include <cmath>

#include "lq_common.cuh"

namespace lq {
namespace {

__global__ void fwht_kernel(const float *__restrict__ x, int d, int log2d, const float *__restrict__ pre,
                            const float *__restrict__ post, float sqrt_d, float *__restrict__ out) {
    extern __shared__ float v[];
    const int64_t base = (int64_t)blockIdx.x * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float a = x[base + i];
        v[i] = pre ? __fmul_rn(a, pre[i]) : a;
    }
    __syncthreads();
    for (int lv = 0; lv < log2d; ++lv) {
        const int h = 1 << lv;
        for (int t = threadIdx.x; t < d / 2; t += blockDim.x) {
            const int i = ((t >> lv) << (lv + 1)) | (t & (h - 1));  // lower index of the pair
            const float a = v[i], b = v[i + h];
            v[i] = __fadd_rn(a, b);
            v[i + h] = __fsub_rn(a, b);
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float r = __fdiv_rn(v[i], sqrt_d);
        out[base + i] = post ? __fmul_rn(r, post[i]) : r;
    }
}

}  // namespace
}  // namespace lq

extern "C" int lq_fwht(const float *x, int64_t n_vec, int d, const float *pre_signs, const float *post_signs,
                       float *out, void *stream) {
    LQ_NVTX_RANGE();
    if (n_vec < 0 || d < 2 || d > 4096 || (d & (d - 1)) != 0) return LQ_ERR_INVALID;
    if (n_vec == 0) return LQ_OK;
    if (!x || !out || n_vec > 0x7fffffff) return LQ_ERR_INVALID;
    int log2d = 0;
    while ((1 << log2d) < d) ++log2d;
    const float sqrt_d = (float)std::sqrt((double)d);  // fp32(sqrt(d)), as torch rounds the scalar
    const int threads = d / 2 < 256 ? (d / 2 < 32 ? 32 : d / 2) : 256;
    lq::fwht_kernel<<<(unsigned)n_vec, threads, (size_t)d * sizeof(float), lq::as_stream(stream)>>>(
        x, d, log2d, pre_signs, post_signs, sqrt_d, out);
    return lq::check_launch();
}
