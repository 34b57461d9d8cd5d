// lq_attn_common.cuh -- pieces shared by the attention kernels over the
// rANS lane layout (lq_attn.cu) and the compact layout (lq_attn_compact.cu):
// softmax constants, the query-group padding, and the launchers of the
// kernels that merge per-CTA partials (lq_attn_merge.cu).
#pragma once

#include "lq_tiledec.cuh"

namespace lq {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <int G>
__host__ __device__ constexpr int padded_g() {
    return (G + 3) & ~3;
}

// Merge the per-CTA partials [heads][nct][G][D + 2] (o unnormalised, m, l in
// base 2) of a head into o[row] (out_dtype) and lse[row] (natural log, may be
// NULL) for the rows heads * G, row order (batch, kv head, g).
int launch_attn_combine(const float *part, uint32_t rows, uint32_t n_kv_heads, uint32_t G, uint32_t D, uint32_t nct,
                        void *out, int out_dtype, float *lse, cudaStream_t st);

}  // namespace lq
