// lq_common.cuh -- shared device helpers for the LatticeQuant B200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/latticequant_b200.h"

#define LQ_LOG2_L 10

namespace lq {

constexpr int kL = LQ_L;
constexpr int kLog2L = LQ_LOG2_L;

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LQ_OK : LQ_ERR_CUDA;
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

__device__ inline void raise_flag(uint32_t *err, uint32_t f) {
    if (err) atomicOr(err, f);
}

// ---- element loads / stores -------------------------------------------
template <int DT>
struct Elem;

template <>
struct Elem<LQ_F32> {
    using T = float;
    __device__ static float load(const void *p, int64_t i) { return static_cast<const float *>(p)[i]; }
    __device__ static void store(void *p, int64_t i, float v) { static_cast<float *>(p)[i] = v; }
};

template <>
struct Elem<LQ_F16> {
    using T = __half;
    __device__ static float load(const void *p, int64_t i) { return __half2float(static_cast<const __half *>(p)[i]); }
    __device__ static void store(void *p, int64_t i, float v) { static_cast<__half *>(p)[i] = __float2half_rn(v); }
};

template <>
struct Elem<LQ_BF16> {
    using T = __nv_bfloat16;
    __device__ static float load(const void *p, int64_t i) {
        return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    }
    __device__ static void store(void *p, int64_t i, float v) {
        static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    }
};

// Load the 8 elements of block `blk` (16-byte aligned vectors for 16-bit
// types, two for fp32).
template <int DT>
__device__ inline void load_block8(const void *x, int64_t blk, float v[8]) {
    if constexpr (DT == LQ_F32) {
        const float4 *p = reinterpret_cast<const float4 *>(x) + 2 * blk;
        float4 a = __ldg(p), b = __ldg(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        uint4 u = __ldg(reinterpret_cast<const uint4 *>(x) + blk);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint16_t lo = (uint16_t)(w[i] & 0xffffu), hi = (uint16_t)(w[i] >> 16);
            if constexpr (DT == LQ_F16) {
                v[2 * i] = __half2float(__ushort_as_half(lo));
                v[2 * i + 1] = __half2float(__ushort_as_half(hi));
            } else {
                v[2 * i] = __bfloat162float(__ushort_as_bfloat16(lo));
                v[2 * i + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
            }
        }
    }
}

template <int DT>
__device__ inline void store_block8(void *y, int64_t blk, const float v[8]) {
    if constexpr (DT == LQ_F32) {
        float4 *p = reinterpret_cast<float4 *>(y) + 2 * blk;
        p[0] = make_float4(v[0], v[1], v[2], v[3]);
        p[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint16_t lo, hi;
            if constexpr (DT == LQ_F16) {
                lo = __half_as_ushort(__float2half_rn(v[2 * i]));
                hi = __half_as_ushort(__float2half_rn(v[2 * i + 1]));
            } else {
                lo = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]));
                hi = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]));
            }
            w[i] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        reinterpret_cast<uint4 *>(y)[blk] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ---- E8 nearest point ---------------------------------------------------
// Bit-exact restatement of core/e8_quantizer.py:20-83 as torch evaluates it
// on the CPU: every operation below is one rounded binary32 op (explicit
// _rn intrinsics keep the compiler from contracting into FMAs), sums run
// left to right, argmin keeps the first index, sign(0) = +1, and
// dist1 <= dist2 keeps the D8 candidate.

// tiebreaker = arange(8, float32) * 1e-7  (core/e8_quantizer.py:42-44)
__device__ __forceinline__ float e8_tie(int i) {
    constexpr uint32_t bits[8] = {0x00000000u, 0x33d6bf95u, 0x3456bf95u, 0x34a10fb0u,
                                  0x34d6bf95u, 0x350637bdu, 0x35210fb0u, 0x353be7a2u};
    return __uint_as_float(bits[i]);
}

__device__ __forceinline__ void d8_nearest(const float x[8], float r[8]) {
    float res[8];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r[i] = rintf(x[i]);
        s = __fadd_rn(s, r[i]);
        res[i] = __fsub_rn(x[i], r[i]);
    }
    // parity = s % 2 != 0; s is integer valued, and even once |s| >= 2^24
    const bool odd = (fabsf(s) < 16777216.0f) && (((int)s) & 1);
    if (odd) {
        int best = 0;
        float bestc = __fsub_rn(1.0f, __fmul_rn(2.0f, fabsf(res[0])));  // + tie(0) == + 0
#pragma unroll
        for (int i = 1; i < 8; ++i) {
            const float c = __fadd_rn(__fsub_rn(1.0f, __fmul_rn(2.0f, fabsf(res[i]))), e8_tie(i));
            if (c < bestc) {
                bestc = c;
                best = i;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i == best) r[i] = __fadd_rn(r[i], res[i] < 0.0f ? -1.0f : 1.0f);
        }
    }
}

__device__ __forceinline__ void e8_nearest(const float x[8], float q[8]) {
    float c1[8], y[8], c2[8];
    d8_nearest(x, c1);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fsub_rn(x[i], 0.5f);
    d8_nearest(y, c2);
    float d1 = 0.0f, d2 = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        c2[i] = __fadd_rn(c2[i], 0.5f);
        const float e1 = __fsub_rn(x[i], c1[i]);
        const float e2 = __fsub_rn(x[i], c2[i]);
        d1 = __fadd_rn(d1, __fmul_rn(e1, e1));
        d2 = __fadd_rn(d2, __fmul_rn(e2, e2));
    }
    const bool use1 = d1 <= d2;
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = use1 ? c1[i] : c2[i];
}

// e8_to_symbols (core/entropy_coder.py:46-68): coset = |q0 - round(q0)| > 0.25,
// ints = round(q - coset/2), sym[0..6] = ints[0..6], sym[7] = floor(ints[7] / 2).
__device__ __forceinline__ int e8_symbols(const float q[8], int sym[8]) {
    const int coset = fabsf(__fsub_rn(q[0], rintf(q[0]))) > 0.25f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float v = coset ? __fsub_rn(q[i], 0.5f) : q[i];
        sym[i] = __float2int_rn(v);
    }
    sym[7] = sym[7] >> 1;  // arithmetic shift == floor division by 2
    return coset;
}

// symbols_to_e8 (core/entropy_coder.py:71-89): coord7 = 2*c8h + parity(sum7).
__device__ __forceinline__ void e8_from_symbols(int coset, const int sym[8], float q[8]) {
    int sum7 = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) sum7 += sym[i];
    const int c7 = 2 * sym[7] + (sum7 & 1);
    const float off = coset ? 0.5f : 0.0f;
#pragma unroll
    for (int i = 0; i < 7; ++i) q[i] = __fadd_rn((float)sym[i], off);
    q[7] = __fadd_rn((float)c7, off);
}

}  // namespace lq
