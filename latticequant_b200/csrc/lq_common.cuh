// lq_common.cuh -- shared device helpers for the LatticeQuant B200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
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

// One NVTX range per C entry point that enqueues work, named after the
// function, in the "latticequant_b200" domain: profilers (Nsight Systems,
// ncu's NVTX filters) see which library call launched each kernel.  NVTX 3
// is header-only; with no tool attached a push or pop is one indirect call
// that returns at once.
inline nvtxDomainHandle_t nvtx_domain() {
    static nvtxDomainHandle_t d = nvtxDomainCreateA("latticequant_b200");
    return d;
}

struct NvtxRange {
    explicit NvtxRange(const char *name) {
        nvtxEventAttributes_t e = {};
        e.version = NVTX_VERSION;
        e.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
        e.messageType = NVTX_MESSAGE_TYPE_ASCII;
        e.message.ascii = name;
        nvtxDomainRangePushEx(nvtx_domain(), &e);
    }
    ~NvtxRange() { nvtxDomainRangePop(nvtx_domain()); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

#define LQ_NVTX_RANGE() const ::lq::NvtxRange lq_nvtx_range_(__func__)

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

// The raw bytes of one block (16-bit types use `a` only), split from the
// conversion so that a loop can issue the next block's load before it works
// on the current one.
struct RawBlock8 {
    uint4 a, b;
};

template <int DT>
__device__ __forceinline__ RawBlock8 load_raw8(const void *x, int64_t blk) {
    RawBlock8 r;
    if constexpr (DT == LQ_F32) {
        const uint4 *p = reinterpret_cast<const uint4 *>(x) + 2 * blk;
        r.a = __ldg(p);
        r.b = __ldg(p + 1);
    } else {
        r.a = __ldg(reinterpret_cast<const uint4 *>(x) + blk);
        r.b = make_uint4(0, 0, 0, 0);
    }
    return r;
}

template <int DT>
__device__ __forceinline__ void raw8_to_float(const RawBlock8 &r, float v[8]) {
    if constexpr (DT == LQ_F32) {
        v[0] = __uint_as_float(r.a.x); v[1] = __uint_as_float(r.a.y);
        v[2] = __uint_as_float(r.a.z); v[3] = __uint_as_float(r.a.w);
        v[4] = __uint_as_float(r.b.x); v[5] = __uint_as_float(r.b.y);
        v[6] = __uint_as_float(r.b.z); v[7] = __uint_as_float(r.b.w);
    } else {
        const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
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
            // paired round-to-nearest-even conversions (one cvt per two values)
            if constexpr (DT == LQ_F16) {
                const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
        reinterpret_cast<uint4 *>(y)[blk] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ---- division by a loop-invariant divisor ---------------------------------
// Round-up multiply-shift method for unsigned division (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994, Fig. 4.1):
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, t = umulhi(m, n),
// n / d = (t + ((n - t) >> min(l, 1))) >> max(l - 1, 0), for d in [1, 2^31).
struct FastDiv {
    uint32_t d, m, sh1, sh2;
    __host__ __device__ FastDiv() : d(1), m(1), sh1(0), sh2(0) {}
    __host__ __device__ explicit FastDiv(uint32_t div) : d(div) {
        uint32_t l = 0;
        while ((1ull << l) < (uint64_t)div) ++l;
        m = (uint32_t)(((1ull << 32) * ((1ull << l) - div)) / div + 1);
        sh1 = l < 1 ? l : 1;
        sh2 = l > 1 ? l - 1 : 0;
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        const uint32_t t = __umulhi(m, n);
        return (t + ((n - t) >> sh1)) >> sh2;
    }
};

// ---- IEEE division by a per-head scale -----------------------------------
// Markstein's theorem (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; also
// Muller et al., Handbook of Floating-Point Arithmetic, FMA-based division):
// with y = RN(1/b), q0 = RN(a*y) and the exact FMA residual r = a - b*q0,
// RN(q0 + r*y) == RN(a/b) in round-to-nearest when nothing over- or
// underflows.  Both |a| (unless 0) and |b| must lie in [2^-40, 2^40], which
// keeps every intermediate normal; anything else takes the IEEE divide.  When
// r == 0, q0 is the exact quotient (this also keeps the sign of zero).
__device__ __forceinline__ bool scale_ok_for_fast_div(float b) {
    const float ab = fabsf(b);
    return ab >= 9.094947e-13f && ab <= 1.0995116e12f;
}

__device__ __forceinline__ float div_by_scale(float a, float b, float y, bool b_ok) {
    const float aa = fabsf(a);
    if (!b_ok || !(aa <= 1.0995116e12f && (aa >= 9.094947e-13f || aa == 0.0f))) return __fdiv_rn(a, b);
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-b, q0, a);
    return r == 0.0f ? q0 : __fmaf_rn(r, y, q0);
}

// The eight quotients of a block.  The FMA path is exact when every nonzero
// |v| of the block lies in [2^-40, 2^40] (a NaN passes through it as NaN);
// otherwise each value takes div_by_scale.  One range test per block keeps
// the common case free of per-value branches.  The select on v == 0 only
// keeps the sign of a zero quotient (a zero input gives r == +0, and
// fma(+0, y, -0) is +0); callers that use the quotient only through the E8
// search, where -0 and +0 give the same lattice point and symbols, pass
// SIGNED_ZERO = false and skip it.
template <bool SIGNED_ZERO = true>
__device__ __forceinline__ void div_block_by_scale(const float v[8], float b, float y, bool b_ok, float xs[8]) {
    // |v| <= 2^40 as a float maximum; 0 < |v| < 2^-40 as an unsigned test
    // on the bits with the sign shifted out: 2*bits - 2 wraps a zero to the
    // top of the range, and a nonzero |v| lands below 2*bits(2^-40) - 2
    // exactly when it is smaller than 2^-40
    float amax = 0.0f;
    uint32_t tmin = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        amax = fmaxf(amax, fabsf(v[i]));
        tmin = min(tmin, __float_as_uint(v[i]) * 2u - 2u);
    }
    if (b_ok && amax <= 1.0995116e12f && tmin >= 0x56fffffeu) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float q0 = __fmul_rn(v[i], y);
            const float r = __fmaf_rn(-b, q0, v[i]);
            if constexpr (SIGNED_ZERO)
                xs[i] = v[i] == 0.0f ? q0 : __fmaf_rn(r, y, q0);  // r == 0 gives q0 as well
            else
                xs[i] = __fmaf_rn(r, y, q0);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = div_by_scale(v[i], b, y, b_ok);
    }
}

// ---- symbol columns between the quantiser and the lane encoder -----------
// One buffer (lq_sym_cols_bytes): int8 columns [tiles][8][TB], then an int16
// plane of the same shape holding the symbols the columns mark with -128
// (those outside [-127, 127]), then one u32 flag per tile (any such symbol).
struct SymCols {
    int8_t *cols;
    int16_t *wide;
    uint32_t *esc;
};

__host__ __device__ inline size_t sym_cols_elems(int64_t n_tiles_total, int64_t tile_blocks) {
    return (size_t)n_tiles_total * (size_t)tile_blocks * 8;
}
__host__ __device__ inline size_t sym_cols_bytes(int64_t n_tiles_total, int64_t tile_blocks) {
    const size_t e = sym_cols_elems(n_tiles_total, tile_blocks);
    return ((3 * e + 15) & ~(size_t)15) + (((size_t)n_tiles_total * 4 + 15) & ~(size_t)15);
}
__host__ __device__ inline SymCols sym_cols_view(void *buf, int64_t n_tiles_total, int64_t tile_blocks) {
    const size_t e = sym_cols_elems(n_tiles_total, tile_blocks);
    char *b = static_cast<char *>(buf);
    return SymCols{reinterpret_cast<int8_t *>(b), reinterpret_cast<int16_t *>(b + e),
                   reinterpret_cast<uint32_t *>(b + ((3 * e + 15) & ~(size_t)15))};
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

// packed fp32x2 ops (sm_100): two independent IEEE binary32 operations, each
// rounded to nearest, in one instruction
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// D8 nearest point (core/e8_quantizer.py:20-58).  Flip cost RN(1 - 2|res|)
// is one FMA because 2|res| is exact; the first-index argmin runs as a
// tree in which the right operand wins only when strictly smaller, which
// selects the same index as a left-to-right scan, and the tree's three
// levels of outcomes select the flipped coordinate.  The flip adds
// sign(res) with sign(0) = +1, i.e. copysign(1, res) (res is never -0:
// x - rint(x) of equal values is +0).
__device__ __forceinline__ void d8_flip(float s, const float c[8], const float res[8], float r[8]) {
    // parity = s % 2 != 0; s is integer valued, and even once |s| >= 2^24
    const bool odd = (fabsf(s) < 16777216.0f) && (((int)s) & 1);
    const bool w01 = c[1] < c[0], w23 = c[3] < c[2], w45 = c[5] < c[4], w67 = c[7] < c[6];
    const float c01 = w01 ? c[1] : c[0], c23 = w23 ? c[3] : c[2];
    const float c45 = w45 ? c[5] : c[4], c67 = w67 ? c[7] : c[6];
    const bool wa = c23 < c01, wb = c67 < c45;
    const float ca = wa ? c23 : c01, cb = wb ? c67 : c45;
    const bool wc = cb < ca;
    const bool lo = odd && !wc, hi = odd && wc;
    const bool f[8] = {lo && !wa && !w01, lo && !wa && w01, lo && wa && !w23, lo && wa && w23,
                       hi && !wb && !w45, hi && !wb && w45, hi && wb && !w67, hi && wb && w67};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (f[i]) r[i] = __fadd_rn(r[i], copysignf(1.0f, res[i]));
    }
}

__device__ __forceinline__ void d8_nearest(const float x[8], float r[8], float res[8]) {
    float c[8];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r[i] = rintf(x[i]);
        s = __fadd_rn(s, r[i]);
        res[i] = __fsub_rn(x[i], r[i]);
        c[i] = __fmaf_rn(-2.0f, fabsf(res[i]), 1.0f);
        if (i) c[i] = __fadd_rn(c[i], e8_tie(i));
    }
    d8_flip(s, c, res, r);
}

// The two D8 searches of the E8 decoder, of x and of y = x - 1/2, in one
// pass: the coordinate sums and the residuals of both run as the two halves
// of packed fp32x2 adds, each half rounded as its scalar op.  The sum starts
// at r[0] instead of 0 + r[0], which differs only in the sign of a zero sum
// and leaves the parity unchanged.
__device__ __forceinline__ void d8_nearest_pair(const float x[8], const float y[8], float r1[8], float r2[8],
                                                float res1[8], float res2[8]) {
    float c1[8], c2[8];
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r1[i] = rintf(x[i]);
        r2[i] = rintf(y[i]);
        const unsigned long long rr = f2_pack(r1[i], r2[i]);
        s = i ? f2_add(s, rr) : rr;
        f2_unpack(f2_sub(f2_pack(x[i], y[i]), rr), res1[i], res2[i]);
        c1[i] = __fmaf_rn(-2.0f, fabsf(res1[i]), 1.0f);
        c2[i] = __fmaf_rn(-2.0f, fabsf(res2[i]), 1.0f);
        if (i) {
            c1[i] = __fadd_rn(c1[i], e8_tie(i));
            c2[i] = __fadd_rn(c2[i], e8_tie(i));
        }
    }
    float s1, s2;
    f2_unpack(s, s1, s2);
    d8_flip(s1, c1, res1, r1);
    d8_flip(s2, c2, res2, r2);
}

// The two squared distances sum((x - c1) ** 2), sum((x - c2) ** 2), each
// left to right with every product and every sum rounded on its own.  The
// squares are scalar __fmul_rn, which is never contracted into an FMA; the
// differences and the running sums of both distances go as the halves of
// packed fp32x2 subtracts and adds.  (A fused square-and-add rounds once
// instead of twice and decides exact ties of dist1 and dist2 the other way:
// seen at full chunk size, a few blocks per million, when the squares were
// packed multiplies.)
__device__ __forceinline__ void e8_dist2(const float x[8], const float c1[8], const float c2[8], float &d1,
                                         float &d2) {
    unsigned long long d = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float e1, e2;
        f2_unpack(f2_sub(f2_pack(x[i], x[i]), f2_pack(c1[i], c2[i])), e1, e2);
        const unsigned long long sq = f2_pack(__fmul_rn(e1, e1), __fmul_rn(e2, e2));
        d = i ? f2_add(d, sq) : sq;  // 0 + v == v exactly
    }
    f2_unpack(d, d1, d2);
}

// E8 nearest point (core/e8_quantizer.py:61-83).
__device__ __forceinline__ void e8_nearest(const float x[8], float q[8]) {
    float c1[8], y[8], c2[8], res1[8], res2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fsub_rn(x[i], 0.5f);
    d8_nearest_pair(x, y, c1, c2, res1, res2);
#pragma unroll
    for (int i = 0; i < 8; ++i) c2[i] = __fadd_rn(c2[i], 0.5f);
    float d1, d2;
    e8_dist2(x, c1, c2, d1, d2);
    const bool use1 = d1 <= d2;
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = use1 ? c1[i] : c2[i];
}

// E8 nearest point fused with e8_to_symbols (core/entropy_coder.py:46-68).
// The winning candidate's D8 coordinates are the symbols directly: for the
// integer coset q = c1 and round(q) = c1; for the half coset q = c2 + 1/2 and
// round(q - 1/2) = c2 (exact while |q| < 2^22, far beyond the symbol range).
// Returns the coset bit; *finite is false when any distance is NaN/inf (a
// non-finite input).  q is written only when WANT_Q.
template <bool WANT_Q>
__device__ __forceinline__ int e8_nearest_symbols(const float x[8], float q[8], int sym[8], bool *finite) {
    float c1[8], y[8], c2[8], res1[8], res2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fsub_rn(x[i], 0.5f);
    d8_nearest_pair(x, y, c1, c2, res1, res2);
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __fadd_rn(c2[i], 0.5f);  // the half-coset point, as the reference forms it
    float d1, d2;
    e8_dist2(x, c1, h, d1, d2);
    *finite = isfinite(d1) && isfinite(d2);
    const bool use1 = d1 <= d2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if constexpr (WANT_Q) q[i] = use1 ? c1[i] : h[i];
        sym[i] = __float2int_rn(use1 ? c1[i] : c2[i]);
    }
    sym[7] = sym[7] >> 1;  // floor(coord8 / 2)
    return use1 ? 0 : 1;
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
