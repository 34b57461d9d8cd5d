// lq_compact.cu -- compact fixed-rate E8 layout and library utilities.
//
// Reference: core/compact_storage.py:87-222 (pack_e8 / unpack_e8) and
// core/triton_dequant.py:45-177 (4-bit unpack + per-head scale -> fp16).
// Layout of one block in b bytes, big-endian:
//   [coset (1) | u0..u6 (b bits each) | u7 >> 1 (b-1 bits)],  u = int + 2^(b-1)
// coord7's low bit is implied by the even sum: lsb = (sum of signed c0..c6)
// mod 2, taken non-negative (the reference's unpack uses Python's %).
#include "lq_common.cuh"

namespace lq {
namespace {

// validate_e8 (core/compact_storage.py:39-80): all coords within 1e-5 of an
// integer (coset 0) or of a half-integer (coset 1), even integer sum.
__device__ inline bool valid_e8(const float q[8], int &coset, int ic[8]) {
    float rint_max = 0.0f, half_max = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        rint_max = fmaxf(rint_max, fabsf(__fsub_rn(q[i], rintf(q[i]))));
        const float h = __fsub_rn(q[i], 0.5f);
        half_max = fmaxf(half_max, fabsf(__fsub_rn(h, rintf(h))));
    }
    const bool is_int = rint_max < 1e-5f;
    const bool is_half = half_max < 1e-5f;
    coset = is_half ? 1 : 0;
    long long s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float v = is_half ? __fsub_rn(q[i], 0.5f) : q[i];
        ic[i] = __float2int_rn(v);
        s += ic[i];
    }
    return (is_int || is_half) && ((s & 1) == 0);
}

__global__ void pack_kernel(const float *__restrict__ q, int64_t n, int b, uint8_t *__restrict__ out,
                            uint32_t *__restrict__ n_bad) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = q[8 * k + i];
    int coset, ic[8];
    const bool ok = valid_e8(v, coset, ic);
    const int R = 1 << (b - 1);
    bool in_range = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) in_range &= (ic[i] >= -R) && (ic[i] <= R - 1);
    if (!ok) atomicAdd(&n_bad[0], 1u);
    else if (!in_range) atomicAdd(&n_bad[1], 1u);
    uint64_t acc = (uint64_t)coset;
#pragma unroll
    for (int i = 0; i < 7; ++i) acc = (acc << b) | (uint64_t)((ic[i] + R) & ((1 << b) - 1));
    acc = (acc << (b - 1)) | (uint64_t)(((ic[7] + R) >> 1) & ((1 << (b - 1)) - 1));
    for (int i = b - 1; i >= 0; --i) {
        out[k * b + i] = (uint8_t)(acc & 0xffu);
        acc >>= 8;
    }
}

__global__ void unpack_kernel(const uint8_t *__restrict__ in, int64_t n, int b, const float *__restrict__ scales,
                              const int32_t *__restrict__ head_idx, float *__restrict__ q_out,
                              uint16_t *__restrict__ f16_out) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    uint64_t acc = 0;
    if (b == 4) {
        const uint32_t w = reinterpret_cast<const uint32_t *>(in)[k];  // 4-byte rows: one aligned load
        acc = __byte_perm(w, 0, 0x0123);                                // big-endian
    } else {
        for (int i = 0; i < b; ++i) acc = (acc << 8) | in[k * b + i];
    }
    const int R = 1 << (b - 1);
    const uint64_t cm = (1ull << b) - 1, um = (1ull << (b - 1)) - 1;
    const int c7u = (int)(acc & um);
    acc >>= (b - 1);
    int s[7];
    int ps = 0;
#pragma unroll
    for (int i = 6; i >= 0; --i) {
        s[i] = (int)(acc & cm) - R;
        acc >>= b;
        ps += s[i];
    }
    const int coset = (int)(acc & 1u);
    const int c7 = c7u * 2 + (ps & 1) - R;
    const float off = coset ? 0.5f : 0.0f;
    float q[8];
#pragma unroll
    for (int i = 0; i < 7; ++i) q[i] = __fadd_rn((float)s[i], off);
    q[7] = __fadd_rn((float)c7, off);
    if (q_out) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q_out[8 * k + i] = q[i];
    }
    if (f16_out) {
        const float sc = scales[head_idx[k]];
#pragma unroll
        for (int i = 0; i < 8; ++i) f16_out[8 * k + i] = __half_as_ushort(__float2half_rn(__fmul_rn(q[i], sc)));
    }
}

// Fused merge of the compact layout with its fp16 fallback
// (llm/fused_triton_merge.py:33-130): block k is representable (mask[k]) and
// stored as code number repr_rank[k] of `packed`, or out of range and stored
// as row fb_rank[k] of `fallback`.  Output fp16 = (point * head scale) for
// coded blocks, the fallback row otherwise.  coord7's low bit is the
// non-negative (sum c0..c6) mod 2; the reference's kernel takes Triton's
// remainder, which is -1 for odd negative sums and then decodes a wrong c7.
__global__ void compact_merge_kernel(const uint8_t *__restrict__ packed, int b, const uint8_t *__restrict__ mask,
                                     const int32_t *__restrict__ repr_rank, const int32_t *__restrict__ fb_rank,
                                     const uint16_t *__restrict__ fallback, const float *__restrict__ scales,
                                     FastDiv bph_div, int64_t n, int64_t n_repr, int64_t n_fb,
                                     uint16_t *__restrict__ out, uint32_t *err) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    uint4 o;
    if (mask[k]) {
        const int64_t r = repr_rank[k];
        if (r < 0 || r >= n_repr) {
            raise_flag(err, LQ_EF_BITSTREAM);
            return;
        }
        uint64_t acc = 0;
        for (int i = 0; i < b; ++i) acc = (acc << 8) | packed[r * b + i];
        const int R = 1 << (b - 1);
        const uint64_t cm = (1ull << b) - 1, um = (1ull << (b - 1)) - 1;
        const int c7u = (int)(acc & um);
        acc >>= (b - 1);
        int s[7], ps = 0;
#pragma unroll
        for (int i = 6; i >= 0; --i) {
            s[i] = (int)(acc & cm) - R;
            acc >>= b;
            ps += s[i];
        }
        const float off = (acc & 1u) ? 0.5f : 0.0f;
        const float sc = scales[bph_div.div((uint32_t)k)];
        float q[8];
#pragma unroll
        for (int i = 0; i < 7; ++i) q[i] = __fmul_rn(__fadd_rn((float)s[i], off), sc);
        q[7] = __fmul_rn(__fadd_rn((float)(c7u * 2 + (ps & 1) - R), off), sc);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h = __floats2half2_rn(q[2 * i], q[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&h);
        }
        o = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        const int64_t f = fb_rank[k];
        if (f < 0 || f >= n_fb) {
            raise_flag(err, LQ_EF_BITSTREAM);
            return;
        }
        o = reinterpret_cast<const uint4 *>(fallback)[f];
    }
    reinterpret_cast<uint4 *>(out)[k] = o;
}

__global__ void selftest_div_kernel(const float *__restrict__ a, const float *__restrict__ b, int64_t n,
                                    float *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float bb = b[i];
    out[i] = div_by_scale(a[i], bb, __frcp_rn(bb), scale_ok_for_fast_div(bb));
}

__global__ void selftest_fastdiv_kernel(const uint32_t *__restrict__ num, int64_t n, FastDiv d,
                                        uint32_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = d.div(num[i]);
}

}  // namespace
}  // namespace lq

extern "C" int lq_selftest(int which, const void *a, const void *b, int64_t n, uint32_t d, void *out, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0 || !out || !a) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    const unsigned g = (unsigned)lq::ceil_div(n, 256);
    cudaStream_t st = lq::as_stream(stream);
    if (which == LQ_SELFTEST_DIV) {
        if (!b) return LQ_ERR_INVALID;
        lq::selftest_div_kernel<<<g, 256, 0, st>>>(static_cast<const float *>(a), static_cast<const float *>(b), n,
                                                    static_cast<float *>(out));
    } else if (which == LQ_SELFTEST_FASTDIV) {
        if (d == 0 || d >= 0x80000000u) return LQ_ERR_INVALID;
        lq::selftest_fastdiv_kernel<<<g, 256, 0, st>>>(static_cast<const uint32_t *>(a), n, lq::FastDiv(d),
                                                        static_cast<uint32_t *>(out));
    } else {
        return LQ_ERR_INVALID;
    }
    return lq::check_launch();
}

extern "C" int lq_version(void) { return 100; }

extern "C" const char *lq_strerror(int status) {
    switch (status) {
        case LQ_OK: return "ok";
        case LQ_ERR_INVALID: return "invalid argument (null pointer, size, dtype or alignment)";
        case LQ_ERR_ALPHABET: return "a stream alphabet exceeds L = 1024 symbols";
        case LQ_ERR_CAPACITY: return "an output or workspace buffer is too small";
        case LQ_ERR_CUDA: return "CUDA launch or runtime error";
        case LQ_ERR_STREAM: return "corrupt bitstream or lane metadata";
        default: return "unknown status";
    }
}

extern "C" int lq_pack_e8(const float *q, int64_t n, int bits, uint8_t *out, uint32_t *n_bad, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0 || bits < 3 || bits > 5) return LQ_ERR_INVALID;
    if (!n_bad) return LQ_ERR_INVALID;
    cudaStream_t st = lq::as_stream(stream);
    if (cudaMemsetAsync(n_bad, 0, 2 * sizeof(uint32_t), st) != cudaSuccess) return LQ_ERR_CUDA;
    if (n == 0) return LQ_OK;
    if (!q || !out) return LQ_ERR_INVALID;
    lq::pack_kernel<<<(unsigned)lq::ceil_div(n, 256), 256, 0, st>>>(q, n, bits, out, n_bad);
    return lq::check_launch();
}

extern "C" int lq_unpack_e8(const uint8_t *packed, int64_t n, int bits, const float *scales, const int32_t *head_idx,
                            float *q_out, uint16_t *f16_out, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0 || bits < 3 || bits > 5) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!packed || (!q_out && !f16_out) || (f16_out && (!scales || !head_idx))) return LQ_ERR_INVALID;
    if (bits == 4 && (reinterpret_cast<uintptr_t>(packed) & 3)) return LQ_ERR_INVALID;
    lq::unpack_kernel<<<(unsigned)lq::ceil_div(n, 256), 256, 0, lq::as_stream(stream)>>>(packed, n, bits, scales,
                                                                                          head_idx, q_out, f16_out);
    return lq::check_launch();
}

extern "C" int lq_compact_merge(const uint8_t *packed, int64_t n_repr, int bits, const uint8_t *repr_mask,
                                const int32_t *repr_rank, const int32_t *fb_rank, const uint16_t *fallback,
                                int64_t n_fallback, const float *scales, int64_t n_heads, int64_t bph, uint16_t *out,
                                uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_heads < 0 || bph <= 0 || bits < 3 || bits > 5 || n_repr < 0 || n_fallback < 0) return LQ_ERR_INVALID;
    const int64_t n = n_heads * bph;
    if (n == 0) return LQ_OK;
    if (!repr_mask || !repr_rank || !fb_rank || !scales || !out || (n_repr && !packed) || (n_fallback && !fallback))
        return LQ_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(out) & 15) || (fallback && (reinterpret_cast<uintptr_t>(fallback) & 15)))
        return LQ_ERR_INVALID;
    if (n >= ((int64_t)1 << 32) || bph >= ((int64_t)1 << 31)) return LQ_ERR_INVALID;
    lq::compact_merge_kernel<<<(unsigned)lq::ceil_div(n, 256), 256, 0, lq::as_stream(stream)>>>(
        packed, bits, repr_mask, repr_rank, fb_rank, fallback, scales, lq::FastDiv((uint32_t)bph), n, n_repr,
        n_fallback, out, err);
    return lq::check_launch();
}
