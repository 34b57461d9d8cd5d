// lq_api.cu -- kernels behind the reference's standalone entry points.
//
// These serve the element-wise API of the reference's core modules
// (quantize_e8, e8_to_symbols, symbols_to_e8, validate_e8 /
// check_representable, pack_coset_bits / unpack_coset_bits, rans_encode of
// single streams).  The KV-cache path does not use them; it runs the fused
// kernels of lq_quantize.cu / lq_rans.cu.
#include "lq_common.cuh"

namespace lq {
namespace {

// quantize_e8 (core/e8_quantizer.py:90-110): q = encode_e8(x / scale), xhat = q * scale
__global__ void quantize_e8_kernel(const float *__restrict__ x, int64_t n, float scale, float *__restrict__ q_out,
                                   float *__restrict__ xhat) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    const float rcp = __frcp_rn(scale);
    const bool fast = scale_ok_for_fast_div(scale);
    float v[8], q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = div_by_scale(x[8 * b + i], scale, rcp, fast);
    e8_nearest(v, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (q_out) q_out[8 * b + i] = q[i];
        if (xhat) xhat[8 * b + i] = __fmul_rn(q[i], scale);
    }
}

// e8_to_symbols (core/entropy_coder.py:46-68) on arbitrary E8 points
__global__ void to_symbols_kernel(const float *__restrict__ q, int64_t n, int32_t *__restrict__ coset,
                                  int32_t *__restrict__ sym) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    float v[8];
    int s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = q[8 * b + i];
    coset[b] = e8_symbols(v, s);
#pragma unroll
    for (int i = 0; i < 8; ++i) sym[8 * b + i] = s[i];
}

// symbols_to_e8 (core/entropy_coder.py:71-89)
__global__ void from_symbols_kernel(const int32_t *__restrict__ coset, const int32_t *__restrict__ sym, int64_t n,
                                    float *__restrict__ q) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    int s[8];
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = sym[8 * b + i];
    e8_from_symbols(coset[b] == 1, s, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[8 * b + i] = v[i];
}

// validate_e8 (core/compact_storage.py:39-80) + the representable range of
// check_representable (:235-249) when bits > 0.
__global__ void check_e8_kernel(const float *__restrict__ q, int64_t n, float atol, int bits,
                                uint8_t *__restrict__ valid, uint8_t *__restrict__ coset,
                                uint8_t *__restrict__ in_range) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    float rmax = 0.0f, hmax = 0.0f;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = q[8 * k + i];
        rmax = fmaxf(rmax, fabsf(__fsub_rn(v[i], rintf(v[i]))));
        const float h = __fsub_rn(v[i], 0.5f);
        hmax = fmaxf(hmax, fabsf(__fsub_rn(h, rintf(h))));
    }
    const bool is_int = rmax < atol, is_half = hmax < atol;
    long long s = 0, lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const long long c = (long long)rintf(is_half ? __fsub_rn(v[i], 0.5f) : v[i]);
        s += c;
        lo = i ? (c < lo ? c : lo) : c;
        hi = i ? (c > hi ? c : hi) : c;
    }
    const bool ok = (is_int || is_half) && ((s & 1) == 0);
    if (valid) valid[k] = ok;
    if (coset) coset[k] = is_half;
    if (in_range) {
        const long long R = bits > 0 ? (1ll << (bits - 1)) : 0;
        in_range[k] = ok && bits > 0 && lo >= -R && hi <= R - 1;
    }
}

// pack_coset_bits / unpack_coset_bits (llm/compressed_kv_cache.py:46-63)
__global__ void pack_bits_kernel(const uint8_t *__restrict__ in, int64_t n, uint8_t *__restrict__ out) {
    const int64_t byte = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (byte * 8 >= n) return;
    uint32_t v = 0;
    for (int i = 0; i < 8; ++i) {
        const int64_t j = byte * 8 + i;
        if (j < n) v |= (uint32_t)(in[j] & 1u) << i;
    }
    out[byte] = (uint8_t)v;
}

__global__ void unpack_bits_kernel(const uint8_t *__restrict__ in, int64_t n, uint8_t *__restrict__ out) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) out[j] = (in[j >> 3] >> (j & 7)) & 1u;
}

// symbol value -> alphabet index, nearest entry, first index on ties
// (core/gpu_ans.py:115-119).  contiguous != 0: alphabet[i] = alphabet[0] + i.
__global__ void map_symbols_kernel(const int64_t *__restrict__ sym, int64_t n, const int64_t *__restrict__ alphabet,
                                   int32_t n_alpha, int contiguous, int32_t *__restrict__ out) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    const int64_t s = sym[k];
    if (contiguous) {
        const int64_t d = s - alphabet[0];
        out[k] = (int32_t)(d < 0 ? 0 : (d >= n_alpha ? n_alpha - 1 : d));
        return;
    }
    int32_t best = 0;
    uint64_t bd = ~0ull;
    for (int32_t i = 0; i < n_alpha; ++i) {
        const int64_t a = alphabet[i];
        const uint64_t d = (uint64_t)(a > s ? a - s : s - a);
        if (d < bd) {
            bd = d;
            best = i;
        }
    }
    out[k] = best;
}

// Independent reference streams, one thread each (core/gpu_ans.py:105-139),
// written backward, MSB-first, end-aligned into a caller-sized slot.
__global__ void encode_streams_kernel(const int32_t *__restrict__ sym_idx, const int64_t *__restrict__ sym_off,
                                      const int64_t *__restrict__ n_sym, const int32_t *__restrict__ table_id,
                                      const int32_t *__restrict__ tab_nsym, const uint32_t *__restrict__ enc_tab,
                                      int64_t n_streams, const int64_t *__restrict__ slot_off,
                                      uint32_t *__restrict__ slots, int64_t *__restrict__ nbits_out,
                                      uint32_t *__restrict__ state_out, uint32_t *err) {
    const int64_t sid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sid >= n_streams) return;
    const int64_t n = n_sym[sid];
    const int32_t t = table_id[sid];
    const int32_t nsym = tab_nsym[t];
    uint32_t *out = slots + slot_off[sid + 1];  // end of this stream's slot
    uint32_t *const out_end = out;
    uint32_t x = LQ_L, acc = 0, cnt = 0;
    if (n > 0 && (nsym <= 0 || nsym > LQ_L)) {
        raise_flag(err, LQ_EF_ALPHABET);
        nbits_out[sid] = 0;
        state_out[sid] = LQ_L;
        return;
    }
    const uint32_t *enc = enc_tab + (size_t)t * LQ_L;
    const int32_t *p = sym_idx + sym_off[sid];
    for (int64_t j = n - 1; j >= 0; --j) {
        const int32_t si = min(max(p[j], 0), nsym - 1);
        const uint32_t e = __ldg(enc + si);
        const uint32_t xmax = e & 0xfffu, k0 = (e >> 12) & 0xfu;  // lq_expand_tables' entry
        const uint32_t k = k0 + (x >= xmax ? 1u : 0u);
        const uint32_t v = x & ~(0xffffffffu << k);
        acc |= v << cnt;
        const uint32_t tt = cnt + k;
        if (tt >= 32u) {
            *--out = acc;
            acc = v >> (32u - cnt);
        }
        cnt = tt & 31u;
        x = (x >> k) + (e >> 16);
    }
    const int64_t nb = 32 * (int64_t)(out_end - out) + cnt;
    if (cnt) *--out = acc;
    nbits_out[sid] = nb;
    state_out[sid] = x;
}

// slot (MSB-first, end-aligned, ceil(nbits/32) words) -> reference words
// (LSB-first, start-aligned) at dst_off, plus the reference's zero spare word.
__global__ void finish_streams_kernel(const uint32_t *__restrict__ slots, const int64_t *__restrict__ slot_off,
                                      const int64_t *__restrict__ nbits, int64_t n_streams,
                                      const int64_t *__restrict__ dst_off, uint32_t *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t sid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (sid >= n_streams) return;
    const int64_t nb = nbits[sid];
    const int64_t nw = (nb + 31) / 32;
    const uint32_t pad = (uint32_t)((32 - (nb & 31)) & 31);
    const uint32_t *src = slots + slot_off[sid + 1] - nw;
    uint32_t *d = dst + dst_off[sid];
    for (int64_t i = lane; i <= nw; i += 32) {
        if (i == nw) {
            d[i] = 0u;
        } else {
            const uint32_t hi = src[i];
            const uint32_t lo = (i + 1 < nw) ? src[i + 1] : 0u;
            d[i] = __brev(__funnelshift_l(lo, hi, pad));
        }
    }
}

}  // namespace
}  // namespace lq

using namespace lq;

static inline unsigned grid_for(int64_t n, int t = 256) { return (unsigned)ceil_div(n, t); }

extern "C" int lq_quantize_e8(const float *x, int64_t n, float scale, float *q_out, float *xhat, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!x || (!q_out && !xhat)) return LQ_ERR_INVALID;
    quantize_e8_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(x, n, scale, q_out, xhat);
    return check_launch();
}

extern "C" int lq_e8_to_symbols(const float *q, int64_t n, int32_t *coset, int32_t *sym, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!q || !coset || !sym) return LQ_ERR_INVALID;
    to_symbols_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(q, n, coset, sym);
    return check_launch();
}

extern "C" int lq_symbols_to_e8(const int32_t *coset, const int32_t *sym, int64_t n, float *q, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!coset || !sym || !q) return LQ_ERR_INVALID;
    from_symbols_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(coset, sym, n, q);
    return check_launch();
}

extern "C" int lq_check_e8(const float *q, int64_t n, float atol, int bits, uint8_t *valid, uint8_t *coset,
                           uint8_t *in_range, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0 || bits < 0 || bits > 30) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!q) return LQ_ERR_INVALID;
    check_e8_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(q, n, atol, bits, valid, coset, in_range);
    return check_launch();
}

extern "C" int lq_pack_bits(const uint8_t *in, int64_t n, uint8_t *out, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!in || !out) return LQ_ERR_INVALID;
    pack_bits_kernel<<<grid_for(ceil_div(n, 8)), 256, 0, as_stream(stream)>>>(in, n, out);
    return check_launch();
}

extern "C" int lq_unpack_bits(const uint8_t *in, int64_t n, uint8_t *out, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!in || !out) return LQ_ERR_INVALID;
    unpack_bits_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(in, n, out);
    return check_launch();
}

extern "C" int lq_map_symbols(const int64_t *sym, int64_t n, const int64_t *alphabet, int32_t n_alpha, int contiguous,
                              int32_t *out, void *stream) {
    LQ_NVTX_RANGE();
    if (n < 0 || n_alpha <= 0) return LQ_ERR_INVALID;
    if (n == 0) return LQ_OK;
    if (!sym || !alphabet || !out) return LQ_ERR_INVALID;
    map_symbols_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(sym, n, alphabet, n_alpha, contiguous, out);
    return check_launch();
}

extern "C" int lq_rans_encode_streams(const int32_t *sym_idx, const int64_t *sym_off, const int64_t *n_sym,
                                      const int32_t *table_id, const int32_t *tab_nsym, const uint32_t *enc_tab,
                                      int64_t n_streams, const int64_t *slot_off, uint32_t *slots, int64_t *nbits,
                                      uint32_t *state, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_streams < 0) return LQ_ERR_INVALID;
    if (n_streams == 0) return LQ_OK;
    if (!sym_idx || !sym_off || !n_sym || !table_id || !tab_nsym || !enc_tab || !slot_off || !slots || !nbits ||
        !state)
        return LQ_ERR_INVALID;
    encode_streams_kernel<<<grid_for(n_streams, 128), 128, 0, as_stream(stream)>>>(
        sym_idx, sym_off, n_sym, table_id, tab_nsym, enc_tab, n_streams, slot_off, slots, nbits, state, err);
    return check_launch();
}

extern "C" int lq_rans_finish_streams(const uint32_t *slots, const int64_t *slot_off, const int64_t *nbits,
                                      int64_t n_streams, const int64_t *dst_off, uint32_t *dst, void *stream) {
    LQ_NVTX_RANGE();
    if (n_streams < 0) return LQ_ERR_INVALID;
    if (n_streams == 0) return LQ_OK;
    if (!slots || !slot_off || !nbits || !dst_off || !dst) return LQ_ERR_INVALID;
    finish_streams_kernel<<<grid_for(n_streams, 8), 256, 0, as_stream(stream)>>>(slots, slot_off, nbits, n_streams,
                                                                                 dst_off, dst);
    return check_launch();
}
