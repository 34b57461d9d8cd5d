/*
 * lq_oracle.c -- CPU restatement of the LatticeQuant KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path in latticequant_b200/csrc.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm may load it.  Nothing in the
 * product package links, imports or calls it.
 *
 * Every function restates one piece of the reference (yoon9728/LatticeQuant)
 * with the exact floating-point operation order the reference gets from
 * torch on the CPU; the file:line of the reference code is given at each
 * function.  The restatement is pinned against fixtures produced by running
 * the reference itself (tests/golden/make_golden.py).
 *
 * Build: oracle/Makefile  ->  oracle/liblq_oracle.so
 * Floating point: compiled with -ffp-contract=off and no fast-math, so each
 * C expression below is one IEEE-754 binary32 operation, rounded to nearest.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define LQ_LOG2_L 10
#define LQ_L (1 << LQ_LOG2_L)

/* ------------------------------------------------------------------------ */
/* half / bfloat16 conversions (round to nearest even)                      */
/* ------------------------------------------------------------------------ */
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (a < 0x38800000u) {                                    /* subnormal half */
        if (a < 0x33000000u) return (uint16_t)sign;           /* < 2^-25 -> 0 */
        uint32_t e = a >> 23;
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 + (113 - e) ... bring to 2^-24 units */
        /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m >> (126 - e) */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (a >> 23) - 127 + 15;
    uint32_t m = a & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* dtype codes shared with the CUDA library: 0 = float32, 1 = float16, 2 = bfloat16 */
static inline float load_elem(const void *x, int dtype, int64_t i) {
    if (dtype == 0) return ((const float *)x)[i];
    if (dtype == 1) return f16_to_f32(((const uint16_t *)x)[i]);
    return bf16_to_f32(((const uint16_t *)x)[i]);
}

static inline void store_elem(void *y, int dtype, int64_t i, float v) {
    if (dtype == 0) ((float *)y)[i] = v;
    else if (dtype == 1) ((uint16_t *)y)[i] = f32_to_f16(v);
    else ((uint16_t *)y)[i] = f32_to_bf16(v);
}

uint16_t lqo_f32_to_f16(float f) { return f32_to_f16(f); }
float lqo_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t lqo_f32_to_bf16(float f) { return f32_to_bf16(f); }

/* ------------------------------------------------------------------------ */
/* torch CPU sum order                                                      */
/* ------------------------------------------------------------------------ */
/*
 * The reference reduces with torch on the CPU:
 *   sigma2 = (t_heads ** 2).mean(dim=(1, 2))      llm/compressed_kv_cache.py:189
 *   dist   = ((x - c) ** 2).sum(dim=-1)            core/e8_quantizer.py:79-80
 * torch's CPU sum of a contiguous row runs a fixed tree: the row is read as
 * vectors of 8 floats, 4 interleaved vector accumulators, each a 4-level
 * cascade with fan-out 2^p (p = max(4, ceil_log2(S)/4), S = row/32); the
 * accumulators are folded row 0 += rows 1..3, then the scalar tail and the 8
 * lanes are added left to right into a zero.  Measured against torch 2.11 on
 * this image (AVX512 capability) for rows of 8 .. 1M elements: identical
 * bits.  An 8-element row reduces strictly left to right.
 */
static int64_t ceil_log2_i64(int64_t x) {
    if (x <= 2) return 1;
    return 64 - __builtin_clzll((uint64_t)(x - 1));
}

float lqo_cascade_sum_f32(const float *a, int64_t n) {
    enum { V = 8, NROWS = 4, NLEV = 4 };
    const int64_t vec_size = n / V;
    const int64_t S = vec_size / NROWS;
    int64_t lp = ceil_log2_i64(S) / NLEV;
    if (lp < 4) lp = 4;
    const int64_t step = (int64_t)1 << lp;
    const int64_t mask = step - 1;
    float acc[NLEV][NROWS][V];
    memset(acc, 0, sizeof(acc));
    int64_t i = 0;
    for (; i + step <= S;) {
        for (int64_t j = 0; j < step; ++j)
            for (int k = 0; k < NROWS; ++k)
                for (int l = 0; l < V; ++l) acc[0][k][l] = acc[0][k][l] + a[((i + j) * NROWS + k) * V + l];
        i += step;
        for (int lv = 1; lv < NLEV; ++lv) {
            for (int k = 0; k < NROWS; ++k)
                for (int l = 0; l < V; ++l) {
                    acc[lv][k][l] = acc[lv][k][l] + acc[lv - 1][k][l];
                    acc[lv - 1][k][l] = 0.0f;
                }
            if ((i & (mask << (lv * lp))) != 0) break;
        }
    }
    for (; i < S; ++i)
        for (int k = 0; k < NROWS; ++k)
            for (int l = 0; l < V; ++l) acc[0][k][l] = acc[0][k][l] + a[(i * NROWS + k) * V + l];
    for (int lv = 1; lv < NLEV; ++lv)
        for (int k = 0; k < NROWS; ++k)
            for (int l = 0; l < V; ++l) acc[0][k][l] = acc[0][k][l] + acc[lv][k][l];
    for (int64_t v = S * NROWS; v < vec_size; ++v)
        for (int l = 0; l < V; ++l) acc[0][0][l] = acc[0][0][l] + a[v * V + l];
    for (int k = 1; k < NROWS; ++k)
        for (int l = 0; l < V; ++l) acc[0][0][l] = acc[0][0][l] + acc[0][k][l];
    float fa = 0.0f;
    for (int64_t e = vec_size * V; e < n; ++e) fa = fa + a[e];
    for (int l = 0; l < V; ++l) fa = fa + acc[0][0][l];
    return fa;
}

/* ------------------------------------------------------------------------ */
/* per-head scale                                                           */
/* ------------------------------------------------------------------------ */
/*
 * llm/compressed_kv_cache.py:183-196
 *   t = tensor.float(); t_heads = t.reshape(n_heads, bph, 8)
 *   sigma2 = (t_heads ** 2).mean(dim=(1, 2))              sum, then / n
 *   target_vol = 2*pi*e * sigma2 * 4**(-bits)             fp32 * fp32(2*pi*e), then * fp32(4**-b)
 *   scales_f32 = target_vol.sqrt(); where(sigma2 < 1e-12, 1, .)
 *   per_head_scale = scales_f32.to(float16)
 * vol_mult is fp32(4 ** -bits), rounded on the host from the double.
 */
#define LQ_TWO_PI_E_F32 17.079468445347132f
#define LQ_SIGMA2_MIN_F32 1e-12f

void lqo_head_scales(const void *x, int dtype, int64_t n_heads, int64_t elems_per_head, float vol_mult,
                     float *sigma2_out, float *scale_f32, uint16_t *scale_f16) {
    float *sq = (float *)malloc(sizeof(float) * (size_t)(elems_per_head > 0 ? elems_per_head : 1));
    for (int64_t h = 0; h < n_heads; ++h) {
        for (int64_t i = 0; i < elems_per_head; ++i) {
            float t = load_elem(x, dtype, h * elems_per_head + i);
            sq[i] = t * t;
        }
        float s = lqo_cascade_sum_f32(sq, elems_per_head);
        float sigma2 = s / (float)elems_per_head;
        float tv = (sigma2 * LQ_TWO_PI_E_F32) * vol_mult;
        float sc = sqrtf(tv);
        if (sigma2 < LQ_SIGMA2_MIN_F32) sc = 1.0f;
        if (sigma2_out) sigma2_out[h] = sigma2;
        if (scale_f32) scale_f32[h] = sc;
        if (scale_f16) scale_f16[h] = f32_to_f16(sc);
    }
    free(sq);
}

/* ------------------------------------------------------------------------ */
/* E8 nearest point                                                         */
/* ------------------------------------------------------------------------ */
/* tiebreaker = arange(8, float32) * 1e-7   (core/e8_quantizer.py:42-44) */
static const uint32_t kTieBits[8] = {0x00000000u, 0x33d6bf95u, 0x3456bf95u, 0x34a10fb0u,
                                     0x34d6bf95u, 0x350637bdu, 0x35210fb0u, 0x353be7a2u};

static inline float tie(int i) {
    float f;
    memcpy(&f, &kTieBits[i], 4);
    return f;
}

/* core/e8_quantizer.py:20-58 -- nearest point of D8 (sum even). */
static void d8_one(const float *x, float *r) {
    float res[8];
    float s = 0.0f;
    for (int i = 0; i < 8; ++i) {
        r[i] = rintf(x[i]);      /* torch.round: half to even */
        s = s + r[i];            /* x_round.sum(dim=-1), left to right */
        res[i] = x[i] - r[i];
    }
    if (fmodf(s, 2.0f) != 0.0f) { /* parity = sum % 2; needs_fix = parity != 0 */
        int best = 0;
        float bestc = 0.0f;
        for (int i = 0; i < 8; ++i) {
            float c = (1.0f - 2.0f * fabsf(res[i])) + tie(i);
            if (i == 0 || c < bestc) { /* argmin: first index wins ties */
                bestc = c;
                best = i;
            }
        }
        float sg = res[best] > 0.0f ? 1.0f : (res[best] < 0.0f ? -1.0f : 1.0f); /* sign(0) -> +1 */
        r[best] = r[best] + sg;
    }
}

void lqo_encode_d8(const float *x, float *out, int64_t n) {
    for (int64_t b = 0; b < n; ++b) d8_one(x + 8 * b, out + 8 * b);
}

/* core/e8_quantizer.py:61-83 -- nearest E8 point; dist1 <= dist2 keeps D8. */
static void e8_one(const float *x, float *q) {
    float c1[8], y[8], c2[8];
    d8_one(x, c1);
    for (int i = 0; i < 8; ++i) y[i] = x[i] - 0.5f;
    d8_one(y, c2);
    float d1 = 0.0f, d2 = 0.0f;
    for (int i = 0; i < 8; ++i) {
        c2[i] = c2[i] + 0.5f;
        float e1 = x[i] - c1[i];
        float e2 = x[i] - c2[i];
        d1 = d1 + e1 * e1;
        d2 = d2 + e2 * e2;
    }
    const float *src = (d1 <= d2) ? c1 : c2;
    for (int i = 0; i < 8; ++i) q[i] = src[i];
}

void lqo_encode_e8(const float *x, float *out, int64_t n) {
    for (int64_t b = 0; b < n; ++b) e8_one(x + 8 * b, out + 8 * b);
}

/* ------------------------------------------------------------------------ */
/* parity-aware symbols                                                     */
/* ------------------------------------------------------------------------ */
/* core/entropy_coder.py:46-68 */
static inline void symbolize_one(const float *q, uint8_t *coset, int32_t *sym) {
    int is_half = fabsf(q[0] - rintf(q[0])) > 0.25f;
    int64_t ic[8];
    for (int i = 0; i < 8; ++i) {
        float v = is_half ? q[i] - 0.5f : q[i];
        ic[i] = (int64_t)rintf(v);
    }
    for (int i = 0; i < 7; ++i) sym[i] = (int32_t)ic[i];
    /* torch.div(coord8, 2, rounding_mode='floor') */
    int64_t c8 = ic[7];
    int64_t fl = c8 >= 0 ? c8 / 2 : -((-c8 + 1) / 2);
    sym[7] = (int32_t)fl;
    *coset = (uint8_t)is_half;
}

void lqo_e8_to_symbols(const float *q, int64_t n, uint8_t *coset, int32_t *sym) {
    for (int64_t b = 0; b < n; ++b) symbolize_one(q + 8 * b, coset + b, sym + 8 * b);
}

/* core/entropy_coder.py:71-89 */
void lqo_symbols_to_e8(const uint8_t *coset, const int32_t *sym, int64_t n, float *q) {
    for (int64_t b = 0; b < n; ++b) {
        const int32_t *s = sym + 8 * b;
        int64_t sum7 = 0;
        for (int i = 0; i < 7; ++i) sum7 += s[i];
        int64_t need = ((sum7 % 2) + 2) % 2;
        int64_t c8 = 2 * (int64_t)s[7] + need;
        float off = coset[b] ? 0.5f : 0.0f;
        for (int i = 0; i < 7; ++i) q[8 * b + i] = (float)s[i] + off;
        q[8 * b + 7] = (float)c8 + off;
    }
}

/* ------------------------------------------------------------------------ */
/* chunk quantisation (the part of _compress_tensor before entropy coding)  */
/* ------------------------------------------------------------------------ */
/*
 * llm/compressed_kv_cache.py:198-204 and :225-228
 *   x_scaled = t_heads / scale_f32[head];  all_q = encode_e8(x_scaled)
 *   decompressed_out = (all_q * scale_f32[head]).to(orig_dtype)
 *   coset, free, c8h = e8_to_symbols(all_q)
 * deq (nullable) is written in out_dtype.
 */
void lqo_quantize_chunk(const void *x, int dtype, int64_t n_heads, int64_t bph, const float *scale_f32,
                        float *q_out, uint8_t *coset, int32_t *sym, void *deq, int out_dtype) {
    float xs[8], q[8];
    for (int64_t h = 0; h < n_heads; ++h) {
        const float sc = scale_f32[h];
        for (int64_t b = 0; b < bph; ++b) {
            const int64_t blk = h * bph + b;
            for (int i = 0; i < 8; ++i) xs[i] = load_elem(x, dtype, blk * 8 + i) / sc;
            e8_one(xs, q);
            if (q_out)
                for (int i = 0; i < 8; ++i) q_out[blk * 8 + i] = q[i];
            if (deq)
                for (int i = 0; i < 8; ++i) store_elem(deq, out_dtype, blk * 8 + i, q[i] * sc);
            if (coset && sym) symbolize_one(q, coset + blk, sym + 8 * blk);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* coset bit packing: llm/compressed_kv_cache.py:46-63 (bit i -> byte i/8,   */
/* bit i%8)                                                                 */
/* ------------------------------------------------------------------------ */
void lqo_pack_coset_bits(const uint8_t *coset, int64_t n, uint8_t *packed) {
    memset(packed, 0, (size_t)((n + 7) / 8));
    for (int64_t i = 0; i < n; ++i) packed[i >> 3] |= (uint8_t)((coset[i] & 1u) << (i & 7));
}

void lqo_unpack_coset_bits(const uint8_t *packed, int64_t n, uint8_t *coset) {
    for (int64_t i = 0; i < n; ++i) coset[i] = (packed[i >> 3] >> (i & 7)) & 1u;
}

/* ------------------------------------------------------------------------ */
/* rANS tables                                                              */
/* ------------------------------------------------------------------------ */
/*
 * core/gpu_ans.py:62-98 build_rans_table, with one change the reference
 * cannot pin: numpy's default argsort order among equal keys depends on the
 * SIMD sort numpy dispatches to, so this C version (like the CUDA table
 * builder) breaks ties by ascending symbol index.  The Python oracle calls
 * numpy's argsort itself when it restates the reference exactly.
 * Returns 0, or -1 when n_sym > L (the reference loops forever there).
 */
static void order_desc_stable(const int64_t *key, int n, int *order) {
    /* insertion sort: key descending, index ascending among equals */
    for (int i = 0; i < n; ++i) order[i] = i;
    for (int i = 1; i < n; ++i) {
        int v = order[i];
        int j = i - 1;
        while (j >= 0 && key[order[j]] < key[v]) {
            order[j + 1] = order[j];
            --j;
        }
        order[j + 1] = v;
    }
}

int lqo_normalize_freqs_stable(const int64_t *counts, int n_sym, int32_t *freqs) {
    if (n_sym <= 0 || n_sym > LQ_L) return -1;
    int64_t total = 0;
    for (int i = 0; i < n_sym; ++i) total += counts[i];
    for (int i = 0; i < n_sym; ++i) {
        if (total == 0) {
            freqs[i] = 1;
        } else {
            double p = (double)counts[i] / (double)total * (double)LQ_L;
            int32_t f = (int32_t)p; /* astype(int32): truncation */
            freqs[i] = f < 1 ? 1 : f;
        }
    }
    int *order = (int *)malloc(sizeof(int) * (size_t)n_sym);
    int64_t *key = (int64_t *)malloc(sizeof(int64_t) * (size_t)n_sym);
    for (;;) {
        int64_t sum = 0;
        for (int i = 0; i < n_sym; ++i) sum += freqs[i];
        if (sum == LQ_L) break;
        int64_t diff = LQ_L - sum;
        if (diff > 0) {
            order_desc_stable(counts, n_sym, order);
            for (int64_t j = 0; j < diff; ++j) freqs[order[j % n_sym]] += 1;
        } else {
            for (int i = 0; i < n_sym; ++i) key[i] = freqs[i];
            order_desc_stable(key, n_sym, order);
            for (int64_t j = 0; j < -diff; ++j) {
                int idx = order[j % n_sym];
                if (freqs[idx] > 1) freqs[idx] -= 1;
            }
        }
    }
    free(order);
    free(key);
    return 0;
}

/* cumfreqs (n_sym+1) and lookup (L) from freqs: core/gpu_ans.py:88-95 */
void lqo_table_from_freqs(const int32_t *freqs, int n_sym, int32_t *cumfreqs, int32_t *lookup) {
    cumfreqs[0] = 0;
    for (int i = 0; i < n_sym; ++i) cumfreqs[i + 1] = cumfreqs[i] + freqs[i];
    for (int s = 0; s < n_sym; ++s)
        for (int j = cumfreqs[s]; j < cumfreqs[s + 1]; ++j) lookup[j] = s;
}

/* ------------------------------------------------------------------------ */
/* rANS encode / decode: core/gpu_ans.py:105-139 and :146-168               */
/* ------------------------------------------------------------------------ */
/*
 * Encode symbol INDICES (already mapped to the table's alphabet).  Writes
 * ceil(n_bits/32)+1 words (the reference keeps one spare word) into words,
 * which must hold cap_words >= ceil(10*n/32)+1.  Returns n_bits, or -1 when
 * the capacity is too small.
 */
int64_t lqo_rans_encode(const int32_t *sym_idx, int64_t n, const int32_t *freqs, const int32_t *cumfreqs,
                        uint32_t *words, int64_t cap_words, uint32_t *state_out) {
    /* bits are emitted LSB-first per symbol in reverse symbol order, then the
     * whole list is reversed; collect into a byte-per-bit scratch. */
    uint8_t *bits = (uint8_t *)malloc((size_t)(10 * n + 1));
    int64_t nb = 0;
    uint64_t x = LQ_L;
    for (int64_t i = n - 1; i >= 0; --i) {
        const uint64_t fs = (uint64_t)freqs[sym_idx[i]];
        const uint64_t cfs = (uint64_t)cumfreqs[sym_idx[i]];
        while (x >= 2 * fs) {
            bits[nb++] = (uint8_t)(x & 1u);
            x >>= 1;
        }
        x = LQ_L * (x / fs) + cfs + (x % fs);
    }
    const int64_t n_words = (nb + 31) / 32 + 1;
    if (n_words > cap_words) {
        free(bits);
        return -1;
    }
    memset(words, 0, sizeof(uint32_t) * (size_t)n_words);
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t b = bits[nb - 1 - i];
        words[i >> 5] |= (uint32_t)b << (i & 31);
    }
    free(bits);
    *state_out = (uint32_t)x;
    return nb;
}

/* Decode n_symbols indices; reading stops at n_bits exactly as the reference
 * does ("while x < L and bit_pos < n_bits").  Bits past n_words read as 0
 * (the reference would raise IndexError there). */
void lqo_rans_decode(const uint32_t *words, int64_t n_words, int64_t n_bits, int64_t state,
                     const int32_t *lookup, const int32_t *freqs, const int32_t *cumfreqs, int64_t n_symbols,
                     int32_t *out_idx) {
    int64_t x = state;
    int64_t pos = 0;
    for (int64_t i = 0; i < n_symbols; ++i) {
        const int64_t slot = x & (LQ_L - 1);
        const int32_t si = lookup[slot];
        out_idx[i] = si;
        x = (int64_t)freqs[si] * (x >> LQ_LOG2_L) + slot - cumfreqs[si];
        while (x < LQ_L && pos < n_bits) {
            const int64_t w = pos >> 5;
            const uint32_t word = w < n_words ? words[w] : 0u;
            x = (x << 1) | ((word >> (pos & 31)) & 1u);
            ++pos;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* compact fixed-rate layout: core/compact_storage.py:87-222                */
/* ------------------------------------------------------------------------ */
/*
 * pack: q must be valid, in-range E8 points (the Python wrapper validates and
 * raises exactly as the reference).  Big-endian b bytes:
 * [coset | u0..u6 (b bits) | u7 >> 1 (b-1 bits)], u = int + 2^(b-1).
 */
void lqo_pack_e8(const float *q, int64_t n, int b, uint8_t *out) {
    const int64_t R = (int64_t)1 << (b - 1);
    for (int64_t k = 0; k < n; ++k) {
        const float *p = q + 8 * k;
        int is_half = fabsf(p[0] - rintf(p[0])) > 0.25f;
        uint64_t acc = (uint64_t)is_half;
        int64_t u[8];
        for (int i = 0; i < 8; ++i) u[i] = (int64_t)rintf(is_half ? p[i] - 0.5f : p[i]) + R;
        for (int i = 0; i < 7; ++i) acc = (acc << b) | (uint64_t)u[i];
        acc = (acc << (b - 1)) | (uint64_t)(u[7] >> 1);
        for (int i = b - 1; i >= 0; --i) {
            out[k * b + i] = (uint8_t)(acc & 0xffu);
            acc >>= 8;
        }
    }
}

void lqo_unpack_e8(const uint8_t *in, int64_t n, int b, float *q) {
    const int64_t R = (int64_t)1 << (b - 1);
    const uint64_t cm = ((uint64_t)1 << b) - 1;
    const uint64_t um = ((uint64_t)1 << (b - 1)) - 1;
    for (int64_t k = 0; k < n; ++k) {
        uint64_t acc = 0;
        for (int i = 0; i < b; ++i) acc = (acc << 8) | in[k * b + i];
        const int64_t c7u = (int64_t)(acc & um);
        acc >>= (b - 1);
        int64_t s[7];
        for (int i = 6; i >= 0; --i) {
            s[i] = (int64_t)(acc & cm) - R;
            acc >>= b;
        }
        const int coset = (int)(acc & 1u);
        int64_t ps = 0;
        for (int i = 0; i < 7; ++i) ps += s[i];
        const int64_t lsb = ((ps % 2) + 2) % 2;
        const int64_t c7 = c7u * 2 + lsb - R;
        const float off = coset ? 0.5f : 0.0f;
        for (int i = 0; i < 7; ++i) q[8 * k + i] = (float)s[i] + off;
        q[8 * k + 7] = (float)c7 + off;
    }
}

/* core/triton_dequant.py:45-132: 4-bit compact -> fp16, fp32 math
 * (c + 0.5*coset) * scale[head_idx[i]], then round to half. */
void lqo_unpack_e8_4bit_f16(const uint8_t *packed, const float *scales, const int32_t *head_idx, int64_t n,
                            uint16_t *out) {
    float q[8];
    for (int64_t k = 0; k < n; ++k) {
        lqo_unpack_e8(packed + 4 * k, 1, 4, q);
        const float sc = scales[head_idx[k]];
        for (int i = 0; i < 8; ++i) out[8 * k + i] = f32_to_f16(q[i] * sc);
    }
}
