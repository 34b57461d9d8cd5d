/*
 * lq_oracle_codec.c -- whole-chunk compress / decompress on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY (see lq_oracle.c).  Restates
 * CompressedKVCache._compress_tensor (llm/compressed_kv_cache.py:176-287) and
 * _decompress_chunk (:289-332) in C, in the tiled lane layout the CUDA
 * library stores, which contains the reference's own layout as the special
 * case tile_blocks >= n_vectors (one tile: lane s is reference stream s).
 *
 * Lane layout of one chunk of N = n_heads * bph E8 blocks:
 *   tile t      = blocks [t*TB, min(N, (t+1)*TB))
 *   stream s    = 8*coset + coord   (coord 7 is coord8_half)
 *   lane l      = 16*t + s: the symbols of stream s whose block lies in tile t,
 *                 in block order, rANS-coded with the chunk's table for s,
 *                 starting from x = L, as core/gpu_ans.py:105-139 does.
 *   words       = lane l occupies words [lane_off[l], lane_off[l+1]),
 *                 ceil(n_bits/32) words, bit i at word i/32, bit i%32.
 * Tables are per (chunk, stream) from the chunk's counts, alphabet
 * [min-2, max+2] as in llm/compressed_kv_cache.py:246-253.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define LQ_L 1024
#define LQ_NSTREAM 16

/* from lq_oracle.c */
void lqo_head_scales(const void *x, int dtype, int64_t n_heads, int64_t elems_per_head, float vol_mult,
                     float *sigma2_out, float *scale_f32, uint16_t *scale_f16);
void lqo_quantize_chunk(const void *x, int dtype, int64_t n_heads, int64_t bph, const float *scale_f32,
                        float *q_out, uint8_t *coset, int32_t *sym, void *deq, int out_dtype);
void lqo_pack_coset_bits(const uint8_t *coset, int64_t n, uint8_t *packed);
int lqo_normalize_freqs_stable(const int64_t *counts, int n_sym, int32_t *freqs);
void lqo_table_from_freqs(const int32_t *freqs, int n_sym, int32_t *cumfreqs, int32_t *lookup);
int64_t lqo_rans_encode(const int32_t *sym_idx, int64_t n, const int32_t *freqs, const int32_t *cumfreqs,
                        uint32_t *words, int64_t cap_words, uint32_t *state_out);
void lqo_rans_decode(const uint32_t *words, int64_t n_words, int64_t n_bits, int64_t state,
                     const int32_t *lookup, const int32_t *freqs, const int32_t *cumfreqs, int64_t n_symbols,
                     int32_t *out_idx);
uint16_t lqo_f32_to_f16(float f);
float lqo_f16_to_f32(uint16_t h);
uint16_t lqo_f32_to_bf16(float f);

/* error codes (same values as the CUDA library's LQ_ERR_*) */
#define LQO_ERR_ALPHABET (-2)
#define LQO_ERR_CAPACITY (-3)

static inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

/*
 * Stream tables of a chunk from its symbols.
 * tab_lo[s], tab_nsym[s] (0 = empty stream) and tab_freq[s*L + i].
 * freqs_in (nullable, same layout) overrides normalisation, so that tables
 * built by numpy on the host can be replayed.
 */
int lqo_chunk_tables(const uint8_t *coset, const int32_t *sym, int64_t N, const int32_t *lo_in,
                     const int32_t *nsym_in, const int32_t *freqs_in, int32_t *tab_lo, int32_t *tab_nsym,
                     int32_t *tab_freq) {
    for (int s = 0; s < LQ_NSTREAM; ++s) {
        const int c = s >> 3, idx = s & 7;
        if (freqs_in) {
            tab_lo[s] = lo_in[s];
            tab_nsym[s] = nsym_in[s];
            memcpy(tab_freq + (size_t)s * LQ_L, freqs_in + (size_t)s * LQ_L, sizeof(int32_t) * LQ_L);
            continue;
        }
        int64_t mn = INT64_MAX, mx = INT64_MIN, cnt = 0;
        for (int64_t b = 0; b < N; ++b) {
            if (coset[b] != c) continue;
            const int64_t v = sym[8 * b + idx];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
            ++cnt;
        }
        if (cnt == 0) {
            tab_lo[s] = 0;
            tab_nsym[s] = 0;
            continue;
        }
        const int64_t lo = mn - 2, hi = mx + 2, n_sym = hi - lo + 1;
        if (n_sym > LQ_L) return LQO_ERR_ALPHABET;
        int64_t counts[LQ_L];
        memset(counts, 0, sizeof(counts));
        for (int64_t b = 0; b < N; ++b)
            if (coset[b] == c) counts[sym[8 * b + idx] - lo]++;
        tab_lo[s] = (int32_t)lo;
        tab_nsym[s] = (int32_t)n_sym;
        if (lqo_normalize_freqs_stable(counts, (int)n_sym, tab_freq + (size_t)s * LQ_L) != 0)
            return LQO_ERR_ALPHABET;
    }
    return 0;
}

/* capacity in words needed for the lanes of a chunk (10 bits/symbol worst case) */
int64_t lqo_lane_capacity_words(int64_t N, int64_t TB) {
    const int64_t n_tiles = ceil_div(N, TB);
    /* sum over lanes of ceil(10 * n / 32) <= 8 * N * 10 / 32 + 16 * n_tiles */
    return (8 * N * 10) / 32 + 16 * n_tiles + 1;
}

/*
 * Entropy-code a quantised chunk in the lane layout.
 * Returns total words, or a negative error.
 */
int64_t lqo_encode_lanes(const uint8_t *coset, const int32_t *sym, int64_t N, int64_t TB, const int32_t *tab_lo,
                         const int32_t *tab_nsym, const int32_t *tab_freq, uint32_t *words, int64_t cap_words,
                         uint32_t *lane_off, uint32_t *lane_nbits, uint32_t *lane_state, uint32_t *tile_n0) {
    const int64_t n_tiles = ceil_div(N, TB);
    int32_t cum[LQ_NSTREAM][LQ_L + 1];
    for (int s = 0; s < LQ_NSTREAM; ++s) {
        cum[s][0] = 0;
        for (int i = 0; i < tab_nsym[s]; ++i) cum[s][i + 1] = cum[s][i] + tab_freq[(size_t)s * LQ_L + i];
    }
    int32_t *idxbuf = (int32_t *)malloc(sizeof(int32_t) * (size_t)(TB > 0 ? TB : 1));
    uint32_t *tmp = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(ceil_div(10 * TB, 32) + 2));
    int64_t w = 0;
    for (int64_t t = 0; t < n_tiles; ++t) {
        const int64_t b0 = t * TB, b1 = (b0 + TB < N) ? b0 + TB : N;
        int64_t n0 = 0;
        for (int64_t b = b0; b < b1; ++b) n0 += (coset[b] == 0);
        tile_n0[t] = (uint32_t)n0;
        for (int s = 0; s < LQ_NSTREAM; ++s) {
            const int c = s >> 3, idx = s & 7;
            const int64_t l = t * LQ_NSTREAM + s;
            int64_t n = 0;
            for (int64_t b = b0; b < b1; ++b)
                if (coset[b] == c) idxbuf[n++] = sym[8 * b + idx] - tab_lo[s];
            lane_off[l] = (uint32_t)w;
            if (n == 0) {
                lane_nbits[l] = 0;
                lane_state[l] = LQ_L;
                continue;
            }
            uint32_t st = 0;
            const int64_t nb = lqo_rans_encode(idxbuf, n, tab_freq + (size_t)s * LQ_L, cum[s], tmp,
                                               ceil_div(10 * TB, 32) + 2, &st);
            const int64_t nw = ceil_div(nb, 32);
            if (nb < 0 || w + nw > cap_words) {
                free(idxbuf);
                free(tmp);
                return LQO_ERR_CAPACITY;
            }
            memcpy(words + w, tmp, sizeof(uint32_t) * (size_t)nw);
            lane_nbits[l] = (uint32_t)nb;
            lane_state[l] = st;
            w += nw;
        }
    }
    lane_off[n_tiles * LQ_NSTREAM] = (uint32_t)w;
    free(idxbuf);
    free(tmp);
    return w;
}

/*
 * Decode the lanes of a chunk back to symbols (coset from the packed bits).
 * Mirrors _decompress_chunk (llm/compressed_kv_cache.py:301-320).
 */
void lqo_decode_lanes(const uint8_t *coset, int64_t N, int64_t TB, const int32_t *tab_lo, const int32_t *tab_nsym,
                      const int32_t *tab_freq, const uint32_t *words, const uint32_t *lane_off,
                      const uint32_t *lane_nbits, const uint32_t *lane_state, int32_t *sym) {
    const int64_t n_tiles = ceil_div(N, TB);
    int32_t *cum = (int32_t *)malloc(sizeof(int32_t) * LQ_NSTREAM * (LQ_L + 1));
    int32_t *lookup = (int32_t *)malloc(sizeof(int32_t) * LQ_NSTREAM * LQ_L);
    for (int s = 0; s < LQ_NSTREAM; ++s)
        if (tab_nsym[s] > 0)
            lqo_table_from_freqs(tab_freq + (size_t)s * LQ_L, tab_nsym[s], cum + s * (LQ_L + 1), lookup + s * LQ_L);
    int32_t *out = (int32_t *)malloc(sizeof(int32_t) * (size_t)(TB > 0 ? TB : 1));
    for (int64_t t = 0; t < n_tiles; ++t) {
        const int64_t b0 = t * TB, b1 = (b0 + TB < N) ? b0 + TB : N;
        for (int s = 0; s < LQ_NSTREAM; ++s) {
            const int c = s >> 3, idx = s & 7;
            const int64_t l = t * LQ_NSTREAM + s;
            int64_t n = 0;
            for (int64_t b = b0; b < b1; ++b) n += (coset[b] == c);
            if (n == 0) continue;
            lqo_rans_decode(words + lane_off[l], (int64_t)lane_off[l + 1] - lane_off[l], lane_nbits[l],
                            lane_state[l], lookup + s * LQ_L, tab_freq + (size_t)s * LQ_L, cum + s * (LQ_L + 1), n,
                            out);
            int64_t j = 0;
            for (int64_t b = b0; b < b1; ++b)
                if (coset[b] == c) sym[8 * b + idx] = out[j++] + tab_lo[s];
        }
    }
    free(out);
    free(cum);
    free(lookup);
}

/* q (fp32 lattice points) * fp16 scale -> out_dtype: llm/compressed_kv_cache.py:322-332 */
void lqo_dequant_symbols(const uint8_t *coset, const int32_t *sym, int64_t n_heads, int64_t bph,
                         const uint16_t *scale_f16, void *out, int out_dtype) {
    for (int64_t h = 0; h < n_heads; ++h) {
        const float sc = lqo_f16_to_f32(scale_f16[h]);
        for (int64_t b = 0; b < bph; ++b) {
            const int64_t blk = h * bph + b;
            const int32_t *s = sym + 8 * blk;
            int64_t sum7 = 0;
            for (int i = 0; i < 7; ++i) sum7 += s[i];
            const int64_t c8 = 2 * (int64_t)s[7] + (((sum7 % 2) + 2) % 2);
            const float off = coset[blk] ? 0.5f : 0.0f;
            for (int i = 0; i < 8; ++i) {
                const float q = (i < 7 ? (float)s[i] : (float)c8) + off;
                const float v = q * sc;
                if (out_dtype == 0) ((float *)out)[blk * 8 + i] = v;
                else if (out_dtype == 1) ((uint16_t *)out)[blk * 8 + i] = lqo_f32_to_f16(v);
                else ((uint16_t *)out)[blk * 8 + i] = lqo_f32_to_bf16(v);
            }
        }
    }
}

/*
 * CPU baseline: full round trip (scales, E8, tables, rANS encode, rANS
 * decode, dequant) of n_chunks equal chunks, chunks handed out to n_threads
 * pthreads.  Returns total compressed bytes counted the way
 * CompressedKVCache.compressed_bytes counts them (4*words + coset bytes +
 * 2*n_heads), or a negative error.
 */
typedef struct {
    const void *x;
    void *out;
    int dtype, out_dtype;
    int64_t n_chunks, n_heads, bph, TB;
    float vol_mult;
    int64_t next; /* guarded by mu */
    int64_t total;
    int err;
    pthread_mutex_t mu;
} batch_job_t;

static int64_t roundtrip_one(batch_job_t *J, int64_t ch) {
    const int64_t N = J->n_heads * J->bph;
    const int esz = J->dtype == 0 ? 4 : 2;
    const int osz = J->out_dtype == 0 ? 4 : 2;
    const char *xc = (const char *)J->x + (size_t)ch * (size_t)N * 8 * esz;
    char *oc = (char *)J->out + (size_t)ch * (size_t)N * 8 * osz;
    const int64_t n_heads = J->n_heads, bph = J->bph, TB = J->TB;
    float *sf32 = (float *)malloc(sizeof(float) * (size_t)n_heads);
    uint16_t *sf16 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n_heads);
    uint8_t *cos = (uint8_t *)malloc((size_t)N);
    int32_t *sym = (int32_t *)malloc(sizeof(int32_t) * 8 * (size_t)N);
    int32_t tab_lo[16], tab_nsym[16];
    int32_t *tab_freq = (int32_t *)malloc(sizeof(int32_t) * 16 * LQ_L);
    const int64_t n_tiles = ceil_div(N, TB);
    const int64_t cap = lqo_lane_capacity_words(N, TB);
    uint32_t *words = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)cap);
    uint32_t *loff = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(n_tiles * 16 + 1));
    uint32_t *lnb = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(n_tiles * 16));
    uint32_t *lst = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(n_tiles * 16));
    uint32_t *tn0 = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n_tiles);
    lqo_head_scales(xc, J->dtype, n_heads, bph * 8, J->vol_mult, NULL, sf32, sf16);
    lqo_quantize_chunk(xc, J->dtype, n_heads, bph, sf32, NULL, cos, sym, NULL, 0);
    int rc = lqo_chunk_tables(cos, sym, N, NULL, NULL, NULL, tab_lo, tab_nsym, tab_freq);
    int64_t nw = rc;
    if (rc == 0) nw = lqo_encode_lanes(cos, sym, N, TB, tab_lo, tab_nsym, tab_freq, words, cap, loff, lnb, lst, tn0);
    int64_t bytes = nw;
    if (nw >= 0) {
        memset(sym, 0, sizeof(int32_t) * 8 * (size_t)N);
        lqo_decode_lanes(cos, N, TB, tab_lo, tab_nsym, tab_freq, words, loff, lnb, lst, sym);
        lqo_dequant_symbols(cos, sym, n_heads, bph, sf16, oc, J->out_dtype);
        bytes = 4 * nw + (N + 7) / 8 + 2 * n_heads;
    }
    free(sf32); free(sf16); free(cos); free(sym); free(tab_freq);
    free(words); free(loff); free(lnb); free(lst); free(tn0);
    return bytes;
}

static void *batch_worker(void *arg) {
    batch_job_t *J = (batch_job_t *)arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        const int64_t ch = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (ch >= J->n_chunks) break;
        const int64_t r = roundtrip_one(J, ch);
        pthread_mutex_lock(&J->mu);
        if (r < 0) J->err = (int)r;
        else J->total += r;
        pthread_mutex_unlock(&J->mu);
    }
    return NULL;
}

int64_t lqo_codec_roundtrip_batch(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph,
                                  float vol_mult, int64_t TB, void *out, int out_dtype, int n_threads) {
    batch_job_t J;
    memset(&J, 0, sizeof(J));
    J.x = x; J.out = out; J.dtype = dtype; J.out_dtype = out_dtype;
    J.n_chunks = n_chunks; J.n_heads = n_heads; J.bph = bph; J.TB = TB; J.vol_mult = vol_mult;
    pthread_mutex_init(&J.mu, NULL);
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, batch_worker, &J);
    for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&J.mu);
    return J.err ? J.err : J.total;
}
