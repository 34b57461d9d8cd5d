// lq_tables.cu -- rANS table construction on the device.
//
// Reference: build_rans_table (core/gpu_ans.py:62-98) with the alphabet of
// llm/compressed_kv_cache.py:246-250:
//   alphabet = [min-2, max+2]; freqs = max(int32(counts/total*L), 1)
//   while sum != L: diff > 0 -> +1 to argsort(-counts)[j % n] for j < diff
//                   diff < 0 -> -1 (if > 1) to argsort(-freqs)[j % n] for j < -diff
// The loop is evaluated in closed form per symbol: position p of the order
// is visited diff/n + (p < diff%n) times.  Orders are stable (ties by
// ascending index); numpy's default argsort order among equal keys depends
// on the SIMD sort it dispatches to, so it cannot be reproduced here.  An
// alphabet larger than L raises LQ_EF_ALPHABET (the reference loops forever).
//
// One CTA per table.  Ranks are computed by counting (O(n^2) over the
// alphabet, n <= 1024).
#include "lq_common.cuh"

namespace lq {
namespace {

constexpr int kTT = 256;  // threads per table

__device__ inline uint64_t block_sum_u64(uint64_t v, uint64_t *sh) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    uint64_t t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += sh[i];
    return t;
}

__device__ inline int block_min_i(int v, int *sh) {
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    int t = sh[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) t = min(t, sh[i]);
    return t;
}

__device__ inline int block_max_i(int v, int *sh) {
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    int t = sh[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) t = max(t, sh[i]);
    return t;
}

__global__ void __launch_bounds__(kTT) build_tables_kernel(const uint32_t *__restrict__ hist, int64_t n_tables,
                                                            int32_t *__restrict__ tab_lo, int32_t *__restrict__ tab_nsym,
                                                            uint16_t *__restrict__ tab_freq, uint32_t *err) {
    __shared__ uint32_t cnt[LQ_L + 4];
    __shared__ int32_t freq[LQ_L];
    __shared__ int32_t rnk[LQ_L];
    __shared__ uint64_t red64[kTT / 32];
    __shared__ int redi[kTT / 32];
    const int64_t t = blockIdx.x;
    const uint32_t *h = hist + t * LQ_HIST_BINS;
    uint16_t *fo = tab_freq + t * LQ_L;

    int mn = LQ_HIST_BINS, mx = -1;
    uint64_t tot = 0;
    for (int i = threadIdx.x; i < LQ_HIST_BINS; i += blockDim.x) {
        const uint32_t c = h[i];
        if (c) {
            mn = min(mn, i);
            mx = max(mx, i);
            tot += c;
        }
    }
    mn = block_min_i(mn, redi);
    mx = block_max_i(mx, redi);
    const uint64_t total = block_sum_u64(tot, red64);
    if (total == 0) {  // empty stream: no table (the reference skips the coset)
        if (threadIdx.x == 0) {
            tab_lo[t] = 0;
            tab_nsym[t] = 0;
        }
        for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) fo[i] = 0;
        return;
    }
    const int lo_bin = mn - 2;
    const int n = mx - mn + 5;
    if (threadIdx.x == 0) {
        tab_lo[t] = lo_bin - LQ_SYM_LIMIT;
        tab_nsym[t] = n;
    }
    if (n > LQ_L) {
        if (threadIdx.x == 0) raise_flag(err, LQ_EF_ALPHABET);
        for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) fo[i] = 0;
        return;
    }
    const double dtotal = (double)total;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int b = lo_bin + i;
        const uint32_t c = (b >= 0 && b < LQ_HIST_BINS) ? h[b] : 0u;
        cnt[i] = c;
        // numpy: (counts / total * L).astype(int32), then max(., 1)
        const int f = (int)__dmul_rn(__ddiv_rn((double)c, dtotal), (double)LQ_L);
        freq[i] = f < 1 ? 1 : f;
    }
    __syncthreads();
    // ranks by (counts desc, index asc): fixed across the loop
    bool have_count_rank = false;
    for (int iter = 0; iter < 64; ++iter) {
        uint64_t part = 0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) part += (uint64_t)freq[i];
        const int64_t sum = (int64_t)block_sum_u64(part, red64);
        if (sum == LQ_L) break;
        const int64_t diff = LQ_L - sum;
        if (diff > 0) {
            if (!have_count_rank) {
                for (int i = threadIdx.x; i < n; i += blockDim.x) {
                    const uint32_t ki = cnt[i];
                    int r = 0;
                    for (int j = 0; j < n; ++j) {
                        const uint32_t kj = cnt[j];
                        r += (kj > ki) || (kj == ki && j < i);
                    }
                    rnk[i] = r;
                }
                have_count_rank = true;
                __syncthreads();
            }
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int p = rnk[i];
                freq[i] += (int)(diff / n) + (p < (int)(diff % n) ? 1 : 0);
            }
        } else {
            have_count_rank = false;  // rnk is reused for the freq order
            __syncthreads();
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int ki = freq[i];
                int r = 0;
                for (int j = 0; j < n; ++j) {
                    const int kj = freq[j];
                    r += (kj > ki) || (kj == ki && j < i);
                }
                rnk[i] = r;
            }
            __syncthreads();
            const int64_t d = -diff;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int p = rnk[i];
                const int visits = (int)(d / n) + (p < (int)(d % n) ? 1 : 0);
                const int f = freq[i];
                freq[i] = f - min(visits, f - 1);
            }
        }
        __syncthreads();
        if (iter == 63 && threadIdx.x == 0) raise_flag(err, LQ_EF_NOCONVERGE);
    }
    for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) fo[i] = (uint16_t)(i < n ? freq[i] : 0);
}

// enc entry: f | cf << 11 | k0 << 21, k0 = max(0, 9 - floor(log2 f)): the
// encoder emits k0 or k0+1 bits from a state in [L, 2L).
// dec entry: si | nb << 10 | (base - L) << 14 for slot in [cf, cf+f):
//   x' = f + slot - cf; nb = bits the decoder reads; base = x' << nb.
__global__ void __launch_bounds__(kTT) expand_tables_kernel(const int32_t *__restrict__ tab_nsym,
                                                             const uint16_t *__restrict__ tab_freq,
                                                             uint32_t *__restrict__ enc_tab,
                                                             uint32_t *__restrict__ dec_tab, uint32_t *err) {
    __shared__ int32_t cf[LQ_L + 1];
    __shared__ int32_t wsum[kTT / 32];
    const int64_t t = blockIdx.x;
    const int n = tab_nsym[t];
    uint32_t *enc = enc_tab ? enc_tab + t * LQ_L : nullptr;
    uint32_t *dec = dec_tab ? dec_tab + t * LQ_L : nullptr;
    if (n <= 0 || n > LQ_L) {
        for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) {
            if (enc) enc[i] = 0;
            if (dec) dec[i] = 0;
        }
        return;
    }
    const uint16_t *f = tab_freq + t * LQ_L;
    // exclusive prefix of f over n entries: 4 entries per thread
    const int per = (LQ_L + kTT - 1) / kTT;
    int loc[(LQ_L + kTT - 1) / kTT];
    int s = 0;
    for (int k = 0; k < per; ++k) {
        const int i = threadIdx.x * per + k;
        loc[k] = (i < n) ? (int)f[i] : 0;
        s += loc[k];
    }
    int inc = s;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) wsum[w] = inc;
    __syncthreads();
    int base = 0;
    for (int i = 0; i < w; ++i) base += wsum[i];
    int run = base + inc - s;
    for (int k = 0; k < per; ++k) {
        const int i = threadIdx.x * per + k;
        if (i < n) cf[i] = run;
        run += loc[k];
    }
    if (threadIdx.x == blockDim.x - 1) cf[n] = run;  // total of all frequencies
    __syncthreads();
    if (threadIdx.x == 0 && cf[n] != LQ_L) raise_flag(err, LQ_EF_ALPHABET);
    for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) {
        if (enc) {
            uint32_t e = 0;
            if (i < n) {
                const int fi = f[i];
                const int g = 31 - __clz(fi > 0 ? fi : 1);
                const int k0 = max(0, 9 - g);
                e = (uint32_t)fi | ((uint32_t)cf[i] << 11) | ((uint32_t)k0 << 21);
            }
            enc[i] = e;
        }
    }
    if (dec) {
        for (int si = threadIdx.x; si < n; si += blockDim.x) {
            const int fi = f[si], c0 = cf[si];
            for (int slot = c0; slot < c0 + fi && slot < LQ_L; ++slot) {
                const uint32_t xp = (uint32_t)(fi + slot - c0);
                const uint32_t nb = xp >= (uint32_t)LQ_L ? 0u : (uint32_t)(__clz(xp) - 21);
                const uint32_t b = xp << nb;
                dec[slot] = (uint32_t)si | (nb << 10) | ((b - LQ_L) << 14);
            }
        }
    }
}

}  // namespace
}  // namespace lq

extern "C" int lq_build_tables(const uint32_t *hist, int64_t n_tables, int32_t *tab_lo, int32_t *tab_nsym,
                               uint16_t *tab_freq, uint32_t *err, void *stream) {
    if (n_tables < 0) return LQ_ERR_INVALID;
    if (n_tables == 0) return LQ_OK;
    if (!hist || !tab_lo || !tab_nsym || !tab_freq) return LQ_ERR_INVALID;
    lq::build_tables_kernel<<<(unsigned)n_tables, lq::kTT, 0, lq::as_stream(stream)>>>(hist, n_tables, tab_lo,
                                                                                        tab_nsym, tab_freq, err);
    return lq::check_launch();
}

extern "C" int lq_expand_tables(const int32_t *tab_nsym, const uint16_t *tab_freq, int64_t n_tables,
                                uint32_t *enc_tab, uint32_t *dec_tab, uint32_t *err, void *stream) {
    if (n_tables < 0) return LQ_ERR_INVALID;
    if (n_tables == 0) return LQ_OK;
    if (!tab_nsym || !tab_freq || (!enc_tab && !dec_tab)) return LQ_ERR_INVALID;
    lq::expand_tables_kernel<<<(unsigned)n_tables, lq::kTT, 0, lq::as_stream(stream)>>>(tab_nsym, tab_freq, enc_tab,
                                                                                         dec_tab, err);
    return lq::check_launch();
}
