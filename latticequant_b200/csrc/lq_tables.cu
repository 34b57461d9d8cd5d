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

// Rank of every entry under (key descending, index ascending): bitonic sort
// of (~key << 32 | index) over the next power of two >= n, in shared memory.
__device__ void stable_desc_ranks(const int32_t *key, int n, uint64_t *sk, int32_t *rnk) {
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    for (int i = threadIdx.x; i < n2; i += blockDim.x)
        sk[i] = i < n ? (((uint64_t)(0xffffffffu - (uint32_t)key[i]) << 32) | (uint32_t)i) : ~0ull;
    __syncthreads();
    for (int k = 2; k <= n2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n2; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = sk[i], b = sk[ixj];
                    if (((i & k) == 0) == (a > b)) {
                        sk[i] = b;
                        sk[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int p = threadIdx.x; p < n; p += blockDim.x) rnk[(uint32_t)(sk[p] & 0xffffffffu)] = p;
    __syncthreads();
}

__global__ void __launch_bounds__(kTT) build_tables_kernel(const uint32_t *__restrict__ hist, int64_t n_tables,
                                                            int32_t *__restrict__ tab_lo, int32_t *__restrict__ tab_nsym,
                                                            uint16_t *__restrict__ tab_freq, uint32_t *err) {
    __shared__ int32_t cnt[LQ_L];
    __shared__ int32_t freq[LQ_L];
    __shared__ int32_t rnk[LQ_L];
    __shared__ uint64_t sk[LQ_L];
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
        cnt[i] = (int32_t)c;  // counts per stream stay below 2^31 (blocks per chunk < 2^31)
        // numpy: (counts / total * L).astype(int32), then max(., 1)
        const int f = (int)__dmul_rn(__ddiv_rn((double)c, dtotal), (double)LQ_L);
        freq[i] = f < 1 ? 1 : f;
    }
    __syncthreads();
    __shared__ int32_t cand[LQ_L];
    __shared__ int n_cand;
    bool have_count_rank = false;
    // Each pass of the reference loop either fixes the sum (diff > 0: one
    // increment pass) or removes at least one from a frequency > 1, so at most
    // L + 1 passes run; the bound only guards against a corrupt histogram.
    for (int iter = 0; iter <= LQ_L + 1; ++iter) {
        uint64_t part = 0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) part += (uint64_t)freq[i];
        const int64_t sum = (int64_t)block_sum_u64(part, red64);
        if (sum == LQ_L) break;
        if (iter == LQ_L + 1) {
            if (threadIdx.x == 0) raise_flag(err, LQ_EF_NOCONVERGE);
            break;
        }
        const int64_t diff = LQ_L - sum;
        if (diff > 0) {
            // argsort(-counts): fixed across iterations
            if (!have_count_rank) {
                stable_desc_ranks(cnt, n, sk, rnk);
                have_count_rank = true;
            }
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int p = rnk[i];
                freq[i] += (int)(diff / n) + (p < (int)(diff % n) ? 1 : 0);
            }
            __syncthreads();
            continue;
        }
        // diff < 0: argsort(-freqs).  Entries at 1 are never decremented and
        // sort after every entry > 1, so only the m entries > 1 matter, at
        // positions 0..m-1 of the order.
        have_count_rank = false;
        if (threadIdx.x == 0) n_cand = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x)
            if (freq[i] > 1) cand[atomicAdd(&n_cand, 1)] = i;
        __syncthreads();
        const int m = n_cand;
        if (m <= 32) {
            // warp 0 finishes every remaining pass in registers
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                // one candidate per lane (lane order is irrelevant: positions
                // compare frequencies and symbol indices)
                const int my = lane < m ? cand[lane] : 0x7fffffff;
                const bool act = lane < m;
                int f = act ? freq[my] : 1;
                int64_t d = -diff;
                for (int pass = 0; pass <= LQ_L + 1 && d > 0; ++pass) {
                    // position among entries > 1: (f desc, index asc)
                    int pos = 0;
                    for (int q = 0; q < 32; ++q) {
                        const int fq = __shfl_sync(0xffffffffu, f, q);
                        const int iq = __shfl_sync(0xffffffffu, my, q);
                        pos += (fq > 1 && (fq > f || (fq == f && iq < my))) ? 1 : 0;
                    }
                    int dec = 0;
                    if (act && f > 1) {
                        const int visits = (int)(d / n) + (pos < (int)(d % n) ? 1 : 0);
                        dec = min(visits, f - 1);
                        f -= dec;
                    }
                    int tot = dec;
                    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
                    d -= tot;
                    if (tot == 0) break;  // cannot happen while sum > L: some entry is > 1
                }
                if (act) freq[my] = f;
            }
            __syncthreads();
            continue;
        }
        stable_desc_ranks(freq, n, sk, rnk);
        const int64_t d = -diff;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const int p = rnk[i];
            const int visits = (int)(d / n) + (p < (int)(d % n) ? 1 : 0);
            const int f = freq[i];
            freq[i] = f - min(visits, f - 1);
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < LQ_L; i += blockDim.x) fo[i] = (uint16_t)(i < n ? freq[i] : 0);
}

// enc entry: (2f << k0) | k0 << 12 | (L + cf - f) << 16, k0 = max(0, 9 -
// floor(log2 f)): from a state x in [L, 2L) the encoder emits k = k0 +
// (x >= 2f << k0) bits (the same test as x >> k0 >= 2f) and moves to
// (x >> k) + L + cf - f.  2f << k0 lies in [L, 2L], so it fits 12 bits.
// dec entry: si | nb << 10 | base << 14 for slot in [cf, cf+f):
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
                e = ((uint32_t)(2 * fi) << k0) | ((uint32_t)k0 << 12) | ((uint32_t)(LQ_L + cf[i] - fi) << 16);
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
                const uint32_t b = xp << nb;  // in [L, 2L)
                dec[slot] = (uint32_t)si | (nb << 10) | (b << 14);
            }
        }
    }
}

}  // namespace
}  // namespace lq

extern "C" int lq_build_tables(const uint32_t *hist, int64_t n_tables, int32_t *tab_lo, int32_t *tab_nsym,
                               uint16_t *tab_freq, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_tables < 0) return LQ_ERR_INVALID;
    if (n_tables == 0) return LQ_OK;
    if (!hist || !tab_lo || !tab_nsym || !tab_freq) return LQ_ERR_INVALID;
    lq::build_tables_kernel<<<(unsigned)n_tables, lq::kTT, 0, lq::as_stream(stream)>>>(hist, n_tables, tab_lo,
                                                                                        tab_nsym, tab_freq, err);
    return lq::check_launch();
}

extern "C" int lq_expand_tables(const int32_t *tab_nsym, const uint16_t *tab_freq, int64_t n_tables,
                                uint32_t *enc_tab, uint32_t *dec_tab, uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_tables < 0) return LQ_ERR_INVALID;
    if (n_tables == 0) return LQ_OK;
    if (!tab_nsym || !tab_freq || (!enc_tab && !dec_tab)) return LQ_ERR_INVALID;
    lq::expand_tables_kernel<<<(unsigned)n_tables, lq::kTT, 0, lq::as_stream(stream)>>>(tab_nsym, tab_freq, enc_tab,
                                                                                         dec_tab, err);
    return lq::check_launch();
}
