// lq_rans.cu -- bit-granular rANS (L = 1024) lane encode / decode.
//
// Reference coder (core/gpu_ans.py):
//   encode (:105-139): x = L; for s in reversed(symbols):
//       while x >= 2f: emit x & 1; x >>= 1
//       x = L*(x // f) + cf + x % f
//     bits reversed, packed LSB-first into u32 words; returns (words, x, n_bits)
//   decode (:146-168): slot = x & (L-1); s = lookup[slot];
//       x = f*(x >> 10) + slot - cf; while x < L and pos < n_bits: x = 2x | bit[pos++]
//
// Encoder, one thread per lane.  With x in [L, 2L) the k emitted bits are
// k0 or k0+1 (k0 from the table entry), so one compare replaces the shift
// loop; the k low bits of x are prepended to a 64-bit accumulator and whole
// 32-bit words leave it toward the FRONT of a per-lane scratch slot, which
// therefore ends up holding the stream MSB-first, end-aligned.  A scan over
// lane sizes and a compaction pass (funnel shift + bit reverse) then lay the
// lanes back to back in the reference's LSB-first word format.
//
// Decoder, one thread per lane, table-driven: for x in [L, 2L) the entry for
// slot gives (symbol, nb, base) and x = base | next nb bits (bit-reversed
// words read MSB-first from a 64-bit buffer).  Near the end of a lane, or for
// a state outside [L, 2L), the reference formula runs literally, including
// its stop at n_bits, so truncated or odd streams decode exactly as the
// reference decodes them.
#include "lq_tiledec.cuh"

namespace lq {
namespace {

// ---------------------------------------------------------------- encode
// Table entry (lq_expand_tables): (2f << k0) | k0 << 12 | (L + cf - f) << 16.
// From x in [L, 2L): k = k0 + (x >= 2f << k0) bits leave (the k low bits of
// x), then x' = (x >> k) + L + cf - f.  The k bits are prepended to a 32-bit
// accumulator; full words are written toward the front of the lane's slot.
//
// A CTA takes kEncTiles tiles of one chunk (16 lanes each) and stages the
// chunk's 16 coder tables (64 KB) in shared memory.  Each lane reads its
// symbols from its int8 coordinate column of the tile (lq_e8_quantize's
// lane-major layout): coset-0 lanes walk the coset-0 prefix backward,
// coset-1 lanes the coset-1 suffix forward, 8 symbols per 8-byte load once
// aligned (a coset-0 lane reverses each loaded vector).  A tile flagged for
// symbols outside [-127, 127] reads them one by one, taking a -128 from the
// int16 plane.
constexpr int kEncTiles = 32;
constexpr size_t kEncSmem = (size_t)LQ_NSTREAMS * LQ_L * 4;

__device__ __forceinline__ uint2 reverse8(uint2 u) {
    return make_uint2(__byte_perm(u.y, 0, 0x0123), __byte_perm(u.x, 0, 0x0123));
}
// byte k of w, sign-extended: prmt's default mode replicates the selected
// byte's top bit where a selector nibble has bit 3 set
template <int K>
__device__ __forceinline__ int sbyte(uint32_t w) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "n"(K | (8 | K) << 4 | (8 | K) << 8 | (8 | K) << 12));
    return r;
}

__global__ void __launch_bounds__(16 * kEncTiles, 2) encode_lanes_kernel(
    SymCols symc, const uint32_t *__restrict__ tile_n0, uint32_t n_tiles, uint32_t N,
    uint32_t TB, const int32_t *__restrict__ tab_lo, const int32_t *__restrict__ tab_nsym,
    const uint32_t *__restrict__ enc_tab, uint32_t *__restrict__ scratch, uint32_t slot_words,
    uint32_t *__restrict__ lane_nbits, uint32_t *__restrict__ lane_state, uint32_t *__restrict__ lane_nwords,
    uint32_t *err) {
    extern __shared__ __align__(16) uint32_t etab[];
    const uint32_t chunk = blockIdx.y;
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(enc_tab + (size_t)chunk * LQ_NSTREAMS * LQ_L);
        uint4 *dst = reinterpret_cast<uint4 *>(etab);
        for (int i = threadIdx.x; i < LQ_NSTREAMS * LQ_L / 4; i += blockDim.x) dst[i] = __ldg(src + i);
    }
    __syncthreads();
    const uint32_t tile = blockIdx.x * kEncTiles + (threadIdx.x >> 4);
    if (tile >= n_tiles) return;
    const uint32_t s = threadIdx.x & 15u, c = s >> 3, idx = s & 7u;
    const uint32_t lg = (chunk * n_tiles + tile) * LQ_NSTREAMS + s;
    const uint32_t tb = (tile * TB + TB <= N) ? TB : N - tile * TB;
    const uint32_t n0 = tile_n0[chunk * n_tiles + tile];
    const int n = (int)(c ? tb - n0 : n0);
    const uint32_t tabi = chunk * LQ_NSTREAMS + s;
    uint32_t *out = scratch + (size_t)lg * slot_words + slot_words;  // written backward
    uint32_t x = LQ_L, nbits = 0;
    if (n > 0) {
        const int lo = tab_lo[tabi];
        const int nsym = tab_nsym[tabi];
        if (nsym <= 0 || nsym > LQ_L) {
            raise_flag(err, LQ_EF_ALPHABET);
            lane_nbits[lg] = 0;
            lane_state[lg] = LQ_L;
            lane_nwords[lg] = 0;
            return;
        }
        const uint32_t tab = smem_addr(etab) + s * (LQ_L * 4);
        const size_t c0 = ((size_t)chunk * n_tiles + tile) * TB * 8 + (size_t)idx * TB;
        const int8_t *col = symc.cols + c0;
        const int16_t *colw = symc.wide + c0;
        const bool esc = symc.esc[(size_t)chunk * n_tiles + tile] != 0u;
        uint32_t acc = 0, cnt = 0, simax = 0;  // simax: largest alphabet index seen (unsigned)
        uint32_t *const out_end = out;
        auto code = [&](int v) {
            const uint32_t si = (uint32_t)(v - lo);
            simax = max(simax, si);
            const uint32_t e = lds_u32(tab + ((si & (LQ_L - 1)) << 2));
            const uint32_t xmax = e & 0xfffu, k0 = (e >> 12) & 0xfu;
            const uint32_t k = k0 + (x >= xmax ? 1u : 0u);
            const uint32_t w = x & ~(0xffffffffu << k);
            acc |= w << cnt;
            const uint32_t t = cnt + k;
            if (t >= 32u) {
                *--out = acc;
                acc = w >> (32u - cnt);
            }
            cnt = t & 31u;
            x = (x >> k) + (e >> 16);
        };
        // symbol j (coding order) sits at col[n0 + j] (coset 1) or col[n0 - 1 - j] (coset 0)
        auto sym_at = [&](int j) {
            const int p = c ? (int)n0 + j : (int)n0 - 1 - j;
            const int v = col[p];
            return v == -128 ? (int)colw[p] : v;
        };
        const int head = min(n, c ? (int)((8u - (n0 & 7u)) & 7u) : (int)(((n0 - 1u) & 7u) + 1u) & 7);
        int j = 0;
        for (; j < head; ++j) code(sym_at(j));
        if (j + 8 <= n) {
            const uint2 *vp = reinterpret_cast<const uint2 *>(col + (c ? (int)n0 + j : (int)n0 - 1 - j - 7));
            const int step = c ? 1 : -1;
            uint2 cur = __ldg(vp);
            for (; j + 8 <= n; j += 8) {
                vp += step;
                const uint2 nxt = (j + 16 <= n) ? __ldg(vp) : cur;
                const uint2 u = c ? cur : reverse8(cur);
                int v[8] = {sbyte<0>(u.x), sbyte<1>(u.x), sbyte<2>(u.x), sbyte<3>(u.x),
                            sbyte<0>(u.y), sbyte<1>(u.y), sbyte<2>(u.y), sbyte<3>(u.y)};
                if (esc) {  // uniform over the tile's 16 lanes
                    const int p = c ? (int)n0 + j : (int)n0 - 1 - j;
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (v[k] == -128) v[k] = colw[c ? p + k : p - k];
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) code(v[k]);
                cur = nxt;
            }
        }
        for (; j < n; ++j) code(sym_at(j));
        if (simax >= (uint32_t)nsym) raise_flag(err, LQ_EF_SYMRANGE);
        nbits = 32u * (uint32_t)(out_end - out) + cnt;
        if (cnt) *--out = acc;
    }
    lane_nbits[lg] = nbits;
    lane_state[lg] = x;
    lane_nwords[lg] = (nbits + 31u) >> 5;
}

// ---------------------------------------------------------------- scan
constexpr int kScanT = 256;
constexpr int kScanItems = 16;
constexpr int64_t kScanTile = (int64_t)kScanT * kScanItems;

__device__ inline uint64_t block_incl_scan(uint64_t v, uint64_t *sh_w) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) sh_w[w] = v;
    __syncthreads();
    uint64_t base = 0;
    for (int i = 0; i < w; ++i) base += sh_w[i];
    __syncthreads();
    return base + v;
}

__global__ void __launch_bounds__(kScanT) scan_reduce_kernel(const uint32_t *__restrict__ cnt, int64_t n,
                                                              uint64_t *__restrict__ block_sums) {
    __shared__ uint64_t sh[kScanT / 32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    uint64_t s = 0;
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + (int64_t)k * kScanT + threadIdx.x;
        if (i < n) s += cnt[i];
    }
    const uint64_t t = block_incl_scan(s, sh);
    if (threadIdx.x == kScanT - 1) block_sums[blockIdx.x] = t;
}

// single CTA: exclusive scan of block sums in place
__global__ void __launch_bounds__(kScanT) scan_blocks_kernel(uint64_t *__restrict__ block_sums, int64_t nb) {
    __shared__ uint64_t sh[kScanT / 32];
    __shared__ uint64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t b0 = 0; b0 < nb; b0 += kScanT) {
        const int64_t i = b0 + threadIdx.x;
        const uint64_t v = i < nb ? block_sums[i] : 0;
        const uint64_t inc = block_incl_scan(v, sh);
        const uint64_t c0 = carry;
        if (i < nb) block_sums[i] = c0 + inc - v;
        __syncthreads();
        if (threadIdx.x == kScanT - 1) carry = c0 + inc;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kScanT) scan_write_kernel(const uint32_t *__restrict__ cnt, int64_t n,
                                                             const uint64_t *__restrict__ block_off,
                                                             uint32_t *__restrict__ off, int64_t cap, uint32_t *err) {
    __shared__ uint64_t sh[kScanT / 32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    // each thread owns kScanItems consecutive entries
    uint32_t v[kScanItems];
    uint64_t s = 0;
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
        v[k] = i < n ? cnt[i] : 0u;
        s += v[k];
    }
    uint64_t run = block_off[blockIdx.x] + block_incl_scan(s, sh) - s;
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
        if (i < n) off[i] = (uint32_t)run;
        run += v[k];
        if (i == n - 1) {
            off[n] = (uint32_t)run;
            if ((int64_t)run > cap || run > 0xffffffffull) raise_flag(err, LQ_EF_CAPACITY);
        }
    }
}

// ---------------------------------------------------------------- compaction
// Output word i of a lane is the bit-reversed funnel of slot words i (high)
// and i + 1 (low) by the lane's pad.  A warp takes kCompactLanes
// consecutive lanes and covers 64 words of each per round: every thread
// loads words i and i + 32 of every lane (thread 31 also word i + 64), all
// before the first store, so that a warp keeps several lanes' loads in
// flight; the low neighbours come by shuffle.  The word count follows from
// the bit count (the encoder stores both); threads 0..kCompactLanes-1 load
// the lanes' metadata at once.
constexpr int kCompactLanes = 4;

__global__ void __launch_bounds__(256) compact_lanes_kernel(const uint32_t *__restrict__ scratch, int64_t slot_words,
                                                             int64_t n_lanes, const uint32_t *__restrict__ lane_off,
                                                             const uint32_t *__restrict__ lane_nbits,
                                                             uint32_t *__restrict__ words, int64_t cap) {
    const int lane = threadIdx.x & 31;
    const int64_t lg0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kCompactLanes;
    if (lg0 >= n_lanes) return;  // warp-uniform
    uint32_t my_nb = 0, my_off = 0;
    if (lane < kCompactLanes && lg0 + lane < n_lanes) {
        my_nb = __ldg(lane_nbits + lg0 + lane);
        my_off = __ldg(lane_off + lg0 + lane);
    }
    int64_t nw[kCompactLanes], dst0[kCompactLanes];
    uint32_t pad[kCompactLanes];
    int64_t nw_max = 0;
#pragma unroll
    for (int k = 0; k < kCompactLanes; ++k) {
        const uint32_t nb = __shfl_sync(0xffffffffu, my_nb, k);
        dst0[k] = __shfl_sync(0xffffffffu, my_off, k);
        nw[k] = (int64_t)((nb + 31u) >> 5);
        if (dst0[k] + nw[k] > cap) nw[k] = 0;  // capacity error already flagged by the scan
        pad[k] = (32u - (nb & 31u)) & 31u;
        nw_max = max(nw_max, nw[k]);
    }
    for (int64_t i0 = 0; i0 < nw_max; i0 += 64) {
        const int64_t i = i0 + lane, i2 = i + 32;
        uint32_t a[kCompactLanes], b[kCompactLanes], t[kCompactLanes];
#pragma unroll
        for (int k = 0; k < kCompactLanes; ++k) {
            const uint32_t *src = scratch + (lg0 + k) * slot_words + (slot_words - nw[k]);
            a[k] = i < nw[k] ? __ldg(src + i) : 0u;
            b[k] = i2 < nw[k] ? __ldg(src + i2) : 0u;
            t[k] = (lane == 31 && i0 + 64 < nw[k]) ? __ldg(src + i0 + 64) : 0u;
        }
#pragma unroll
        for (int k = 0; k < kCompactLanes; ++k) {
            const uint32_t a_next = __shfl_down_sync(0xffffffffu, a[k], 1);
            const uint32_t b_first = __shfl_sync(0xffffffffu, b[k], 0);
            const uint32_t b_next = __shfl_down_sync(0xffffffffu, b[k], 1);
            const uint32_t lo_a = lane == 31 ? b_first : a_next;  // word i + 1 (0 past the end)
            const uint32_t lo_b = lane == 31 ? t[k] : b_next;     // word i + 33
            uint32_t *dst = words + dst0[k];
            if (i < nw[k]) dst[i] = __brev(__funnelshift_l(lo_a, a[k], pad[k]));
            if (i2 < nw[k]) dst[i2] = __brev(__funnelshift_l(lo_b, b[k], pad[k]));
        }
    }
}

// ---------------------------------------------------------------- decode
// MSB-first reader over a lane's words (reference words bit-reversed).
struct BitReader {
    const uint32_t *w;
    int64_t nw, wi;
    uint64_t buf;  // next bits at the top
    int cnt;       // valid bits in buf
    __device__ void init(const uint32_t *words, int64_t n_words) {
        w = words;
        nw = n_words;
        wi = 0;
        buf = 0;
        cnt = 0;
        refill();
    }
    __device__ __forceinline__ void refill() {
        while (cnt <= 32 && wi < nw) {
            buf |= (uint64_t)__brev(__ldg(w + wi)) << (32 - cnt);
            ++wi;
            cnt += 32;
        }
    }
    // nb in [0, 32]; bits past the end of the words read as 0
    __device__ __forceinline__ uint32_t read(int nb) {
        const uint32_t v = nb ? (uint32_t)(buf >> (64 - nb)) : 0u;
        buf = nb == 64 ? 0 : buf << nb;
        cnt -= nb;
        if (cnt < 0) cnt = 0;
        if (cnt <= 32) refill();
        return v;
    }
};

// Decode n symbols of one lane into out[j*ostride] (alphabet index).
// dec: fast table (or nullptr), freq/cf source for the literal path.
struct LaneTables {
    const uint32_t *dec;    // [L] si | nb << 10 | base << 14
    const uint32_t *enc;    // [nsym] f | cf << 11 (literal path), or nullptr
    const uint16_t *freq;   // [nsym] frequencies (literal path when enc == nullptr)
};

__device__ inline void literal_step(uint32_t &x, int64_t &pos, int64_t n_bits, uint32_t si, uint32_t f, uint32_t cf,
                                    uint32_t slot, BitReader &br) {
    x = f * (x >> LQ_LOG2_L) + slot - cf;
    while (x < (uint32_t)LQ_L && pos < n_bits) {
        x = (x << 1) | br.read(1);
        ++pos;
    }
}

template <typename Emit>
__device__ inline void decode_lane(const uint32_t *words, int64_t n_words, int64_t n_bits, uint32_t state, int64_t n,
                                   const uint32_t *dec, const uint16_t *freq, Emit emit) {
    BitReader br;
    br.init(words, n_words);
    uint32_t x = state;
    int64_t pos = 0;
    for (int64_t j = 0; j < n; ++j) {
        const uint32_t slot = x & (LQ_L - 1);
        const uint32_t e = dec[slot];
        const uint32_t si = e & 0x3ffu;
        emit(j, si);
        if ((x >> LQ_LOG2_L) == 1u && pos + 10 <= n_bits) {
            const int nb = (int)((e >> 10) & 0xfu);
            x = (e >> 14) | br.read(nb);
            pos += nb;
        } else {
            // literal reference semantics (end of lane, or state outside [L, 2L))
            const uint32_t f = freq[si];
            const uint32_t xp = (e >> 14) >> ((e >> 10) & 0xfu);  // f + slot - cf
            const uint32_t cf = f + slot - xp;
            literal_step(x, pos, n_bits, si, f, cf, slot, br);
        }
    }
}

// General path: thread per lane, symbols to the encoder's row layout.
__global__ void __launch_bounds__(256) decode_lanes_kernel(
    const uint32_t *__restrict__ words, int64_t n_words, const uint32_t *__restrict__ lane_off,
    const uint32_t *__restrict__ lane_nbits, const uint32_t *__restrict__ lane_state,
    const uint32_t *__restrict__ tile_n0, int64_t n_lanes, int64_t n_tiles, int64_t N, int64_t TB,
    const int32_t *__restrict__ tab_lo, const int32_t *__restrict__ tab_nsym, const uint16_t *__restrict__ tab_freq,
    const uint32_t *__restrict__ dec_tab, int16_t *__restrict__ sym_rows, uint32_t *err) {
    const int64_t lg = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (lg >= n_lanes) return;
    const int64_t per_chunk = n_tiles * LQ_NSTREAMS;
    const int64_t chunk = lg / per_chunk;
    const int64_t rem = lg - chunk * per_chunk;
    const int64_t tile = rem >> 4;
    const int s = (int)(rem & 15), c = s >> 3, idx = s & 7;
    const int64_t tb = (tile * TB + TB <= N) ? TB : N - tile * TB;
    const int64_t n0 = tile_n0[chunk * n_tiles + tile];
    const int64_t n = c ? tb - n0 : n0;
    if (n <= 0) return;
    const int64_t tabi = chunk * LQ_NSTREAMS + s;
    const int lo = tab_lo[tabi];
    const int nsym = tab_nsym[tabi];
    int16_t *rows = sym_rows + (chunk * n_tiles + tile) * TB * 8 + idx;
    if (nsym <= 0 || nsym > LQ_L) {
        raise_flag(err, LQ_EF_ALPHABET);
        return;
    }
    const int64_t w0 = lane_off[lg];
    const int64_t nb = lane_nbits[lg];
    const int64_t nw = ceil_div(nb, 32);
    if (w0 + nw > n_words) {
        raise_flag(err, LQ_EF_BITSTREAM);
        return;
    }
    // rank r of coset 0 -> row r; of coset 1 -> row tb-1-r
    decode_lane(words + w0, nw, nb, lane_state[lg], n, dec_tab + tabi * LQ_L, tab_freq + tabi * LQ_L,
                [&](int64_t r, uint32_t si) {
                    const int64_t row = c ? tb - 1 - r : r;
                    rows[row * 8] = (int16_t)((int)si + lo);
                });
}

// Exclusive count of coset-1 blocks before each coset word, within its tile.
__global__ void __launch_bounds__(256) coset_rank_kernel(const uint32_t *__restrict__ coset_words, int64_t n_chunks,
                                                          int64_t words_per_chunk, int64_t words_per_tile,
                                                          uint32_t *__restrict__ rank1) {
    // one thread per tile, sequential over the tile's words
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t tiles_per_chunk = ceil_div(words_per_chunk, words_per_tile);
    if (g >= n_chunks * tiles_per_chunk) return;
    const int64_t chunk = g / tiles_per_chunk, tile = g % tiles_per_chunk;
    const int64_t w0 = tile * words_per_tile;
    const int64_t w1 = (w0 + words_per_tile < words_per_chunk) ? w0 + words_per_tile : words_per_chunk;
    const uint32_t *cw = coset_words + chunk * words_per_chunk;
    uint32_t *r = rank1 + chunk * words_per_chunk;
    uint32_t run = 0;
    for (int64_t w = w0; w < w1; ++w) {
        r[w] = run;
        run += __popc(cw[w]);
    }
}

template <int DO>
__global__ void __launch_bounds__(256) reconstruct_kernel(const int16_t *__restrict__ sym_rows,
                                                           const uint32_t *__restrict__ coset_words,
                                                           const uint32_t *__restrict__ rank1, int64_t n_chunks,
                                                           int64_t n_heads, int64_t bph, int64_t TB, int64_t n_tiles,
                                                           const uint16_t *__restrict__ scale_f16, void *out,
                                                           int32_t *sym_out, FastDiv n_div, FastDiv tb_div,
                                                           FastDiv bph_div) {
    const int64_t gb = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t N = n_heads * bph;
    if (gb >= n_chunks * N) return;
    // gb < 2^31 * 65535: split into chunk and block with 32-bit divisions
    const int64_t chunk = (gb >> 31) == 0 ? (int64_t)n_div.div((uint32_t)gb) : gb / N;
    const int64_t b = gb - chunk * N;
    const int64_t tile = tb_div.div((uint32_t)b), p = b - tile * TB;
    const int64_t tb = (tile * TB + TB <= N) ? TB : N - tile * TB;
    const int64_t wpc = ceil_div(N, 32);
    const uint32_t word = coset_words[chunk * wpc + (b >> 5)];
    const int bit = (int)(b & 31);
    const uint32_t below = __popc(word & ((1u << bit) - 1u));
    const int64_t r1 = rank1[chunk * wpc + (b >> 5)] + below;  // coset-1 blocks before b in the tile
    const int c = (word >> bit) & 1u;
    const int64_t row = c ? tb - 1 - r1 : p - r1;
    const uint4 u = reinterpret_cast<const uint4 *>(sym_rows + (chunk * n_tiles + tile) * TB * 8)[row];
    int sym[8];
    sym[0] = (int16_t)(u.x & 0xffffu); sym[1] = (int16_t)(u.x >> 16);
    sym[2] = (int16_t)(u.y & 0xffffu); sym[3] = (int16_t)(u.y >> 16);
    sym[4] = (int16_t)(u.z & 0xffffu); sym[5] = (int16_t)(u.z >> 16);
    sym[6] = (int16_t)(u.w & 0xffffu); sym[7] = (int16_t)(u.w >> 16);
    if (sym_out) {
        int4 *so = reinterpret_cast<int4 *>(sym_out) + 2 * gb;
        so[0] = make_int4(sym[0], sym[1], sym[2], sym[3]);
        so[1] = make_int4(sym[4], sym[5], sym[6], sym[7]);
    }
    if constexpr (DO >= 0) {
        float q[8];
        e8_from_symbols(c, sym, q);
        const float sc = __half2float(__ushort_as_half(scale_f16[chunk * n_heads + bph_div.div((uint32_t)b)]));
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(q[i], sc);
        store_block8<DO>(out, gb, q);
    }
}

// ---------------------------------------------------------------- fused decode
// Decode + dequantise: lq_tiledec.cuh's position-ordered tile decoder with
// an epilogue that rebuilds the E8 point (symbols_to_e8) and writes it times
// the fp16 head scale; a half-warp writes 16 consecutive blocks per step.
constexpr int kDecR = 48;                                             // ring rows per round
constexpr size_t kDecRingBytes = (size_t)(kDecR + 2) * kRingStride * 2;  // + 2 carried rows
__host__ __device__ inline size_t fused_smem_bytes(int nwarps) { return kTablesSmem + (size_t)nwarps * kDecRingBytes; }

template <int DO>
__global__ void __launch_bounds__(1024, 1) decode_fused_kernel(ChunkDev a, FastDiv bph_div, void *__restrict__ out,
                                                              int32_t *__restrict__ sym_out, uint32_t *err) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t *dtab = reinterpret_cast<uint32_t *>(smem);
    const int nwarps = blockDim.x >> 5;
    const uint32_t ring = smem_addr(smem + kTablesSmem + (size_t)(threadIdx.x >> 5) * kDecRingBytes);
    const uint32_t chunk = blockIdx.y;
    stage_tables(a, chunk, dtab);
    __syncthreads();
    const uint32_t tile0 = (blockIdx.x * nwarps + (threadIdx.x >> 5)) * 2;
    if (tile0 >= a.n_tiles) return;
    const uint32_t N = a.n_heads * a.bph;
    auto epi = [&](bool ok, int t, uint32_t grp, uint32_t j, uint32_t cc, const uint4 blk) {
        if (!ok) return;
        const uint32_t b = (tile0 + t) * a.TB + grp * 16 + j;
        const size_t gb = (size_t)chunk * N + b;
        if (sym_out) {
            int sym[8];
            ring_symbols(blk, cc, sym);
            int4 *so = reinterpret_cast<int4 *>(sym_out) + 2 * gb;
            so[0] = make_int4(sym[0], sym[1], sym[2], sym[3]);
            so[1] = make_int4(sym[4], sym[5], sym[6], sym[7]);
        }
        if constexpr (DO >= 0) {
            const float sc = __half2float(__ushort_as_half(a.scale_f16[chunk * a.n_heads + bph_div.div(b)]));
            unsigned long long q2[4];
            ring_point_scaled2(blk, sc, q2);
            float q[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) f2_unpack(q2[i], q[2 * i], q[2 * i + 1]);
            store_block8<DO>(out, gb, q);
        }
    };
    // optimistic decode; a warp whose lanes read past their bits writes its
    // blocks again from the exact decode (every block is overwritten)
    if (decode_two_tiles_ordered<kDecR, false>(a, chunk, tile0, true, true, smem_addr(dtab), ring, epi, err))
        decode_two_tiles_ordered<kDecR, true>(a, chunk, tile0, true, true, smem_addr(dtab), ring, epi, err);
}

// ---------------------------------------------------------------- reference streams
__global__ void __launch_bounds__(128) decode_streams_kernel(
    const uint32_t *__restrict__ bits, int64_t n_words, const int64_t *__restrict__ bit_offsets,
    const int64_t *__restrict__ n_bits, const int64_t *__restrict__ init_states, const int64_t *__restrict__ n_decode,
    const int32_t *__restrict__ lookup, const int32_t *__restrict__ freqs, const int32_t *__restrict__ cumfreqs,
    const int32_t *__restrict__ alphabet, const int32_t *__restrict__ table_id, int64_t max_sym, int64_t n_streams,
    int64_t *__restrict__ out, const int64_t *__restrict__ out_offsets, uint32_t *err) {
    const int64_t sid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sid >= n_streams) return;
    const int64_t tid = table_id[sid];
    const int32_t *lk = lookup + tid * LQ_L;
    const int32_t *fr = freqs + tid * max_sym;
    const int32_t *cfr = cumfreqs + tid * max_sym;
    const int32_t *al = alphabet + tid * max_sym;
    const int64_t b0 = bit_offsets[sid];
    const int64_t nb = n_bits[sid];
    const int64_t nd = n_decode[sid];
    int64_t *o = out + out_offsets[sid];
    // the reference reads bit (b0 + pos) of the flat int32 word array
    if (b0 < 0 || nb < 0 || ((b0 + nb + 31) >> 5) > n_words || init_states[sid] < 0 ||
        init_states[sid] > 0xffffffffll) {
        raise_flag(err, LQ_EF_BITSTREAM);
        return;
    }
    uint32_t x = (uint32_t)init_states[sid];
    int64_t pos = 0;
    for (int64_t i = 0; i < nd; ++i) {
        const uint32_t slot = x & (LQ_L - 1);
        const int32_t si = lk[slot];
        if (si < 0 || si >= max_sym) {
            raise_flag(err, LQ_EF_BITSTREAM);
            return;
        }
        o[i] = (int64_t)al[si];
        x = (uint32_t)fr[si] * (x >> LQ_LOG2_L) + slot - (uint32_t)cfr[si];
        while (x < (uint32_t)LQ_L && pos < nb) {
            const int64_t ab = b0 + pos;
            x = (x << 1) | ((__ldg(bits + (ab >> 5)) >> (ab & 31)) & 1u);
            ++pos;
        }
    }
}

}  // namespace
}  // namespace lq

using namespace lq;

static int64_t slot_words_for(int64_t TB) { return ceil_div(10 * TB, 32) + 1; }

extern "C" size_t lq_rans_encode_workspace(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks) {
    if (n_chunks <= 0 || n_vectors <= 0 || tile_blocks <= 0) return 0;
    const int64_t n_tiles = ceil_div(n_vectors, tile_blocks);
    const int64_t n_lanes = n_chunks * n_tiles * LQ_NSTREAMS;
    const int64_t nblk = ceil_div(n_lanes, kScanTile);
    size_t b = sizeof(uint32_t) * (size_t)(n_lanes * slot_words_for(tile_blocks));  // scratch slots
    b += sizeof(uint32_t) * (size_t)n_lanes;                                        // lane word counts
    b = (b + 15) & ~(size_t)15;
    b += sizeof(uint64_t) * (size_t)(nblk + 1);                                     // scan block sums
    return b;
}

extern "C" int lq_rans_encode(const void *sym_cols, const uint32_t *tile_n0, int64_t n_chunks, int64_t n_vectors,
                              int64_t tile_blocks, const int32_t *tab_lo, const int32_t *tab_nsym,
                              const uint32_t *enc_tab, uint32_t *words, int64_t words_cap, uint32_t *lane_off,
                              uint32_t *lane_nbits, uint32_t *lane_state, void *workspace, size_t workspace_bytes,
                              uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_chunks < 0 || n_vectors < 0 || tile_blocks <= 0 || (tile_blocks % 32) != 0 || words_cap < 0)
        return LQ_ERR_INVALID;
    if (!lane_off) return LQ_ERR_INVALID;
    cudaStream_t st = as_stream(stream);
    if (n_chunks == 0 || n_vectors == 0) {
        if (cudaMemsetAsync(lane_off, 0, sizeof(uint32_t), st) != cudaSuccess) return LQ_ERR_CUDA;
        return LQ_OK;
    }
    if (!sym_cols || !tile_n0 || !tab_lo || !tab_nsym || !enc_tab || !words || !lane_nbits || !lane_state ||
        !workspace)
        return LQ_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(sym_cols) & 15) return LQ_ERR_INVALID;  // vector symbol loads
    if (workspace_bytes < lq_rans_encode_workspace(n_chunks, n_vectors, tile_blocks)) return LQ_ERR_CAPACITY;
    const int64_t n_tiles = ceil_div(n_vectors, tile_blocks);
    const int64_t n_lanes = n_chunks * n_tiles * LQ_NSTREAMS;
    const int64_t sw = slot_words_for(tile_blocks);
    uint32_t *scratch = static_cast<uint32_t *>(workspace);
    uint32_t *nwords = scratch + n_lanes * sw;
    size_t off = ((sizeof(uint32_t) * (size_t)(n_lanes * sw + n_lanes)) + 15) & ~(size_t)15;
    uint64_t *bsum = reinterpret_cast<uint64_t *>(static_cast<char *>(workspace) + off);
    const int64_t nblk = ceil_div(n_lanes, kScanTile);
    if (n_chunks > 65535) return LQ_ERR_INVALID;
    if (cudaFuncSetAttribute(encode_lanes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kEncSmem) !=
        cudaSuccess)
        return LQ_ERR_CUDA;
    encode_lanes_kernel<<<dim3((unsigned)ceil_div(n_tiles, kEncTiles), (unsigned)n_chunks), 16 * kEncTiles, kEncSmem,
                          st>>>(sym_cols_view(const_cast<void *>(sym_cols), n_chunks * n_tiles, tile_blocks), tile_n0,
                                (uint32_t)n_tiles, (uint32_t)n_vectors, (uint32_t)tile_blocks,
                                tab_lo, tab_nsym, enc_tab, scratch, (uint32_t)sw, lane_nbits, lane_state, nwords, err);
    scan_reduce_kernel<<<(unsigned)nblk, kScanT, 0, st>>>(nwords, n_lanes, bsum);
    scan_blocks_kernel<<<1, kScanT, 0, st>>>(bsum, nblk);
    scan_write_kernel<<<(unsigned)nblk, kScanT, 0, st>>>(nwords, n_lanes, bsum, lane_off, words_cap, err);
    compact_lanes_kernel<<<(unsigned)ceil_div(n_lanes, 8 * kCompactLanes), 256, 0, st>>>(
        scratch, sw, n_lanes, lane_off, lane_nbits, words, words_cap);
    return check_launch();
}

extern "C" size_t lq_rans_decode_workspace(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks) {
    if (n_chunks <= 0 || n_vectors <= 0 || tile_blocks <= 0) return 0;
    const int64_t n_tiles = ceil_div(n_vectors, tile_blocks);
    size_t b = sizeof(int16_t) * 8 * (size_t)(n_chunks * n_tiles * tile_blocks);  // symbol rows
    b += sizeof(uint32_t) * (size_t)(n_chunks * ceil_div(n_vectors, 32));         // coset ranks
    return (b + 15) & ~(size_t)15;
}

extern "C" int lq_rans_decode(const uint32_t *words, int64_t n_words, const uint32_t *lane_off,
                                 const uint32_t *lane_nbits, const uint32_t *lane_state, const uint32_t *coset_words,
                                 const uint32_t *tile_n0, int64_t n_chunks, int64_t n_heads, int64_t bph,
                                 int64_t tile_blocks, const int32_t *tab_lo, const int32_t *tab_nsym,
                                 const uint16_t *tab_freq, const uint32_t *dec_tab, const uint16_t *scale_f16,
                                 void *out, int out_dtype, int32_t *sym_out, void *workspace, size_t workspace_bytes,
                                 uint32_t *err, void *stream) {
    LQ_NVTX_RANGE();
    if (n_chunks < 0 || n_heads < 0 || bph < 0 || tile_blocks <= 0 || (tile_blocks % 32) != 0 || n_words < 0)
        return LQ_ERR_INVALID;
    const int64_t N = n_heads * bph;
    if (n_chunks == 0 || N == 0) return LQ_OK;
    if (!lane_off || !lane_nbits || !lane_state || !coset_words || !tile_n0 || !tab_lo || !tab_nsym || !tab_freq ||
        !dec_tab || !workspace || (!out && !sym_out) || (n_words > 0 && !words))
        return LQ_ERR_INVALID;
    if (out && (reinterpret_cast<uintptr_t>(out) & 15)) return LQ_ERR_INVALID;
    if (out && !scale_f16) return LQ_ERR_INVALID;
    if (workspace_bytes < lq_rans_decode_workspace(n_chunks, N, tile_blocks)) return LQ_ERR_CAPACITY;
    cudaStream_t st = as_stream(stream);
    const int64_t n_tiles = ceil_div(N, tile_blocks);
    const int64_t n_lanes = n_chunks * n_tiles * LQ_NSTREAMS;
    // fused path: tables + per-warp rank lists + rings fit in shared memory
    const int nwarps = 32;  // one CTA of 32 warps per SM
    if (n_chunks <= 65535 && n_lanes < ((int64_t)1 << 32)) {
        const size_t sm = fused_smem_bytes(nwarps);
        dim3 grid((unsigned)ceil_div(n_tiles, 2 * nwarps), (unsigned)n_chunks);
        const FastDiv bd((uint32_t)bph);
        const ChunkDev cv{words,     (uint32_t)n_words, lane_off,          lane_nbits,           lane_state,
                          coset_words, tile_n0,         (uint32_t)n_heads, (uint32_t)bph,        (uint32_t)tile_blocks,
                          (uint32_t)n_tiles, tab_lo,    tab_nsym,          tab_freq,             dec_tab,
                          scale_f16};
#define LQ_LAUNCH_FUSED(DOV)                                                                                    \
    do {                                                                                                        \
        if (cudaFuncSetAttribute(decode_fused_kernel<DOV>, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                 (int)sm) != cudaSuccess)                                                       \
            return LQ_ERR_CUDA;                                                                                 \
        decode_fused_kernel<DOV><<<grid, 32 * nwarps, sm, st>>>(cv, bd, out, sym_out, err);                   \
    } while (0)
        if (!out) LQ_LAUNCH_FUSED(-1);
        else if (out_dtype == LQ_F32) LQ_LAUNCH_FUSED(LQ_F32);
        else if (out_dtype == LQ_F16) LQ_LAUNCH_FUSED(LQ_F16);
        else if (out_dtype == LQ_BF16) LQ_LAUNCH_FUSED(LQ_BF16);
        else return LQ_ERR_INVALID;
#undef LQ_LAUNCH_FUSED
        return check_launch();
    }
    int16_t *rows = static_cast<int16_t *>(workspace);
    uint32_t *rank1 = reinterpret_cast<uint32_t *>(rows + 8 * n_chunks * n_tiles * tile_blocks);
    decode_lanes_kernel<<<(unsigned)ceil_div(n_lanes, 256), 256, 0, st>>>(
        words, n_words, lane_off, lane_nbits, lane_state, tile_n0, n_lanes, n_tiles, N, tile_blocks, tab_lo, tab_nsym,
        tab_freq, dec_tab, rows, err);
    const int64_t wpc = ceil_div(N, 32);
    const int64_t wpt = tile_blocks / 32;
    coset_rank_kernel<<<(unsigned)ceil_div(n_chunks * n_tiles, 256), 256, 0, st>>>(coset_words, n_chunks, wpc, wpt,
                                                                                   rank1);
    const unsigned g = (unsigned)ceil_div(n_chunks * N, 256);
    const FastDiv nd((uint32_t)N), td((uint32_t)tile_blocks), bd((uint32_t)bph);
    if (!out) {
        reconstruct_kernel<-1><<<g, 256, 0, st>>>(rows, coset_words, rank1, n_chunks, n_heads, bph, tile_blocks,
                                                  n_tiles, scale_f16, out, sym_out, nd, td, bd);
    } else if (out_dtype == LQ_F32) {
        reconstruct_kernel<LQ_F32><<<g, 256, 0, st>>>(rows, coset_words, rank1, n_chunks, n_heads, bph, tile_blocks,
                                                      n_tiles, scale_f16, out, sym_out, nd, td, bd);
    } else if (out_dtype == LQ_F16) {
        reconstruct_kernel<LQ_F16><<<g, 256, 0, st>>>(rows, coset_words, rank1, n_chunks, n_heads, bph, tile_blocks,
                                                      n_tiles, scale_f16, out, sym_out, nd, td, bd);
    } else if (out_dtype == LQ_BF16) {
        reconstruct_kernel<LQ_BF16><<<g, 256, 0, st>>>(rows, coset_words, rank1, n_chunks, n_heads, bph, tile_blocks,
                                                       n_tiles, scale_f16, out, sym_out, nd, td, bd);
    } else {
        return LQ_ERR_INVALID;
    }
    return check_launch();
}

extern "C" int lq_rans_decode_streams(const uint32_t *bitstream, int64_t n_words, const int64_t *bit_offsets,
                                      const int64_t *n_bits, const int64_t *init_states, const int64_t *n_decode,
                                      const int32_t *lookup, const int32_t *freqs, const int32_t *cumfreqs,
                                      const int32_t *alphabet, const int32_t *table_id, int64_t max_sym,
                                      int64_t n_streams, int64_t *out, const int64_t *out_offsets, uint32_t *err,
                                      void *stream) {
    LQ_NVTX_RANGE();
    if (n_streams < 0 || max_sym < 0 || n_words < 0) return LQ_ERR_INVALID;
    if (n_streams == 0) return LQ_OK;
    if (!bitstream || !bit_offsets || !n_bits || !init_states || !n_decode || !lookup || !freqs || !cumfreqs ||
        !alphabet || !table_id || !out || !out_offsets)
        return LQ_ERR_INVALID;
    decode_streams_kernel<<<(unsigned)ceil_div(n_streams, 128), 128, 0, as_stream(stream)>>>(
        bitstream, n_words, bit_offsets, n_bits, init_states, n_decode, lookup, freqs, cumfreqs, alphabet, table_id,
        max_sym, n_streams, out, out_offsets, err);
    return check_launch();
}
