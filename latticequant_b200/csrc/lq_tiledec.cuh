// lq_tiledec.cuh -- the shared rANS tile decoder.
//
// One warp decodes two tiles of a chunk: lanes 0-15 the 16 lanes (streams) of
// the first tile, lanes 16-31 those of the second.  Per round each lane
// decodes up to kRing symbols of its lane into a shared ring; then the warp
// hands every block whose 8 symbols just arrived (rank r of coset c in tile
// t -> block position via a rank->position list built from the coset bits)
// to an epilogue: write it out dequantised, or fold it into attention scores
// or value sums.  The chunk's 16 decode tables live in shared memory.
//
// Decoder step (reference: core/gpu_ans.py:146-168): for x in [L, 2L) the
// table entry for slot = x & (L-1) gives (symbol, k, base) and
// x = base | next k bits, read MSB-first from a 64-bit buffer over the
// bit-reversed reference words.  Near the end of a lane, or for a state
// outside [L, 2L), the reference formula runs literally, including its stop
// at n_bits, so truncated or odd streams decode exactly as the reference does.
#pragma once

#include "lq_common.cuh"

namespace lq {

constexpr int kRing = 32;
constexpr int kRingStride = 40;  // int16 per ring row: 80 B keeps 8-symbol groups 16-B aligned, conflict-free

// Device view of a batch of equal chunks in the lane layout.
struct ChunkDev {
    const uint32_t *words;
    uint32_t n_words;
    const uint32_t *lane_off, *lane_nbits, *lane_state, *coset_words, *tile_n0;
    uint32_t n_heads, bph, TB, n_tiles;
    const int32_t *tab_lo, *tab_nsym;
    const uint16_t *tab_freq;
    const uint32_t *dec_tab;
    const uint16_t *scale_f16;
};

// per-warp shared memory of the decoder: rank lists for 2 tiles + the ring
__host__ __device__ inline size_t tiledec_warp_smem(uint32_t TB) {
    return (size_t)2 * TB * 2 + (size_t)kRing * kRingStride * 2;
}
constexpr size_t kTablesSmem = (size_t)LQ_NSTREAMS * LQ_L * 4;

// all threads of the CTA: the chunk's 16 decode tables into shared memory
__device__ inline void stage_tables(const ChunkDev &a, uint32_t chunk, uint32_t *dtab) {
    const uint4 *src = reinterpret_cast<const uint4 *>(a.dec_tab + (size_t)chunk * LQ_NSTREAMS * LQ_L);
    uint4 *dst = reinterpret_cast<uint4 *>(dtab);
    for (int i = threadIdx.x; i < LQ_NSTREAMS * LQ_L / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// the 8 int16 symbols of one block, 16-byte aligned in shared memory
__device__ __forceinline__ void ring_block(const int16_t *p, int *sym) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    sym[0] = (int16_t)(u.x & 0xffffu);
    sym[1] = (int16_t)(u.x >> 16);
    sym[2] = (int16_t)(u.y & 0xffffu);
    sym[3] = (int16_t)(u.y >> 16);
    sym[4] = (int16_t)(u.z & 0xffffu);
    sym[5] = (int16_t)(u.z >> 16);
    sym[6] = (int16_t)(u.w & 0xffffu);
    sym[7] = (int16_t)(u.w >> 16);
}

// Decoder state of one lane (one stream of one tile).
struct LaneDec {
    const uint32_t *wp;
    const uint32_t *dt;
    const uint16_t *fr;
    uint64_t bb;  // 64-bit MSB-first bit buffer, `avail` valid bits
    uint32_t x, nb, nw, wi;
    int lo, avail, budget;
    bool fast_ok;

    // Set up lane `s` of tile `tile`; returns the symbol count n (0 on a bad
    // table or a lane running past the word array, with the flag raised).
    __device__ __forceinline__ int init(const ChunkDev &a, uint32_t chunk, uint32_t tile, uint32_t s,
                                        const uint32_t *dtab, int n, uint32_t *err) {
        const uint32_t tabi = chunk * LQ_NSTREAMS + s;
        lo = 0;
        x = LQ_L;
        nb = 0;
        nw = 0;
        wp = a.words;
        if (n > 0) {
            const int nsym = a.tab_nsym[tabi];
            lo = a.tab_lo[tabi];
            const uint32_t lg = (chunk * a.n_tiles + tile) * LQ_NSTREAMS + s;
            const uint32_t w0 = a.lane_off[lg];
            nb = a.lane_nbits[lg];
            nw = (nb + 31u) >> 5;
            x = a.lane_state[lg];
            if (nsym <= 0 || nsym > LQ_L) {
                raise_flag(err, LQ_EF_ALPHABET);
                n = 0;
            } else if ((uint64_t)w0 + nw > a.n_words) {
                raise_flag(err, LQ_EF_BITSTREAM);
                n = 0;
            }
            wp = a.words + w0;
        }
        dt = dtab + s * LQ_L;
        fr = a.tab_freq + (size_t)tabi * LQ_L;
        bb = 0;
        avail = 0;
        wi = 0;
        refill();
        refill();
        // the table-driven step is exact while x is in [L, 2L) and 10 more bits exist
        budget = (int)nb - 10;
        fast_ok = (x >> LQ_LOG2_L) == 1u;
        return n;
    }

    // A step takes at most 10 bits, so after a refill (avail >= 33) three
    // table-driven steps can run before the next refill, which is predicated
    // rather than branched.
    __device__ __forceinline__ void refill() {
        const bool need = avail <= 32;
        const uint32_t w = (need && wi < nw) ? __brev(__ldg(wp + wi)) : 0u;
        if (need) {
            bb |= (uint64_t)w << (32 - avail);
            avail += 32;
            ++wi;
        }
    }

    __device__ __forceinline__ void fast_step(int16_t *dst) {
        const uint32_t slot = x & (LQ_L - 1);
        const uint32_t e = dt[slot];
        *dst = (int16_t)((int)(e & 0x3ffu) + lo);
        const uint32_t k = (e >> 10) & 0xfu;
        x = (e >> 14) | __funnelshift_lc((uint32_t)(bb >> 32), 0u, k);
        bb <<= k;
        avail -= (int)k;
        budget -= (int)k;
    }

    __device__ __forceinline__ void slow_step(int16_t *dst) {
        const uint32_t slot = x & (LQ_L - 1);
        const uint32_t e = dt[slot];
        const uint32_t si = e & 0x3ffu;
        *dst = (int16_t)((int)si + lo);
        const uint32_t k = (e >> 10) & 0xfu;
        if (fast_ok && budget >= 0) {
            x = (e >> 14) | __funnelshift_lc((uint32_t)(bb >> 32), 0u, k);
            bb <<= k;
            avail -= (int)k;
            budget -= (int)k;
        } else {
            // literal reference step (end of lane, or a state outside [L, 2L))
            uint32_t pos = (uint32_t)((int)nb - 10 - budget);
            const uint32_t f = fr[si];
            const uint32_t cf = f + slot - ((e >> 14) >> k);  // (e >> 14) >> k == f + slot - cf
            x = f * (x >> LQ_LOG2_L) + slot - cf;
            while (x < (uint32_t)LQ_L && pos < nb) {
                x = (x << 1) | (uint32_t)(bb >> 63);
                bb <<= 1;
                --avail;
                ++pos;
                refill();
            }
            budget = (int)nb - 10 - (int)pos;
            fast_ok = (x >> LQ_LOG2_L) == 1u;
        }
        refill();
    }

    // decode `cnt` symbols into col[0], col[stride], ...
    __device__ __forceinline__ void run(int cnt, int16_t *col, int stride) {
        int j = 0;
        // groups of three table-driven steps while every step of the group is exact
        for (; j + 3 <= cnt && fast_ok && budget >= 20; j += 3) {
            fast_step(col + j * stride);
            fast_step(col + (j + 1) * stride);
            fast_step(col + (j + 2) * stride);
            refill();
        }
        for (; j < cnt; ++j) slow_step(col + j * stride);
    }
};

// One warp: decode tiles tile0 and tile0+1 (when they exist) of `chunk` and
// call epi(t, coset, position_in_tile, sym[8]) once per block, in rank order;
// `rows` holds 2*TB u16, `ring` kRing*kRingStride int16 of this warp's
// shared memory.
template <class Epi>
__device__ __forceinline__ void decode_two_tiles(const ChunkDev &a, uint32_t chunk, uint32_t tile0,
                                                 const uint32_t *dtab, uint16_t *rows, int16_t *ring, Epi &&epi,
                                                 uint32_t *err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t TB = a.TB, n_tiles = a.n_tiles;
    const uint32_t N = a.n_heads * a.bph;
    const uint32_t wpc = (N + 31) >> 5;
    const uint32_t lt = (1u << lane) - 1u;

    uint32_t tbv[2], n0v[2];
    bool tact[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const uint32_t tile = tile0 + t;
        tact[t] = tile < n_tiles;
        tbv[t] = tact[t] ? ((tile * TB + TB <= N) ? TB : N - tile * TB) : 0u;
        n0v[t] = tact[t] ? a.tile_n0[chunk * n_tiles + tile] : 0u;
        if (!tact[t]) continue;
        // rank -> position lists: coset-0 rank r at r, coset-1 rank r at tb-1-r
        const uint32_t *cw = a.coset_words + (size_t)chunk * wpc + (size_t)tile * (TB >> 5);
        uint32_t c0 = 0, c1 = 0;
        const uint32_t tb = tbv[t];
        for (uint32_t off = 0; off < tb; off += 32) {
            const uint32_t word = __ldg(cw + (off >> 5));
            const uint32_t left = tb - off;
            const uint32_t actm = left >= 32 ? 0xffffffffu : ((1u << left) - 1u);
            const uint32_t w1 = word & actm, w0 = ~word & actm;
            if (lane < left) {
                const uint32_t pos = ((word >> lane) & 1u) ? tb - 1 - (c1 + __popc(w1 & lt)) : c0 + __popc(w0 & lt);
                rows[t * TB + pos] = (uint16_t)(off + lane);
            }
            c1 += __popc(w1);
            c0 += __popc(w0);
        }
    }
    __syncwarp();

    // lane setup: lanes 0-15 -> tile0, 16-31 -> tile0+1; stream s = lane & 15
    const uint32_t lt_tile = lane >> 4, s = lane & 15u, c = s >> 3;
    const bool my_act = lt_tile ? tact[1] : tact[0];
    const uint32_t my_tb = lt_tile ? tbv[1] : tbv[0], my_n0 = lt_tile ? n0v[1] : n0v[0];
    LaneDec d;
    const int n = d.init(a, chunk, tile0 + lt_tile, s, dtab, my_act ? (int)(c ? my_tb - my_n0 : my_n0) : 0, err);
    const int maxn = (int)__reduce_max_sync(0xffffffffu, (unsigned)n);

    for (int base = 0; base < maxn; base += kRing) {
        d.run(min(kRing, n - base), ring + lane, kRingStride);
        __syncwarp();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int t = g >> 1, cc = g & 1;
            if (!tact[t]) continue;
            const int nc = (int)(cc ? tbv[t] - n0v[t] : n0v[t]);
            const int r = base + (int)lane;
            if (r < nc) {
                const uint32_t p = rows[t * TB + (cc ? tbv[t] - 1 - r : r)];
                int sym[8];
                ring_block(ring + lane * kRingStride + t * 16 + cc * 8, sym);
                epi(t, cc, p, sym);
            }
        }
        __syncwarp();
    }
}

// One warp: decode tiles tile0 (lanes 0-15, if act0) and tile0+1 (lanes
// 16-31, if act1) in POSITION order.  Each round a half-warp takes the next
// groups of 16 block positions of its tile, as many as keep both cosets'
// new symbols within R (at least one group, since a group holds 16 blocks):
// the 8 lanes of each coset decode exactly the symbols of those groups into
// ring rows 0.., and then every lane j of the half takes block 16*group + j.
// All 32 lanes call epi(ok, t, group, j, coset, sym) together once per group
// step (ok = false for a lane without a block), so the epilogue may use
// warp shuffles; blocks reach it in increasing position order per lane.
template <int R, class Epi>
__device__ __forceinline__ void decode_two_tiles_ordered(const ChunkDev &a, uint32_t chunk, uint32_t tile0, bool act0,
                                                         bool act1, const uint32_t *dtab, int16_t *ring, Epi &&epi,
                                                         uint32_t *err) {
    static_assert(R >= 16 && R * kRingStride * 2 < 65536, "ring rows");
    const uint32_t lane = threadIdx.x & 31, hb = lane & 16u, j = lane & 15u, c = j >> 3;
    const uint32_t TB = a.TB, N = a.n_heads * a.bph;
    const uint32_t wpc = (N + 31) >> 5;
    const uint32_t tile = tile0 + (hb >> 4);
    const bool act = (hb ? act1 : act0) && tile < a.n_tiles;
    const uint32_t tb = act ? min(TB, N - tile * TB) : 0u;
    const uint32_t ngroups = (tb + 15u) >> 4;
    const uint32_t n0 = act ? a.tile_n0[chunk * a.n_tiles + tile] : 0u;
    const uint32_t *cw = a.coset_words + (size_t)chunk * wpc + (size_t)(act ? tile : 0u) * (TB >> 5);
    LaneDec d;
    const int n = d.init(a, chunk, act ? tile : 0u, j, dtab, act ? (int)(c ? tb - n0 : n0) : 0, err);
    uint32_t gpos = 0;
    for (;;) {
        // coset bits of this half's next 16 groups, one per lane, and their prefix counts
        const uint32_t gk = gpos + j;
        const bool gv = gk < ngroups;
        uint32_t bits = 0;
        int glen = 0;
        if (gv) {
            glen = min(16, (int)(tb - 16u * gk));
            bits = (__ldg(cw + (gk >> 1)) >> ((gk & 1u) * 16u)) & ((1u << glen) - 1u);
        }
        const int ones = __popc(bits), zeros = glen - ones;
        int p1 = ones, p0 = zeros;
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) {
            const int u1 = __shfl_up_sync(0xffffffffu, p1, off, 16);
            const int u0 = __shfl_up_sync(0xffffffffu, p0, off, 16);
            if ((int)j >= off) {
                p1 += u1;
                p0 += u0;
            }
        }
        // prefix sums only grow, so the groups that fit form a prefix of the lanes
        const bool fit = gv && p1 <= R && p0 <= R;
        const int ng = __popc((__ballot_sync(0xffffffffu, fit) >> hb) & 0xffffu);
        const int ngmax = max(ng, __shfl_xor_sync(0xffffffffu, ng, 16));
        if (ngmax == 0) break;
        const int last = (int)hb + max(ng, 1) - 1;
        const int n1r = __shfl_sync(0xffffffffu, p1, last);
        const int n0r = __shfl_sync(0xffffffffu, p0, last);
        const int cnt = (ng > 0 && n > 0) ? (c ? n1r : n0r) : 0;
        d.run(cnt, ring + lane, kRingStride);
        __syncwarp();
        for (int it = 0; it < ngmax; ++it) {
            const int src = (int)hb + it;
            const uint32_t bi = __shfl_sync(0xffffffffu, bits, src);
            const int gl = __shfl_sync(0xffffffffu, glen, src);
            const int b1 = __shfl_sync(0xffffffffu, p1 - ones, src);
            const int b0 = __shfl_sync(0xffffffffu, p0 - zeros, src);
            const bool ok = it < ng && (int)j < gl;
            const uint32_t cc = (bi >> j) & 1u;
            const uint32_t below = (1u << j) - 1u;
            const int rr = cc ? b1 + __popc(bi & below) : b0 + __popc(~bi & below);
            int sym[8];
            if (ok) {
                ring_block(ring + rr * kRingStride + hb + cc * 8u, sym);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) sym[i] = 0;
            }
            epi(ok, (int)(hb >> 4), gpos + (uint32_t)it, j, cc, sym);
        }
        __syncwarp();
        gpos += (uint32_t)ng;
    }
}

}  // namespace lq
