// lq_tiledec.cuh -- the shared rANS tile decoder.
//
// One warp decodes two tiles of a chunk: lanes 0-15 the 16 lanes (streams) of
// the first tile, lanes 16-31 those of the second.  Per round each lane
// decodes a run of symbols of its lane into a shared ring; then the warp
// hands the blocks whose 8 symbols just arrived, in block order, to an
// epilogue: write them out dequantised, or fold them into attention scores
// or value sums.  The chunk's 16 decode tables live in shared memory.
//
// Decoder step (reference: core/gpu_ans.py:146-168): for x in [L, 2L) the
// table entry for slot = x & (L-1) gives (symbol, k, xs) and
// x = xs << k | next k bits, read MSB-first from a 64-bit buffer over the
// bit-reversed reference words.  Near the end of a lane, or for a state
// outside [L, 2L), the reference formula runs literally, including its stop
// at n_bits, so truncated or odd streams decode exactly as the reference does.
//
// Shared memory is addressed with 32-bit shared-window addresses and moved
// with ld.shared / st.shared, so the hot loop carries no generic-pointer
// arithmetic.
#pragma once

#include "lq_common.cuh"

namespace lq {

constexpr int kRingStride = 40;  // u16 per ring row: 80 B keeps 8-symbol groups 16-B aligned, conflict-free

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts_u16(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "r"(v));
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

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
    const uint32_t *staged_tab;  // optional: the tables in shared-memory form (staged_tables_kernel)
};

constexpr size_t kTablesSmem = (size_t)LQ_NSTREAMS * LQ_L * 4;

// Shared-memory form of a decode-table entry, for x in [L, 2L):
//   bits  0-15  the symbol as a biased doubled lattice coordinate:
//               2*sym + c + 2^15 for coordinates 0-6, 4*sym + c + 2^15 for
//               coordinate 7 (c = the stream's coset), i.e. 2*q + 2^15 before
//               the parity bit of q7 (entropy_coder.py:71-89 inverted later)
//   bits 16-26  xs = f + slot - cf, the state before renormalisation
//   bits 27-31  k, the bits renormalisation reads (x' = xs << k | next k bits)
// Built from lq_expand_tables' entry (si | k << 10 | (xs << k) << 14).
__device__ __forceinline__ uint32_t smem_entry(uint32_t e, int lo, int c, int mul) {
    const uint32_t si = e & 0x3ffu, k = (e >> 10) & 0xfu, xs = (e >> 14) >> k;
    const uint32_t v = (uint32_t)(((int)si + lo) * mul + c + 32768) & 0xffffu;
    return v | (xs << 16) | (k << 27);
}

// ---- bulk (TMA engine) copies into shared memory, completed on an mbarrier
__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar), "r"(count) : "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// one thread: expect `bytes` on the barrier and copy them global -> shared
// (both addresses 16-byte aligned, bytes a multiple of 16); no multicast
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t mbar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic reads of dst before the async write
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Wait for phase `parity` of the barrier, at most about a second; false
// (with LQ_EF_TIMEOUT raised) if it did not complete.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, uint32_t *err) {
    const uint64_t t0 = global_ns();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(mbar), "r"(parity)
            : "memory");
        if (done) return true;
        if (global_ns() - t0 > 1000000000ull) {
            raise_flag(err, LQ_EF_TIMEOUT);
            return false;
        }
    }
}

// all threads of the CTA: the chunk's 16 decode tables into shared memory
__device__ inline void stage_tables(const ChunkDev &a, uint32_t chunk, uint32_t *dtab) {
    const uint4 *src = reinterpret_cast<const uint4 *>(a.dec_tab + (size_t)chunk * LQ_NSTREAMS * LQ_L);
    uint4 *dst = reinterpret_cast<uint4 *>(dtab);
    for (int i = threadIdx.x; i < LQ_NSTREAMS * LQ_L / 4; i += blockDim.x) {
        const int s = i >> 8;  // 256 uint4 per table
        const int lo = __ldg(a.tab_lo + chunk * LQ_NSTREAMS + s);
        const int c = s >> 3, mul = (s & 7) == 7 ? 4 : 2;
        uint4 u = __ldg(src + i);
        u.x = smem_entry(u.x, lo, c, mul);
        u.y = smem_entry(u.y, lo, c, mul);
        u.z = smem_entry(u.z, lo, c, mul);
        u.w = smem_entry(u.w, lo, c, mul);
        dst[i] = u;
    }
}

// ---- blocks in the ring: 8 u16 = 2q + 2^15 (q7 without its parity bit)
// Exact E8 point of a ring block.  A value v < 2^16 placed in the mantissa of
// 1.5 * 2^22 (where the spacing is 0.5) reads back as 1.5 * 2^22 + v / 2, so
// one byte permute and one subtraction give q exactly.
__device__ __forceinline__ float ring_value(uint32_t w, bool hi, float off) {
    return __int_as_float(__byte_perm(w, 0x4AC00000u, hi ? 0x7632u : 0x7610u)) - off;
}

__device__ __forceinline__ uint32_t ring_parity(const uint4 u) {
    // parity of sum(sym[0..6]) = xor of bit 1 of the seven stored values
    const uint32_t x = u.x ^ u.y ^ u.z ^ (u.w & 0xffffu);
    return ((x ^ (x >> 16)) >> 1) & 1u;
}

__device__ __forceinline__ void ring_point(const uint4 u, float q[8]) {
    constexpr float kOff = 6307840.0f;  // 1.5 * 2^22 + 2^15 / 2
    q[0] = ring_value(u.x, false, kOff);
    q[1] = ring_value(u.x, true, kOff);
    q[2] = ring_value(u.y, false, kOff);
    q[3] = ring_value(u.y, true, kOff);
    q[4] = ring_value(u.z, false, kOff);
    q[5] = ring_value(u.z, true, kOff);
    q[6] = ring_value(u.w, false, kOff);
    // q7 = (4*sym7 + c)/2 + parity
    q[7] = ring_value(u.w, true, __int_as_float(0x4AC08000 - 2 * (int)ring_parity(u)));
}

// ring_point as four packed fp32x2 pairs (channels 2i, 2i+1), by packed
// subtractions (exact, as the scalar ones)
__device__ __forceinline__ void ring_point2(const uint4 u, unsigned long long q2[4]) {
    constexpr float kOff = 6307840.0f;  // 1.5 * 2^22 + 2^15 / 2
    const float off7 = __int_as_float(0x4AC08000 - 2 * (int)ring_parity(u));
    const unsigned long long off = f2_pack(kOff, kOff);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const unsigned long long raw = f2_pack(__int_as_float(__byte_perm(w[i], 0x4AC00000u, 0x7610u)),
                                               __int_as_float(__byte_perm(w[i], 0x4AC00000u, 0x7632u)));
        q2[i] = f2_sub(raw, i == 3 ? f2_pack(kOff, off7) : off);
    }
}
// ring_point2 times s: packed multiplies, each half rounded as its scalar op
__device__ __forceinline__ void ring_point_scaled2(const uint4 u, float s, unsigned long long q2[4]) {
    ring_point2(u, q2);
    const unsigned long long ss = f2_pack(s, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) q2[i] = f2_mul(q2[i], ss);
}

// the reference's integer symbols (entropy_coder.py:46-68) of a ring block
__device__ __forceinline__ void ring_symbols(const uint4 u, int c, int sym[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int v = (int)((w[i >> 1] >> (16 * (i & 1))) & 0xffffu) - 32768 - c;
        sym[i] = v >> (i == 7 ? 2 : 1);
    }
}

// Decoder state of one lane (one stream of one tile).
//
// Bits are read MSB-first from a 64-bit buffer bh:bl over the bit-reversed
// reference words (`avail` valid bits from the top of bh), with the word
// after them already loaded in `nxt`, so the load of a word is issued a full
// word of symbols before it is needed.  A table-driven ("fast") step is exact
// while x is in [L, 2L) and the k bits it reads exist (consumed + 10 <=
// n_bits); during a run of fast steps only x's low 10 bits (the next slot)
// are kept exact and x is rebuilt as (x & (L-1)) | L before a literal step.
struct LaneDec {
    const uint32_t *wp;
    const uint16_t *fr;
    uint32_t dtb;  // shared address of this stream's table
    uint32_t bh, bl;
    uint32_t x, nb, nw, wi, nxt;
    int lo, avail, c, shift;
    bool fast_ok;

    // bits consumed so far: words moved into the buffer minus what is left there
    __device__ __forceinline__ int consumed() const { return 32 * (int)(wi - 1u) - avail; }

    // Set up lane `s` of tile `tile`; returns the symbol count n (0 on a bad
    // table or a lane running past the word array, with the flag raised).
    __device__ __forceinline__ int init(const ChunkDev &a, uint32_t chunk, uint32_t tile, uint32_t s, uint32_t dtab,
                                        int n, uint32_t *err) {
        const uint32_t tabi = chunk * LQ_NSTREAMS + s;
        lo = 0;
        x = LQ_L;
        nb = 0;
        nw = 0;
        wp = a.words;
        c = (int)(s >> 3);
        shift = (s & 7) == 7 ? 2 : 1;
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
                nw = 0;
            } else if ((uint64_t)w0 + nw > a.n_words) {
                raise_flag(err, LQ_EF_BITSTREAM);
                n = 0;
                nw = 0;
            }
            wp = a.words + w0;
        }
        dtb = dtab + s * (LQ_L * 4);
        fr = a.tab_freq + (size_t)tabi * LQ_L;
        bh = __brev(nw > 0 ? __ldg(wp) : 0u);
        bl = __brev(nw > 1 ? __ldg(wp + 1) : 0u);
        nxt = nw > 2 ? __ldg(wp + 2) : 0u;
        avail = 64;
        wi = 3;
        fast_ok = (x >> LQ_LOG2_L) == 1u;
        return n;
    }

    // drop the top k (<= 31) bits of the buffer
    __device__ __forceinline__ void take(uint32_t k) {
        bh = __funnelshift_l(bl, bh, k);
        bl = __funnelshift_l(0u, bl, k);  // bl << k for k < 32, without clamping code
        avail -= (int)k;
    }

    // move the prefetched word into the buffer once 32 bits are free (no branch)
    __device__ __forceinline__ void refill() {
        const bool r = avail <= 32;
        const uint32_t w = __brev(nxt);
        bh |= r ? __funnelshift_rc(w, 0u, (uint32_t)avail) : 0u;  // w >> avail, 0 when avail == 32
        bl |= r ? __funnelshift_l(0u, w, (uint32_t)(32 - avail)) : 0u;
        avail += r ? 32 : 0;
        uint32_t v = 0;
        if (r && wi < nw) v = __ldg(wp + wi);
        nxt = r ? v : nxt;
        wi += r ? 1u : 0u;
    }

    __device__ __forceinline__ void fast_step(uint32_t dst) {
        const uint32_t e = lds_u32(dtb + ((x & (LQ_L - 1)) << 2));
        sts_u16(dst, e);
        const uint32_t k = e >> 27;
        // (xs << k) | next k bits; the k-field above xs lands above bit 10
        x = __funnelshift_l(bh, e >> 16, k);
        take(k);
    }

    // one step, table-driven when exact, else the reference formula literally
    // (including its stop at n_bits: core/gpu_ans.py:160-166)
    __device__ __forceinline__ void single_step(uint32_t dst) {
        if (fast_ok && consumed() + 10 <= (int)nb) {
            fast_step(dst);
        } else {
            if (fast_ok) x = (x & (LQ_L - 1)) | LQ_L;
            const uint32_t slot = x & (LQ_L - 1);
            const uint32_t e = lds_u32(dtb + (slot << 2));
            sts_u16(dst, e);
            const int sym = ((int)(e & 0xffffu) - 32768 - c) >> shift;
            const uint32_t si = (uint32_t)(sym - lo) & 0x3ffu;
            const uint32_t f = fr[si];
            const uint32_t cf = f + slot - ((e >> 16) & 0x7ffu);
            x = f * (x >> LQ_LOG2_L) + slot - cf;
            while (x < (uint32_t)LQ_L && consumed() < (int)nb) {
                x = (x << 1) | (bh >> 31);
                take(1);
                refill();
            }
            fast_ok = (x >> LQ_LOG2_L) == 1u;
        }
        refill();
    }

    // Three table-driven steps and a refill, written out in PTX so the group
    // costs what its arithmetic costs: per step a slot lookup, the ring
    // store, two shifts out of the entry, three funnel shifts (the new state
    // and the 64-bit buffer) and the bit count; the refill is predicated, not
    // branched.  Variable shifts are funnel shifts whose amount the hardware
    // takes as given (wrap) or clamps itself, so no range fix-up is emitted.
    // Ring rows are kRingStride u16 apart.
    __device__ __forceinline__ void fast_group(uint32_t dst) {
        static_assert(kRingStride * 2 == 80, "ring row offsets below");
        asm volatile(
            "{\n\t"
            ".reg .b32 e, k, t, a, w, z;\n\t"
            ".reg .pred p, q;\n\t"
            ".reg .b64 ad;\n\t"
            "mov.b32 z, 0;\n\t"
            "and.b32 a, %0, 1023;\n\t"
            "mad.lo.u32 a, a, 4, %6;\n\t"
            "ld.shared.u32 e, [a];\n\t"
            "st.shared.u16 [%7], e;\n\t"
            "shr.u32 k, e, 27;\n\t"
            "shr.u32 t, e, 16;\n\t"
            "shf.l.wrap.b32 %0, %1, t, k;\n\t"
            "shf.l.wrap.b32 %1, %2, %1, k;\n\t"
            "shf.l.wrap.b32 %2, z, %2, k;\n\t"
            "sub.s32 %3, %3, k;\n\t"
            "and.b32 a, %0, 1023;\n\t"
            "mad.lo.u32 a, a, 4, %6;\n\t"
            "ld.shared.u32 e, [a];\n\t"
            "st.shared.u16 [%7+80], e;\n\t"
            "shr.u32 k, e, 27;\n\t"
            "shr.u32 t, e, 16;\n\t"
            "shf.l.wrap.b32 %0, %1, t, k;\n\t"
            "shf.l.wrap.b32 %1, %2, %1, k;\n\t"
            "shf.l.wrap.b32 %2, z, %2, k;\n\t"
            "sub.s32 %3, %3, k;\n\t"
            "and.b32 a, %0, 1023;\n\t"
            "mad.lo.u32 a, a, 4, %6;\n\t"
            "ld.shared.u32 e, [a];\n\t"
            "st.shared.u16 [%7+160], e;\n\t"
            "shr.u32 k, e, 27;\n\t"
            "shr.u32 t, e, 16;\n\t"
            "shf.l.wrap.b32 %0, %1, t, k;\n\t"
            "shf.l.wrap.b32 %1, %2, %1, k;\n\t"
            "shf.l.wrap.b32 %2, z, %2, k;\n\t"
            "sub.s32 %3, %3, k;\n\t"
            // refill: when at most 32 bits are left, append the prefetched word
            // below them and prefetch the next one (0 past the lane's end)
            "setp.le.s32 p, %3, 32;\n\t"
            "@p brev.b32 w, %4;\n\t"
            "@p sub.s32 t, 32, %3;\n\t"
            "@p shf.l.wrap.b32 t, z, w, t;\n\t"
            "@p or.b32 %2, %2, t;\n\t"
            "@p shf.r.clamp.b32 t, w, z, %3;\n\t"
            "@p or.b32 %1, %1, t;\n\t"
            "@p add.s32 %3, %3, 32;\n\t"
            "setp.lt.and.u32 q, %5, %8, p;\n\t"
            "@p mov.b32 %4, 0;\n\t"
            "@q mad.wide.u32 ad, %5, 4, %9;\n\t"
            "@q ld.global.nc.u32 %4, [ad];\n\t"
            "@p add.u32 %5, %5, 1;\n\t"
            "}"
            : "+r"(x), "+r"(bh), "+r"(bl), "+r"(avail), "+r"(nxt), "+r"(wi)
            : "r"(dtb), "r"(dst), "r"(nw), "l"(wp));
    }

    // decode `cnt` symbols to shared addresses dst, dst + sb, dst + 2*sb, ...
    // (sb = one ring row).  CHECKED: a group runs table-driven only while all
    // three steps stay inside the lane, the rest literally, so every stream
    // decodes exactly as the reference decodes it.  Unchecked: table-driven
    // groups throughout (single steps for a remainder of one or two), which
    // is exact for every stream whose decode never reads past n_bits -- every
    // stream an encoder wrote; consumed() > nb after the lane's last symbol
    // tells afterwards that it did not hold.
    template <bool CHECKED>
    __device__ __forceinline__ void run(int cnt, uint32_t dst) {
        constexpr uint32_t sb = kRingStride * 2;
        int j = 0;
        if (fast_ok) {
            const int lim = CHECKED ? (int)nb - 30 : 0x7fffffff;
#pragma unroll 1
            for (; j + 3 <= cnt && (!CHECKED || consumed() <= lim); j += 3) {
                fast_group(dst);
                dst += 3 * sb;
            }
        }
        for (; j < cnt; ++j) {
            single_step(dst);
            dst += sb;
        }
    }
};

// One warp: decode tiles tile0 (lanes 0-15, if act0) and tile0+1 (lanes
// 16-31, if act1) in POSITION order.  Each round a half-warp takes the next
// groups of 16 block positions of its tile, as many as keep both cosets'
// new symbols within R (at least one group, since a group holds 16 blocks):
// the 8 lanes of each coset own exactly the symbols of those groups in ring
// rows 0.., and then every lane j of the half takes block 16*group + j.
// Lanes decode in whole groups of three steps (except at the lane's end); the
// one or two symbols a lane decodes past the round's need are carried to rows
// 0.. of the next round.
// All 32 lanes call epi(ok, t, group, j, coset, block) together once per
// group step (ok = false for a lane without a block), so the epilogue may
// use warp shuffles; blocks reach it in increasing position order per lane.
// CHECKED = false decodes optimistically (LaneDec::run) and returns whether
// any lane of the warp read past its n_bits, in which case the blocks it
// handed out may differ from the reference decode and the caller decodes the
// same tiles again with CHECKED = true (which always returns false).
// `ring` is (R + 2) rows of kRingStride u16.
template <int R, bool CHECKED, class Epi>
__device__ __forceinline__ bool decode_two_tiles_ordered(const ChunkDev &a, uint32_t chunk, uint32_t tile0, bool act0,
                                                         bool act1, uint32_t dtab, uint32_t ring, Epi &&epi,
                                                         uint32_t *err) {
    static_assert(R >= 16 && (R + 2) * kRingStride * 2 < 65536, "ring rows");
    constexpr uint32_t kRow = kRingStride * 2;
    const uint32_t lane = threadIdx.x & 31, hb = lane & 16u, j = lane & 15u, c = j >> 3;
    const uint32_t TB = a.TB, N = a.n_heads * a.bph;
    const uint32_t wpc = (N + 31) >> 5;
    const uint32_t tile = tile0 + (hb >> 4);
    const bool act = (hb ? act1 : act0) && tile < a.n_tiles;
    const uint32_t tb = act ? min(TB, N - tile * TB) : 0u;
    const uint32_t ngroups = (tb + 15u) >> 4;
    const uint32_t n0 = act ? a.tile_n0[chunk * a.n_tiles + tile] : 0u;
    const uint32_t *cw = a.coset_words + (size_t)chunk * wpc + (size_t)(act ? tile : 0u) * (TB >> 5);
    const uint32_t col = ring + lane * 2;
    LaneDec d;
    // symbols of the lane not yet decoded (0 for a lane without symbols or
    // with a bad table or word range: it decodes nothing)
    int left = d.init(a, chunk, act ? tile : 0u, j, dtab, act ? (int)(c ? tb - n0 : n0) : 0, err);
    uint32_t gpos = 0;
    int ahead = 0, prev = 0;  // symbols decoded past the last round's need, at rows prev..
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
        // a lane with symbols still to decode or to hand out takes its coset's count
        const int cnt = (ng > 0 && (left > 0 || ahead > 0)) ? (c ? n1r : n0r) : 0;
        if (ahead > 0 && prev > 0) {  // carried symbols to rows 0, 1 (forward copy)
            sts_u16(col, lds_u16(col + (uint32_t)prev * kRow));
            if (ahead > 1) sts_u16(col + kRow, lds_u16(col + (uint32_t)(prev + 1) * kRow));
        }
        const int need = cnt - ahead;
        if (need > 0) {
            // whole groups of three, but never past the lane's last symbol,
            // so a lane reads no bit beyond its stream unless it is malformed
            const int dec = min((need + 2) / 3 * 3, left);
            d.run<CHECKED>(dec, col + (uint32_t)ahead * kRow);
            left -= dec;
            ahead += dec - cnt;
        } else {
            ahead = -need;
        }
        prev = cnt;
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
            uint4 blk = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);  // q = 0
            if (ok) blk = lds_v4(ring + (uint32_t)rr * kRow + (hb + cc * 8u) * 2u);
            epi(ok, (int)(hb >> 4), gpos + (uint32_t)it, j, cc, blk);
        }
        __syncwarp();
        gpos += (uint32_t)ng;
    }
    // (a lane without symbols has consumed 0 bits)
    return !CHECKED && __any_sync(0xffffffffu, d.consumed() > (int)d.nb);
}

}  // namespace lq
