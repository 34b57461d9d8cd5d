// lq_scale.cu -- per-head sigma^2 and lattice scale.
//
// Reference: llm/compressed_kv_cache.py:183-196
//   sigma2 = (t_heads ** 2).mean(dim=(1, 2)); scale = sqrt(2*pi*e*sigma2*4^-b)
//   scale = 1 where sigma2 < 1e-12; per_head_scale = scale.to(float16)
//
// torch sums a contiguous row on the CPU with a fixed tree, and the sum is
// reproduced here bit for bit so that the scales (and with them every
// lattice point) agree with the reference.  The tree, for a row of E
// elements read as vec_size = E/8 vectors of 8 lanes:
//   * 32 chains: chain t = 8k + l sums elements 32*i + t, i in [0, S),
//     S = vec_size / 4 (k = interleaved accumulator row, l = vector lane);
//   * each chain is a 4-level cascade with fan-out G = 2^max(4, ceil_log2(S)/4):
//     level-0 sums G consecutive elements left to right, level-1 sums G
//     level-0 sums, level-2 sums G level-1 sums, level-3 sums all level-2
//     sums; leftovers: chain = ((tail + part1) + part2) + acc3;
//   * vectors 4S..vec_size-1 are added to row k = 0, then row 0 += rows 1..3
//     lane by lane; finally a zero accumulates the E%8 scalar tail and then
//     lanes 0..7, left to right.
// One warp evaluates one (head, level-1 block): lane t owns chain t, so every
// warp-wide load reads 32 consecutive elements.  A second pass folds the
// level-1 sums of each head.  Heads whose chain fits in one level-1 block
// (S < G^2) are finished by a single pass.
#include <mutex>

#include "lq_common.cuh"

namespace lq {
namespace {

__host__ __device__ inline int64_t ceil_log2_i64(int64_t x) {
    if (x <= 2) return 1;
#ifdef __CUDA_ARCH__
    return 64 - __clzll((long long)(x - 1));
#else
    return 64 - __builtin_clzll((unsigned long long)(x - 1));
#endif
}

struct Cascade {
    int64_t E, vec_size, S, G, n_l1;
    __host__ __device__ explicit Cascade(int64_t e) : E(e) {
        vec_size = E / 8;
        S = vec_size / 4;
        int64_t lp = ceil_log2_i64(S) / 4;
        if (lp < 4) lp = 4;
        G = (int64_t)1 << lp;
        n_l1 = ceil_div(S, G * G);
        if (n_l1 < 1) n_l1 = 1;
    }
};

template <int DT>
__device__ __forceinline__ float sq(const void *x, int64_t i) {
    const float t = Elem<DT>::load(x, i);
    return __fmul_rn(t, t);
}

// Sum of chain `lane` over i in [i0, i1) as complete level-0 groups, plus the
// trailing partial group separately.  Returns the level-1 partial; *tail gets
// the partial group's sum.
template <int DT>
__device__ __forceinline__ float chain_block(const void *xh, int64_t i0, int64_t i1, int64_t G, int lane,
                                             float *tail) {
    float acc1 = 0.0f;
    const int64_t full = (i1 - i0) / G;
    int64_t i = i0;
    int64_t g = 0;
    if (G == 16) {
        // two level-0 groups per batch: 32 loads in flight, adds still in order
        for (; g + 1 < full; g += 2) {
            float v[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) v[u] = sq<DT>(xh, 32 * (i + u) + lane);
            float a = 0.0f, b = 0.0f;
#pragma unroll
            for (int u = 0; u < 16; ++u) a = __fadd_rn(a, v[u]);
#pragma unroll
            for (int u = 16; u < 32; ++u) b = __fadd_rn(b, v[u]);
            acc1 = __fadd_rn(__fadd_rn(acc1, a), b);
            i += 32;
        }
    }
    for (; g < full; ++g) {
        float a0 = 0.0f;
        // 16 loads in flight before the dependent adds
        for (int64_t j = 0; j < G; j += 16) {
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = sq<DT>(xh, 32 * (i + j + u) + lane);
#pragma unroll
            for (int u = 0; u < 16; ++u) a0 = __fadd_rn(a0, v[u]);
        }
        acc1 = __fadd_rn(acc1, a0);
        i += G;
    }
    float t = 0.0f;
    for (; i < i1; ++i) t = __fadd_rn(t, sq<DT>(xh, 32 * i + lane));
    *tail = t;
    return acc1;
}

// Final fold of one head, given per-chain (tail, part1, part2, acc3) in lane t.
template <int DT>
__device__ __forceinline__ float fold_head(const void *xh, const Cascade &c, float chain, int lane) {
    // extra vectors 4S .. vec_size-1 go into row 0 (lanes 0..7)
    float r = chain;
    if (lane < 8)
        for (int64_t v = c.S * 4; v < c.vec_size; ++v) r = __fadd_rn(r, sq<DT>(xh, v * 8 + lane));
    // row 0 += row 1, += row 2, += row 3 (lane-wise)
    const float r1 = __shfl_sync(0xffffffffu, r, lane + 8);
    const float r2 = __shfl_sync(0xffffffffu, r, lane + 16);
    const float r3 = __shfl_sync(0xffffffffu, r, lane + 24);
    r = __fadd_rn(__fadd_rn(__fadd_rn(r, r1), r2), r3);
    // scalar tail then lanes 0..7, left to right, from zero
    float fa = 0.0f;
    if (lane == 0)
        for (int64_t e = c.vec_size * 8; e < c.E; ++e) fa = __fadd_rn(fa, sq<DT>(xh, e));
#pragma unroll
    for (int l = 0; l < 8; ++l) {
        const float rl = __shfl_sync(0xffffffffu, r, l);
        fa = __fadd_rn(fa, rl);
    }
    return fa;  // valid in every lane
}

__device__ __forceinline__ void write_scale(int64_t h, float sum, int64_t E, float vol_mult, float *sigma2,
                                            float *scale_f32, uint16_t *scale_f16) {
    // 2*pi*e as a Python double, cast to fp32 by torch
    constexpr float kTwoPiE = 17.079468445347132f;
    const float s2 = __fdiv_rn(sum, (float)E);
    float sc = __fsqrt_rn(__fmul_rn(__fmul_rn(s2, kTwoPiE), vol_mult));
    if (s2 < 1e-12f) sc = 1.0f;
    if (sigma2) sigma2[h] = s2;
    if (scale_f32) scale_f32[h] = sc;
    if (scale_f16) scale_f16[h] = __half_as_ushort(__float2half_rn(sc));
}

// Heads with a single level-1 block: one warp does everything.
template <int DT>
__global__ void __launch_bounds__(256) scale_small_kernel(const void *x, int64_t n_heads, int64_t E, float vol_mult,
                                                           float *sigma2, float *scale_f32, uint16_t *scale_f16) {
    const int lane = threadIdx.x & 31;
    const int64_t h = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (h >= n_heads) return;
    const Cascade c(E);
    const char *xh = static_cast<const char *>(x) + h * E * (DT == LQ_F32 ? 4 : 2);
    float tail;
    const float part1 = chain_block<DT>(xh, 0, c.S, c.G, lane, &tail);
    // single block: complete level-1 block goes to level 2, else it is part1
    float chain;
    if (c.S == c.G * c.G) {
        chain = __fadd_rn(__fadd_rn(__fadd_rn(tail, 0.0f), part1), 0.0f);
    } else {
        chain = __fadd_rn(__fadd_rn(__fadd_rn(tail, part1), 0.0f), 0.0f);
    }
    const float sum = fold_head<DT>(xh, c, chain, lane);
    if (lane == 0) write_scale(h, sum, E, vol_mult, sigma2, scale_f32, scale_f16);
}

// 16-bit input, complete level-1 block with G = 16 (256 rows of 32 chains):
// 64-row batches arrive as 16-byte loads (4 KB per warp in flight), are
// transposed through shared memory, and each lane sums its chain in order.
template <int DT>
__device__ __forceinline__ float chain_block_vec16(const char *xh, int64_t i0, int lane, uint4 *stage) {
    const uint4 *src = reinterpret_cast<const uint4 *>(xh + i0 * 64);  // 32 chains x 2 B per row
    const uint16_t *st16 = reinterpret_cast<const uint16_t *>(stage);
    uint4 buf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) buf[k] = __ldg(src + k * 32 + lane);
    float acc1 = 0.0f;
#pragma unroll 1
    for (int b = 0; b < 4; ++b) {
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) stage[k * 32 + lane] = buf[k];
        __syncwarp();
        if (b < 3) {
#pragma unroll
            for (int k = 0; k < 8; ++k) buf[k] = __ldg(src + (b + 1) * 256 + k * 32 + lane);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float a0 = 0.0f;
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const uint16_t u = st16[(g * 16 + r) * 32 + lane];
                const float t = DT == LQ_F16 ? __half2float(__ushort_as_half(u)) : __bfloat162float(__ushort_as_bfloat16(u));
                a0 = __fadd_rn(a0, __fmul_rn(t, t));
            }
            acc1 = __fadd_rn(acc1, a0);
        }
    }
    return acc1;
}

// Pass 1 (large heads): one warp per (head, level-1 block).
template <int DT>
__global__ void __launch_bounds__(256) scale_l1_kernel(const void *x, int64_t n_heads, int64_t E, float *l1,
                                                        float *tails) {
    __shared__ uint4 stage_all[8][256];  // 4 KB per warp
    const int lane = threadIdx.x & 31;
    const Cascade c(E);
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= n_heads * c.n_l1) return;
    const int64_t h = w / c.n_l1, j = w % c.n_l1;
    const char *xh = static_cast<const char *>(x) + h * E * (DT == LQ_F32 ? 4 : 2);
    const int64_t i0 = j * c.G * c.G;
    const int64_t i1 = (i0 + c.G * c.G < c.S) ? i0 + c.G * c.G : c.S;
    float tail;
    float part;
    const bool aligned = (reinterpret_cast<uintptr_t>(xh) & 15) == 0;
    if (DT != LQ_F32 && c.G == 16 && i1 - i0 == 256 && aligned) {
        part = chain_block_vec16<DT>(xh, i0, lane, stage_all[threadIdx.x >> 5]);
        tail = 0.0f;
    } else {
        part = chain_block<DT>(xh, i0, i1, c.G, lane, &tail);
    }
    l1[w * 32 + lane] = part;
    if (j == c.n_l1 - 1) tails[h * 32 + lane] = tail;
}

// Pass 2: fold level-1 sums into levels 2 and 3, then the head.
template <int DT>
__global__ void __launch_bounds__(256) scale_fold_kernel(const void *x, int64_t n_heads, int64_t E, float vol_mult,
                                                          const float *l1, const float *tails, float *sigma2,
                                                          float *scale_f32, uint16_t *scale_f16) {
    const int lane = threadIdx.x & 31;
    const int64_t h = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (h >= n_heads) return;
    const Cascade c(E);
    const char *xh = static_cast<const char *>(x) + h * E * (DT == LQ_F32 ? 4 : 2);
    const int64_t n_full = c.S / (c.G * c.G);  // complete level-1 blocks
    float acc2 = 0.0f, acc3 = 0.0f;
    const float *hl = l1 + h * c.n_l1 * 32;
    for (int64_t j = 0; j < n_full; ++j) {
        acc2 = __fadd_rn(acc2, hl[j * 32 + lane]);
        if (((j + 1) % c.G) == 0) {
            acc3 = __fadd_rn(acc3, acc2);
            acc2 = 0.0f;
        }
    }
    const float part1 = (n_full < c.n_l1) ? hl[n_full * 32 + lane] : 0.0f;
    const float tail = tails[h * 32 + lane];
    const float chain = __fadd_rn(__fadd_rn(__fadd_rn(tail, part1), acc2), acc3);
    const float sum = fold_head<DT>(xh, c, chain, lane);
    if (lane == 0) write_scale(h, sum, E, vol_mult, sigma2, scale_f32, scale_f16);
}

template <int DT>
int launch_scales(const void *x, int64_t n_heads, int64_t E, float vol_mult, float *sigma2, float *scale_f32,
                  uint16_t *scale_f16, void *ws, size_t ws_bytes, cudaStream_t st) {
    const Cascade c(E);
    const int wpb = 8;
    if (c.n_l1 == 1) {
        const int64_t blocks = ceil_div(n_heads, wpb);
        scale_small_kernel<DT><<<(unsigned)blocks, 32 * wpb, 0, st>>>(x, n_heads, E, vol_mult, sigma2, scale_f32,
                                                                        scale_f16);
        return check_launch();
    }
    const size_t need = sizeof(float) * 32 * (size_t)(n_heads * c.n_l1 + n_heads);
    if (ws == nullptr || ws_bytes < need) return LQ_ERR_CAPACITY;
    float *l1 = static_cast<float *>(ws);
    float *tails = l1 + 32 * n_heads * c.n_l1;
    const int64_t warps = n_heads * c.n_l1;
    scale_l1_kernel<DT><<<(unsigned)ceil_div(warps, wpb), 32 * wpb, 0, st>>>(x, n_heads, E, l1, tails);
    scale_fold_kernel<DT><<<(unsigned)ceil_div(n_heads, wpb), 32 * wpb, 0, st>>>(x, n_heads, E, vol_mult, l1, tails,
                                                                                 sigma2, scale_f32, scale_f16);
    return check_launch();
}

}  // namespace
}  // namespace lq

extern "C" size_t lq_head_scales_workspace(int64_t n_heads_total, int64_t elems_per_head) {
    const lq::Cascade c(elems_per_head);
    if (c.n_l1 == 1) return 0;
    return sizeof(float) * 32 * (size_t)(n_heads_total * c.n_l1 + n_heads_total);
}

extern "C" int lq_head_scales(const void *x, int dtype, int64_t n_heads_total, int64_t elems_per_head,
                              float vol_mult, float *sigma2, float *scale_f32, uint16_t *scale_f16, void *workspace,
                              size_t workspace_bytes, void *stream) {
    LQ_NVTX_RANGE();
    if (n_heads_total < 0 || elems_per_head < 0) return LQ_ERR_INVALID;
    if (n_heads_total == 0) return LQ_OK;
    if (x == nullptr || elems_per_head == 0) return LQ_ERR_INVALID;
    cudaStream_t st = lq::as_stream(stream);
    switch (dtype) {
        case LQ_F32:
            return lq::launch_scales<LQ_F32>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32, scale_f16,
                                             workspace, workspace_bytes, st);
        case LQ_F16:
            return lq::launch_scales<LQ_F16>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32, scale_f16,
                                             workspace, workspace_bytes, st);
        case LQ_BF16:
            return lq::launch_scales<LQ_BF16>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32,
                                              scale_f16, workspace, workspace_bytes, st);
        default:
            return LQ_ERR_INVALID;
    }
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  The level-1 partial sums go to a scratch array
// that is part of this library's own device image, so the caller passes no
// workspace and nothing is allocated per call.  Host code cannot use the
// array's name as a device address: the address is looked up once per device
// with cudaGetSymbolAddress and cached here.  Every call on a device shares
// the array; nothing in it needs to start at zero (each call writes every
// entry it later reads).
// ---------------------------------------------------------------------------
static __device__ __align__(256) float lq_scales_static_scratch[LQ_HEAD_SCALES_STATIC_FLOATS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float *g_static_scratch[kMaxDevices] = {};
void *g_static_ctx[kMaxDevices] = {};  // the context the cached address belongs to

// The current driver context (CUcontext), fetched through the runtime so the
// library needs no link-time dependency on libcuda; nullptr if unavailable.
void *current_context() {
    using CtxGetCurrent = int (*)(void **);
    static CtxGetCurrent fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (CtxGetCurrent) nullptr;
        return reinterpret_cast<CtxGetCurrent>(f);
    }();
    void *ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != 0) return nullptr;
    return ctx;
}

// The scratch array's device address on the current device.  The address is
// looked up once per (device, context) and cached; a new context on the same
// device (after cudaDeviceReset, or a context the caller created) makes the
// next call look it up again.
int static_scratch_for_current_device(float **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return LQ_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return LQ_ERR_INVALID;
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_scratch[dev] == nullptr || ctx == nullptr || ctx != g_static_ctx[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, lq_scales_static_scratch) != cudaSuccess || p == nullptr) return LQ_ERR_CUDA;
        g_static_scratch[dev] = static_cast<float *>(p);
        g_static_ctx[dev] = ctx;
    }
    *out = g_static_scratch[dev];
    return LQ_OK;
}
}  // namespace

extern "C" int lq_head_scales_static(const void *x, int dtype, int64_t n_heads_total, int64_t elems_per_head,
                                     float vol_mult, float *sigma2, float *scale_f32, uint16_t *scale_f16,
                                     void *stream) {
    LQ_NVTX_RANGE();
    if (n_heads_total < 0 || elems_per_head < 0) return LQ_ERR_INVALID;
    if (n_heads_total == 0) return LQ_OK;
    if (x == nullptr || elems_per_head == 0) return LQ_ERR_INVALID;
    if (dtype != LQ_F32 && dtype != LQ_F16 && dtype != LQ_BF16) return LQ_ERR_INVALID;
    const size_t cap = sizeof(float) * (size_t)LQ_HEAD_SCALES_STATIC_FLOATS;
    // a head takes 32 * (n_l1 + 1) scratch floats when its sum needs a second
    // pass (none otherwise); compared by division so no product can overflow
    const lq::Cascade c(elems_per_head);
    if (c.n_l1 > 1 && n_heads_total > (int64_t)(LQ_HEAD_SCALES_STATIC_FLOATS / 32) / (c.n_l1 + 1))
        return LQ_ERR_CAPACITY;
    if (lq_head_scales_workspace(n_heads_total, elems_per_head) > cap) return LQ_ERR_CAPACITY;
    float *ws = nullptr;
    const int rc = static_scratch_for_current_device(&ws);
    if (rc != LQ_OK) return rc;
    cudaStream_t st = lq::as_stream(stream);
    switch (dtype) {
        case LQ_F32:
            return lq::launch_scales<LQ_F32>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32, scale_f16,
                                             ws, cap, st);
        case LQ_F16:
            return lq::launch_scales<LQ_F16>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32, scale_f16,
                                             ws, cap, st);
        default:
            return lq::launch_scales<LQ_BF16>(x, n_heads_total, elems_per_head, vol_mult, sigma2, scale_f32,
                                              scale_f16, ws, cap, st);
    }
}
