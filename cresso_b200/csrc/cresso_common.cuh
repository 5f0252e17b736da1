// Shared device / host helpers of the B200 CRESSO5 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#include "../../include/cresso_b200.h"

namespace cresso {

constexpr int kThreads = 256;  // every kernel of the library runs 256-thread blocks
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRank = 16;       // the fused float32 spectral path
constexpr int kMaxRankPlain = 64;  // the float64-arithmetic spectral path with its modes in registers
constexpr int kMaxRankWide = 4096; // the same path with its modes in memory (rank 65 to 4096)
constexpr int kChunkW = 32;        // modes per projection chunk of the wide-rank kernels
constexpr int kMaxTB = 8192;   // hash_tables * hash_bins held in shared memory
constexpr int kMaxBins = 4096; // same bound as the reference CUDA hash path (cresso_v5.py:1002)

// Salted three-round int64 coordinate hash, remainder taken Python-style.
// Restates _hash_index_tensor (cresso_v5.py:495-516): torch int64 arithmetic
// wraps modulo 2^64 (done here in uint64), `>>` is an arithmetic shift of the
// signed value, and torch.remainder returns a value in [0, bins).
__host__ __device__ __forceinline__ int64_t hash_bin(int64_t i, int64_t bins, int64_t salt) {
    const uint64_t s = (uint64_t)(salt + 1);
    uint64_t h = (uint64_t)i * (uint64_t)(1103515245ULL + 97ULL * s) + (12345ULL + 0x9E3779B1ULL * s);
    int64_t v = (int64_t)h;
    v ^= (v >> 16);
    h = (uint64_t)v * (2246822519ULL + 1315423911ULL * s);
    v = (int64_t)h;
    v ^= (v >> 13);
    h = (uint64_t)v * (3266489917ULL + 374761393ULL * s);
    v = (int64_t)h;
    v ^= (v >> 16);
    if ((bins & (bins - 1)) == 0) return v & (bins - 1);
    int64_t r = v % bins;
    return r < 0 ? r + bins : r;
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__host__ __device__ __forceinline__ int pow2_ceil(int64_t v) {
    int p = 1;
    while (p < v && p < (1 << 30)) p <<= 1;
    return p;
}

// Mode kinds of the carrier pack (cresso_v5.py:302-348): mode % 4 == 1 uses
// per-axis products of cos and of sin; every other mode (and the zero mode,
// whose tables are (1, 0)) is a complex exponential product.
__host__ __device__ constexpr bool mode_is_product(int k) { return (k & 3) == 1; }

// ---------------------------------------------------------------------------
// Per-shape workspace layout (built by cresso_shape_workspace_init).
//   rowtab : float [grows][RM][2]   (a1, a2) of mode k on global row i
//   coltab : float [RM][2][gcols]   (b1, b2) of mode k on global column j
//   stats  : double [RM][8]         mu_c, inv_c, mu_s, inv_s, mhat_c, mhat_s
//   gram   : double [2RM][2RM]      mean(basis_p * basis_q), p = 2k (cos) / 2k+1 (sin)
//   counts : float [T][B]           elements of the tensor in each hash bin
//   tmp    : double                 table sums used while building stats / gram
// For a 1-D tensor of n elements grows = 1 and gcols = n.
// ---------------------------------------------------------------------------
struct ShapeWsHeader {
    int64_t magic, ndim, grows, gcols, rank, rm, bins, tables;
    int64_t off_rowtab, off_coltab, off_stats, off_gram, off_counts, off_tmp, bytes, n;
};
constexpr int64_t kShapeWsMagic = 0x43524553534f3542LL;  // "CRESSO5B"

__host__ __device__ inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

__host__ inline ShapeWsHeader shape_ws_layout(int64_t ndim, int64_t grows, int64_t gcols, int64_t rank, int64_t rm,
                                             int64_t bins, int64_t tables) {
    ShapeWsHeader h{};
    h.magic = kShapeWsMagic;
    h.ndim = ndim;
    h.grows = grows;
    h.gcols = gcols;
    h.rank = rank;
    h.rm = rm;
    h.bins = bins;
    h.tables = tables;
    h.n = grows * gcols;
    int64_t off = align_up((int64_t)sizeof(ShapeWsHeader), 256);
    h.off_rowtab = off;
    off = align_up(off + grows * rm * 2 * 4, 256);
    h.off_coltab = off;
    off = align_up(off + rm * 2 * gcols * 4, 256);
    h.off_stats = off;
    off = align_up(off + rm * 8 * 8, 256);
    h.off_gram = off;
    off = align_up(off + (2 * rm) * (2 * rm) * 8, 256);
    h.off_counts = off;
    off = align_up(off + (bins > 0 ? bins * tables * 4 : 0), 256);
    // set-up scratch: per-axis sums S1[p] and cross sums S2[p][q] of the tables
    h.off_tmp = off;
    off = align_up(off + 2 * ((2 * rm) * (2 * rm) + 2 * rm) * 8, 256);
    h.bytes = off;
    return h;
}

// Float64 shape workspace (float64 parameters on the spectral route): float64
// axis tables rowtab [grows][rm][2] and coltab [2 rm][gcols], the carrier stats
// and Gram from them; no hash counts.
constexpr int64_t kModeParamBytes = 512;  // room for one mode's carrier parameters (basis_ws.cu ModeParam)
constexpr int64_t kShapeWs64Magic = 0x43524553534f3544LL;  // "CRESSO5D"
__host__ inline ShapeWsHeader shape_ws64_layout(int64_t ndim, int64_t grows, int64_t gcols, int64_t rank, int64_t rm) {
    ShapeWsHeader h{};
    h.magic = kShapeWs64Magic;
    h.ndim = ndim;
    h.grows = grows;
    h.gcols = gcols;
    h.rank = rank;
    h.rm = rm;
    h.n = grows * gcols;
    int64_t off = align_up((int64_t)sizeof(ShapeWsHeader), 256);
    h.off_rowtab = off;
    off = align_up(off + grows * rm * 2 * 8, 256);
    h.off_coltab = off;
    off = align_up(off + 2 * rm * gcols * 8, 256);
    h.off_stats = off;
    off = align_up(off + 64 * (rm > kMaxRankPlain ? rm : kMaxRankPlain), 256);  // ModeStats: 8 doubles per mode
    h.off_gram = off;
    if (rm <= kMaxRankPlain) {
        off = align_up(off + (2 * rm) * (2 * rm) * 8, 256);
        h.off_tmp = off;
        off = align_up(off + 2 * (2 * rm + 4 * rm * rm) * 8, 256);
    } else {
        // wide rank: no carrier Gram (the float64 path does not use it); per axis the
        // table sums S1[2 rm] and each mode's own 2 x 2 block of cross sums, then the
        // mode parameters (kModeParamBytes per mode) uploaded for the set-up kernels
        h.off_tmp = off;
        off = align_up(off + 2 * (2 * rm + 4 * rm) * 8, 256);
        off = align_up(off + kModeParamBytes * rm, 256);
    }
    h.off_counts = off;
    h.bytes = off;
    return h;
}

__host__ __device__ inline int rank_pad(int64_t rank) {
    if (rank > kMaxRankPlain) return (int)align_up(rank, kChunkW);  // wide rank: whole projection chunks
    return rank <= 4 ? 4 : (rank <= 8 ? 8 : (rank <= 16 ? 16 : (rank <= 32 ? 32 : 64)));
}

// ---------------------------------------------------------------------------
// Warp / block reductions (fixed order => run-to-run deterministic)
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sums N per-thread values across the block in a fixed order.  `red` is
// shared scratch of N * kWarps doubles and `out` shared memory of N doubles,
// readable by every thread on return; all threads must call.
template <int N>
__device__ __forceinline__ void block_sum_to(double (&v)[N], double* red, double* out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        double s = warp_sum(v[j]);
        if (lane == 0) red[j * kWarps + warp] = s;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < N; j += blockDim.x) {
        double s = 0.0;
        for (int w = 0; w < kWarps; ++w) s += red[j * kWarps + w];
        out[j] = s;
    }
    __syncthreads();
}

__device__ __forceinline__ double block_sum(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double s = warp_sum(v);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w) t += red[w];
        red[kWarps] = t;
    }
    __syncthreads();
    t = red[kWarps];
    __syncthreads();
    return t;
}

__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

// Per-element transcendentals of the streaming kernels.
//
// log(1 + x) for x >= 0.  For x <= 1: log(1 + x) = 2 atanh(z) with
// z = x / (x + 2) in [0, 1/3], summed as its Taylor series
// 2 z (1 + z^2/3 + z^4/5 + ... + z^12/13), truncation below 2e-8 relative and
// no cancellation near x = 0.  For x > 1: ln 2 * log2(1 + x) on the
// special-function unit, within 2 ulp for arguments above 2.
__device__ __forceinline__ float log1p_pos(float x) {
    const float z = __fdividef(x, x + 2.0f);  // divisor in [2, 3] on the branch that uses it
    const float w = z * z;
    float p = 1.0f / 13.0f;
    p = fmaf(p, w, 1.0f / 11.0f);
    p = fmaf(p, w, 1.0f / 9.0f);
    p = fmaf(p, w, 1.0f / 7.0f);
    p = fmaf(p, w, 1.0f / 5.0f);
    p = fmaf(p, w, 1.0f / 3.0f);
    const float series = 2.0f * fmaf(z * w, p, z);
    const float lg = 0.693147180559945309f * __log2f(1.0f + x);
    return x <= 1.0f ? series : lg;
}
// Square root of a positive normal number, approximate (relative error ~2^-22).
__device__ __forceinline__ float sqrt_sfu(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}


// Element e of a parameter / gradient of type dt (float32 work, cresso_v5.py:119-124).
// -lr rounded (once, from double) to the parameter type dt; float32: -lr.
__device__ __forceinline__ float neg_lr_in(double lr, int dt) {
    if (dt == CRESSO_DTYPE_F16) return __half2float(__double2half(-lr));
    if (dt == CRESSO_DTYPE_BF16) return __bfloat162float(__double2bfloat16(-lr));
    return (float)(-lr);
}

__device__ __forceinline__ float load_elem(const void* p, int64_t e, int dt) {
    if (dt == CRESSO_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[e]);
    if (dt == CRESSO_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[e]);
    return __ldg(reinterpret_cast<const float*>(p) + e);
}
// param.add_(update.to(param.dtype), alpha=-lr)  (cresso_v5.py:1582).  float32:
// p + (-lr) u.  16-bit: round(p + round(-lr) round(u)), every rounding to the
// parameter's type, as PyTorch's vectorised CPU kernel computes it (alpha
// converted to the tensor's type, the sum formed in float32); neg_lr16 is
// -lr rounded to that type.
__device__ __forceinline__ void apply_update(void* p, int64_t e, int dt, float neg_lr, float neg_lr16,
                                             float update) {
    if (dt == CRESSO_DTYPE_F16) {
        __half* h = reinterpret_cast<__half*>(p);
        const float u = __half2float(__float2half_rn(update));
        h[e] = __float2half_rn(__half2float(h[e]) + neg_lr16 * u);
    } else if (dt == CRESSO_DTYPE_BF16) {
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p);
        const float u = __bfloat162float(__float2bfloat16_rn(update));
        h[e] = __float2bfloat16_rn(__bfloat162float(h[e]) + neg_lr16 * u);
    } else {
        float* f = reinterpret_cast<float*>(p);
        f[e] = f[e] + neg_lr * update;
    }
}

// EMA with a copy on the first step (reference _update_reservoir,
// cresso_v5.py:900-905): old * decay + cur * (1 - decay).
// decay is the Python float of the group; torch multiplies a float32 tensor
// by (float)decay and adds with alpha (float)(1 - decay).
__device__ __forceinline__ float reservoir(float old, float cur, double decay, int64_t step) {
    if (step <= 1) return cur;
    return old * (float)decay + cur * (float)(1.0 - decay);
}
// float64 state (float64 parameters): the decay and 1 - decay stay float64.
__device__ __forceinline__ double reservoir(double old, double cur, double decay, int64_t step) {
    if (step <= 1) return cur;
    return old * decay + cur * (1.0 - decay);
}

// Work-type overloads (float: the float32 functions; double: the float64 ones) for
// the kernels that run in the parameter's work type (float32 for float32 / float16 /
// bfloat16 parameters, float64 for float64 ones; cresso_v5.py:119-124).
__device__ __forceinline__ float w_exp(float x) { return expf(x); }
__device__ __forceinline__ double w_exp(double x) { return exp(x); }
__device__ __forceinline__ float w_log(float x) { return logf(x); }
__device__ __forceinline__ double w_log(double x) { return log(x); }
__device__ __forceinline__ float w_log1p(float x) { return log1pf(x); }
__device__ __forceinline__ double w_log1p(double x) { return log1p(x); }
__device__ __forceinline__ float w_pow(float x, float y) { return powf(x, y); }
__device__ __forceinline__ double w_pow(double x, double y) { return pow(x, y); }
__device__ __forceinline__ float w_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double w_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float w_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double w_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float w_abs(float x) { return fabsf(x); }
__device__ __forceinline__ double w_abs(double x) { return fabs(x); }
__device__ __forceinline__ float w_min(float x, float y) { return fminf(x, y); }
__device__ __forceinline__ double w_min(double x, double y) { return fmin(x, y); }
__device__ __forceinline__ float w_max(float x, float y) { return fmaxf(x, y); }
__device__ __forceinline__ double w_max(double x, double y) { return fmax(x, y); }
__device__ __forceinline__ float w_div(float x, float y) { return __fdiv_rn(x, y); }
__device__ __forceinline__ double w_div(double x, double y) { return __ddiv_rn(x, y); }
template <typename W>
__device__ __forceinline__ W clampw(W v, W lo, W hi) { return w_min(w_max(v, lo), hi); }
template <typename W>
__device__ __forceinline__ W w_sgn(W x) { return x > W(0) ? W(1) : (x < W(0) ? W(-1) : W(0)); }

// Element e of a float64 parameter / gradient.
__device__ __forceinline__ double load_f64(const void* p, int64_t e) {
    return __ldg(reinterpret_cast<const double*>(p) + e);
}
template <typename W>
__device__ __forceinline__ W load_w(const void* p, int64_t e, int dt);
template <>
__device__ __forceinline__ float load_w<float>(const void* p, int64_t e, int dt) { return load_elem(p, e, dt); }
template <>
__device__ __forceinline__ double load_w<double>(const void* p, int64_t e, int) { return load_f64(p, e); }
// -lr in the parameter's type: float32 / 16-bit as neg_lr_in, float64: -lr.
template <typename W>
__device__ __forceinline__ W neg_lr_w(double lr, int dt);
template <>
__device__ __forceinline__ float neg_lr_w<float>(double lr, int dt) { return neg_lr_in(lr, dt); }
template <>
__device__ __forceinline__ double neg_lr_w<double>(double lr, int) { return -lr; }
// param.add_(update, alpha=-lr): float64 parameters p + (-lr) u in float64.
template <typename W>
__device__ __forceinline__ void apply_update_w(void* p, int64_t e, int dt, W neg_lr, W neg_lr16, W update);
template <>
__device__ __forceinline__ void apply_update_w<float>(void* p, int64_t e, int dt, float neg_lr, float neg_lr16,
                                                      float update) {
    apply_update(p, e, dt, neg_lr, neg_lr16, update);
}
template <>
__device__ __forceinline__ void apply_update_w<double>(void* p, int64_t e, int, double neg_lr, double, double update) {
    double* d = reinterpret_cast<double*>(p);
    d[e] = d[e] + neg_lr * update;
}

}  // namespace cresso
