// Per-shape workspace (separable carrier tables, stats, Gram, hash bin
// counts), the shared hash bin-index cache, and the op-level entry points
// (hash index / reduce / gather, basis project / reconstruct, instant metric)
// that mirror the reference's per-op extension functions.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "basis_dev.cuh"
#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

// ---------------------------------------------------------------------------
// Host-side carrier parameters
// ---------------------------------------------------------------------------

// _hash_unit (cresso_v5.py:127-135).  Inputs are small, so the Python integer
// arithmetic fits in uint64; the 32-bit masks make the wrapped products exact.
static double hash_unit_host(int64_t n, int64_t salt) {
    uint64_t x = (uint64_t)(n + 1) * 0x9E3779B1ULL + (uint64_t)(salt + 11) * 0x85EBCA77ULL;
    x ^= x >> 16;
    x = (x * 0x7FEB352DULL) & 0xFFFFFFFFULL;
    x ^= x >> 15;
    x = (x * 0x846CA68BULL) & 0xFFFFFFFFULL;
    x ^= x >> 16;
    return (double)(x & 0xFFFFFFULL) / (double)(1 << 24);
}

struct AxisParam {
    double f, chirp, center, width;
    int32_t pad0, pad1;
};
// A tensor of rank n >= 2 is handled as (product of the n - 1 leading axes) x
// (last axis): every carrier factorises so, the leading axes composing into
// the row table (complex products of (cos, sin) pairs, or component-wise
// products for the product kind).  A 1-D tensor has no leading axis.
struct ModeParam {
    int32_t zero, kind, nlead, pad;
    AxisParam lead[CRESSO_MAX_NDIM - 1];
    AxisParam col;
};
struct ModePack {
    ModeParam m[kMaxRankPlain];
    int64_t ldim[CRESSO_MAX_NDIM];  // leading axis lengths
};

static AxisParam axis_param(int64_t mode, int64_t axis, int64_t f) {
    AxisParam a{};
    a.f = (double)f;
    a.chirp = 0.25 + 1.75 * hash_unit_host(mode, 17 + axis);
    a.center = 0.15 + 0.70 * hash_unit_host(mode, 101 + axis);
    a.width = 0.18 + 0.20 * hash_unit_host(mode, 151 + axis);
    return a;
}

static_assert(sizeof(ModeParam) <= kModeParamBytes, "mode parameters fit their workspace slot");

// Carrier parameters of mode k (frequencies freqs[k][ndim]).
static void fill_mode(ModeParam& m, int64_t ndim, int64_t k, const int64_t* freqs) {
    int64_t fsum = 0;
    for (int64_t a = 0; a < ndim; ++a) fsum += freqs[k * ndim + a] < 0 ? -freqs[k * ndim + a] : freqs[k * ndim + a];
    m.zero = fsum == 0;
    m.kind = (int32_t)(k % 4);
    m.nlead = (int32_t)(ndim - 1);
    for (int64_t a = 0; a + 1 < ndim; ++a) m.lead[a] = axis_param(k, a, freqs[k * ndim + a]);
    m.col = axis_param(k, ndim - 1, freqs[k * ndim + ndim - 1]);
}

static ModePack make_modes(int64_t ndim, const int64_t* shape, int64_t rank, const int64_t* freqs) {
    ModePack p;
    memset(&p, 0, sizeof(p));
    for (int64_t a = 0; a + 1 < ndim; ++a) p.ldim[a] = shape[a];
    for (int64_t k = 0; k < rank; ++k) fill_mode(p.m[k], ndim, k, freqs);
    return p;
}

// Leading axis lengths, passed by value to the wide-rank set-up kernels.
struct Ldim {
    int64_t d[CRESSO_MAX_NDIM];
};

// ---------------------------------------------------------------------------
// Set-up kernels
// ---------------------------------------------------------------------------

// One axis value (x1, x2) of mode k at coordinate idx of an axis of length dim.
// Mirrors _axis_coord / _additive_phase / _basis_pair (cresso_v5.py:237-348)
// in float64.
__device__ void axis_value(const ModeParam& m, const AxisParam& ax, int64_t idx, int64_t dim, double& x1, double& x2) {
    if (m.zero) {
        x1 = 1.0;
        x2 = 0.0;
        return;
    }
    const double pi = 3.14159265358979323846;
    const double u = ((double)idx + 0.5) / (double)dim;
    const double f = ax.f;
    if (m.kind == 1) {
        if (f == 0.0) {  // axis skipped in the products
            x1 = 1.0;
            x2 = 1.0;
        } else {
            sincos(pi * f * u, &x2, &x1);
        }
        return;
    }
    double ph = pi * f * u;
    if (m.kind >= 2) ph += pi * ax.chirp * fmax(1.0, f) * (u - 0.5) * (u - 0.5);
    sincos(ph, &x2, &x1);
    if (m.kind == 3) {
        const double z = (u - ax.center) / ax.width;
        const double w = exp(-0.5 * z * z);
        x1 *= w;
        x2 *= w;
    }
}

// Table value (x1, x2) of mode m at table index idx: a global row (idx < grows,
// the composition of the leading axes) or column idx - grows.
__device__ __forceinline__ void table_value(const ModeParam& m, const int64_t* ldim, int64_t idx, int64_t grows,
                                            int64_t gcols, double& x1, double& x2) {
    if (idx >= grows) {
        axis_value(m, m.col, idx - grows, gcols, x1, x2);
    } else if (m.zero) {
        x1 = 1.0;
        x2 = 0.0;
    } else {
        // leading axes, last one fastest; start from the identity of the composition
        x1 = 1.0;
        x2 = m.kind == 1 ? 1.0 : 0.0;
        int64_t rem = idx;
        for (int a = m.nlead - 1; a >= 0; --a) {
            const int64_t dim = ldim[a];
            const int64_t coord = rem % dim;
            rem /= dim;
            double y1, y2;
            axis_value(m, m.lead[a], coord, dim, y1, y2);
            if (m.kind == 1) {
                x1 *= y1;
                x2 *= y2;
            } else {
                const double t1 = x1 * y1 - x2 * y2;
                x2 = x1 * y2 + x2 * y1;
                x1 = t1;
            }
        }
    }
}

// Axis tables in T (float for the float32 path, double for float64 tensors).
template <typename T>
__global__ void build_tables_kernel(ModePack modes, int rank, int rm, int64_t grows, int64_t gcols, T* rowtab,
                                    T* coltab) {
    const int64_t total = (grows + gcols) * rm;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(t % rm);
        const int64_t idx = t / rm;
        double x1 = 0.0, x2 = 0.0;
        if (k < rank) table_value(modes.m[k], modes.ldim, idx, grows, gcols, x1, x2);
        if (idx < grows) {
            rowtab[(idx * rm + k) * 2 + 0] = (T)x1;
            rowtab[(idx * rm + k) * 2 + 1] = (T)x2;
        } else {
            const int64_t j = idx - grows;
            coltab[(2 * k) * gcols + j] = (T)x1;
            coltab[(2 * k + 1) * gcols + j] = (T)x2;
        }
    }
}

// Block 0 sums the row table, block 1 the column table: S1[p] = sum x_p and
// S2[p][q] = sum x_p x_q over the axis, p = 2k + (0 | 1), in float64.
template <typename T>
__global__ void table_sums_kernel(const T* rowtab, const T* coltab, int rm, int64_t grows, int64_t gcols,
                                  double* tmp) {
    const int P = 2 * rm;
    const bool rows = blockIdx.x == 0;
    const int64_t len = rows ? grows : gcols;
    double* S1 = tmp + (rows ? 0 : (P + P * P));
    double* S2 = S1 + P;
    for (int w = threadIdx.x; w < P + P * P; w += blockDim.x) {
        int p, q;
        if (w < P) {
            p = w;
            q = -1;
        } else {
            p = (w - P) / P;
            q = (w - P) % P;
            if (q < p) continue;
        }
        double s = 0.0;
        for (int64_t i = 0; i < len; ++i) {
            double xp, xq = 1.0;
            if (rows) {
                xp = rowtab[i * P + p];
                if (q >= 0) xq = rowtab[i * P + q];
            } else {
                xp = coltab[(int64_t)p * gcols + i];
                if (q >= 0) xq = coltab[(int64_t)q * gcols + i];
            }
            s += xp * xq;
        }
        if (q < 0) {
            S1[p] = s;
        } else {
            S2[p * P + q] = s;
            S2[q * P + p] = s;
        }
    }
}

struct Term {
    double c;
    int p, q;
};

// Separable terms of raw basis function X = 2k + comp (comp 0 cos, 1 sin):
// raw_X(i, j) = sum_t c_t * rowtab_{p_t}(i) * coltab_{q_t}(j).
__device__ int basis_terms(int X, Term* t) {
    const int k = X >> 1;
    const int c0 = 2 * k, s0 = 2 * k + 1;
    if (mode_is_product(k)) {
        const int p = (X & 1) ? s0 : c0;
        t[0].c = 1.0;
        t[0].p = p;
        t[0].q = p;
        return 1;
    }
    if ((X & 1) == 0) {  // a1 b1 - a2 b2
        t[0].c = 1.0;
        t[0].p = c0;
        t[0].q = c0;
        t[1].c = -1.0;
        t[1].p = s0;
        t[1].q = s0;
    } else {  // a1 b2 + a2 b1
        t[0].c = 1.0;
        t[0].p = c0;
        t[0].q = s0;
        t[1].c = 1.0;
        t[1].p = s0;
        t[1].q = c0;
    }
    return 2;
}

// Stats of raw basis function X = 2k + comp with mean m and mean square m2
// over the tensor: its mean and inverse RMS (zero-mode carriers stay (1, 0)).
__device__ void store_stat(ModeStats* stats, int X, int rank, bool zero, double m, double m2, double& mu_x,
                           double& inv_x) {
    const int k = X >> 1;
    double mhat = 0.0;
    mu_x = 0.0;
    inv_x = 0.0;
    if (k < rank) {
        if (zero) {
            inv_x = 1.0;
            mhat = m;  // unnormalised (1, 0) carrier: mean 1 for cos, 0 for sin
        } else {
            const double var = fmax(m2 - m * m, 0.0);
            // A carrier that is constant over the tensor (an axis of length 1)
            // normalises to zero (the reference divides fp32 rounding noise
            // by 1e-6 there); everything else follows the reference formula.
            if (var <= 1e-10 * m2) {
                inv_x = 0.0;
            } else {
                inv_x = 1.0 / fmax(sqrt(var + 1e-12), 1e-6);
            }
            mu_x = m;
        }
    }
    if ((X & 1) == 0) {
        stats[k].mu_c = mu_x;
        stats[k].inv_c = inv_x;
        stats[k].mhat_c = mhat;
        stats[k].rawmean_c = k < rank ? m : 0.0;
    } else {
        stats[k].mu_s = mu_x;
        stats[k].inv_s = inv_x;
        stats[k].mhat_s = mhat;
        stats[k].rawmean_s = k < rank ? m : 0.0;
    }
}

// Normalisation stats and the Gram matrix of the normalised carriers, from
// the table sums.  _normalize_basis (cresso_v5.py:138-142): zero mean, divide
// by max(sqrt(mean(x^2) + 1e-12), 1e-6).  The zero mode stays (1, 0).
__global__ void stats_gram_kernel(ModePack modes, int rank, int rm, double n, const double* tmp, ModeStats* stats,
                                  double* gram) {
    const int P = 2 * rm;
    const double* A1 = tmp;
    const double* A2 = tmp + P;
    const double* B1 = tmp + P + P * P;
    const double* B2 = B1 + P;
    __shared__ double mu[2 * kMaxRankPlain], inv[2 * kMaxRankPlain], ex2[2 * kMaxRankPlain];
    for (int X = threadIdx.x; X < P; X += blockDim.x) {
        const int k = X >> 1;
        Term t[2];
        const int nt = basis_terms(X, t);
        double m = 0.0, m2 = 0.0;
        for (int a = 0; a < nt; ++a) {
            m += t[a].c * A1[t[a].p] * B1[t[a].q];
            for (int b = 0; b < nt; ++b) m2 += t[a].c * t[b].c * A2[t[a].p * P + t[b].p] * B2[t[a].q * P + t[b].q];
        }
        m /= n;
        m2 /= n;
        double mu_x, inv_x;
        store_stat(stats, X, rank, k < rank && modes.m[k].zero, m, m2, mu_x, inv_x);
        mu[X] = mu_x;
        inv[X] = inv_x;
        ex2[X] = m;
    }
    __syncthreads();
    for (int w = threadIdx.x; w < P * P; w += blockDim.x) {
        const int X = w / P, Y = w % P;
        Term tx[2], ty[2];
        const int nx = basis_terms(X, tx), ny = basis_terms(Y, ty);
        double e = 0.0;
        for (int a = 0; a < nx; ++a)
            for (int b = 0; b < ny; ++b) e += tx[a].c * ty[b].c * A2[tx[a].p * P + ty[b].p] * B2[tx[a].q * P + ty[b].q];
        e /= n;
        // mean((raw_X - mu_X)(raw_Y - mu_Y)) = E[XY] - mu_X E[Y] - mu_Y E[X] + mu_X mu_Y
        const double cov = e - mu[X] * ex2[Y] - mu[Y] * ex2[X] + mu[X] * mu[Y];
        gram[w] = inv[X] * inv[Y] * cov;
    }
}

// ---- Wide rank (65 to 4096 modes, float64 workspace): the mode parameters are
// read from device memory, and only each mode's own table sums are formed (the
// float64 spectral path needs no carrier Gram).

__global__ void build_tables_wide_kernel(const ModeParam* __restrict__ modes, Ldim ldim, int rank, int rm,
                                         int64_t grows, int64_t gcols, double* rowtab, double* coltab) {
    const int64_t total = (grows + gcols) * rm;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(t % rm);
        const int64_t idx = t / rm;
        double x1 = 0.0, x2 = 0.0;
        if (k < rank) table_value(modes[k], ldim.d, idx, grows, gcols, x1, x2);
        if (idx < grows) {
            rowtab[(idx * rm + k) * 2 + 0] = x1;
            rowtab[(idx * rm + k) * 2 + 1] = x2;
        } else {
            const int64_t j = idx - grows;
            coltab[(2 * k) * gcols + j] = x1;
            coltab[(2 * k + 1) * gcols + j] = x2;
        }
    }
}

// Per axis (blockIdx.y: 0 rows, 1 columns) and mode k: S1[2k + c] = sum x_c and
// the mode's block D[k][2c + c'] = sum x_c x_c' (c, c' = 0 cos, 1 sin), summed
// in index order.  Axis a's sums start at tmp + 6 rm a: S1[2 rm], then D[rm][4].
__global__ void table_sums_blocks_kernel(const double* __restrict__ rowtab, const double* __restrict__ coltab, int rm,
                                         int64_t grows, int64_t gcols, double* tmp) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= rm) return;
    const bool rows = blockIdx.y == 0;
    const int64_t len = rows ? grows : gcols;
    double s1 = 0.0, s2 = 0.0, s11 = 0.0, s12 = 0.0, s22 = 0.0;
    for (int64_t i = 0; i < len; ++i) {
        double x1, x2;
        if (rows) {
            x1 = rowtab[(i * rm + k) * 2];
            x2 = rowtab[(i * rm + k) * 2 + 1];
        } else {
            x1 = coltab[(int64_t)(2 * k) * gcols + i];
            x2 = coltab[(int64_t)(2 * k + 1) * gcols + i];
        }
        s1 += x1;
        s2 += x2;
        s11 += x1 * x1;
        s12 += x1 * x2;
        s22 += x2 * x2;
    }
    double* S1 = tmp + (rows ? 0 : 6 * rm);
    double* Dk = S1 + 2 * rm + 4 * k;
    S1[2 * k] = s1;
    S1[2 * k + 1] = s2;
    Dk[0] = s11;
    Dk[1] = s12;
    Dk[2] = s12;
    Dk[3] = s22;
}

// Normalisation stats from the per-mode table sums: the terms of a raw basis
// function only pair the tables of its own mode.
__global__ void stats_wide_kernel(const ModeParam* __restrict__ modes, int rank, int rm, double n,
                                  const double* __restrict__ tmp, ModeStats* stats) {
    const int P = 2 * rm;
    const double* A1 = tmp;
    const double* AD = tmp + P;
    const double* B1 = tmp + 6 * rm;
    const double* BD = B1 + P;
    for (int X = blockIdx.x * blockDim.x + threadIdx.x; X < P; X += gridDim.x * blockDim.x) {
        const int k = X >> 1;
        Term t[2];
        const int nt = basis_terms(X, t);
        auto blk = [&](const double* Dm, int p, int q) { return Dm[4 * k + 2 * (p - 2 * k) + (q - 2 * k)]; };
        double m = 0.0, m2 = 0.0;
        for (int a = 0; a < nt; ++a) {
            m += t[a].c * A1[t[a].p] * B1[t[a].q];
            for (int b = 0; b < nt; ++b) m2 += t[a].c * t[b].c * blk(AD, t[a].p, t[b].p) * blk(BD, t[a].q, t[b].q);
        }
        m /= n;
        m2 /= n;
        double mu_x, inv_x;
        store_stat(stats, X, rank, k < rank && modes[k].zero, m, m2, mu_x, inv_x);
    }
}

__global__ void hash_count_kernel(int64_t n, int64_t bins, int64_t tables, unsigned int* counts) {
    extern __shared__ unsigned int hist[];
    const int64_t tb = bins * tables;
    for (int64_t b = threadIdx.x; b < tb; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        for (int64_t t = 0; t < tables; ++t) atomicAdd(&hist[t * bins + hash_bin(i, bins, t)], 1u);
    __syncthreads();
    for (int64_t b = threadIdx.x; b < tb; b += blockDim.x)
        if (hist[b]) atomicAdd(&counts[b], hist[b]);
}

__global__ void counts_to_float_kernel(int64_t tb, unsigned int* counts) {
    for (int64_t b = threadIdx.x; b < tb; b += blockDim.x) {
        const unsigned int c = counts[b];
        reinterpret_cast<float*>(counts)[b] = (float)c;
    }
}

template <typename IdxT>
__global__ void hash_cache_kernel(int64_t n, int64_t bins, int64_t tables, IdxT* cache) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        for (int64_t t = 0; t < tables; ++t) cache[t * n + i] = (IdxT)hash_bin(i, bins, t);
}

// Joint section of a two-table cache with at most 64 bins: j = b0 + 64 b1 per
// flat index, one 16-bit load for both bins.
__global__ void hash_joint_kernel(int64_t n, int64_t bins, uint16_t* joint) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        joint[i] = (uint16_t)(hash_bin(i, bins, 0) + 64 * hash_bin(i, bins, 1));
}

// ---------------------------------------------------------------------------
// Op-level kernels (single-block reductions: they back the op parity tests)
// ---------------------------------------------------------------------------

__global__ void hash_index_kernel(int64_t offset, int64_t n, int64_t bins, int64_t salt, int64_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = hash_bin(offset + i, bins, salt);
}

__global__ void hash_gather_kernel(const float* values, int64_t bins, int64_t n, int64_t salt, float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = values[hash_bin(i, bins, salt)];
}

// Bin sums in float64 (one block; per-bin fixed-order combine of per-warp
// partial bins), then mean = sum / max(count, 1)  (cresso_v5.py:519-526).
__global__ void hash_reduce_mean_kernel(const float* x, int64_t n, int64_t bins, int64_t salt, float* out) {
    extern __shared__ double sb[];  // [kWarps][bins] sums followed by [kWarps][bins] counts
    double* sums = sb;
    double* cnts = sb + kWarps * bins;
    for (int64_t b = threadIdx.x; b < 2 * kWarps * bins; b += blockDim.x) sb[b] = 0.0;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        int64_t b = -1;
        double v = 0.0;
        if (i < n) {
            b = hash_bin(i, bins, salt);
            v = x[i];
        }
        // lanes of a warp add in lane order: deterministic
        for (int l = 0; l < 32; ++l) {
            const int64_t bl = __shfl_sync(0xffffffffu, b, l);
            const double vl = __shfl_sync(0xffffffffu, v, l);
            if (lane == 0 && bl >= 0) {
                sums[warp * bins + bl] += vl;
                cnts[warp * bins + bl] += 1.0;
            }
        }
    }
    __syncthreads();
    for (int64_t b = threadIdx.x; b < bins; b += blockDim.x) {
        double s = 0.0, c = 0.0;
        for (int w = 0; w < kWarps; ++w) {
            s += sums[w * bins + b];
            c += cnts[w * bins + b];
        }
        out[b] = (float)s / fmaxf((float)c, 1.0f);
    }
}

template <int RM>
__global__ void basis_project_kernel(const float* x, const ShapeWsHeader* hdr_dev, const float* rowtab, const float* coltab,
                                     const ModeStats* stats, int64_t grows, int64_t gcols, int rank, float* out_cos,
                                     float* out_sin) {
    double C[RM], S[RM];
    double sx = 0.0;
#pragma unroll
    for (int k = 0; k < RM; ++k) C[k] = S[k] = 0.0;
    for (int64_t j = threadIdx.x; j < gcols; j += blockDim.x) {
        float z1[RM], z2[RM];
#pragma unroll
        for (int k = 0; k < RM; ++k) z1[k] = z2[k] = 0.0f;
        double colsum = 0.0;
        double Z1[RM], Z2[RM];
#pragma unroll
        for (int k = 0; k < RM; ++k) Z1[k] = Z2[k] = 0.0;
        for (int64_t i = 0; i < grows; ++i) {
            float a1[RM], a2[RM];
            load_row<RM>(rowtab, i, a1, a2);
            const double v = x[i * gcols + j];
            colsum += v;
#pragma unroll
            for (int k = 0; k < RM; ++k) {
                Z1[k] += v * (double)a1[k];
                Z2[k] += v * (double)a2[k];
            }
        }
        float b1[RM], b2[RM];
        load_col<RM>(coltab, gcols, j, b1, b2);
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            if (mode_is_product(k)) {
                C[k] += (double)b1[k] * Z1[k];
                S[k] += (double)b2[k] * Z2[k];
            } else {
                C[k] += (double)b1[k] * Z1[k] - (double)b2[k] * Z2[k];
                S[k] += (double)b2[k] * Z1[k] + (double)b1[k] * Z2[k];
            }
        }
        sx += colsum;
        (void)z1;
        (void)z2;
    }
    __shared__ double red[(2 * RM + 1) * kWarps];
    __shared__ double tot[2 * RM + 1];
    double v[2 * RM + 1];
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        v[k] = C[k];
        v[RM + k] = S[k];
    }
    v[2 * RM] = sx;
    block_sum_to<2 * RM + 1>(v, red, tot);
    if (threadIdx.x < rank) {
        const int k = threadIdx.x;
        const double n = (double)grows * (double)gcols;
        const ModeStats st = stats[k];
        out_cos[k] = (float)(st.inv_c * (tot[k] - st.mu_c * tot[2 * RM]) / n);
        out_sin[k] = (float)(st.inv_s * (tot[RM + k] - st.mu_s * tot[2 * RM]) / n);
    }
    (void)hdr_dev;
}

template <int RM>
__global__ void basis_reconstruct_kernel(const float* cc, const float* cs, const float* gates, const float* rowtab,
                                         const float* coltab, const ModeStats* stats, int64_t grows, int64_t gcols,
                                         int rank, float* out) {
    __shared__ float al[RM], be[RM];
    __shared__ float Ksh;
    if (threadIdx.x == 0) {
        const double shrink = recon_shrink(rank);
        double K = 0.0;
        for (int k = 0; k < RM; ++k) {
            double a = 0.0, b = 0.0;
            if (k < rank) {
                const double g = gates ? (double)gates[k] : 1.0;
                // _reconstruct uses alpha = float(coeff) * shrink * gate (cresso_v5.py:374)
                a = (double)cc[k] * shrink * g * stats[k].inv_c;
                b = (double)cs[k] * shrink * g * stats[k].inv_s;
                K -= a * stats[k].mu_c + b * stats[k].mu_s;
            }
            al[k] = (float)a;
            be[k] = (float)b;
        }
        Ksh = (float)K;
    }
    __syncthreads();
    const int64_t n = grows * gcols;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / gcols, j = e % gcols;
        float a1[RM], a2[RM], b1[RM], b2[RM], U[RM], V[RM];
        load_row<RM>(rowtab, i, a1, a2);
        load_col<RM>(coltab, gcols, j, b1, b2);
        make_uv<RM>(b1, b2, al, be, U, V);
        out[e] = recon_dot<RM>(Ksh, a1, a2, U, V);
    }
}

// Instant axial metric of a 1-D or 2-D field (cresso_v5.py:243-262), one
// block: float64 axis sums in shared memory, then the per-element metric.
__global__ void instant_metric_kernel(const float* rel, int64_t rows, int64_t cols, int ndim, float power, float coupling,
                                      float eps, float* out) {
    extern __shared__ double axs[];  // rows row-sums then cols col-sums (2-D)
    __shared__ double red[kWarps + 1];
    const int64_t n = rows * cols;
    const float pw = fmaxf(power, 0.25f);
    if (coupling == 0.0f || n <= 1) {
        for (int64_t e = threadIdx.x; e < n; e += blockDim.x) out[e] = 1.0f;
        return;
    }
    if (ndim == 2)
        for (int64_t t = threadIdx.x; t < rows + cols; t += blockDim.x) axs[t] = 0.0;
    __syncthreads();
    double tot = 0.0;
    if (ndim == 2) {
        for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
            double cs = 0.0;
            for (int64_t i = 0; i < rows; ++i) cs += fminf(powf(fmaxf(rel[i * cols + j], eps), pw), 1.0e6f);
            axs[rows + j] = cs;
        }
        for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
            double rs = 0.0;
            for (int64_t j = 0; j < cols; ++j) rs += fminf(powf(fmaxf(rel[i * cols + j], eps), pw), 1.0e6f);
            axs[i] = rs;
            tot += rs;
        }
    } else {
        for (int64_t e = threadIdx.x; e < n; e += blockDim.x) tot += fminf(powf(fmaxf(rel[e], eps), pw), 1.0e6f);
    }
    tot = block_sum(tot, red);
    const float gm = fmaxf((float)(tot / (double)n), eps);
    const float kk = coupling / ((float)ndim * pw);
    for (int64_t e = threadIdx.x; e < n; e += blockDim.x) {
        float lg;
        if (ndim == 2) {
            const int64_t i = e / cols, j = e % cols;
            const float rm = (float)(axs[i] / (double)cols), cm = (float)(axs[rows + j] / (double)rows);
            lg = logf(fmaxf(rm / gm, eps)) + logf(fmaxf(cm / gm, eps));
        } else {
            const float d = fminf(powf(fmaxf(rel[e], eps), pw), 1.0e6f);
            lg = logf(fmaxf(d / gm, eps));
        }
        out[e] = clampf(expf(kk * lg), 0.08f, 12.0f);
    }
}

static int checked_shape(int64_t ndim, const int64_t* shape, int64_t* grows, int64_t* gcols) {
    CRESSO_REQUIRE(shape != nullptr, CRESSO_EINVAL, "shape pointer is NULL");
    CRESSO_REQUIRE(ndim >= 1 && ndim <= CRESSO_MAX_NDIM, CRESSO_EUNSUPPORTED,
                   "spectral carriers support tensors of rank 1 to %d (got ndim=%lld)", CRESSO_MAX_NDIM, (long long)ndim);
    for (int64_t a = 0; a < ndim; ++a) CRESSO_REQUIRE(shape[a] > 0, CRESSO_EINVAL, "shape[%lld] must be > 0", (long long)a);
    // (product of the leading axes) x (last axis)
    int64_t lead = 1;
    for (int64_t a = 0; a + 1 < ndim; ++a) lead *= shape[a];
    *grows = lead;
    *gcols = shape[ndim - 1];
    return CRESSO_OK;
}

int launch_project(int rm, const float* x, const ShapeWsHeader& h, const char* base, float* oc, float* os,
                   cudaStream_t st) {
    const float* rowtab = reinterpret_cast<const float*>(base + h.off_rowtab);
    const float* coltab = reinterpret_cast<const float*>(base + h.off_coltab);
    const ModeStats* stats = reinterpret_cast<const ModeStats*>(base + h.off_stats);
    switch (rm) {
        case 4:
            basis_project_kernel<4><<<1, kThreads, 0, st>>>(x, nullptr, rowtab, coltab, stats, h.grows, h.gcols,
                                                             (int)h.rank, oc, os);
            break;
        case 8:
            basis_project_kernel<8><<<1, kThreads, 0, st>>>(x, nullptr, rowtab, coltab, stats, h.grows, h.gcols,
                                                             (int)h.rank, oc, os);
            break;
        default:
            basis_project_kernel<16><<<1, kThreads, 0, st>>>(x, nullptr, rowtab, coltab, stats, h.grows, h.gcols,
                                                              (int)h.rank, oc, os);
    }
    CRESSO_LAUNCHED("basis_project_kernel");
    return CRESSO_OK;
}

}  // namespace cresso

using namespace cresso;

static int read_ws_header(const void* ws, ShapeWsHeader* h) {
    CRESSO_REQUIRE(ws != nullptr, CRESSO_EINVAL, "shape workspace pointer is NULL");
    CRESSO_CUDA(cudaMemcpy(h, ws, sizeof(ShapeWsHeader), cudaMemcpyDeviceToHost));
    CRESSO_REQUIRE(h->magic == kShapeWsMagic, CRESSO_EINVAL, "shape workspace is not initialised");
    return CRESSO_OK;
}

extern "C" {

int cresso_hash_index(int64_t offset, int64_t n, int64_t bins, int64_t salt, int64_t* idx, cresso_stream_t stream) {
    CRESSO_REQUIRE(n >= 0 && offset >= 0, CRESSO_EINVAL, "hash_index: n and offset must be >= 0");
    CRESSO_REQUIRE(bins > 0, CRESSO_EINVAL, "hash_index: bins must be > 0");
    CRESSO_REQUIRE(salt >= 0, CRESSO_EINVAL, "hash_index: salt must be >= 0");
    if (n == 0) return CRESSO_OK;
    CRESSO_REQUIRE(idx != nullptr, CRESSO_EINVAL, "hash_index: output pointer is NULL");
    const int blocks = (int)std::min<int64_t>(ceil_div(n, kThreads), 65535);
    hash_index_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(offset, n, bins, salt, idx);
    CRESSO_LAUNCHED("hash_index_kernel");
    return CRESSO_OK;
}

int cresso_hash_gather(const float* values, int64_t bins, int64_t n, int64_t salt, float* out, cresso_stream_t stream) {
    CRESSO_REQUIRE(n >= 0 && bins > 0 && salt >= 0, CRESSO_EINVAL, "hash_gather: bad n / bins / salt");
    if (n == 0) return CRESSO_OK;
    CRESSO_REQUIRE(values && out, CRESSO_EINVAL, "hash_gather: NULL pointer");
    const int blocks = (int)std::min<int64_t>(ceil_div(n, kThreads), 65535);
    hash_gather_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(values, bins, n, salt, out);
    CRESSO_LAUNCHED("hash_gather_kernel");
    return CRESSO_OK;
}

int cresso_hash_reduce_mean(const float* x, int64_t n, int64_t bins, int64_t salt, float* out, cresso_stream_t stream) {
    CRESSO_REQUIRE(n >= 0 && salt >= 0, CRESSO_EINVAL, "hash_reduce_mean: bad n / salt");
    CRESSO_REQUIRE(bins > 0 && bins <= 1024, CRESSO_EUNSUPPORTED,
                   "hash_reduce_mean: bins must be in [1, 1024] (got %lld)", (long long)bins);
    CRESSO_REQUIRE(out != nullptr && (n == 0 || x != nullptr), CRESSO_EINVAL, "hash_reduce_mean: NULL pointer");
    const size_t smem = (size_t)2 * kWarps * bins * sizeof(double);
    if (smem > 48 * 1024)
        CRESSO_CUDA(cudaFuncSetAttribute(hash_reduce_mean_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    hash_reduce_mean_kernel<<<1, kThreads, smem, (cudaStream_t)stream>>>(x, n, bins, salt, out);
    CRESSO_LAUNCHED("hash_reduce_mean_kernel");
    return CRESSO_OK;
}

int cresso_hash_cache_bytes(int64_t n, int64_t bins, int64_t tables, int64_t* bytes) {
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "hash_cache_bytes: NULL output");
    CRESSO_REQUIRE(n >= 0 && bins > 0 && bins <= 65536 && tables >= 1, CRESSO_EINVAL,
                   "hash_cache_bytes: need n >= 0, 1 <= bins <= 65536, tables >= 1");
    *bytes = align_up(n * tables * (bins <= 256 ? 1 : 2), 256);
    if (tables == 2 && bins <= 64) *bytes += align_up(2 * n, 256);  // the joint section
    return CRESSO_OK;
}

int cresso_hash_cache_init(int64_t n, int64_t bins, int64_t tables, void* cache, cresso_stream_t stream) {
    CRESSO_REQUIRE(n >= 0 && bins > 0 && bins <= 65536 && tables >= 1, CRESSO_EINVAL,
                   "hash_cache_init: need n >= 0, 1 <= bins <= 65536, tables >= 1");
    if (n == 0) return CRESSO_OK;
    CRESSO_REQUIRE(cache != nullptr, CRESSO_EINVAL, "hash_cache_init: NULL cache");
    const int blocks = (int)std::min<int64_t>(ceil_div(n, kThreads), 148 * 16);
    if (bins <= 256)
        hash_cache_kernel<uint8_t><<<blocks, kThreads, 0, (cudaStream_t)stream>>>(n, bins, tables, (uint8_t*)cache);
    else
        hash_cache_kernel<uint16_t><<<blocks, kThreads, 0, (cudaStream_t)stream>>>(n, bins, tables, (uint16_t*)cache);
    CRESSO_LAUNCHED("hash_cache_kernel");
    if (tables == 2 && bins <= 64) {
        uint16_t* joint = reinterpret_cast<uint16_t*>((char*)cache + align_up(2 * n, 256));
        hash_joint_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(n, bins, joint);
        CRESSO_LAUNCHED("hash_joint_kernel");
    }
    return CRESSO_OK;
}

int cresso_shape_workspace_bytes(int64_t ndim, const int64_t* shape, int64_t rank, int64_t bins, int64_t tables,
                                 int64_t* bytes) {
    int64_t grows, gcols;
    int st = checked_shape(ndim, shape, &grows, &gcols);
    if (st) return st;
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "shape_workspace_bytes: NULL output");
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRank, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA path (got %lld)", kMaxRank, (long long)rank);
    CRESSO_REQUIRE(bins >= 0 && tables >= 0, CRESSO_EINVAL, "bins / tables must be >= 0");
    *bytes = shape_ws_layout(ndim, grows, gcols, rank, rank_pad(rank), bins, tables).bytes;
    return CRESSO_OK;
}

int cresso_shape_workspace_init(int64_t ndim, const int64_t* shape, int64_t rank, const int64_t* freqs, int64_t bins,
                                int64_t tables, void* ws, cresso_stream_t stream) {
    int64_t grows, gcols;
    int st = checked_shape(ndim, shape, &grows, &gcols);
    if (st) return st;
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRank, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA path (got %lld)", kMaxRank, (long long)rank);
    CRESSO_REQUIRE(freqs != nullptr && ws != nullptr, CRESSO_EINVAL, "shape_workspace_init: NULL pointer");
    CRESSO_REQUIRE(bins >= 0 && tables >= 0, CRESSO_EINVAL, "bins / tables must be >= 0");
    const int rm = rank_pad(rank);
    ShapeWsHeader h = shape_ws_layout(ndim, grows, gcols, rank, rm, bins, tables);
    cudaStream_t s = (cudaStream_t)stream;
    char* base = (char*)ws;
    ModePack modes = make_modes(ndim, shape, rank, freqs);
    float* rowtab = reinterpret_cast<float*>(base + h.off_rowtab);
    float* coltab = reinterpret_cast<float*>(base + h.off_coltab);
    double* tmp = reinterpret_cast<double*>(base + h.off_tmp);
    const int64_t cells = (grows + gcols) * rm;
    build_tables_kernel<float><<<(int)std::min<int64_t>(ceil_div(cells, kThreads), 4096), kThreads, 0, s>>>(
        modes, (int)rank, rm, grows, gcols, rowtab, coltab);
    CRESSO_LAUNCHED("build_tables_kernel");
    table_sums_kernel<float><<<2, kThreads, 0, s>>>(rowtab, coltab, rm, grows, gcols, tmp);
    CRESSO_LAUNCHED("table_sums_kernel");
    stats_gram_kernel<<<1, kThreads, 0, s>>>(modes, (int)rank, rm, (double)grows * (double)gcols, tmp,
                                              reinterpret_cast<ModeStats*>(base + h.off_stats),
                                              reinterpret_cast<double*>(base + h.off_gram));
    CRESSO_LAUNCHED("stats_gram_kernel");
    if (bins > 0 && tables > 0) {
        CRESSO_REQUIRE(bins * tables <= kMaxTB, CRESSO_EUNSUPPORTED,
                       "hash_bins * hash_tables must be <= %d on the CUDA path", kMaxTB);
        unsigned int* counts = reinterpret_cast<unsigned int*>(base + h.off_counts);
        CRESSO_CUDA(cudaMemsetAsync(counts, 0, bins * tables * 4, s));
        const size_t smem = (size_t)bins * tables * 4;
        if (smem > 48 * 1024)
            CRESSO_CUDA(cudaFuncSetAttribute(hash_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        const int blocks = (int)std::min<int64_t>(ceil_div(h.n, kThreads * 16), 148 * 8);
        hash_count_kernel<<<blocks, kThreads, smem, s>>>(h.n, bins, tables, counts);
        CRESSO_LAUNCHED("hash_count_kernel");
        counts_to_float_kernel<<<1, kThreads, 0, s>>>(bins * tables, counts);
        CRESSO_LAUNCHED("counts_to_float_kernel");
    }
    CRESSO_CUDA(cudaMemcpyAsync(ws, &h, sizeof(h), cudaMemcpyHostToDevice, s));
    // the header lives on this stack frame: finish the copy before returning
    CRESSO_CUDA(cudaStreamSynchronize(s));
    return CRESSO_OK;
}

int cresso_shape_workspace64_bytes(int64_t ndim, const int64_t* shape, int64_t rank, int64_t* bytes) {
    int64_t grows, gcols;
    int st = checked_shape(ndim, shape, &grows, &gcols);
    if (st) return st;
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "shape_workspace64_bytes: NULL output");
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRankWide, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA path (got %lld)", kMaxRankWide, (long long)rank);
    *bytes = shape_ws64_layout(ndim, grows, gcols, rank, rank_pad(rank)).bytes;
    return CRESSO_OK;
}

int cresso_shape_workspace64_init(int64_t ndim, const int64_t* shape, int64_t rank, const int64_t* freqs, void* ws,
                                  cresso_stream_t stream) {
    int64_t grows, gcols;
    int st = checked_shape(ndim, shape, &grows, &gcols);
    if (st) return st;
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRankWide, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA path (got %lld)", kMaxRankWide, (long long)rank);
    CRESSO_REQUIRE(freqs != nullptr && ws != nullptr, CRESSO_EINVAL, "shape_workspace64_init: NULL pointer");
    const int rm = rank_pad(rank);
    ShapeWsHeader h = shape_ws64_layout(ndim, grows, gcols, rank, rm);
    cudaStream_t s = (cudaStream_t)stream;
    char* base = (char*)ws;
    double* rowtab = reinterpret_cast<double*>(base + h.off_rowtab);
    double* coltab = reinterpret_cast<double*>(base + h.off_coltab);
    double* tmp = reinterpret_cast<double*>(base + h.off_tmp);
    const int64_t cells = (grows + gcols) * rm;
    if (rm > kMaxRankPlain) {
        // wide rank: the mode parameters go to the workspace (after the table sums)
        std::vector<ModeParam> mv((size_t)rm);
        memset(mv.data(), 0, sizeof(ModeParam) * mv.size());
        for (int64_t k = 0; k < rank; ++k) fill_mode(mv[(size_t)k], ndim, k, freqs);
        Ldim ld{};
        for (int64_t a = 0; a + 1 < ndim; ++a) ld.d[a] = shape[a];
        ModeParam* d_modes = reinterpret_cast<ModeParam*>(base + h.off_tmp + align_up(2 * (2 * rm + 4 * rm) * 8, 256));
        // pageable source: the copy has staged its bytes when it returns
        CRESSO_CUDA(cudaMemcpyAsync(d_modes, mv.data(), sizeof(ModeParam) * mv.size(), cudaMemcpyHostToDevice, s));
        build_tables_wide_kernel<<<(int)std::min<int64_t>(ceil_div(cells, kThreads), 4096), kThreads, 0, s>>>(
            d_modes, ld, (int)rank, rm, grows, gcols, rowtab, coltab);
        CRESSO_LAUNCHED("build_tables_wide_kernel");
        table_sums_blocks_kernel<<<dim3((unsigned)ceil_div(rm, kThreads), 2), kThreads, 0, s>>>(rowtab, coltab, rm, grows,
                                                                                                 gcols, tmp);
        CRESSO_LAUNCHED("table_sums_blocks_kernel");
        stats_wide_kernel<<<(int)ceil_div(2 * rm, kThreads), kThreads, 0, s>>>(
            d_modes, (int)rank, rm, (double)grows * (double)gcols, tmp, reinterpret_cast<ModeStats*>(base + h.off_stats));
        CRESSO_LAUNCHED("stats_wide_kernel");
        CRESSO_CUDA(cudaMemcpyAsync(ws, &h, sizeof(h), cudaMemcpyHostToDevice, s));
        CRESSO_CUDA(cudaStreamSynchronize(s));
        return CRESSO_OK;
    }
    ModePack modes = make_modes(ndim, shape, rank, freqs);
    build_tables_kernel<double><<<(int)std::min<int64_t>(ceil_div(cells, kThreads), 4096), kThreads, 0, s>>>(
        modes, (int)rank, rm, grows, gcols, rowtab, coltab);
    CRESSO_LAUNCHED("build_tables_kernel<double>");
    table_sums_kernel<double><<<2, kThreads, 0, s>>>(rowtab, coltab, rm, grows, gcols, tmp);
    CRESSO_LAUNCHED("table_sums_kernel<double>");
    stats_gram_kernel<<<1, kThreads, 0, s>>>(modes, (int)rank, rm, (double)grows * (double)gcols, tmp,
                                              reinterpret_cast<ModeStats*>(base + h.off_stats),
                                              reinterpret_cast<double*>(base + h.off_gram));
    CRESSO_LAUNCHED("stats_gram_kernel");
    CRESSO_CUDA(cudaMemcpyAsync(ws, &h, sizeof(h), cudaMemcpyHostToDevice, s));
    // the header lives on this stack frame: finish the copy before returning
    CRESSO_CUDA(cudaStreamSynchronize(s));
    return CRESSO_OK;
}

int cresso_basis_project(const float* x, const void* ws, float* out_cos, float* out_sin, cresso_stream_t stream) {
    ShapeWsHeader h;
    int st = read_ws_header(ws, &h);
    if (st) return st;
    CRESSO_REQUIRE(x && out_cos && out_sin, CRESSO_EINVAL, "basis_project: NULL pointer");
    return launch_project((int)h.rm, x, h, (const char*)ws, out_cos, out_sin, (cudaStream_t)stream);
}

int cresso_basis_reconstruct(const float* coef_cos, const float* coef_sin, const float* gates, const void* ws, float* out,
                             cresso_stream_t stream) {
    ShapeWsHeader h;
    int st = read_ws_header(ws, &h);
    if (st) return st;
    CRESSO_REQUIRE(coef_cos && coef_sin && out, CRESSO_EINVAL, "basis_reconstruct: NULL pointer");
    const char* base = (const char*)ws;
    const float* rowtab = reinterpret_cast<const float*>(base + h.off_rowtab);
    const float* coltab = reinterpret_cast<const float*>(base + h.off_coltab);
    const ModeStats* stats = reinterpret_cast<const ModeStats*>(base + h.off_stats);
    cudaStream_t s = (cudaStream_t)stream;
    const int blocks = (int)std::min<int64_t>(ceil_div(h.n, kThreads), 148 * 8);
    switch (h.rm) {
        case 4:
            basis_reconstruct_kernel<4><<<blocks, kThreads, 0, s>>>(coef_cos, coef_sin, gates, rowtab, coltab, stats,
                                                                     h.grows, h.gcols, (int)h.rank, out);
            break;
        case 8:
            basis_reconstruct_kernel<8><<<blocks, kThreads, 0, s>>>(coef_cos, coef_sin, gates, rowtab, coltab, stats,
                                                                     h.grows, h.gcols, (int)h.rank, out);
            break;
        default:
            basis_reconstruct_kernel<16><<<blocks, kThreads, 0, s>>>(coef_cos, coef_sin, gates, rowtab, coltab, stats,
                                                                      h.grows, h.gcols, (int)h.rank, out);
    }
    CRESSO_LAUNCHED("basis_reconstruct_kernel");
    return CRESSO_OK;
}

int cresso_instant_axis_metric(const float* rel, int64_t ndim, const int64_t* shape, double power, double coupling,
                               double eps, float* out, cresso_stream_t stream) {
    CRESSO_REQUIRE(ndim == 1 || ndim == 2, CRESSO_EUNSUPPORTED,
                   "instant_axis_metric: 1-D and 2-D fields (got ndim=%lld)", (long long)ndim);
    int64_t rows, cols;
    int st = checked_shape(ndim, shape, &rows, &cols);
    if (st) return st;
    CRESSO_REQUIRE(rel && out, CRESSO_EINVAL, "instant_axis_metric: NULL pointer");
    const size_t smem = ndim == 2 ? (size_t)(rows + cols) * sizeof(double) : 0;
    CRESSO_REQUIRE(smem <= 200 * 1024, CRESSO_EUNSUPPORTED, "instant_axis_metric: rows + cols too large for the op kernel");
    if (smem > 48 * 1024)
        CRESSO_CUDA(cudaFuncSetAttribute(instant_metric_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    instant_metric_kernel<<<1, kThreads, smem, (cudaStream_t)stream>>>(rel, rows, cols, (int)ndim, (float)power,
                                                                        (float)coupling, (float)eps, out);
    CRESSO_LAUNCHED("instant_metric_kernel");
    return CRESSO_OK;
}

}  // extern "C"
