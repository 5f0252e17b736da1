// Spectral-route CRESSO5 step for float64 parameters (cresso_v5.py:945-1353
// with float64 work and state, cresso_v5.py:119-124), and for float32 /
// float16 / bfloat16 parameters of rank 17 to 4096 (float32 state).
//
// The float32 path (spectral.cu) is built around float32 tiles, tf32 tensor-core
// reconstructions, fixed-point bin sums and at most 16 modes held in registers;
// these tensors instead run this plain float64 pipeline (modes padded to 4, 8,
// 16, 32 or 64), with the same five passes and the same reductions between
// them, each pass one launch over the blocks of a whole group of tensors and
// each finalize one launch of a block per tensor:
//   P1 force energy | fin1 scale
//   P2 density, hash-bin sums and counts, density projections
//      (+ row sums / column sums of the instant-metric density, rank >= 2)
//      | fin2 hash energy and bin log-metric, metric oscillator, instant factors
//   P3 tangent (kept in the scratch), error, port and tangent projections,
//      port bin sums | fin3 surprise, hash impulse, confidence, contact
//      oscillators, second prediction and echo coefficients
//   P4 drive Gram of (rational, bounded, root, tangent, prediction, novelty,
//      echo, hash prediction) | fin4 drive coefficients, drive energy, gain
//   P5 parameter update
// Carriers come from the float64 axis tables of a float64 shape workspace
// (cresso_shape_workspace64_init).  Block partial sums are written per block and
// added in block order by the one-block finalize kernels; the bin sums inside a
// block are exact integer sums (exact_bins_add), so every sum of the pipeline
// is the same from run to run.  Above rank 64 the modes leave the
// registers (the wide-rank kernels s64w_*, RM == 0 in the launch templates).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <string.h>

#include <algorithm>
#include <vector>

#include "basis_dev.cuh"
#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

namespace {

constexpr int kMaxTB64 = 2048;  // hash_bins * hash_tables on the float64 path
constexpr int kGram64 = 36;     // pair sums of 8 drive vectors
constexpr int kMaxBlocks64 = 256;
constexpr int kMaxLeadSum64 = 4096;  // sum of the leading axis lengths (rank >= 3)

enum {
    Q_LR, Q_WD, Q_EP, Q_DT, Q_IF, Q_CG, Q_REST, Q_CUBIC, Q_MDT, Q_MF, Q_MC, Q_LS, Q_IC, Q_IP, Q_RCM, Q_EM, Q_TM,
    Q_HD, Q_HID, Q_HMC, Q_HDM, Q_DFM, Q_RFM, Q_RD, Q_REFD, Q_RG, Q_CD, Q_CONFG, Q_SG, Q_SD, Q_PM, Q_NM, Q_WS, Q_SB,
    Q_TGT, Q_MING, Q_MAXG, Q_CLIP, Q_SPIKE, Q_EPS, Q_MAX, Q_RANK, Q_MAXF, Q_BINS, Q_TABLES, Q_HARDMIN, Q_THINCUT,
    Q_MD, Q_MID, Q_MDM, Q_COUNT
};
static_assert(sizeof(cresso_hparams) == Q_COUNT * sizeof(double), "cresso_hparams field order");

// P: storage type of the state (double for float64 tensors, float for float32,
// float16 and bfloat16 tensors of rank > 16); the arithmetic is float64.  The
// parameter and gradient keep their own type, pdt (CRESSO_DTYPE_*).
template <typename P>
struct alignas(16) T64 {
    int64_t ndim, N, rows, cols, step;
    int64_t dims[CRESSO_MAX_NDIM];
    void* param;
    const void* grad;
    const double* rowtab;  // [rows][rm][2]
    const double* coltab;  // [2 rm][cols]
    const ModeStats* stats;
    P *omega, *q_cos, *q_sin, *p_cos, *p_sin, *m_cos, *m_sin, *mp_cos, *mp_sin, *ca_cos, *ca_sin, *conf;
    P *h_energy, *h_impulse, *h_refractory, *force_rms, *drive_energy, *surprise, *action;
    int32_t R, T, B, hard, hash_on, echo_on, inst, local_on, f32, pdt;
    int32_t RW, pad_;  // padded rank: the mode stride of the tables and coefficient vectors
    double hp[64];
};

// Per-tensor values passed from the finalize kernels to the pass kernels.
struct C64 {
    double scale, gm, kk, meanL, S, clip;
    double m_al[kMaxRankPlain], m_be[kMaxRankPlain];  // log-metric reconstruction (shrink * metric oscillator)
    double p_al[kMaxRankPlain], p_be[kMaxRankPlain];  // prediction (shrink * gate * q), P3: old q, P4/P5: new q
    double e_al[kMaxRankPlain], e_be[kMaxRankPlain];  // echo reconstruction (shrink * tangent projection)
    double c[8], gain;                      // drive = sum c_i v_i
};

struct alignas(16) Buf64 {
    C64* cst;
    double* rec;     // [blocks][L]
    double* lterm;   // [T * B] per-bin log hash metric (P3)
    double* impv;    // [T * B] hash impulse per bin (P4 / P5)
    double* counts;  // [T * B] elements per bin
    double* rowsum;  // [rows] instant-metric density per row, then its log factor
    double* colsum;  // [cols] same per column
    double* tbuf;    // [N] tangent
    // wide rank only (rank > kMaxRankPlain):
    double* wcoef;   // [W_COUNT][RW] reconstruction coefficients and contact temporaries
    double* pbuf;    // [N] port field (P3)
    double* rec2;    // [chunks][blocks][kRec2] per-chunk projection records
    int blocks;      // blocks of this tensor in the element passes (records in rec)
};

// The tensors of one launch group: per-tensor descriptors and buffers in device
// memory, and for each launch kind the first block of every tensor (blk[n] is
// the grid).  Every kernel first finds its tensor and copies the two records
// into shared memory.
template <typename P>
struct G64 {
    const T64<P>* ts;
    const Buf64* bufs;
    const int* blk;      // [n + 1] element passes
    const int* blk_row;  // [n + 1] row sums of the instant-metric density
    const int* blk_col;  // [n + 1] column sums
    int n;
};

// Tensor t with blk[t] <= b < blk[t + 1] (blk ascending; empty ranges skipped).
__device__ __forceinline__ int find_tensor(const int* blk, int n, int b) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(blk + mid) <= b)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// Every thread: tensor t's descriptor and buffers into shared memory.
template <typename P>
__device__ __forceinline__ void bind_tensor(const G64<P>& G, int t, T64<P>& sD, Buf64& sB) {
    static_assert(sizeof(T64<P>) % 16 == 0 && sizeof(Buf64) % 16 == 0, "16-byte records");
    const int4* d = reinterpret_cast<const int4*>(G.ts + t);
    for (int i = threadIdx.x; i < (int)(sizeof(T64<P>) / 16); i += blockDim.x) reinterpret_cast<int4*>(&sD)[i] = d[i];
    const int4* b = reinterpret_cast<const int4*>(G.bufs + t);
    for (int i = threadIdx.x; i < (int)(sizeof(Buf64) / 16); i += blockDim.x) reinterpret_cast<int4*>(&sB)[i] = b[i];
    __syncthreads();
}

// Prologue of a kernel over the blocks of a group: D / Bf are this block's
// tensor, lb its block within the tensor, gb the tensor's blocks.
#define S64_BIND_BLOCKS(BLK)                                     \
    __shared__ T64<P> sD;                                        \
    __shared__ Buf64 sB;                                         \
    const int t_ = find_tensor(G.BLK, G.n, (int)blockIdx.x);     \
    bind_tensor(G, t_, sD, sB);                                  \
    const T64<P>& D = sD;                                        \
    const Buf64& Bf = sB;                                        \
    const int64_t lb = (int64_t)blockIdx.x - G.BLK[t_];          \
    const int64_t gb = (int64_t)(G.BLK[t_ + 1] - G.BLK[t_]);     \
    (void)lb;                                                    \
    (void)gb

// Prologue of a finalize kernel: one block per tensor.
#define S64_BIND_TENSOR()                                        \
    __shared__ T64<P> sD;                                        \
    __shared__ Buf64 sB;                                         \
    bind_tensor(G, (int)blockIdx.x, sD, sB);                     \
    const T64<P>& D = sD;                                        \
    const Buf64& Bf = sB

__device__ __forceinline__ double clampd(double v, double lo, double hi) { return fmin(fmax(v, lo), hi); }
__device__ __forceinline__ double sigmoidd(double x) { return 1.0 / (1.0 + exp(-x)); }
__device__ __forceinline__ double sgnd(double x) { return x > 0.0 ? 1.0 : (x < 0.0 ? -1.0 : 0.0); }

// Normalised carrier (cos, sin) of mode k at row r, column c; the row table
// holds rm modes per row.
template <typename P>
__device__ __forceinline__ void carrier_at(const T64<P>& D, int64_t rm, int64_t r, int64_t c, int k, double& ch,
                                           double& sh) {
    const double a1 = D.rowtab[(r * rm + k) * 2], a2 = D.rowtab[(r * rm + k) * 2 + 1];
    const double b1 = D.coltab[(int64_t)(2 * k) * D.cols + c], b2 = D.coltab[(int64_t)(2 * k + 1) * D.cols + c];
    double rc, rs;
    if (mode_is_product(k)) {
        rc = a1 * b1;
        rs = a2 * b2;
    } else {
        rc = a1 * b1 - a2 * b2;
        rs = a1 * b2 + a2 * b1;
    }
    const ModeStats& m = D.stats[k];
    ch = (rc - m.mu_c) * m.inv_c;
    sh = (rs - m.mu_s) * m.inv_s;
}

template <int RM, typename P>
__device__ __forceinline__ void carrier(const T64<P>& D, int64_t r, int64_t c, int k, double& ch, double& sh) {
    carrier_at(D, RM, r, c, k, ch, sh);
}

// Normalised carriers (cos, sin) of modes 0..RM-1 at row r, column c.
template <int RM, typename P>
__device__ __forceinline__ void carriers(const T64<P>& D, int64_t r, int64_t c, double (&ch)[RM], double (&sh)[RM]) {
#pragma unroll
    for (int k = 0; k < RM; ++k) carrier<RM>(D, r, c, k, ch[k], sh[k]);
}

// The prediction and (when echo) the echo reconstruction at row r, column c in
// one sweep over the modes, each carrier formed once: the same sums, in the
// same order, as recon() over stored carriers.
template <int RM, typename P>
__device__ __forceinline__ void recon_pred_echo(const T64<P>& D, const C64& C, int64_t r, int64_t c, bool echo,
                                                double& pred, double& ech) {
    double a = 0.0, b = 0.0;
#pragma unroll(RM > 16 ? 8 : RM)
    for (int k = 0; k < RM; ++k) {
        double chk, shk;
        carrier<RM>(D, r, c, k, chk, shk);
        a += chk * C.p_al[k];
        a += shk * C.p_be[k];
        if (echo) {
            b += chk * C.e_al[k];
            b += shk * C.e_be[k];
        }
    }
    pred = a;
    ech = echo ? b : 0.0;
}

template <int RM>
__device__ __forceinline__ double recon(const double* al, const double* be, const double (&ch)[RM],
                                        const double (&sh)[RM]) {
    double out = 0.0;
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        out += ch[k] * al[k];
        out += sh[k] * be[k];
    }
    return out;
}

// Parameter / gradient element e as float64 (every storage type converts exactly).
__device__ __forceinline__ double load_pg(const void* p, int64_t e, int dt) {
    if (dt == CRESSO_DTYPE_F64) return static_cast<const double*>(p)[e];
    return (double)load_elem(p, e, dt);
}

template <typename P>
__device__ __forceinline__ double force_of(const T64<P>& D, int64_t e) {
    double f = (D.hp[Q_MAX] != 0.0 ? -1.0 : 1.0) * load_pg(D.grad, e, D.pdt);
    if (D.hp[Q_WD] != 0.0) f = f + D.hp[Q_WD] * load_pg(D.param, e, D.pdt);
    return f;
}

template <typename P>
__device__ __forceinline__ double rel_of(const T64<P>& D, double scale, double f) {
    return fmin(fabs(f) / scale + D.hp[Q_EPS], 1.0e4);
}

template <typename P>
__device__ __forceinline__ double idens_of(const T64<P>& D, double rel) {
    const double pw = fmax(D.hp[Q_IP], 0.25);
    return fmin(pow(fmax(rel, D.hp[Q_EPS]), pw), 1.0e6);
}

// Block sum of v[0..L) into rec[0..L); every thread calls.
template <int L>
__device__ __forceinline__ void block_record(double (&v)[L], double* red, double* rec) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int j = 0; j < L; ++j) {
        const double s = warp_sum(v[j]);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < kWarps; ++w) t += red[w];
            rec[j] = t;
        }
        __syncthreads();
    }
}

// ---- Exact hash-bin sums.  A value v with |v| < 2^66 is the integer
// s = round(|v| 2^60) split into three limbs of 42 bits (high, middle, low; each
// negated for negative v), each added into the bin with a native 64-bit
// shared-memory integer atomic.  Integer sums do not depend on the order of the
// additions, and a block's limb sums (exact for up to 2^21 values per bin) turn
// into one double by a fixed formula, so the bin sums are the same in every run;
// the only rounding is that of s (at most 2^-61 per value).  Values out of that
// range, and non-finite ones, go to a float64 side sum of the bin (so that they
// still propagate as they do in the reference).
// Shared layout for tb bins: long long limbs [3][tb], then double side [tb].
__host__ __device__ constexpr size_t exact_bins_bytes(int tb) { return (size_t)tb * 4 * 8; }

__device__ __forceinline__ void exact_bins_zero(unsigned char* base, int tb) {
    long long* lim = reinterpret_cast<long long*>(base);
    double* side = reinterpret_cast<double*>(lim + 3 * tb);
    for (int i = threadIdx.x; i < 3 * tb; i += blockDim.x) lim[i] = 0;
    for (int i = threadIdx.x; i < tb; i += blockDim.x) side[i] = 0.0;
}

__device__ __forceinline__ void exact_bins_add(unsigned char* base, int tb, int b, double v) {
    unsigned long long* lim = reinterpret_cast<unsigned long long*>(base);
    const double a = fabs(v);
    if (a < 0x1p66) {
        const double sc = a * 0x1p60;                 // exact (power-of-two scaling)
        const double h = floor(sc * 0x1p-84);
        const double r1 = sc - h * 0x1p84;            // exact, in [0, 2^84)
        const double m = floor(r1 * 0x1p-42);
        const double r0 = r1 - m * 0x1p42;            // exact, in [0, 2^42)
        long long hi = (long long)h, mid = (long long)m, lo = llrint(r0);
        if (v < 0.0) {
            hi = -hi;
            mid = -mid;
            lo = -lo;
        }
        atomicAdd(&lim[b], (unsigned long long)hi);
        atomicAdd(&lim[tb + b], (unsigned long long)mid);
        atomicAdd(&lim[2 * tb + b], (unsigned long long)lo);
    } else {
        double* side = reinterpret_cast<double*>(lim + 3 * tb);
        atomicAdd(&side[b], v);
    }
}

__device__ __forceinline__ double exact_bins_value(const unsigned char* base, int tb, int b) {
    const long long* lim = reinterpret_cast<const long long*>(base);
    const double* side = reinterpret_cast<const double*>(lim + 3 * tb);
    return ((double)lim[b] * 0x1p24 + (double)lim[tb + b] * 0x1p-18 + (double)lim[2 * tb + b] * 0x1p-60) + side[b];
}

// ---- P1: force energy
template <typename P>
__global__ void __launch_bounds__(kThreads) s64_p1(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    double v[1] = {0.0};
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const double f = force_of(D, e);
        v[0] += f * f;
    }
    block_record<1>(v, red, Bf.rec + lb * 1);
}

template <typename P>
__global__ void s64_fin1(G64<P> G) {
    S64_BIND_TENSOR();
    if (threadIdx.x != 0) return;
    double s = 0.0;
    for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[b];
    const double eps = D.hp[Q_EPS];
    const double frn = sqrt(s / (double)D.N + eps);
    const double fr = reservoir((double)*D.force_rms, frn, D.hp[Q_RD], D.step);
    *D.force_rms = fr;
    Bf.cst->scale = fmax(fr, eps);
}

// ---- P2: density, bins, projections.  Record: [sum L, sum dens, sum L c_k (RM), sum L s_k (RM),
// bin sums (TB), bin counts (TB)]
template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_p2(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    extern __shared__ __align__(16) unsigned char s64_smem[];  // exact bin sums, then [TB] counts
    const int TB = D.T * D.B;
    const bool hash_on = D.hash_on != 0;
    double* cnt = reinterpret_cast<double*>(s64_smem + exact_bins_bytes(TB));
    if (hash_on) {
        exact_bins_zero(s64_smem, TB);
        for (int i = threadIdx.x; i < TB; i += kThreads) cnt[i] = 0.0;
    }
    __syncthreads();
    const double scale = Bf.cst->scale, ep = D.hp[Q_EP];
    double v[2 + 2 * RM];
#pragma unroll
    for (int j = 0; j < 2 + 2 * RM; ++j) v[j] = 0.0;
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const double rel = rel_of(D, scale, force_of(D, e));
        const double ds = pow(rel, ep);
        const double L = log1p(ds);
        v[0] += L;
        if (D.inst) v[1] += idens_of(D, rel);
        double ch[RM], sh[RM];
        carriers<RM>(D, e / D.cols, e % D.cols, ch, sh);
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            v[2 + k] += L * ch[k];
            v[2 + RM + k] += L * sh[k];
        }
        if (hash_on)
            for (int t = 0; t < D.T; ++t) {
                const int b = (int)hash_bin(e, D.B, t);
                exact_bins_add(s64_smem, TB, t * D.B + b, ds);
                atomicAdd(&cnt[t * D.B + b], 1.0);  // whole numbers: exact in any order
            }
    }
    const int RL = 2 + 2 * RM + 2 * TB;
    double* rec = Bf.rec + lb * RL;
    block_record<2 + 2 * RM>(v, red, rec);  // its barriers order the bin atomics before the reads
    if (hash_on)
        for (int i = threadIdx.x; i < TB; i += kThreads) {
            rec[2 + 2 * RM + i] = exact_bins_value(s64_smem, TB, i);
            rec[2 + 2 * RM + TB + i] = cnt[i];
        }
}

// Row sums of the instant-metric density: one warp per row (rank >= 2).
template <typename P>
__global__ void __launch_bounds__(kThreads) s64_rowsum(G64<P> G) {
    S64_BIND_BLOCKS(blk_row);
    const int lane = threadIdx.x & 31;
    const double scale = Bf.cst->scale;
    for (int64_t r = lb * kWarps + (threadIdx.x >> 5); r < D.rows; r += gb * kWarps) {
        double s = 0.0;
        for (int64_t c = lane; c < D.cols; c += 32) s += idens_of(D, rel_of(D, scale, force_of(D, r * D.cols + c)));
        s = warp_sum(s);
        if (lane == 0) Bf.rowsum[r] = s;
    }
}

// Column sums of the instant-metric density (rank >= 2), in col_chunks(rows)
// row chunks: block (chunk, tile) sums its chunk of rows for the 256 columns of
// its tile, one thread per column, into tbuf[chunk][cols] (the tangent field
// is written only later, by P3); the finalize adds the chunks in order.
__host__ __device__ inline int64_t col_chunks(int64_t rows) { return (rows + 31) / 32 < 64 ? (rows + 31) / 32 : 64; }

template <typename P>
__global__ void __launch_bounds__(kThreads) s64_colsum(G64<P> G) {
    S64_BIND_BLOCKS(blk_col);
    const double scale = Bf.cst->scale;
    const int64_t tiles = (D.cols + kThreads - 1) / kThreads, chunks = col_chunks(D.rows);
    const int64_t per = (D.rows + chunks - 1) / chunks;
    const int64_t chunk = lb / tiles, c = (lb % tiles) * kThreads + threadIdx.x;
    if (c >= D.cols) return;
    const int64_t r0 = chunk * per, r1 = r0 + per < D.rows ? r0 + per : D.rows;
    double s = 0.0;
    for (int64_t r = r0; r < r1; ++r) s += idens_of(D, rel_of(D, scale, force_of(D, r * D.cols + c)));
    Bf.tbuf[chunk * D.cols + c] = s;
}

// Hash energy reservoirs and the per-bin log metric (cresso_v5.py:995-1056)
// from the blocks' bin sums and counts: block b's sums at rec[b * L + off + i],
// its counts TB further on.  Every thread calls.
template <typename P>
__device__ void fin2_hash(const T64<P>& D, const Buf64& Bf, int64_t L, int64_t off) {
    __shared__ double emean[8];
    const int tid = threadIdx.x;
    const int TB = D.T * D.B;
    const double eps = D.hp[Q_EPS];
    for (int i = tid; i < TB; i += kThreads) {
        double s = 0.0, n = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) {
            s += Bf.rec[(int64_t)b * L + off + i];
            n += Bf.rec[(int64_t)b * L + off + TB + i];
        }
        Bf.counts[i] = n;
        const double cell = s / fmax(n, 1.0);
        D.h_energy[i] = reservoir((double)D.h_energy[i], cell, D.hp[Q_HD], D.step);
    }
    __syncthreads();
    if (tid < D.T) {
        double s = 0.0;
        for (int b = 0; b < D.B; ++b) s += D.h_energy[tid * D.B + b];
        emean[tid] = fmax(s / (double)D.B, eps);
    }
    __syncthreads();
    const double xp = D.hp[Q_HMC] / fmax(0.25, D.hp[Q_EP]);
    for (int i = tid; i < TB; i += kThreads) {
        const double hm = fmax(D.h_energy[i] / emean[i / D.B], eps);
        Bf.lterm[i] = log(fmax(clampd(pow(hm, xp), 0.08, 12.0), eps));
    }
}

// Thread 0: the density mean, the instant-metric mean and exponent.
template <typename P>
__device__ void fin2_scalars(const T64<P>& D, C64& C, double sum_l, double sum_dens) {
    const double N = (double)D.N, eps = D.hp[Q_EPS];
    C.meanL = fmax(sum_l / N, eps);
    C.gm = fmax(sum_dens / N, eps);
    const double pw = fmax(D.hp[Q_IP], 0.25);
    const double ic = D.hard ? D.hp[Q_IC] : 0.0;
    C.kk = ic / ((double)D.ndim * pw);
}

// Metric oscillator of mode k < R driven by the density projection (pc, ps)
// (cresso_v5.py:1057-1093), and the mode's log-metric and prediction
// coefficients (the prediction from the old oscillators, cresso_v5.py:1125-1129).
template <typename P>
__device__ void fin2_mode(const T64<P>& D, int k, double pc, double ps, double shrink, double& m_al, double& m_be,
                          double& p_al, double& p_be) {
    const double mdt = D.hp[Q_MDT];
    const double damp = fmax(0.0, 1.0 - mdt * D.hp[Q_MF]);
    const double om2 = D.omega[k] * D.omega[k];
    double mp = D.mp_cos[k] * damp + mdt * (pc - om2 * D.m_cos[k]);
    double mq = clampd(D.m_cos[k] + mdt * mp, -3.0, 3.0);
    D.mp_cos[k] = mp;
    D.m_cos[k] = mq;
    m_al = mq * shrink;
    mp = D.mp_sin[k] * damp + mdt * (ps - om2 * D.m_sin[k]);
    mq = clampd(D.m_sin[k] + mdt * mp, -3.0, 3.0);
    D.mp_sin[k] = mp;
    D.m_sin[k] = mq;
    m_be = mq * shrink;
    const double g = sigmoidd(D.hp[Q_CONFG] * D.conf[k]);
    p_al = D.q_cos[k] * shrink * g;
    p_be = D.q_sin[k] * shrink * g;
}

// Instant-metric factors (cresso_v5.py:243-262): logs of the axis means over the
// mean.  Every thread calls, after C.gm is set.
template <typename P>
__device__ void fin2_axes(const T64<P>& D, const Buf64& Bf, double gm) {
    __shared__ double s_lax[kMaxLeadSum64];
    const int tid = threadIdx.x;
    const double N = (double)D.N, eps = D.hp[Q_EPS];
    const int64_t chunks = col_chunks(D.rows);
    for (int64_t c = tid; c < D.cols; c += kThreads) {
        double s = 0.0;
        for (int64_t ch = 0; ch < chunks; ++ch) s += Bf.tbuf[ch * D.cols + c];
        Bf.colsum[c] = log(fmax((s / (double)D.rows) / gm, eps));
    }
    if (D.ndim == 2) {
        for (int64_t r = tid; r < D.rows; r += kThreads)
            Bf.rowsum[r] = log(fmax((Bf.rowsum[r] / (double)D.cols) / gm, eps));
        return;
    }
    // rank >= 3: per leading axis and coordinate the marginal mean (a fixed-order sum of
    // the row sums with that coordinate); a row's log factor sums its axes' logs
    const int nl = (int)D.ndim - 1;
    int lead_sum = 0;
    for (int a = 0; a < nl; ++a) lead_sum += (int)D.dims[a];
    for (int j = tid; j < lead_sum; j += kThreads) {
        int a = 0, c = j;
        while (c >= D.dims[a]) {
            c -= (int)D.dims[a];
            ++a;
        }
        int64_t inner = 1;
        for (int b = a + 1; b < nl; ++b) inner *= D.dims[b];
        const int64_t outer = D.rows / (D.dims[a] * inner);
        double m = 0.0;
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) m += Bf.rowsum[(o * D.dims[a] + c) * inner + i];
        s_lax[j] = log(fmax((m / (N / (double)D.dims[a])) / gm, eps));
    }
    __syncthreads();
    for (int64_t r = tid; r < D.rows; r += kThreads) {
        double lsum = 0.0;
        int64_t rem = r;
        int off = lead_sum;
        for (int a = nl - 1; a >= 0; --a) {
            off -= (int)D.dims[a];
            lsum += s_lax[off + (int)(rem % D.dims[a])];
            rem /= D.dims[a];
        }
        Bf.rowsum[r] = lsum;
    }
}

template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_fin2(G64<P> G) {
    S64_BIND_TENSOR();
    __shared__ double tot[2 + 2 * RM];
    const int tid = threadIdx.x;
    const int TB = D.T * D.B;
    const int L = 2 + 2 * RM + 2 * TB;
    const double N = (double)D.N;
    C64& C = *Bf.cst;
    for (int j = tid; j < 2 + 2 * RM; j += kThreads) {
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[(int64_t)b * L + j];
        tot[j] = s;
    }
    if (D.hash_on) fin2_hash(D, Bf, L, 2 + 2 * RM);
    __syncthreads();
    const double shrink = 1.0 / sqrt(fmax(1.0, 0.7 * log2((double)D.R + 1.0)));
    if (tid == 0) fin2_scalars(D, C, tot[0], tot[1]);
    __syncthreads();
    if (tid < RM) {
        const int k = tid;
        if (k < D.R) {
            const ModeStats& m = D.stats[k];
            const double pc = tot[2 + k] / N / C.meanL - m.mhat_c;
            const double ps = tot[2 + RM + k] / N / C.meanL - m.mhat_s;
            fin2_mode(D, k, pc, ps, shrink, C.m_al[k], C.m_be[k], C.p_al[k], C.p_be[k]);
        } else {
            C.m_al[k] = C.m_be[k] = C.p_al[k] = C.p_be[k] = 0.0;
        }
    }
    if (D.inst && D.ndim >= 2) {
        __syncthreads();
        fin2_axes(D, Bf, C.gm);
    }
}

// Tangent of element e (row r, column c) with force f, relative magnitude rel
// and clamped log metric lm (cresso_v5.py:1095-1123).
template <typename P>
__device__ __forceinline__ double tangent_of(const T64<P>& D, const Buf64& Bf, const C64& C, int64_t e, int64_t r,
                                             int64_t c, double f, double rel, double lm) {
    const double eps = D.hp[Q_EPS];
    const double metric = clampd(exp(D.hp[Q_MC] * lm), 0.06, 16.0);
    const double local = D.local_on ? clampd(1.0 + D.hp[Q_LS] * sqrt(fmin(rel, 100.0)), 1.0, 8.0) : 1.0;
    double inst = 1.0;
    if (D.inst) {
        const double lg = D.ndim >= 2 ? Bf.rowsum[r] + Bf.colsum[c] : log(fmax(idens_of(D, rel) / C.gm, eps));
        inst = clampd(exp(C.kk * lg), 0.08, 12.0);
    }
    double hm = 1.0;
    if (D.hash_on) {
        double lsum = 0.0;
        for (int t = 0; t < D.T; ++t) lsum += Bf.lterm[t * D.B + (int)hash_bin(e, D.B, t)];
        hm = clampd(exp(lsum / (double)D.T), 0.08, 12.0);
    }
    return clampd(f / (C.scale * metric * local * inst * hm + eps), -1.0e4, 1.0e4);
}

// ---- P3: tangent, error, projections of the port and of the tangent, port bins.
// Record: [sum err^2, sum port c_k (RM), sum port s_k (RM), sum t c_k (RM), sum t s_k (RM), port bins (TB)]
template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_p3(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    extern __shared__ __align__(16) unsigned char s64_smem[];  // exact bin sums
    const int TB = D.T * D.B;
    const bool hash_on = D.hash_on != 0;
    if (hash_on) exact_bins_zero(s64_smem, TB);
    __syncthreads();
    const C64& C = *Bf.cst;
    const double scale = C.scale, tm = D.hp[Q_TM];
    double v[1 + 4 * RM];
#pragma unroll
    for (int j = 0; j < 1 + 4 * RM; ++j) v[j] = 0.0;
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const int64_t r = e / D.cols, c = e % D.cols;
        const double f = force_of(D, e);
        const double rel = rel_of(D, scale, f);
        double ch[RM], sh[RM];
        carriers<RM>(D, r, c, ch, sh);
        const double lm = clampd(recon<RM>(C.m_al, C.m_be, ch, sh), -3.0, 3.0);
        const double t = tangent_of(D, Bf, C, e, r, c, f, rel, lm);
        Bf.tbuf[e] = t;
        const double err = t - recon<RM>(C.p_al, C.p_be, ch, sh);
        v[0] += err * err;
        const double port = err + tm * t;
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            v[1 + k] += port * ch[k];
            v[1 + RM + k] += port * sh[k];
            v[1 + 2 * RM + k] += t * ch[k];
            v[1 + 3 * RM + k] += t * sh[k];
        }
        if (hash_on)
            for (int tb = 0; tb < D.T; ++tb) exact_bins_add(s64_smem, TB, tb * D.B + (int)hash_bin(e, D.B, tb), port);
    }
    const int RL = 1 + 4 * RM + TB;
    double* rec = Bf.rec + lb * RL;
    block_record<1 + 4 * RM>(v, red, rec);
    if (hash_on)
        for (int i = threadIdx.x; i < TB; i += kThreads) rec[1 + 4 * RM + i] = exact_bins_value(s64_smem, TB, i);
}

// Hash impulse reservoirs (cresso_v5.py:1140-1184) from the blocks' port bin
// sums at rec[b * L + off + i].  Every thread calls.
template <typename P>
__device__ void fin3_hash(const T64<P>& D, const Buf64& Bf, int64_t L, int64_t off) {
    const int TB = D.T * D.B;
    const double hd = D.hp[Q_HD], hid = D.hp[Q_HID], rg = D.hp[Q_RG];
    for (int i = threadIdx.x; i < TB; i += kThreads) {
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[(int64_t)b * L + off + i];
        const double cell = s / fmax(Bf.counts[i], 1.0);
        const double href = D.h_refractory[i] * hd + (1.0 - hd) * fabs(cell);
        D.h_refractory[i] = href;
        const double hg = 1.0 / (1.0 + rg * href);
        const double himp = D.h_impulse[i] * hid + (1.0 - hid) * (cell * hg);
        D.h_impulse[i] = himp;
        Bf.impv[i] = himp;
    }
}

// Thread 0: confidence from the old oscillators (cresso_v5.py:1186-1202), then
// the contact oscillators, cos half then sin half (cresso_v5.py:914-943,
// 1204-1250), driven by the port projection (pc, ps); gp is R doubles of room.
template <typename P>
__device__ void fin3_contact(const T64<P>& D, double S, const double* pc, const double* ps, double* gp) {
    const int R = D.R;
    const double eps = D.hp[Q_EPS];
    const double cd = D.hp[Q_CD];
    for (int k = 0; k < R; ++k) {
        const double qc = D.q_cos[k], qs = D.q_sin[k];
        const double pe = sqrt(pc[k] * pc[k] + ps[k] * ps[k] + eps);
        const double support = (pc[k] * qc + ps[k] * qs) / (pe * sqrt(qc * qc + qs * qs + eps) + eps);
        D.conf[k] = clampd(D.conf[k] * cd + (1.0 - cd) * clampd(support, -1.0, 1.0), -4.0, 4.0);
    }
    const double dt = D.hp[Q_DT], rd = D.hp[Q_REFD], rg = D.hp[Q_RG];
    const double plast = 1.0 + D.hp[Q_SG] * S / (1.0 + S);
    const double brake = 1.0 / (1.0 + D.hp[Q_SB] * S);
    double action = *D.action;
    for (int half = 0; half < 2; ++half) {
        P* q = half ? D.q_sin : D.q_cos;
        P* p = half ? D.p_sin : D.p_cos;
        P* ca = half ? D.ca_sin : D.ca_cos;
        const double* port = half ? ps : pc;
        double p2 = 0.0, oq2 = 0.0, pp = 0.0;
        for (int k = 0; k < R; ++k) {
            ca[k] = ca[k] * rd + (1.0 - rd) * fabs(port[k]);
            const double rgate = 1.0 / (1.0 + rg * ca[k]);
            gp[k] = port[k] * rgate * plast * brake;
            p2 += p[k] * p[k];
            const double oq = D.omega[k] * q[k];
            oq2 += oq * oq;
            pp += gp[k] * p[k];
        }
        const double energy = 0.5 * (p2 / R + oq2 / R);
        action = action * 0.985 + dt * (pp / R - energy);
        const double fr = D.hp[Q_IF] + D.hp[Q_CG] * tanh(fabs(action));
        const double damp = fmax(1.0 - dt * fr, 0.0);
        for (int k = 0; k < R; ++k) {
            const double om2 = D.omega[k] * D.omega[k];
            p[k] = p[k] * damp + dt * (gp[k] - D.hp[Q_REST] * om2 * q[k] - D.hp[Q_CUBIC] * (q[k] * q[k] * q[k]));
            q[k] = clampd(q[k] + dt * p[k], -8.0, 8.0);
        }
    }
    *D.action = action;
}

template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_fin3(G64<P> G) {
    S64_BIND_TENSOR();
    __shared__ double tot[1 + 4 * RM];
    const int tid = threadIdx.x;
    const int TB = D.T * D.B;
    const int L = 1 + 4 * RM + TB;
    const double N = (double)D.N, eps = D.hp[Q_EPS];
    C64& C = *Bf.cst;
    for (int j = tid; j < 1 + 4 * RM; j += kThreads) {
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[(int64_t)b * L + j];
        tot[j] = s;
    }
    if (D.hash_on) fin3_hash(D, Bf, L, 1 + 4 * RM);
    __syncthreads();
    if (tid != 0) return;
    // ---- surprise (cresso_v5.py:1132-1134)
    const double S = reservoir((double)*D.surprise, sqrt(tot[0] / N + eps), D.hp[Q_SD], D.step);
    *D.surprise = S;
    C.S = S;
    const int R = D.R;
    const double shrink = 1.0 / sqrt(fmax(1.0, 0.7 * log2((double)R + 1.0)));
    double pc[kMaxRankPlain], ps[kMaxRankPlain], gp[kMaxRankPlain];
    for (int k = 0; k < R; ++k) {
        pc[k] = tot[1 + k] / N;
        ps[k] = tot[1 + RM + k] / N;
    }
    fin3_contact(D, S, pc, ps, gp);
    // ---- second prediction and echo coefficients (cresso_v5.py:1252-1258)
    for (int k = 0; k < RM; ++k) {
        if (k < R) {
            const double g = sigmoidd(D.hp[Q_CONFG] * D.conf[k]);
            C.p_al[k] = D.q_cos[k] * shrink * g;
            C.p_be[k] = D.q_sin[k] * shrink * g;
            C.e_al[k] = D.echo_on ? (tot[1 + 2 * RM + k] / N) * shrink : 0.0;
            C.e_be[k] = D.echo_on ? (tot[1 + 3 * RM + k] / N) * shrink : 0.0;
        } else {
            C.p_al[k] = C.p_be[k] = C.e_al[k] = C.e_be[k] = 0.0;
        }
    }
    C.clip = D.hp[Q_CLIP];
}

// ---- Wide rank (kMaxRankPlain < rank <= kMaxRankWide)
// The modes no longer fit registers.  Reconstructions loop over the modes with
// their coefficients in the scratch (Bf.wcoef); projections run in chunks of
// kChunkW modes, chunk y of a pass being the blocks with blockIdx.y == y, each
// block writing one record per chunk (Bf.rec2).  P3 is split: an element pass
// stores the tangent and the port, and a chunked pass projects both from the
// stored fields, so every pass costs O(rank) per element.
enum { W_MAL, W_MBE, W_PAL, W_PBE, W_EAL, W_EBE, W_PC, W_PS, W_GP, W_COUNT };
constexpr int kRec2 = 4 * kChunkW;  // doubles per (chunk, block) record

// Prediction and (when echo) echo at row r, column c from the wide coefficients.
template <typename P>
__device__ __forceinline__ void recon_pred_echo_w(const T64<P>& D, const Buf64& Bf, int64_t r, int64_t c, bool echo,
                                                  double& pred, double& ech) {
    const int RW = D.RW;
    const double* pal = Bf.wcoef + W_PAL * RW;
    const double* pbe = Bf.wcoef + W_PBE * RW;
    const double* eal = Bf.wcoef + W_EAL * RW;
    const double* ebe = Bf.wcoef + W_EBE * RW;
    double a = 0.0, b = 0.0;
    for (int k = 0; k < D.R; ++k) {
        double chk, shk;
        carrier_at(D, RW, r, c, k, chk, shk);
        a += chk * pal[k];
        a += shk * pbe[k];
        if (echo) {
            b += chk * eal[k];
            b += shk * ebe[k];
        }
    }
    pred = a;
    ech = echo ? b : 0.0;
}

// P2, chunk y = blockIdx.y: the density sums and the hash bins (chunk 0) and the
// density projection on modes [y kChunkW, (y + 1) kChunkW).  rec2 record: [sum L,
// sum dens, cos (kChunkW), sin (kChunkW)]; bin sums and counts in rec ([blocks][2 TB]).
template <typename P>
__global__ void __launch_bounds__(kThreads) s64w_p2(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    extern __shared__ __align__(16) unsigned char s64_smem[];  // exact bin sums, then [TB] counts
    const int TB = D.T * D.B;
    const int y = blockIdx.y;
    const bool bins = D.hash_on != 0 && y == 0;
    double* cnt = reinterpret_cast<double*>(s64_smem + exact_bins_bytes(TB));
    if (bins) {
        exact_bins_zero(s64_smem, TB);
        for (int i = threadIdx.x; i < TB; i += kThreads) cnt[i] = 0.0;
    }
    __syncthreads();
    const double scale = Bf.cst->scale, ep = D.hp[Q_EP];
    const int k0 = y * kChunkW;
    const int kn = min(kChunkW, D.R - k0);  // modes of this chunk below the rank
    double v[2 + 2 * kChunkW];
#pragma unroll
    for (int j = 0; j < 2 + 2 * kChunkW; ++j) v[j] = 0.0;
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const double rel = rel_of(D, scale, force_of(D, e));
        const double ds = pow(rel, ep);
        const double L = log1p(ds);
        v[0] += L;
        if (D.inst) v[1] += idens_of(D, rel);
        const int64_t r = e / D.cols, c = e % D.cols;
#pragma unroll
        for (int j = 0; j < kChunkW; ++j) {
            if (j < kn) {
                double ch, sh;
                carrier_at(D, D.RW, r, c, k0 + j, ch, sh);
                v[2 + j] += L * ch;
                v[2 + kChunkW + j] += L * sh;
            }
        }
        if (bins)
            for (int t = 0; t < D.T; ++t) {
                const int b = (int)hash_bin(e, D.B, t);
                exact_bins_add(s64_smem, TB, t * D.B + b, ds);
                atomicAdd(&cnt[t * D.B + b], 1.0);
            }
    }
    block_record<2 + 2 * kChunkW>(v, red, Bf.rec2 + ((int64_t)y * Bf.blocks + lb) * kRec2);
    if (bins)
        for (int i = threadIdx.x; i < TB; i += kThreads) {
            Bf.rec[lb * 2 * TB + i] = exact_bins_value(s64_smem, TB, i);
            Bf.rec[lb * 2 * TB + TB + i] = cnt[i];
        }
}

template <typename P>
__global__ void __launch_bounds__(kThreads) s64w_fin2(G64<P> G) {
    S64_BIND_TENSOR();
    __shared__ double tot[2];
    const int tid = threadIdx.x;
    const int TB = D.T * D.B;
    const int RW = D.RW;
    const double N = (double)D.N;
    C64& C = *Bf.cst;
    if (tid < 2) {  // chunk 0's records
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec2[(int64_t)b * kRec2 + tid];
        tot[tid] = s;
    }
    if (D.hash_on) fin2_hash(D, Bf, 2 * TB, 0);
    __syncthreads();
    const double shrink = 1.0 / sqrt(fmax(1.0, 0.7 * log2((double)D.R + 1.0)));
    if (tid == 0) fin2_scalars(D, C, tot[0], tot[1]);
    __syncthreads();
    double* w = Bf.wcoef;
    for (int k = tid; k < RW; k += kThreads) {
        if (k < D.R) {
            const int64_t y = k / kChunkW, j = k % kChunkW;
            double sc = 0.0, ss = 0.0;
            for (int b = 0; b < Bf.blocks; ++b) {
                const double* r2 = Bf.rec2 + (y * Bf.blocks + b) * kRec2;
                sc += r2[2 + j];
                ss += r2[2 + kChunkW + j];
            }
            const ModeStats& m = D.stats[k];
            fin2_mode(D, k, sc / N / C.meanL - m.mhat_c, ss / N / C.meanL - m.mhat_s, shrink, w[W_MAL * RW + k],
                      w[W_MBE * RW + k], w[W_PAL * RW + k], w[W_PBE * RW + k]);
        } else {
            w[W_MAL * RW + k] = w[W_MBE * RW + k] = w[W_PAL * RW + k] = w[W_PBE * RW + k] = 0.0;
        }
    }
    if (D.inst && D.ndim >= 2) {
        __syncthreads();
        fin2_axes(D, Bf, C.gm);
    }
}

// P3 element pass: the tangent and the port stored (tbuf, pbuf), sum err^2 and
// the port bins.  rec record: [sum err^2, port bins (TB)].
template <typename P>
__global__ void __launch_bounds__(kThreads) s64w_p3a(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    extern __shared__ __align__(16) unsigned char s64_smem[];  // exact bin sums
    const int TB = D.T * D.B;
    const bool hash_on = D.hash_on != 0;
    if (hash_on) exact_bins_zero(s64_smem, TB);
    __syncthreads();
    const C64& C = *Bf.cst;
    const double scale = C.scale, tm = D.hp[Q_TM];
    const int RW = D.RW;
    const double* mal = Bf.wcoef + W_MAL * RW;
    const double* mbe = Bf.wcoef + W_MBE * RW;
    const double* pal = Bf.wcoef + W_PAL * RW;
    const double* pbe = Bf.wcoef + W_PBE * RW;
    double v[1] = {0.0};
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const int64_t r = e / D.cols, c = e % D.cols;
        const double f = force_of(D, e);
        const double rel = rel_of(D, scale, f);
        double lm = 0.0, pr = 0.0;
        for (int k = 0; k < D.R; ++k) {
            double ch, sh;
            carrier_at(D, RW, r, c, k, ch, sh);
            lm += ch * mal[k];
            lm += sh * mbe[k];
            pr += ch * pal[k];
            pr += sh * pbe[k];
        }
        const double t = tangent_of(D, Bf, C, e, r, c, f, rel, clampd(lm, -3.0, 3.0));
        Bf.tbuf[e] = t;
        const double err = t - pr;
        v[0] += err * err;
        const double port = err + tm * t;
        Bf.pbuf[e] = port;
        if (hash_on)
            for (int tb = 0; tb < D.T; ++tb) exact_bins_add(s64_smem, TB, tb * D.B + (int)hash_bin(e, D.B, tb), port);
    }
    double* rec = Bf.rec + lb * (1 + TB);
    block_record<1>(v, red, rec);
    if (hash_on)
        for (int i = threadIdx.x; i < TB; i += kThreads) rec[1 + i] = exact_bins_value(s64_smem, TB, i);
}

// P3 projections, chunk y = blockIdx.y: the stored port and tangent on modes
// [y kChunkW, (y + 1) kChunkW).  rec2 record: [port cos, port sin, t cos, t sin]
// (kChunkW each).
template <typename P>
__global__ void __launch_bounds__(kThreads) s64w_p3b(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    const int y = blockIdx.y;
    const int k0 = y * kChunkW;
    const int kn = min(kChunkW, D.R - k0);
    double v[4 * kChunkW];
#pragma unroll
    for (int j = 0; j < 4 * kChunkW; ++j) v[j] = 0.0;
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        const int64_t r = e / D.cols, c = e % D.cols;
        const double port = Bf.pbuf[e], t = Bf.tbuf[e];
#pragma unroll
        for (int j = 0; j < kChunkW; ++j) {
            if (j < kn) {
                double ch, sh;
                carrier_at(D, D.RW, r, c, k0 + j, ch, sh);
                v[j] += port * ch;
                v[kChunkW + j] += port * sh;
                v[2 * kChunkW + j] += t * ch;
                v[3 * kChunkW + j] += t * sh;
            }
        }
    }
    block_record<4 * kChunkW>(v, red, Bf.rec2 + ((int64_t)y * Bf.blocks + lb) * kRec2);
}

template <typename P>
__global__ void __launch_bounds__(kThreads) s64w_fin3(G64<P> G) {
    S64_BIND_TENSOR();
    __shared__ double tot0;
    const int tid = threadIdx.x;
    const int TB = D.T * D.B;
    const int RW = D.RW;
    const double N = (double)D.N, eps = D.hp[Q_EPS];
    C64& C = *Bf.cst;
    double* w = Bf.wcoef;
    if (tid == 0) {
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[(int64_t)b * (1 + TB)];
        tot0 = s;
    }
    if (D.hash_on) fin3_hash(D, Bf, 1 + TB, 1);
    // per mode: the port projection (contact drive) and the tangent projection (echo)
    for (int k = tid; k < RW; k += kThreads) {
        const int64_t y = k / kChunkW, j = k % kChunkW;
        double pc = 0.0, ps = 0.0, tc = 0.0, ts = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) {
            const double* r2 = Bf.rec2 + (y * Bf.blocks + b) * kRec2;
            pc += r2[j];
            ps += r2[kChunkW + j];
            tc += r2[2 * kChunkW + j];
            ts += r2[3 * kChunkW + j];
        }
        w[W_PC * RW + k] = pc / N;
        w[W_PS * RW + k] = ps / N;
        w[W_EAL * RW + k] = tc / N;
        w[W_EBE * RW + k] = ts / N;
    }
    __syncthreads();
    if (tid == 0) {
        // ---- surprise (cresso_v5.py:1132-1134), confidence and contact oscillators
        const double S = reservoir((double)*D.surprise, sqrt(tot0 / N + eps), D.hp[Q_SD], D.step);
        *D.surprise = S;
        C.S = S;
        fin3_contact(D, S, w + W_PC * RW, w + W_PS * RW, w + W_GP * RW);
        C.clip = D.hp[Q_CLIP];
    }
    __syncthreads();
    // ---- second prediction and echo coefficients (cresso_v5.py:1252-1258)
    const double shrink = 1.0 / sqrt(fmax(1.0, 0.7 * log2((double)D.R + 1.0)));
    for (int k = tid; k < RW; k += kThreads) {
        if (k < D.R) {
            const double g = sigmoidd(D.hp[Q_CONFG] * D.conf[k]);
            w[W_PAL * RW + k] = D.q_cos[k] * shrink * g;
            w[W_PBE * RW + k] = D.q_sin[k] * shrink * g;
            w[W_EAL * RW + k] = D.echo_on ? w[W_EAL * RW + k] * shrink : 0.0;
            w[W_EBE * RW + k] = D.echo_on ? w[W_EBE * RW + k] * shrink : 0.0;
        } else {
            w[W_PAL * RW + k] = w[W_PBE * RW + k] = w[W_EAL * RW + k] = w[W_EBE * RW + k] = 0.0;
        }
    }
}

// The eight drive vectors of one element (cresso_v5.py:1303-1326):
// rational, bounded, root (before its normalisation), tangent, prediction,
// novelty, echo (raw), hash prediction (raw).
// RM == 0: wide rank (the coefficients in Bf.wcoef).
template <int RM, typename P>
__device__ __forceinline__ void drive_vectors(const T64<P>& D, const Buf64& Bf, int64_t e, double (&v)[8]) {
    const C64& C = *Bf.cst;
    const double eps = D.hp[Q_EPS], clip = C.clip;
    const double t = Bf.tbuf[e];
    double pred, echo;
    if constexpr (RM == 0)
        recon_pred_echo_w(D, Bf, e / D.cols, e % D.cols, D.echo_on != 0, pred, echo);
    else
        recon_pred_echo<RM>(D, C, e / D.cols, e % D.cols, D.echo_on != 0, pred, echo);
    v[0] = t / (1.0 + fabs(t) / clip);
    v[1] = tanh(t / clip) * clip;
    v[2] = sgnd(t) * sqrt(fmin(fabs(t), clip * clip) + eps);
    v[3] = t;
    v[4] = pred;
    v[5] = tanh((t - pred) / (clip * (1.0 + C.S))) * clip;
    v[6] = echo;
    double hp = 0.0;
    if (D.hash_on) {
        for (int t2 = 0; t2 < D.T; ++t2) hp += Bf.impv[t2 * D.B + (int)hash_bin(e, D.B, t2)];
        hp = hp / (double)D.T;
    }
    v[7] = hp;
}

__host__ __device__ constexpr int g8(int a, int b) { return a * 8 - (a * (a - 1)) / 2 + (b - a); }

template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_p4(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    __shared__ double red[kWarps];
    double g[kGram64];
#pragma unroll
    for (int j = 0; j < kGram64; ++j) g[j] = 0.0;
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        double v[8];
        drive_vectors<RM>(D, Bf, e, v);
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = a; b < 8; ++b) g[g8(a, b)] += v[a] * v[b];
    }
    block_record<kGram64>(g, red, Bf.rec + lb * kGram64);
}

// Drive coefficients from the Gram (cresso_v5.py:1303-1353).
template <typename P>
__global__ void s64_fin4(G64<P> G) {
    S64_BIND_TENSOR();
    __shared__ double Gs[kGram64];
    const int tid = threadIdx.x;
    for (int j = tid; j < kGram64; j += kThreads) {
        double s = 0.0;
        for (int b = 0; b < Bf.blocks; ++b) s += Bf.rec[(int64_t)b * kGram64 + j];
        Gs[j] = s;
    }
    __syncthreads();
    if (tid != 0) return;
    C64& C = *Bf.cst;
    const double N = (double)D.N, eps = D.hp[Q_EPS], S = C.S;
    auto Gm = [&](int a, int b) { return a <= b ? Gs[g8(a, b)] : Gs[g8(b, a)]; };
    enum { RAT, BND, ROOT, TT, PR, NOV, ECHO, HASH };
    auto rms_of = [&](const double* c8) {  // sqrt(mean((sum c_i v_i)^2) + eps)
        double s = 0.0;
        for (int i = 0; i < 8; ++i)
            for (int j = 0; j < 8; ++j) s += c8[i] * c8[j] * Gm(i, j);
        return sqrt(fmax(s, 0.0) / N + eps);
    };
    const double frms = sqrt(Gm(TT, TT) / N + eps);
    const double prms = sqrt(Gm(PR, PR) / N + eps);
    const double align = clampd((Gm(TT, PR) / N) / (frms * prms + eps), -1.0, 1.0);
    const double align_gate = prms > sqrt(eps) ? clampd((align + 1.0) * 0.5, 0.0, 1.0) : 0.0;
    const int ws = (int)D.hp[Q_WS];
    const double warm = ws == 0 ? 1.0 : (1.0 - exp(-(double)D.step / (double)(ws > 1 ? ws : 1)));
    const double mix = D.hp[Q_PM] * warm * align_gate * (1.0 / (1.0 + S));
    const double rat_rms = sqrt(Gm(RAT, RAT) / N + eps);
    const double k_root = rat_rms / fmax(sqrt(Gm(ROOT, ROOT) / N + eps), eps);
    const double spike = D.hp[Q_SPIKE] / (1.0 + S);
    const double root_mix = (D.hard ? D.hp[Q_RCM] : 0.0) / (1.0 + 0.5 * S);
    double shaped[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    shaped[RAT] = (1.0 - root_mix) * (1.0 - spike);
    shaped[BND] = (1.0 - root_mix) * spike;
    shaped[ROOT] = root_mix * k_root;
    const double shaped_rms = rms_of(shaped);
    const double dm = D.hp[Q_DFM] / (1.0 + 0.35 * S);
    double core[8];
    for (int i = 0; i < 8; ++i) core[i] = (1.0 - dm) * shaped[i];
    core[TT] += dm * (shaped_rms / fmax(frms, eps));
    const double core_rms = rms_of(core);
    const double resm = D.hp[Q_RFM] / (1.0 + S);
    const double err_rms = sqrt(fmax(Gm(TT, TT) - 2.0 * Gm(TT, PR) + Gm(PR, PR), 0.0) / N + eps);
    const double k_res = core_rms / fmax(err_rms, eps);
    double c[8];
    for (int i = 0; i < 8; ++i) c[i] = (1.0 - mix) * core[i];
    c[PR] += mix;
    c[NOV] += D.hp[Q_NM];
    c[TT] += resm * k_res;
    c[PR] -= resm * k_res;
    if (D.hard && D.echo_on) {
        const double k_e = shaped_rms / fmax(sqrt(Gm(ECHO, ECHO) / N + eps), eps);
        c[ECHO] += D.hp[Q_EM] * k_e;
    }
    if (D.hard && D.hash_on) {
        const double k_h = shaped_rms / fmax(sqrt(Gm(HASH, HASH) / N + eps), eps);
        c[HASH] += D.hp[Q_HDM] * k_h;
    }
    double d2 = 0.0;
    for (int i = 0; i < 8; ++i)
        for (int j = 0; j < 8; ++j) d2 += c[i] * c[j] * Gm(i, j);
    const double DE = reservoir((double)*D.drive_energy, fmax(d2, 0.0) / N, D.hp[Q_RD], D.step);
    *D.drive_energy = DE;
    C.gain = clampd(D.hp[Q_TGT] / sqrt(DE + eps), D.hp[Q_MING], D.hp[Q_MAXG]);
    for (int i = 0; i < 8; ++i) C.c[i] = c[i];
}

template <int RM, typename P>
__global__ void __launch_bounds__(kThreads) s64_p5(G64<P> G) {
    S64_BIND_BLOCKS(blk);
    const C64& C = *Bf.cst;
    const double neg_lr = -D.hp[Q_LR], gain = C.gain;
    const float neg_lr16 = neg_lr_in(D.hp[Q_LR], D.pdt);
    for (int64_t e = lb * kThreads + threadIdx.x; e < D.N; e += gb * kThreads) {
        double v[8];
        drive_vectors<RM>(D, Bf, e, v);
        double drive = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) drive += C.c[i] * v[i];
        if (D.pdt == CRESSO_DTYPE_F64) {
            double* p = static_cast<double*>(D.param);
            p[e] = p[e] + neg_lr * (drive * gain);
        } else if (D.pdt == CRESSO_DTYPE_F32) {
            float* p = static_cast<float*>(D.param);
            p[e] = (float)((double)p[e] + neg_lr * (drive * gain));
        } else {
            // 16-bit: the update rounded to the parameter type, then param.add_(u, alpha=-lr)
            apply_update(D.param, e, D.pdt, 0.0f, neg_lr16, (float)(drive * gain));
        }
    }
}

// Both storage types have the same layout (every pointer the same size), so the
// plan keeps T64<double> and the tensors of a float32-state group are uploaded
// as T64<float> records (the same bytes).
static_assert(sizeof(T64<float>) == sizeof(T64<double>), "T64 layout");

// Tensors are launched in groups: consecutive tensors of one state type whose
// scratch (tables, block records, bin and axis buffers, the tangent field)
// stays within kGroupBytes64; a larger tensor forms a group of its own.  The
// groups run one after another and reuse the same scratch.
constexpr int64_t kGroupBytes64 = 1LL << 30;
constexpr int kGroupTensors64 = 4096;

struct Item64 {
    int blocks, rblocks, cblocks;  // element passes, row sums, column sums
    int64_t L;                     // doubles per block record
    int64_t bytes;                 // scratch of this tensor
};
struct Group64 {
    int first, count;
    bool f32;
    int64_t bytes;
};
struct Plan64 {
    std::vector<T64<double>> ts;
    std::vector<Item64> items;
    std::vector<Group64> groups;
    int64_t bytes;
};

int64_t tensor_scratch64(const T64<double>& T, const Item64& it) {
    const int64_t TB = std::max<int64_t>((int64_t)T.T * T.B, 1);
    int64_t b = align_up((int64_t)sizeof(C64), 256);
    b += align_up(8 * it.L * it.blocks, 256);
    b += 3 * align_up(8 * TB, 256);
    b += align_up(8 * T.rows, 256) + align_up(8 * T.cols, 256);
    b += align_up(8 * T.N, 256);
    if (T.RW > kMaxRankPlain) {  // wcoef, pbuf, rec2
        b += align_up(8 * (int64_t)W_COUNT * T.RW, 256);
        b += align_up(8 * T.N, 256);
        b += align_up(8 * (int64_t)(T.RW / kChunkW) * it.blocks * kRec2, 256);
    }
    return b;
}

int64_t group_tables64(int n) {
    return align_up((int64_t)sizeof(T64<double>) * n, 256) + align_up((int64_t)sizeof(Buf64) * n, 256) +
           align_up(3 * 4 * (int64_t)(n + 1), 256);
}

int plan64(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, Plan64& P) {
    CRESSO_REQUIRE(descs != nullptr && hp != nullptr && n >= 1, CRESSO_EINVAL, "spectral64: need tensors and hparams");
    const int64_t rank = (int64_t)hp->rank, bins = (int64_t)hp->hash_bins, tables = (int64_t)hp->hash_tables;
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRankWide, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA spectral path (got %lld)", kMaxRankWide, (long long)rank);
    CRESSO_REQUIRE(bins >= 0 && tables >= 1, CRESSO_EINVAL, "hash_bins must be >= 0, hash_tables >= 1");
    CRESSO_REQUIRE(bins * tables <= kMaxTB64, CRESSO_EUNSUPPORTED,
                   "hash_bins * hash_tables must be <= %d for float64 parameters", kMaxTB64);
    const int rm = rank_pad(rank);
    P.ts.assign(n, T64<double>{});
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        CRESSO_REQUIRE(d.dtype == CRESSO_DTYPE_F64 || ((d.dtype == CRESSO_DTYPE_F32 || d.dtype == CRESSO_DTYPE_F16 ||
                                                         d.dtype == CRESSO_DTYPE_BF16) &&
                                                        rank > kMaxRank),
                       CRESSO_EINVAL,
                       "tensor %lld: spectral64 takes float64 tensors, and float32 / float16 / bfloat16 tensors "
                       "when rank > %d",
                       (long long)i, kMaxRank);
        CRESSO_REQUIRE(d.ndim >= 1 && d.ndim <= CRESSO_MAX_NDIM, CRESSO_EUNSUPPORTED,
                       "tensor %lld: spectral route supports tensors of rank 1 to %d", (long long)i, CRESSO_MAX_NDIM);
        int64_t rows = 1, lead_sum = 0;
        for (int64_t a = 0; a < d.ndim; ++a)
            CRESSO_REQUIRE(d.shape[a] >= 1, CRESSO_EINVAL, "tensor %lld: empty dimension", (long long)i);
        for (int64_t a = 0; a + 1 < d.ndim; ++a) {
            rows *= d.shape[a];
            lead_sum += d.shape[a];
        }
        const int64_t cols = d.shape[d.ndim - 1];
        CRESSO_REQUIRE(d.row0 == 0 && d.col0 == 0 && d.rows == rows && d.cols == cols, CRESSO_EUNSUPPORTED,
                       "tensor %lld: float64 tensors are not sharded", (long long)i);
        CRESSO_REQUIRE(rows * cols < (1LL << 40), CRESSO_EUNSUPPORTED, "tensor %lld: too many elements", (long long)i);
        CRESSO_REQUIRE(d.ndim <= 2 || lead_sum <= kMaxLeadSum64, CRESSO_EUNSUPPORTED,
                       "tensor %lld: leading axes sum to %lld (at most %d)", (long long)i, (long long)lead_sum,
                       kMaxLeadSum64);
        CRESSO_REQUIRE(d.step >= 1, CRESSO_EINVAL, "tensor %lld: step must be >= 1", (long long)i);
        CRESSO_REQUIRE(d.param && d.grad && d.shape_ws && d.omega && d.q_cos && d.q_sin && d.p_cos && d.p_sin &&
                           d.metric_cos && d.metric_sin && d.metric_p_cos && d.metric_p_sin && d.calcium_cos &&
                           d.calcium_sin && d.mode_confidence && d.force_rms && d.drive_energy && d.surprise && d.action,
                       CRESSO_EINVAL, "tensor %lld: NULL param / grad / workspace / state pointer", (long long)i);
        T64<double>& T = P.ts[i];
        T.ndim = d.ndim;
        T.rows = rows;
        T.cols = cols;
        T.N = rows * cols;
        T.step = d.step;
        for (int64_t a = 0; a < CRESSO_MAX_NDIM; ++a) T.dims[a] = a < d.ndim ? d.shape[a] : 0;
        T.param = (void*)d.param;
        T.grad = (const void*)d.grad;
        T.pdt = (int32_t)d.dtype;
        T.f32 = d.dtype != CRESSO_DTYPE_F64;  // state storage: float (see as_f32) unless float64
        const ShapeWsHeader wh = shape_ws64_layout(d.ndim, rows, cols, rank, rm);
        const char* ws = (const char*)d.shape_ws;
        T.rowtab = (const double*)(ws + wh.off_rowtab);
        T.coltab = (const double*)(ws + wh.off_coltab);
        T.stats = (const ModeStats*)(ws + wh.off_stats);
        T.omega = (double*)d.omega;
        T.q_cos = (double*)d.q_cos;
        T.q_sin = (double*)d.q_sin;
        T.p_cos = (double*)d.p_cos;
        T.p_sin = (double*)d.p_sin;
        T.m_cos = (double*)d.metric_cos;
        T.m_sin = (double*)d.metric_sin;
        T.mp_cos = (double*)d.metric_p_cos;
        T.mp_sin = (double*)d.metric_p_sin;
        T.ca_cos = (double*)d.calcium_cos;
        T.ca_sin = (double*)d.calcium_sin;
        T.conf = (double*)d.mode_confidence;
        T.h_energy = (double*)d.hash_energy;
        T.h_impulse = (double*)d.hash_impulse;
        T.h_refractory = (double*)d.hash_refractory;
        T.force_rms = (double*)d.force_rms;
        T.drive_energy = (double*)d.drive_energy;
        T.surprise = (double*)d.surprise;
        T.action = (double*)d.action;
        T.R = (int32_t)rank;
        T.RW = (int32_t)rm;
        T.T = (int32_t)tables;
        T.B = (int32_t)bins;
        // hard channel: numel >= hard_channel_min_size and not a thin 2-D matrix (cresso_v5.py:983-989)
        const int64_t cutoff = (int64_t)hp->thin_matrix_hard_cutoff;
        const bool thin = d.ndim == 2 && cutoff > 0 && std::min(d.shape[0], d.shape[1]) <= cutoff;
        const bool hard = T.N >= (int64_t)hp->hard_channel_min_size && !thin;
        T.hard = hard;
        T.hash_on = hard && bins > 0 && d.hash_energy && d.hash_impulse && d.hash_refractory;
        if (!T.hash_on) T.T = 1, T.B = 0;
        T.echo_on = hard && hp->echo_mix != 0.0;
        T.inst = hard && hp->instant_metric_coupling != 0.0 && T.N > 1;
        T.local_on = hp->local_sharpness != 0.0;
        memcpy(T.hp, hp, sizeof(cresso_hparams));
    }
    int dev = 0, sms = 148;
    CRESSO_CUDA(cudaGetDevice(&dev));
    CRESSO_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    P.items.assign(n, Item64{});
    P.groups.clear();
    P.bytes = 0;
    for (int64_t i = 0; i < n; ++i) {
        const T64<double>& T = P.ts[i];
        Item64& it = P.items[i];
        it.blocks = (int)std::max<int64_t>(
            1, std::min<int64_t>(std::min<int64_t>(ceil_div(T.N, kThreads * 4), kMaxBlocks64), 2 * sms));
        const bool axes = T.inst && T.ndim >= 2;
        it.rblocks = axes ? (int)std::min<int64_t>(ceil_div(T.rows, kWarps), 4096) : 0;
        it.cblocks = axes ? (int)(ceil_div(T.cols, kThreads) * col_chunks(T.rows)) : 0;
        const int64_t TBi = (int64_t)T.T * T.B;
        if (rm > kMaxRankPlain)  // wide rank: the projections go to rec2
            it.L = std::max<int64_t>(std::max<int64_t>(2 * TBi, 1 + TBi), kGram64);
        else
            it.L = std::max<int64_t>(std::max<int64_t>(2 + 2 * rm + 2 * TBi, 1 + 4 * rm + TBi), kGram64);
        it.bytes = tensor_scratch64(T, it);
        const bool f32 = T.f32 != 0;
        if (P.groups.empty() || P.groups.back().f32 != f32 || P.groups.back().count == kGroupTensors64 ||
            group_tables64(P.groups.back().count + 1) + P.groups.back().bytes + it.bytes > kGroupBytes64)
            P.groups.push_back(Group64{(int)i, 0, f32, 0});
        Group64& g = P.groups.back();
        ++g.count;
        g.bytes += it.bytes;  // the tensors' scratch; the tables are added below
    }
    for (const Group64& g : P.groups) P.bytes = std::max(P.bytes, group_tables64(g.count) + g.bytes);
    return CRESSO_OK;
}

// Dynamic shared memory beyond the default 48 KB needs the kernel's opt-in.
template <typename K>
cudaError_t set_smem(K* kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// One group: its tables uploaded to the front of the scratch, then every pass
// as one launch over the blocks of all its tensors and every finalize as one
// launch of a block per tensor.
template <int RM, typename P>
int run_group(const Plan64& PL, const Group64& Gr, char* base, cudaStream_t s) {
    const int n = Gr.count;
    std::vector<T64<P>> ts(n);
    std::vector<Buf64> bufs(n);
    std::vector<int> blk(3 * (n + 1));
    T64<P>* d_ts = reinterpret_cast<T64<P>*>(base);
    int64_t off = align_up((int64_t)sizeof(T64<P>) * n, 256);
    Buf64* d_bufs = reinterpret_cast<Buf64*>(base + off);
    off += align_up((int64_t)sizeof(Buf64) * n, 256);
    int* d_blk = reinterpret_cast<int*>(base + off);
    off += align_up(3 * 4 * (int64_t)(n + 1), 256);
    int g = 0, gr = 0, gc = 0;
    bool any_axes = false;
    size_t smem2 = 0, smem3 = 0;
    for (int j = 0; j < n; ++j) {
        const int i = Gr.first + j;
        const T64<double>& T = PL.ts[i];
        const Item64& it = PL.items[i];
        memcpy(&ts[j], &T, sizeof(T64<P>));
        const int64_t TB = std::max<int64_t>((int64_t)T.T * T.B, 1);
        char* q = base + off;
        Buf64& bf = bufs[j];
        bf.cst = reinterpret_cast<C64*>(q);
        q += align_up((int64_t)sizeof(C64), 256);
        bf.rec = reinterpret_cast<double*>(q);
        q += align_up(8 * it.L * it.blocks, 256);
        bf.lterm = reinterpret_cast<double*>(q);
        q += align_up(8 * TB, 256);
        bf.impv = reinterpret_cast<double*>(q);
        q += align_up(8 * TB, 256);
        bf.counts = reinterpret_cast<double*>(q);
        q += align_up(8 * TB, 256);
        bf.rowsum = reinterpret_cast<double*>(q);
        q += align_up(8 * T.rows, 256);
        bf.colsum = reinterpret_cast<double*>(q);
        q += align_up(8 * T.cols, 256);
        bf.tbuf = reinterpret_cast<double*>(q);
        q += align_up(8 * T.N, 256);
        bf.wcoef = bf.pbuf = bf.rec2 = nullptr;
        if (T.RW > kMaxRankPlain) {
            bf.wcoef = reinterpret_cast<double*>(q);
            q += align_up(8 * (int64_t)W_COUNT * T.RW, 256);
            bf.pbuf = reinterpret_cast<double*>(q);
            q += align_up(8 * T.N, 256);
            bf.rec2 = reinterpret_cast<double*>(q);
            q += align_up(8 * (int64_t)(T.RW / kChunkW) * it.blocks * kRec2, 256);
        }
        bf.blocks = it.blocks;
        off += it.bytes;
        blk[j] = g;
        blk[n + 1 + j] = gr;
        blk[2 * (n + 1) + j] = gc;
        g += it.blocks;
        gr += it.rblocks;
        gc += it.cblocks;
        if (T.hash_on) {
            smem2 = std::max(smem2, exact_bins_bytes(T.T * T.B) + (size_t)T.T * T.B * 8);
            smem3 = std::max(smem3, exact_bins_bytes(T.T * T.B));
        }
        any_axes = any_axes || it.rblocks > 0;
    }
    blk[n] = g;
    blk[2 * n + 1] = gr;
    blk[3 * n + 2] = gc;
    // pageable sources: each copy returns once its bytes are staged, so the vectors may go
    CRESSO_CUDA(cudaMemcpyAsync(d_ts, ts.data(), sizeof(T64<P>) * n, cudaMemcpyHostToDevice, s));
    CRESSO_CUDA(cudaMemcpyAsync(d_bufs, bufs.data(), sizeof(Buf64) * n, cudaMemcpyHostToDevice, s));
    CRESSO_CUDA(cudaMemcpyAsync(d_blk, blk.data(), sizeof(int) * blk.size(), cudaMemcpyHostToDevice, s));
    const G64<P> G{d_ts, d_bufs, d_blk, d_blk + (n + 1), d_blk + 2 * (n + 1), n};
    {
        NvtxRange r("cresso64 P1 force energy");
        s64_p1<P><<<g, kThreads, 0, s>>>(G);
        CRESSO_LAUNCHED("s64_p1");
        s64_fin1<P><<<n, 32, 0, s>>>(G);
        CRESSO_LAUNCHED("s64_fin1");
    }
    const unsigned chunks = RM == 0 ? (unsigned)(PL.ts[Gr.first].RW / kChunkW) : 1u;  // one rank per group
    {
        NvtxRange r("cresso64 P2 density / bins / projection");
        if constexpr (RM == 0) {
            CRESSO_CUDA(set_smem(s64w_p2<P>, smem2));
            s64w_p2<P><<<dim3(g, chunks), kThreads, smem2, s>>>(G);
            CRESSO_LAUNCHED("s64w_p2");
        } else {
            CRESSO_CUDA(set_smem(s64_p2<RM, P>, smem2));
            s64_p2<RM, P><<<g, kThreads, smem2, s>>>(G);
            CRESSO_LAUNCHED("s64_p2");
        }
        if (any_axes) {
            s64_rowsum<P><<<gr, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64_rowsum");
            s64_colsum<P><<<gc, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64_colsum");
        }
        if constexpr (RM == 0) {
            s64w_fin2<P><<<n, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64w_fin2");
        } else {
            s64_fin2<RM, P><<<n, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64_fin2");
        }
    }
    {
        NvtxRange r("cresso64 P3 tangent / port");
        if constexpr (RM == 0) {
            CRESSO_CUDA(set_smem(s64w_p3a<P>, smem3));
            s64w_p3a<P><<<g, kThreads, smem3, s>>>(G);
            CRESSO_LAUNCHED("s64w_p3a");
            s64w_p3b<P><<<dim3(g, chunks), kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64w_p3b");
            s64w_fin3<P><<<n, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64w_fin3");
        } else {
            CRESSO_CUDA(set_smem(s64_p3<RM, P>, smem3));
            s64_p3<RM, P><<<g, kThreads, smem3, s>>>(G);
            CRESSO_LAUNCHED("s64_p3");
            s64_fin3<RM, P><<<n, kThreads, 0, s>>>(G);
            CRESSO_LAUNCHED("s64_fin3");
        }
    }
    {
        NvtxRange r("cresso64 P4 drive Gram / P5 update");
        s64_p4<RM, P><<<g, kThreads, 0, s>>>(G);
        CRESSO_LAUNCHED("s64_p4");
        s64_fin4<P><<<n, kThreads, 0, s>>>(G);
        CRESSO_LAUNCHED("s64_fin4");
        s64_p5<RM, P><<<g, kThreads, 0, s>>>(G);
        CRESSO_LAUNCHED("s64_p5");
    }
    return CRESSO_OK;
}

}  // namespace

}  // namespace cresso

using namespace cresso;

extern "C" {

int cresso_spectral64_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                    int64_t* bytes) {
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "spectral64_scratch_bytes: NULL output");
    Plan64 P;
    int st = plan64(descs, n, hp, P);
    if (st) return st;
    *bytes = P.bytes;
    return CRESSO_OK;
}

int cresso_spectral64_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                          int64_t scratch_bytes, cresso_stream_t stream) {
    Plan64 P;
    int st = plan64(descs, n, hp, P);
    if (st) return st;
    CRESSO_REQUIRE(scratch != nullptr, CRESSO_EINVAL, "spectral64_run: NULL scratch");
    CRESSO_REQUIRE(scratch_bytes >= P.bytes, CRESSO_ESCRATCH, "spectral64_run: scratch of %lld bytes, need %lld",
                   (long long)scratch_bytes, (long long)P.bytes);
    NvtxRange range("cresso_spectral64_run %lld tensors", (long long)n);
    char* base = (char*)scratch;
    cudaStream_t s = (cudaStream_t)stream;
    const int rm = rank_pad((int64_t)hp->rank);
    // groups one after another on the stream: each reuses the same scratch
    for (const Group64& G : P.groups) {
        if (G.f32) {
            switch (rm) {
                case 4: st = run_group<4, float>(P, G, base, s); break;
                case 8: st = run_group<8, float>(P, G, base, s); break;
                case 16: st = run_group<16, float>(P, G, base, s); break;
                case 32: st = run_group<32, float>(P, G, base, s); break;
                case 64: st = run_group<64, float>(P, G, base, s); break;
                default: st = run_group<0, float>(P, G, base, s); break;  // wide rank
            }
        } else {
            switch (rm) {
                case 4: st = run_group<4, double>(P, G, base, s); break;
                case 8: st = run_group<8, double>(P, G, base, s); break;
                case 16: st = run_group<16, double>(P, G, base, s); break;
                case 32: st = run_group<32, double>(P, G, base, s); break;
                case 64: st = run_group<64, double>(P, G, base, s); break;
                default: st = run_group<0, double>(P, G, base, s); break;  // wide rank
            }
        }
        if (st) return st;
    }
    return CRESSO_OK;
}

}  // extern "C"
