// Fused CRESSO5 spectral-route step for a group of tensors.
//
// The reference step (cresso_v5.py:945-1353) is a chain of dense field ops
// separated by global reductions.  Here it runs as five streaming passes over
// each tensor, every pass a single grouped launch for all tensors:
//
//   P1  f = g (+wd p)                     -> sum f^2                    (force_rms)
//   P2  rel, rel^p, log1p, axis density   -> hash bin sums, projection of log1p,
//                                            row / column sums of the density
//   P3  metric, instant and hash metrics  -> tangent t (stored), prediction error,
//                                            projection of t, hash bin sums of the port
//   P4  t, new prediction, echo, shapes   -> Gram of the drive components
//   P5  t, drive                          -> p -= lr * gain * drive
//
// After each of P1..P4 a reduce kernel sums the per-block records of every
// tensor in a fixed order into a float64 "reduction vector" (the only data a
// row-sharded run all-reduces across GPUs), and a finalize kernel (one block
// per tensor) updates the persistent rank / hash / scalar state and writes
// the per-tensor constants the next pass needs.  No host synchronisation.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "basis_dev.cuh"
#include "cresso_common.cuh"
#include "cresso_status.h"
#include "tcgen05.cuh"

namespace cresso {

constexpr int kStages = 14;  // see launch_stage
constexpr int kNSRec = 36;  // float64 scalars per block record (>= 2 + 2 * kMaxRank, >= 29)
constexpr int kGram = 29;   // 28 pair sums of (u, root, t, pred, nov, echo, hp) + sum rat^2
constexpr int kMaxLeadSum = 4096;  // sum of the leading axis lengths of an N-d tensor with the instant metric

enum : int32_t {
    F_MAXIMIZE = 1,
    F_WD = 2,
    F_HARD = 4,
    F_HASH = 8,
    F_LOCAL = 16,
    F_ECHO = 32,
    F_INST2D = 64,
    F_INST1D = 128,
    F_IPOW1 = 256,  // instant_metric_power == 1 (density = rel)
    F_VEC = 512,    // rows 16-byte aligned: streaming tiles are staged with cp.async
    F_F16 = 1024,   // float16 parameter and gradient (float32 copies in the scratch)
    F_BF16 = 2048,  // bfloat16 parameter and gradient (float32 copies in the scratch)
};

struct TensorConsts {
    float scale, inv_scale;
    float m_al[kMaxRank], m_be[kMaxRank], m_K;     // metric field reconstruction (inv folded)
    float p0_al[kMaxRank], p0_be[kMaxRank], p0_K;  // prediction from the old oscillators
    float pr_al[kMaxRank], pr_be[kMaxRank], pr_K;  // prediction from the new oscillators
    float ec_al[kMaxRank], ec_be[kMaxRank], ec_K;  // echo = reconstruction of proj(t)
    float cb_al[kMaxRank], cb_be[kMaxRank], cb_K;  // c_pred * pred + c_echo * echo
    float inst_k, inst_gm;
    float S, sp, invD, clip, inv_clip, clip2;
    float c_u, c_root, c_t, c_nov, c_hp, gain, neg_lr;
    float pad[3];
    double pv[2 * kMaxRank];  // old prediction coefficients on the normalised carriers
};

// The tensors of a group fall in three launch classes: class 0 ("full") holds
// the float32 tensors whose every item is a full, 16-byte aligned 256-column
// tile with 8-bit bin indices; class 2 the 16-bit tensors of that form; class
// 1 the rest.  Each pass runs one launch per non-empty class over that class's
// item list; only P5 differs between classes 0 and 2.
struct GroupHdr {
    int64_t n_tensors, n_items, rm, bins, tables, tb, iters, idx_bytes, rb_max;
    int32_t* status;                  // device word, OR of failure bits (1: a bounded wait gave up,
                                      // 2: products still in flight when the block freed its TMEM)
    int64_t cls_items[3], cls_nt[3];  // items and tensors of each class
    int64_t grid[3][6];               // blocks of pass 1..5 per class (index 0 unused)
    double hp[64];                    // cresso_hparams
};

struct DevTensor {
    int64_t rows, cols, row0, col0, gcols, N;
    int64_t dims[CRESSO_MAX_NDIM];  // global shape (rank >= 3: leading-axis factors of the instant metric)
    int64_t item_base, n_items, step, hidx_n;  // item_base: first item in the class's item list
    int32_t ndim, R, TC, RPI, RB, n_ct, n_bands, flags;
    int32_t cfirst[6], recbase[6], nrec[6];
    // 1: the pass-2 column sums of the lean kernel, one float64 per (block record,
    // column) summed over the bands of the block's run of that column tile; 0: one
    // float per (row band, column)
    int32_t col_runs;
    float* param;   // float32 parameter (the caller's, or the scratch copy of a 16-bit one)
    const float* grad;  // float32 gradient (the caller's, or the scratch copy in tbuf)
    float* tbuf;
    void* param_h;  // the caller's 16-bit parameter and gradient (F_F16 / F_BF16)
    const void* grad_h;
    const float* rowtab;
    const float* coltab;
    const ModeStats* stats;
    const double* gram;
    const float* counts;
    const void* hidx;
    float *omega, *q_cos, *q_sin, *p_cos, *p_sin, *m_cos, *m_sin, *mp_cos, *mp_sin, *ca_cos, *ca_sin, *conf;
    float *h_energy, *h_impulse, *h_refractory, *force_rms, *drive_energy, *surprise, *action;
    TensorConsts* cst;
    float* htab;
    float* rowf;
    float* colf;
    float* rowpart;
    float* colpart;
    double* red[5];  // slices of reduction vectors 1..4 (index 0 unused)
};

// hparams indices (field order of cresso_hparams)
enum HP {
    H_LR, H_WD, H_EP, H_DT, H_IF, H_CG, H_REST, H_CUBIC, H_MDT, H_MF, H_MC, H_LS, H_IC, H_IP, H_RCM, H_EM, H_TM,
    H_HD, H_HID, H_HMC, H_HDM, H_DFM, H_RFM, H_RD, H_REFD, H_RG, H_CD, H_CONFG, H_SG, H_SD, H_PM, H_NM, H_WS, H_SB,
    H_TGT, H_MING, H_MAXG, H_CLIP, H_SPIKE, H_EPS, H_MAX, H_RANK, H_MAXF, H_BINS, H_TABLES, H_HARDMIN, H_THINCUT,
    H_MD, H_MID, H_MDM, H_COUNT
};
static_assert(sizeof(cresso_hparams) == H_COUNT * sizeof(double), "cresso_hparams field order");

__device__ __forceinline__ int gram_idx(int a, int b) { return a * 7 - (a * (a - 1)) / 2 + (b - a); }

__device__ __forceinline__ int find_tensor(const int64_t* __restrict__ item_base, int n, int64_t item) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (item_base[mid] <= item) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int load_bin(const void* hidx, int idx_bytes, int64_t stride, int t, int64_t gflat) {
    if (idx_bytes == 1) return __ldg(reinterpret_cast<const uint8_t*>(hidx) + t * stride + gflat);
    return __ldg(reinterpret_cast<const uint16_t*>(hidx) + t * stride + gflat);
}

__device__ __forceinline__ float sgnf(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }

// Per-element drive components shared by P4 and P5 (cresso_v5.py:1315-1326).
struct DriveK {
    float clip, inv_clip, clip2, sp, invD, eps;
};
struct DriveParts {
    float u, root, nov, rat;
};
__device__ __forceinline__ DriveParts drive_parts(float t, float pred, const DriveK& c) {
    DriveParts d;
    const float at = fabsf(t);
    d.rat = __fdividef(t, 1.0f + at * c.inv_clip);  // denominator in [1, 1 + 1e4 / clip]
    const float bnd = tanhf(t * c.inv_clip) * c.clip;
    d.root = sgnf(t) * sqrt_sfu(fminf(at, c.clip2) + c.eps);
    d.u = (1.0f - c.sp) * d.rat + c.sp * bnd;
    d.nov = tanhf((t - pred) * c.invD) * c.clip;
    return d;
}

// Sum of each of v[0..3] over aligned groups of `w` lanes (w a power of two,
// 4 <= w <= 32) in 1.5 shuffles per value: after the call, lane l of a group
// holds the sum of v[2 * ((l & (w/2)) != 0) + ((l & (w/4)) != 0)].
__device__ __forceinline__ float group_sum4(const float (&v)[4], int w) {
    const int lane = threadIdx.x & 31;
    const int o1 = w >> 1, o2 = w >> 2;
    const bool hi1 = (lane & o1) != 0;
    const float s0 = hi1 ? v[0] : v[2], s1 = hi1 ? v[1] : v[3];
    const float k0 = hi1 ? v[2] : v[0], k1 = hi1 ? v[3] : v[1];
    const float w0 = k0 + __shfl_xor_sync(0xffffffffu, s0, o1);
    const float w1 = k1 + __shfl_xor_sync(0xffffffffu, s1, o1);
    const bool hi2 = (lane & o2) != 0;
    float x = (hi2 ? w1 : w0) + __shfl_xor_sync(0xffffffffu, hi2 ? w0 : w1, o2);
    for (int o = w >> 3; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// ---------------------------------------------------------------------------
// Pass kernel
//
// Thread mapping: a block processes "items" of one tensor: TC columns x RB
// rows (TC = min(256, next_pow2(cols)), RB = RPI * ITERS, RPI = 256 / TC).
// Thread (lc, rs) owns column ct * TC + lc and rows rs, rs + RPI, ... of the
// item, so per-column carrier factors stay in registers and per-row factors
// are warp-uniform.  Blocks walk a contiguous range of the group's item list
// (a static persistent schedule) and emit one record of partial sums per
// tensor they touch.
//
// Staging: for tensors whose rows are 16-byte aligned (cols, col0 and the
// global row length multiples of 16) the streaming tiles of an item -- the
// gradient or tangent, the parameter when needed, the hash-bin bytes of the
// first two tables and the item's rows of the carrier row table -- are copied
// into shared memory with cp.async 16-byte copies, double buffered: the copies
// of item i+1 are in flight while item i computes out of shared memory.  Other
// tensors read the same tiles straight from global memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Sum over the 32 lanes of a warp of each of v[0..31], by a transposing
// butterfly (31 shuffles in all): on return lane l holds the sum of v[l].
// v is used as scratch.
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool hi = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; ++i) {
            const float send = hi ? v[i] : v[i + s];
            const float keep = hi ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return v[0];
}

template <int PASS, int RM>
struct PassCfg {
    // float64 block-state sums in shared memory: the projection contractions of
    // P2 / P3 per thread, the drive Gram of P4 per warp (one entry per lane)
    static constexpr int kAccDoubles = PASS == 4 ? kWarps * 32 : (PASS == 2 || PASS == 3 ? 2 * RM * kThreads : 0);
    static constexpr int kMinBlocks = RM > 8 ? 1 : 2;
    static constexpr int kUnroll = PASS == 3 ? 2 : 4;  // rows computed together
    static constexpr bool kP = PASS == 5;              // parameter tile always staged
};

// Hash-bin sums of P2 (density) and P3 (port) in shared memory.
//
// Values are added as int32 fixed point (value * 2^S, rounded to nearest) with
// native shared-memory integer atomics, into `bin_copies` copies of the bins
// (thread tid adds into copy tid % copies; copies padded by one word so that
// they sit in different banks).  After every item the copies are emptied into
// an exact int64 per-bin block sum, so the count of values one copy's bin can
// take between flushes is at most (threads / copies) * ITERS = 2^lg_cnt.  The
// scale S = max(16, 26 - lg_cnt) and the bound |value| < V = 2^(30 - lg_cnt - S)
// keep every copy below 2^30 + 2^lg_cnt < 2^31; values at or above V (and
// non-finite ones) go to a float32 per-bin sum with float atomics instead.
// The fixed-point part is exact and order independent; its rounding error is
// at most 2^-(S+1) per value.
__host__ __device__ inline int bin_copies(int tb) {
    int c = 4096 / (tb + 1);  // 16 KB of int32 copies
    c = c < 1 ? 1 : (c > 16 ? 16 : c);
    while (c & (c - 1)) c &= c - 1;  // power of two
    return c;
}
struct BinFix {
    int s;        // scale exponent S
    float scale;  // 2^S
    float vmax;   // values with |v| < vmax take the fixed-point path
};
__host__ __device__ inline BinFix bin_fix(int copies, int iters) {
    int lg = 0;
    while ((1 << lg) < (kThreads / copies) * iters) ++lg;
    const int S = 26 - lg > 16 ? 26 - lg : 16;
    BinFix f;
    f.s = S;
    f.scale = (float)(1 << (S - 16)) * 65536.0f;
    f.vmax = (float)(1 << (30 - lg - S));
    return f;
}

// Shared-memory bytes of one staging buffer of an item.
__host__ __device__ inline int stage_bytes(int iters, int rm, int tables2, int idx_bytes, bool with_p, int rb_max) {
    const int tile = 256 * iters;
    int b = tile * 4;  // gradient or tangent
    if (with_p) b += tile * 4;
    b += tables2 * tile * idx_bytes;
    b += rb_max * 2 * rm * 4;  // the item's rows of the row table
    return (int)align_up(b, 16);
}

// Column factors of both reconstructions for global column gc, as tf32 hi / lo
// splits into TMEM: reconstruction j at columns taddr + 64 j (hi) and + 16 (lo),
// slots (K_j, 0, U_1, V_1, ..., U_7, V_7) (mode 0 is the carrier (1, 0), so its
// slot pair carries the constant term).  Not inlined: it runs once per column
// tile, and keeping it out of the item loop keeps that loop free of spills.
template <int RM>
__device__ __noinline__ void tc_column_factors(const float* __restrict__ coltab, int64_t gcols, int64_t gc,
                                               const float* __restrict__ s_coef, uint32_t taddr) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        float b1[RM], b2[RM];
        load_col<RM>(coltab, gcols, gc, b1, b2);
        float U[RM], V[RM];
        make_uv<RM>(b1, b2, s_coef + 2 * j * RM, s_coef + (2 * j + 1) * RM, U, V);
        U[0] = s_coef[4 * RM + j];
        V[0] = 0.0f;
        float w[2 * RM];
#pragma unroll
        for (int q = 0; q < RM; ++q) {
            w[2 * q] = tf32_rna(U[q]);
            w[2 * q + 1] = tf32_rna(V[q]);
        }
        tc_st16(taddr + 64 * j, w);
#pragma unroll
        for (int q = 0; q < RM; ++q) {
            w[2 * q] = tf32_rna(U[q] - tf32_rna(U[q]));
            w[2 * q + 1] = tf32_rna(V[q] - tf32_rna(V[q]));
        }
        tc_st16(taddr + 64 * j + 16, w);
        tc_wait_st();
    }
}

// TMEM columns of a block of the tensor-core kernels (two blocks per SM at most):
// A operands [0, 128), two D buffers [128, 256).
constexpr uint32_t kTcCols = 256;
constexpr uint64_t kTcWaitNs = 1000000000ull;  // bound of one MMA wait (1 s)

// TCR ("tensor-core reconstruction"): the two per-element reconstructions of P3
// (metric, prediction), P4 (prediction, echo) and P5 (prediction, drive
// combination) of a class-0 item (256 columns x 16 rows, rank pad 8) are one
// 3xTF32 tcgen05 product each,
// D[col][row] = sum_k A[col][k] B[row][k] with A the column factors
// (K, 0, U_1, V_1, ..., U_7, V_7) in TMEM and B the 16 carrier rows
// (a1_k, a2_k) in shared memory; hi / lo tf32 splits of both operands give
// A_hi B_hi + A_hi B_lo + A_lo B_hi, float32-level accuracy.  The products of
// item i+1 are issued at the start of item i into the other D buffer, so the
// tensor core runs under the CUDA-core work of the item.
template <int PASS, int RM, int NT, bool FULL, bool TCR, bool H16 = false>
__global__ void __launch_bounds__(kThreads, PassCfg<PASS, RM>::kMinBlocks)
spectral_pass_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts,
                     const int64_t* __restrict__ item_lists, const int32_t* __restrict__ tensor_lists,
                     double* __restrict__ rec_scal, float* __restrict__ rec_bins, int cls) {
    static_assert(!TCR || (FULL && RM == 8 && PASS >= 3), "tensor-core reconstruction: class 0, rank pad 8, P3-P5");
    constexpr int NACC = PassCfg<PASS, RM>::kAccDoubles;
    // rows computed together; P3 keeps two on the CUDA-core form (register budget)
    constexpr int UNR = (TCR && PASS == 3) ? 4 : PassCfg<PASS, RM>::kUnroll;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // group constants, once per block
    // this launch's class: its item list (prefix sums over its tensors) and tensor indices
    // (item_lists / tensor_lists point at this class's lists; H16: P5 of class 2)
    static_assert(!H16 || (FULL && PASS == 5), "16-bit kernel form: class-2 P5 only");
    const int64_t n_items = hdr->cls_items[cls];
    const int nt = (int)hdr->cls_nt[cls];
    const int64_t* __restrict__ item_base = item_lists;
    const int32_t* __restrict__ tmap = tensor_lists;
    const int TB = (int)hdr->tb, B = (int)hdr->bins;
    const int T = NT > 0 ? NT : (int)hdr->tables;  // hash tables (compile-time 1 or 2 on the fast path)
    const int T2 = T < 2 ? T : 2;                    // tables whose bin bytes are staged
    const int ITERS = TCR ? 16 : (int)hdr->iters;  // the host launches TCR kernels only when iters == 16
    const bool idx8 = FULL || hdr->idx_bytes == 1;
    const int ib = idx8 ? 1 : 2;
    const bool stage_p_any = PassCfg<PASS, RM>::kP || (PASS <= 3 && hdr->hp[H_WD] != 0.0);
    const float eps = (float)hdr->hp[H_EPS];
    const float wd = (float)hdr->hp[H_WD];
    const float ep = (float)hdr->hp[H_EP];
    const float ipw = fmaxf((float)hdr->hp[H_IP], 0.25f);
    const float mcpl = (float)hdr->hp[H_MC];
    const float lsh = (float)hdr->hp[H_LS];
    const float tmix = (float)hdr->hp[H_TM];
    const float invT = 1.0f / (float)T;
    const int64_t it0 = (int64_t)blockIdx.x * n_items / gridDim.x;
    const int64_t it1 = ((int64_t)blockIdx.x + 1) * n_items / gridDim.x;

    // shared memory carve-up
    constexpr bool kBins = PASS == 2 || PASS == 3;
    constexpr bool kTab = PASS >= 3;
    // hash-bin sums: int32 fixed-point copies, int64 block sums, float32 sums of the large values
    const int ncopies = kBins ? bin_copies(TB) : 1;
    const int cstride = TB + 1;
    const BinFix fix = bin_fix(ncopies, ITERS);
    const int tile = 256 * ITERS;
    const int sbytes = stage_bytes(ITERS, RM, PASS >= 2 ? T2 : 0, ib, stage_p_any, (int)hdr->rb_max);
    unsigned char* s_stage = smem_raw;                                        // 2 * sbytes
    double* s_red = reinterpret_cast<double*>(smem_raw + 2 * sbytes);         // kNSRec * kWarps
    double* s_tot = s_red + kNSRec * kWarps;                                  // kNSRec
    double* s_acc = s_tot + kNSRec;                                           // NACC
    float* s_coef = reinterpret_cast<float*>(s_acc + NACC);                   // 4 * RM + 4
    long long* s_lbin = reinterpret_cast<long long*>(s_coef + 4 * RM + 4);   // TB (kBins)
    float* s_fbin = reinterpret_cast<float*>(s_lbin + (kBins ? TB : 0));      // TB (kBins)
    int* s_ibin = reinterpret_cast<int*>(s_fbin + (kBins ? TB : 0));          // ncopies * (TB + 1) (kBins)
    float* s_tab = reinterpret_cast<float*>(s_ibin + (kBins ? ncopies * cstride : 0));  // TB
    float* s_rowred = s_tab + (kTab ? TB : 0);                                // 8 * ITERS
    float* s_colred = s_rowred + (PASS == 2 ? 8 * ITERS : 0);                 // kThreads
    // TCR: B tiles [buffer][hi, lo] (128-byte aligned), the MMA mbarrier, TMEM base, wait flag
    unsigned char* s_tcb = nullptr;
    uint64_t* s_tcbar = nullptr;
    uint32_t* s_tcslot = nullptr;
    int* s_tcflag = nullptr;
    uint32_t tc_base = 0, tc_parity = 0;
    bool tc_abort = false;
    if constexpr (TCR) {
        const uint32_t raw = smem_u32(smem_raw);
        const uint32_t end = smem_u32(s_colred + (PASS == 2 ? kThreads : 0));
        s_tcb = smem_raw + (((end + 127u) & ~127u) - raw);
        s_tcbar = reinterpret_cast<uint64_t*>(s_tcb + 4 * kTcTileBytes);
        s_tcslot = reinterpret_cast<uint32_t*>(s_tcbar + 1);
        s_tcflag = reinterpret_cast<int*>(s_tcslot + 1);
        if (warp == 0) tc_alloc(s_tcslot, kTcCols);
        if (tid == 0) mbar_init(s_tcbar, 4);  // one arrival per issuing thread
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tc_base = *s_tcslot;
    }

    int k = find_tensor(item_base, nt, it0);
    int64_t it = it0;
    while (it < it1) {
        // ---- tensor descriptor and constants into registers
        const DevTensor* __restrict__ Dp = dts + tmap[k];
        const int64_t rows = Dp->rows, cols = Dp->cols, row0 = Dp->row0, col0 = Dp->col0, gcols = Dp->gcols;
        const int64_t ibase = item_base[k], hidx_n = Dp->hidx_n;
        const int64_t seg_end = min(it1, item_base[k + 1]);
        const int flags = Dp->flags;
        // class 0: 256-column tiles (one thread per column, RPI = 1), no partial tiles
        const int TC = FULL ? 256 : Dp->TC, RPI = FULL ? 1 : Dp->RPI, RB = FULL ? ITERS : Dp->RB;
        const int n_bands = Dp->n_bands;
        const int rows32 = (int)rows, cols32 = (int)cols, row032 = (int)row0, gcols32 = (int)gcols;
        const bool hash_on = (flags & F_HASH) != 0;
        const bool vec = FULL || (flags & F_VEC) != 0;
        const bool wd_on = (flags & F_WD) != 0;
        // 16-bit parameter: compile-time in class 0 / 2 (H16), run-time in class 1
        const bool half16 = FULL ? H16 : (flags & (F_F16 | F_BF16)) != 0;
        const bool stage_p = PassCfg<PASS, RM>::kP || (PASS <= 3 && wd_on);
        // P5 of a 16-bit tensor stages its parameter in that type (16-byte chunks of 8
        // elements; aligned tensors) or widened to float32 (the per-element path)
        const bool stage_p16 = PASS == 5 && half16;
        const float* __restrict__ grad = Dp->grad;
        float* __restrict__ param = Dp->param;
        float* __restrict__ tbuf = Dp->tbuf;
        const float* __restrict__ rowtab = Dp->rowtab;
        const float* __restrict__ coltab = Dp->coltab;
        const unsigned char* __restrict__ hidx = reinterpret_cast<const unsigned char*>(Dp->hidx);
        const float* __restrict__ rowf = Dp->rowf;
        const float* __restrict__ xsrc = PASS <= 3 ? grad : tbuf;
        const TensorConsts* __restrict__ Cp = Dp->cst;
        const float sgn = (flags & F_MAXIMIZE) ? -1.0f : 1.0f;
        float scale = 0.f, inv_scale = 0.f, inst_k = 0.f, inst_gm = 1.f;
        DriveK dk{};
        float c_u = 0.f, c_root = 0.f, c_t = 0.f, c_nov = 0.f, c_hp = 0.f, gain = 0.f, neg_lr = 0.f;
        float neg_lr16 = 0.f;
        if constexpr (PASS >= 2 && PASS <= 3) {
            scale = Cp->scale;
            inv_scale = Cp->inv_scale;
            inst_k = Cp->inst_k;
            inst_gm = Cp->inst_gm;
        }
        if constexpr (PASS >= 4) {
            dk = DriveK{Cp->clip, Cp->inv_clip, Cp->clip2, Cp->sp, Cp->invD, eps};
        }
        if constexpr (PASS == 5) {
            c_u = Cp->c_u;
            c_root = Cp->c_root;
            c_t = Cp->c_t;
            c_nov = Cp->c_nov;
            c_hp = Cp->c_hp;
            gain = Cp->gain;
            neg_lr = Cp->neg_lr;
            // -lr in the parameter's 16-bit type (rounded once from double), as
            // param.add_(update.to(param.dtype), alpha=-lr) converts alpha
            if constexpr (!FULL || H16) {
                if (flags & F_BF16)
                    neg_lr16 = __bfloat162float(__double2bfloat16(-hdr->hp[H_LR]));
                else if (flags & F_F16)
                    neg_lr16 = __half2float(__double2half(-hdr->hp[H_LR]));
            }
        }
        // reconstruction coefficients of this pass into shared memory
        if constexpr (PASS >= 3) {
            const float* al1 = PASS == 3 ? Cp->m_al : Cp->pr_al;
            const float* be1 = PASS == 3 ? Cp->m_be : Cp->pr_be;
            const float* al2 = PASS == 3 ? Cp->p0_al : (PASS == 4 ? Cp->ec_al : Cp->cb_al);
            const float* be2 = PASS == 3 ? Cp->p0_be : (PASS == 4 ? Cp->ec_be : Cp->cb_be);
            if (tid < RM) {
                s_coef[tid] = al1[tid];
                s_coef[RM + tid] = be1[tid];
                s_coef[2 * RM + tid] = al2[tid];
                s_coef[3 * RM + tid] = be2[tid];
            }
            if (tid == 0) {
                s_coef[4 * RM] = PASS == 3 ? Cp->m_K : Cp->pr_K;
                s_coef[4 * RM + 1] = PASS == 3 ? Cp->p0_K : (PASS == 4 ? Cp->ec_K : Cp->cb_K);
            }
        }
        if constexpr (kBins) {
            for (int b = tid; b < ncopies * cstride; b += kThreads) s_ibin[b] = 0;
            for (int b = tid; b < TB; b += kThreads) {
                s_lbin[b] = 0;
                s_fbin[b] = 0.0f;
            }
        }
        if constexpr (kTab) {
            if (hash_on) {
                const float* src = Dp->htab;
                for (int b = tid; b < TB; b += kThreads) s_tab[b] = src[b];
            }
        }
        if constexpr (NACC > 0) {
            for (int j = tid; j < NACC; j += kThreads) s_acc[j] = 0.0;
        }
        __syncthreads();
        int* my_bins = s_ibin + (tid & (ncopies - 1)) * cstride;
        const float K1 = kTab ? s_coef[4 * RM] : 0.f, K2 = kTab ? s_coef[4 * RM + 1] : 0.f;
        double acc0 = 0.0, acc1 = 0.0;
        const int lc = tid & (TC - 1), rs = tid / TC;
        const int wseg = min(TC, 32);

        // stage layout inside one buffer: x tile, p tile, bin tiles, row-table rows
        const int off_p = tile * 4;
        const int off_b = off_p + (stage_p_any ? tile * 4 : 0);
        const int off_r = off_b + (PASS >= 2 ? T2 * tile * ib : 0);
        const int lg_tc = 31 - __clz(TC);
        const int lg_cpr = lg_tc - 2;                  // log2 of 16-byte chunks per tile row (floats)
        const int lg_cprb = lg_tc + (ib == 2) - 4;     // same for the bin bytes
        const int lg_rbcprb = 31 - __clz(RB) + lg_cprb;
        const int lg_rm2 = 31 - __clz(RM) - 1;         // 16-byte chunks per row-table row = RM / 2
        // Copies the tiles of item (ct, band) into buffer `buf`: cp.async 16-byte
        // copies for aligned tensors, per-element loads for the others.
        auto stage_item = [&](int ct, int band, int buf) {
            unsigned char* sb = s_stage + buf * sbytes;
            const int rb = band * RB;
            const int cb = ct * TC;
            if (vec) {
                for (int c = tid; c < (RB << lg_cpr); c += kThreads) {
                    const int lr = c >> lg_cpr, cc = c & ((1 << lg_cpr) - 1);
                    const int r = rb + lr, col = cb + 4 * cc;
                    const bool ok = FULL || (r < rows32 && col < cols32);
                    const int64_t e = ok ? (int64_t)r * cols32 + col : 0;
                    cp_async16(sb + (lr * TC + 4 * cc) * 4, xsrc + e, ok ? 16 : 0);
                    if (stage_p && !stage_p16) cp_async16(sb + off_p + (lr * TC + 4 * cc) * 4, param + e, ok ? 16 : 0);
                }
                if (stage_p16) {
                    const int lg_cph = lg_tc - 3;  // 16-byte chunks of 8 elements per tile row
                    for (int c = tid; c < (RB << lg_cph); c += kThreads) {
                        const int lr = c >> lg_cph, cc = c & ((1 << lg_cph) - 1);
                        const int r = rb + lr, col = cb + 8 * cc;
                        const bool ok = FULL || (r < rows32 && col < cols32);
                        const int64_t e = ok ? (int64_t)r * cols32 + col : 0;
                        cp_async16(sb + off_p + (lr * TC + 8 * cc) * 2,
                                   reinterpret_cast<const unsigned char*>(Dp->param_h) + 2 * e, ok ? 16 : 0);
                    }
                }
                if (PASS >= 2 && hash_on) {
                    for (int c = tid; c < (T2 << lg_rbcprb); c += kThreads) {
                        const int t = c >> lg_rbcprb;
                        const int c2 = c & ((1 << lg_rbcprb) - 1);
                        const int lr = c2 >> lg_cprb, cc = c2 & ((1 << lg_cprb) - 1);
                        const int r = rb + lr;
                        const bool ok = FULL || (r < rows32 && cb + (cc << (4 - (ib == 2))) < cols32);
                        const int64_t g = ok ? ((int64_t)(row032 + r) * gcols32 + col0 + cb) * ib + 16 * cc : 0;
                        cp_async16(sb + off_b + (t * tile + lr * TC) * ib + 16 * cc, hidx + t * hidx_n * ib + g,
                                   ok ? 16 : 0);
                    }
                }
                if (PASS >= 2) {
                    for (int c = tid; c < (RB << lg_rm2); c += kThreads) {
                        const bool ok = FULL || rb + (c >> lg_rm2) < rows32;
                        const int64_t g = ok ? (int64_t)(row032 + rb) * 2 * RM + 4 * c : 0;
                        cp_async16(sb + off_r + 16 * c, rowtab + g, ok ? 16 : 0);
                    }
                }
                cp_async_commit();
            } else {
                const int col = cb + lc;
                for (int m = 0; m < ITERS; ++m) {
                    const int lr = rs + RPI * m, r = rb + lr;
                    const bool ok = r < rows32 && col < cols32;
                    const int64_t e = (int64_t)r * cols32 + col;
                    const int o = lr * TC + lc;
                    reinterpret_cast<float*>(sb)[o] = ok ? xsrc[e] : 0.0f;
                    if (stage_p) {
                        float pv = 0.0f;
                        if (ok) {
                            if (!stage_p16)
                                pv = param[e];
                            else if (flags & F_BF16)
                                pv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(Dp->param_h)[e]);
                            else
                                pv = __half2float(reinterpret_cast<const __half*>(Dp->param_h)[e]);
                        }
                        reinterpret_cast<float*>(sb + off_p)[o] = pv;
                    }
                    if (PASS >= 2 && hash_on) {
                        const int64_t g = ((int64_t)(row032 + r) * gcols32 + col0 + col);
                        for (int t = 0; t < T2; ++t) {
                            if (idx8)
                                sb[off_b + t * tile + o] = ok ? hidx[t * hidx_n + g] : 0;
                            else
                                reinterpret_cast<uint16_t*>(sb + off_b)[t * tile + o] =
                                    ok ? reinterpret_cast<const uint16_t*>(hidx)[t * hidx_n + g] : 0;
                        }
                    }
                }
            }
        };

        float g32[PASS == 4 ? kGram : 1];
#pragma unroll
        for (int q = 0; q < (PASS == 4 ? kGram : 1); ++q) g32[q] = 0.0f;
        int buf = 0;
        int ct = (int)((it - ibase) / n_bands);
        int band = (int)((it - ibase) - (int64_t)ct * n_bands);
        if (vec && it < seg_end) stage_item(ct, band, 0);
        int items_since_flush = 0;
        // Per-column state carried across the items of one column tile (items are
        // column-tile major, so a block walks down the bands of a tile): the
        // reconstruction factors of the column, and the float32 projection
        // partials, contracted into the float64 block state every 4 items and
        // whenever the tile changes.
        float U1[RM], V1[RM], U2[RM], V2[RM];
        float colf = 1.0f;
        int uv_ct = -1;
        int tcb = 0;    // TCR: D and B buffer of the current item
        int a_ct = -1;  // TCR: column tile whose factors are in TMEM
        const int tc_h = tid >> 7;                               // TCR: column half = M tile
        const uint32_t tc_lane = (uint32_t)(tid & 96) << 16;     // TCR: this warp's TMEM lane quarter
        // TCR helpers: the column factors of tile c into TMEM (A, both reconstructions, hi
        // and lo); the 16 carrier rows of band bnd into B buffer bb; the products of one
        // item into D buffer bb (one thread) and their commit to the mbarrier.
        auto tc_build_a = [&](int c) {
            if constexpr (TCR) tc_column_factors<RM>(coltab, gcols, col0 + (int64_t)c * 256 + lc, s_coef, tc_base + tc_lane + 32 * tc_h);
        };
        // this thread's value of the carrier rows of band bnd (row tid / 16, slot tid % 16)
        auto tc_load_b = [&](int bnd) -> float {
            if constexpr (TCR) return __ldg(rowtab + ((int64_t)row032 + bnd * 16 + (tid >> 4)) * 16 + (tid & 15));
            return 0.0f;
        };
        auto tc_store_b = [&](float v, int bb) {
            if constexpr (TCR) {
                const float hi = tf32_rna(v);
                unsigned char* tb = s_tcb + bb * 2 * kTcTileBytes;
                const int o = tc_kmajor_off(tid >> 4, tid & 15);
                *reinterpret_cast<float*>(tb + o) = hi;
                *reinterpret_cast<float*>(tb + kTcTileBytes + o) = tf32_rna(v - hi);
            }
        };
        // issued by the four threads tid % 64 == 0 (warps 0, 2, 4, 6), one reconstruction j and
        // one column half each, so no single warp carries all 24 products of an item
        auto tc_issue = [&](int bb) {
            if constexpr (TCR) {
                tc_fence_after();
                const int j = (tid >> 6) & 1, hh = tid >> 7;
                const uint32_t bhi = smem_u32(s_tcb + bb * 2 * kTcTileBytes), blo = bhi + kTcTileBytes;
                constexpr uint32_t idesc = tc_idesc_tf32(128, 16);
                const uint32_t d = tc_base + 128 + 64 * bb + 32 * j + 16 * hh;
                const uint32_t ahi = tc_base + 16 * (4 * j + 2 * hh), alo = ahi + 16;
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const uint32_t bo = 2 * kTcLBO * ks;
                    tc_mma_tf32_ts(d, ahi + 8 * ks, tc_smem_desc(bhi + bo), idesc, ks > 0);
                    tc_mma_tf32_ts(d, ahi + 8 * ks, tc_smem_desc(blo + bo), idesc, 1);
                    tc_mma_tf32_ts(d, alo + 8 * ks, tc_smem_desc(bhi + bo), idesc, 1);
                }
                tc_commit(smem_u32(s_tcbar));
            }
        };
        // TCR pipeline: the products of item i + 1 are issued at the start of item i and run
        // under its CUDA-core work; the carrier rows of item i + 2 are fetched into a register
        // at the start of item i and stored as B operand at its end.
        float tc_bnext = 0.0f;
        if constexpr (TCR) {  // segment prologue: B of the first two items, the first item's products
            tc_build_a(ct);
            a_ct = ct;
            tc_store_b(tc_load_b(band), 0);
            if (it + 1 < seg_end) tc_store_b(tc_load_b(band + 1 == n_bands ? 0 : band + 1), 1);
            tc_fence_smem();
            tc_fence_before();
            __syncthreads();
            if ((tid & 63) == 0) tc_issue(0);
        }
        // projection partials (a1_q, a2_q) x field, summed over this thread's rows; packed
        // pairs for the two-lane fp32 FMA of sm_100 (each lane rounds as fmaf)
        float2 z12[RM];
        float zc = 0.0f;
#pragma unroll
        for (int q = 0; q < RM; ++q) z12[q] = make_float2(0.0f, 0.0f);
        for (; it < seg_end; ++it) {
            const int col = ct * TC + lc;
            const bool cvalid = FULL || col < cols32;
            const int gc = (int)col0 + (cvalid ? col : 0);
            const int rbase = band * RB;
            const int nband = band + 1 == n_bands ? 0 : band + 1;
            const int nct = band + 1 == n_bands ? ct + 1 : ct;
            if (vec) {
                if (it + 1 < seg_end) {
                    stage_item(nct, nband, buf ^ 1);
                    cp_async_wait<1>();
                } else {
                    cp_async_wait<0>();
                }
            } else {
                stage_item(ct, band, buf);
            }
            if constexpr (TCR) {
                // this item's products were issued one item earlier (or in the segment prologue)
                if (tid == 0) *s_tcflag = mbar_wait_bounded(smem_u32(s_tcbar), tc_parity, kTcWaitNs) ? 0 : 1;
                tc_parity ^= 1;
            }
            __syncthreads();
            // tiles of this item in shared memory (row table: staged, or global for unaligned tensors)
            const unsigned char* sb = s_stage + buf * sbytes;
            const float* xb = reinterpret_cast<const float*>(sb);
            const float* pb = reinterpret_cast<const float*>(sb + off_p);
            const unsigned char* bb = sb + off_b;
            const float* rtb = vec ? reinterpret_cast<const float*>(sb + off_r)
                                   : rowtab + (int64_t)(row032 + rbase) * 2 * RM;

            if constexpr (PASS >= 3) {
                if (ct != uv_ct) {
                    uv_ct = ct;
                    if constexpr (!TCR) {
                        float b1[RM], b2[RM];
                        load_col<RM>(coltab, gcols, gc, b1, b2);
                        make_uv<RM>(b1, b2, s_coef, s_coef + RM, U1, V1);
                        make_uv<RM>(b1, b2, s_coef + 2 * RM, s_coef + 3 * RM, U2, V2);
                    }
                    if constexpr (PASS == 3) {
                        if (flags & F_INST2D) colf = Dp->colf[cvalid ? col : 0];
                    }
                }
            }
            // TCR: this item's two reconstructions are in D buffer tcb (read per row group below)
            if constexpr (TCR) {
                if (*s_tcflag) {  // a product never completed: stop this block (uniform after the barrier)
                    if (tid == 0) atomicOr(hdr->status, 1);
                    tc_abort = true;
                    break;
                }
                tc_fence_after();
                if (it + 1 < seg_end) {
                    if (nct != a_ct) {  // the next item starts a new column tile (block-uniform)
                        tc_build_a(nct);
                        a_ct = nct;
                        tc_fence_before();
                        __syncthreads();
                    }
                    if ((tid & 63) == 0) tc_issue(tcb ^ 1);
                }
                if (it + 2 < seg_end) tc_bnext = tc_load_b(nband + 1 == n_bands ? 0 : nband + 1);
            }
            float s0 = 0.0f, s1 = 0.0f, colacc = 0.0f;

            for (int m0 = 0; m0 < ITERS; m0 += UNR) {
                float dv[UNR];
                // TCR: rows m0 .. m0 + UNR - 1 of both reconstructions for this thread's column
                float R1[TCR ? UNR : 1], R2[TCR ? UNR : 1];
                if constexpr (TCR) {
                    const uint32_t ta = tc_base + tc_lane + 128 + 64 * tcb + 16 * tc_h + m0;
                    tc_ld<UNR>(ta, R1);
                    tc_ld<UNR>(ta + 32, R2);
                    tc_wait_ld();
                }
#pragma unroll
                for (int u = 0; u < UNR; ++u) {
                    dv[u] = 0.0f;
                    const int lr = rs + RPI * (m0 + u);
                    const int r = rbase + lr;
                    if (!FULL && !(cvalid && r < rows32)) continue;
                    const int o = lr * TC + lc;  // offset inside the item tiles
                    const float xval = xb[o];
                    auto bin_of = [&](int t) -> int {
                        if (NT > 0 || t < 2) {
                            return idx8 ? (int)bb[t * tile + o] : (int)reinterpret_cast<const uint16_t*>(bb)[t * tile + o];
                        }
                        const int64_t g = ((int64_t)(row032 + r) * gcols32 + gc) * ib + t * hidx_n * ib;
                        return idx8 ? (int)__ldg(hidx + g) : (int)__ldg(reinterpret_cast<const uint16_t*>(hidx + g));
                    };
                    if constexpr (PASS == 1) {
                        float f = sgn * xval;
                        if (wd_on) f = f + wd * pb[o];
                        s0 = fmaf(f, f, s0);
                    } else if constexpr (PASS == 2) {
                        float f = sgn * xval;
                        if (wd_on) f = f + wd * pb[o];
                        float a1[RM], a2[RM];
                        load_row<RM>(rtb, lr, a1, a2);
                        const float rel = fminf(fabsf(f) * inv_scale + eps, 1.0e4f);
                        const float ds = exp2f(ep * __log2f(rel));  // rel >= eps > 0 (normal)
                        // log1p(ds) - 1/2: the density is centred before the float32 partial sums
                        // (the constant is added back exactly in the finalize)
                        const float L = log1p_pos(ds);
                        const float Lc = L - 0.5f;
                        const float d = (flags & F_IPOW1) ? rel : fminf(powf(fmaxf(rel, eps), ipw), 1.0e6f);
                        dv[u] = d;
                        s0 += L;
                        s1 += d;
                        colacc += d;
                        const float2 Lc2 = make_float2(Lc, Lc);
#pragma unroll
                        for (int q = 1; q < RM; ++q) z12[q] = __ffma2_rn(make_float2(a1[q], a2[q]), Lc2, z12[q]);
                        zc += Lc;
                        if (hash_on) {
                            // fixed-point path for every value (zero for the large ones), one
                            // rarely taken branch for the float path of the large values
                            const bool fx = ds < fix.vmax;
                            const int qv = fx ? __float2int_rn(ds * fix.scale) : 0;
#pragma unroll
                            for (int t = 0; t < (NT > 0 ? NT : T); ++t) atomicAdd(&my_bins[t * B + bin_of(t)], qv);
                            if (!fx) {
                                for (int t = 0; t < (NT > 0 ? NT : T); ++t) atomicAdd(&s_fbin[t * B + bin_of(t)], ds);
                            }
                        }
                    } else if constexpr (PASS == 3) {
                        float f = sgn * xval;
                        if (wd_on) f = f + wd * pb[o];
                        float a1[RM], a2[RM];
                        load_row<RM>(rtb, lr, a1, a2);
                        const float rel = fminf(fabsf(f) * inv_scale + eps, 1.0e4f);
                        float lm_raw;
                        if constexpr (TCR) lm_raw = R1[u]; else lm_raw = recon_dot_nz<RM>(K1, a1, a2, U1, V1);
                        const float lm = clampf(lm_raw, -3.0f, 3.0f);
                        const float metric = clampf(__expf(mcpl * lm), 0.06f, 16.0f);  // |mcpl * lm| <= 3 mcpl
                        float den = scale * metric;
                        if (flags & F_LOCAL) den = den * clampf(1.0f + lsh * sqrt_sfu(fminf(rel, 100.0f)), 1.0f, 8.0f);
                        if (flags & F_INST2D) {
                            den = den * clampf(rowf[r] * colf, 0.08f, 12.0f);
                        } else if (!FULL && (flags & F_INST1D)) {  // 1-D tensors are never in class 0
                            const float dd = (flags & F_IPOW1) ? rel : fminf(powf(fmaxf(rel, eps), ipw), 1.0e6f);
                            den = den * clampf(expf(inst_k * logf(fmaxf(dd / inst_gm, eps))), 0.08f, 12.0f);
                        }
                        int bi[NT > 0 ? NT : 2];
                        if (hash_on) {
                            // hash metric exp(mean_t log m_t) = prod_t m_t^(1/T), roots tabulated per bin
                            float hm = 1.0f;
#pragma unroll
                            for (int t = 0; t < (NT > 0 ? NT : T); ++t) {
                                const int bt = bin_of(t);
                                if (NT > 0 || t < 2) bi[NT > 0 ? t : (t & 1)] = bt;
                                hm *= s_tab[t * B + bt];
                            }
                            den = den * clampf(hm, 0.08f, 12.0f);
                        }
                        const float t = clampf(__fdividef(f, den + eps), -1.0e4f, 1.0e4f);
                        tbuf[(int64_t)r * cols32 + col] = t;
                        float pred;
                        if constexpr (TCR) pred = R2[u]; else pred = recon_dot_nz<RM>(K2, a1, a2, U2, V2);
                        const float err = t - pred;
                        s0 = fmaf(err, err, s0);
                        s1 += t;
                        const float2 t2 = make_float2(t, t);
#pragma unroll
                        for (int q = 1; q < RM; ++q) z12[q] = __ffma2_rn(make_float2(a1[q], a2[q]), t2, z12[q]);
                        zc += t;
                        if (hash_on) {
                            const float port = err + tmix * t;
                            const bool fx = fabsf(port) < fix.vmax;  // false for non-finite values
                            const int qv = fx ? __float2int_rn(port * fix.scale) : 0;
#pragma unroll
                            for (int t2 = 0; t2 < (NT > 0 ? NT : T); ++t2) {
                                const int bt = (NT > 0 || t2 < 2) ? bi[NT > 0 ? t2 : (t2 & 1)] : bin_of(t2);
                                atomicAdd(&my_bins[t2 * B + bt], qv);
                            }
                            if (!fx) {
                                for (int t2 = 0; t2 < (NT > 0 ? NT : T); ++t2) {
                                    const int bt = (NT > 0 || t2 < 2) ? bi[NT > 0 ? t2 : (t2 & 1)] : bin_of(t2);
                                    atomicAdd(&s_fbin[t2 * B + bt], port);
                                }
                            }
                        }
                    } else if constexpr (PASS == 4) {
                        float pred, echo;
                        if constexpr (TCR) {
                            pred = R1[u];
                            echo = (flags & F_ECHO) ? R2[u] : 0.0f;
                        } else {
                            float a1[RM], a2[RM];
                            load_row<RM>(rtb, lr, a1, a2);
                            pred = recon_dot_nz<RM>(K1, a1, a2, U1, V1);
                            echo = (flags & F_ECHO) ? recon_dot_nz<RM>(K2, a1, a2, U2, V2) : 0.0f;
                        }
                        const float t = xval;
                        float hpv = 0.0f;
                        if (hash_on) {
#pragma unroll
                            for (int t2 = 0; t2 < (NT > 0 ? NT : T); ++t2) hpv += s_tab[t2 * B + bin_of(t2)];
                            hpv = hpv * invT;
                        }
                        const DriveParts dp = drive_parts(t, pred, dk);
                        const float v[7] = {dp.u, dp.root, t, pred, dp.nov, echo, hpv};
#pragma unroll
                        for (int a = 0; a < 7; ++a)
#pragma unroll
                            for (int b = a; b < 7; ++b) g32[gram_idx(a, b)] = fmaf(v[a], v[b], g32[gram_idx(a, b)]);
                        g32[28] = fmaf(dp.rat, dp.rat, g32[28]);
                    } else {  // PASS 5
                        float pred, comb;
                        if constexpr (TCR) {
                            pred = R1[u];
                            comb = R2[u];
                        } else {
                            float a1[RM], a2[RM];
                            load_row<RM>(rtb, lr, a1, a2);
                            pred = recon_dot_nz<RM>(K1, a1, a2, U1, V1);
                            comb = recon_dot_nz<RM>(K2, a1, a2, U2, V2);
                        }
                        const float t = xval;
                        float hpv = 0.0f;
                        if (hash_on) {
#pragma unroll
                            for (int t2 = 0; t2 < (NT > 0 ? NT : T); ++t2) hpv += s_tab[t2 * B + bin_of(t2)];
                            hpv = hpv * invT;
                        }
                        const DriveParts dp = drive_parts(t, pred, dk);
                        const float drive = c_u * dp.u + c_root * dp.root + c_t * t + comb + c_nov * dp.nov + c_hp * hpv;
                        const float upd = drive * gain;
                        const int64_t pe = (int64_t)r * cols32 + col;
                        if (!half16) {
                            param[pe] = pb[o] + neg_lr * upd;
                        } else {
                            // round(p + round(-lr) round(u)), every rounding to the 16-bit type
                            const bool bf = (flags & F_BF16) != 0;
                            const unsigned short raw = reinterpret_cast<const unsigned short*>(pb)[o];
                            const float p0 = !vec ? pb[o]
                                             : (bf ? __bfloat162float(__ushort_as_bfloat16(raw))
                                                   : __half2float(__ushort_as_half(raw)));
                            if (bf) {
                                const float u = __bfloat162float(__float2bfloat16_rn(upd));
                                reinterpret_cast<__nv_bfloat16*>(Dp->param_h)[pe] = __float2bfloat16_rn(p0 + neg_lr16 * u);
                            } else {
                                const float u = __half2float(__float2half_rn(upd));
                                reinterpret_cast<__half*>(Dp->param_h)[pe] = __float2half_rn(p0 + neg_lr16 * u);
                            }
                        }
                    }
                }
                if constexpr (PASS == 2) {
                    // row sums of the axis density over the TC lanes of each row
                    if (UNR == 4 && wseg >= 4) {
                        float dv4[4] = {dv[0], dv[UNR > 1 ? 1 : 0], dv[UNR > 2 ? 2 : 0], dv[UNR > 3 ? 3 : 0]};
                        const float x = group_sum4(dv4, wseg);
                        const int sl = lane & (wseg - 1);
                        const int o1 = wseg >> 1, o2 = wseg >> 2;
                        const int ur = 2 * ((sl & o1) != 0) + ((sl & o2) != 0);
                        if ((sl & (o2 - 1)) == 0) {  // lowest lane of its class writes row ur
                            const int r = rbase + rs + RPI * (m0 + ur);
                            if (TC <= 32) {
                                if (r < rows32) Dp->rowpart[(int64_t)ct * rows + r] = x;
                            } else {
                                s_rowred[(rs + RPI * (m0 + ur)) * (TC >> 5) + (lc >> 5)] = x;
                            }
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < UNR; ++u) {
                            float x = dv[u];
                            for (int o = wseg >> 1; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
                            const int r = rbase + rs + RPI * (m0 + u);
                            if (TC <= 32) {
                                if (lc == 0 && r < rows32) Dp->rowpart[(int64_t)ct * rows + r] = x;
                            } else if (lane == 0) {
                                s_rowred[(rs + RPI * (m0 + u)) * (TC >> 5) + (lc >> 5)] = x;
                            }
                        }
                    }
                }
            }  // rows of the item

            // ---- item epilogue: float32 item partials into float64 block state
            if constexpr (PASS == 1) {
                acc0 += (double)s0;
            } else if constexpr (PASS == 2 || PASS == 3) {
                acc0 += (double)s0;
                acc1 += (double)s1;
                if (nct != ct || it + 1 == seg_end || ++items_since_flush == 4) {
                    if (cvalid) {
                        float b1[RM], b2[RM];
                        load_col<RM>(coltab, gcols, gc, b1, b2);
                        s_acc[tid] += (double)zc;  // zero mode: sum of the projected field
#pragma unroll
                        for (int q = 1; q < RM; ++q) {
                            const double B1 = b1[q], B2 = b2[q], Z1 = z12[q].x, Z2 = z12[q].y;
                            double c, s;
                            if (mode_is_product(q)) {
                                c = B1 * Z1;
                                s = B2 * Z2;
                            } else {
                                c = B1 * Z1 - B2 * Z2;
                                s = B2 * Z1 + B1 * Z2;
                            }
                            s_acc[q * kThreads + tid] += c;
                            s_acc[(RM + q) * kThreads + tid] += s;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < RM; ++q) z12[q] = make_float2(0.0f, 0.0f);
                    zc = 0.0f;
                    items_since_flush = 0;
                }
            } else if constexpr (PASS == 4) {
                // float32 Gram partials over up to 2 items, summed across the warp (lane q
                // ends with entry q) into the warp's float64 sums
                if (++items_since_flush == 2 || it + 1 == seg_end) {
                    float v[32];
#pragma unroll
                    for (int q = 0; q < 32; ++q) v[q] = q < kGram ? g32[q < kGram ? q : 0] : 0.0f;
                    const float x = warp_transpose_sum32(v);
                    if (lane < kGram) s_acc[warp * 32 + lane] += (double)x;
#pragma unroll
                    for (int q = 0; q < kGram; ++q) g32[q] = 0.0f;
                    items_since_flush = 0;
                }
            }
            if constexpr (PASS == 2) {
                if (TC > 32) {
                    __syncthreads();
                    const int nw = TC >> 5;
                    for (int lr = tid; lr < RB; lr += kThreads) {
                        float s = 0.0f;
                        for (int w = 0; w < nw; ++w) s += s_rowred[lr * nw + w];
                        if (rbase + lr < rows32) Dp->rowpart[(int64_t)ct * rows + rbase + lr] = s;
                    }
                }
                // column sums: combine the RPI threads that share a column
                s_colred[tid] = colacc;
                __syncthreads();
                if (rs == 0 && cvalid) {
                    float s = 0.0f;
                    for (int q = 0; q < RPI; ++q) s += s_colred[q * TC + lc];
                    Dp->colpart[(int64_t)band * cols + col] = s;
                }
            }
            if constexpr (TCR) {  // item i + 2's carrier rows into this item's B buffer (its products are done)
                if (it + 2 < seg_end) {
                    tc_store_b(tc_bnext, tcb);
                    tc_fence_smem();
                }
                tc_fence_before();
            }
            __syncthreads();  // this buffer (and the reduction scratch) is free again
            if constexpr (TCR) tcb ^= 1;
            if constexpr (kBins) {
                // empty the fixed-point copies into the exact block sums (ordered before the
                // next item's atomics by the barrier that precedes its compute)
                if (hash_on) {
                    for (int b = tid; b < TB; b += kThreads) {
                        long long s = 0;
                        for (int c = 0; c < ncopies; ++c) {
                            s += s_ibin[c * cstride + b];
                            s_ibin[c * cstride + b] = 0;
                        }
                        s_lbin[b] += s;
                    }
                }
            }
            if (vec) buf ^= 1;
            ct = nct;
            band = nband;
        }  // items of the segment

        // ---- segment flush: one record per (block, tensor)
        if constexpr (PASS <= 4) {
            const int rec = Dp->recbase[PASS] + ((int)blockIdx.x - Dp->cfirst[PASS]);
            double* out = rec_scal + (int64_t)rec * kNSRec;
            if constexpr (PASS == 1) {
                double v[1] = {acc0};
                block_sum_to<1>(v, s_red, s_tot);
                if (tid == 0) out[0] = s_tot[0];
            } else if constexpr (PASS == 4) {
                // the warps' sums in a fixed order (the item loop ended with a barrier)
                if (tid < kGram) {
                    double v = 0.0;
                    for (int w = 0; w < kWarps; ++w) v += s_acc[w * 32 + tid];
                    out[tid] = v;
                }
            } else {
                constexpr int NS = 2 + 2 * RM;
                double v[NS];
                v[0] = acc0;
                v[1] = acc1;
#pragma unroll
                for (int q = 0; q < 2 * RM; ++q) v[2 + q] = s_acc[q * kThreads + tid];
                block_sum_to<NS>(v, s_red, s_tot);
                for (int j = tid; j < NS; j += kThreads) out[j] = s_tot[j];
                if constexpr (kBins) {
                    if (hash_on) {
                        const double inv_scale = ldexp(1.0, -fix.s);
                        for (int b = tid; b < TB; b += kThreads)
                            rec_bins[(int64_t)rec * TB + b] = (float)((double)s_lbin[b] * inv_scale + (double)s_fbin[b]);
                    }
                }
            }
        }
        __syncthreads();
        ++k;
        if (tc_abort) break;
    }
    if constexpr (TCR) {
        cp_async_wait<0>();
        // after a give-up, the products of the next item may still be in flight: wait for
        // them (bounded) before the TMEM is freed, and record bit 2 if they never completed
        // (the tensor core may then still write TMEM that another block can claim)
        if (tc_abort && tid == 0 && !mbar_wait_bounded(smem_u32(s_tcbar), tc_parity ^ 1, kTcWaitNs))
            atomicOr(hdr->status, 2);
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tc_dealloc(tc_base, kTcCols);
        }
    }
}

}  // namespace cresso

#include "spectral_fast.cuh"

namespace cresso {

// ---------------------------------------------------------------------------
// Reduce: fixed-order sums of block records into the reduction vectors
// ---------------------------------------------------------------------------
__host__ __device__ inline int64_t red_len(int pass, int64_t rm, int64_t tb, int64_t cols, int ndim) {
    switch (pass) {
        case 1: return 1;
        case 2: return 2 + 2 * rm + tb + (ndim >= 2 ? cols : 0);
        case 3: return 2 + 2 * rm + tb;
        default: return kGram;
    }
}

// The per-block records of a pass summed into D.red[pass] in float64.  Every
// output is added in one fixed order - G interleaved partial sums (records g,
// g + G, g + 2G, ... in increasing order), then the G partials in order - so
// the result does not depend on the launch or the GPU.  Block kinds: the
// scalar and hash-bin outputs (records of the blocks that covered the tensor)
// take 8 outputs x 32 groups per block; the column sums of pass 2 (one
// partial per row band) take 64 outputs x 4 groups, or 256 outputs of one
// group when the partials are per block run (col_runs).  grid.x = the largest
// number of scalar blocks over the tensors + the largest number of column
// blocks; grid.y = tensors.
constexpr int kRedOutA = 8, kRedGrpA = kThreads / kRedOutA;   // 8 x 32
constexpr int kRedOutB = 64, kRedGrpB = kThreads / kRedOutB;  // 64 x 4

__host__ __device__ inline int64_t red_scal_len(int pass, int64_t rm, int64_t tb) {
    return pass == 1 ? 1 : (pass == 4 ? kGram : 2 + 2 * rm + tb);
}

__global__ void reduce_kernel(int pass, int blocks_a, const GroupHdr* __restrict__ hdr,
                              const DevTensor* __restrict__ dts, const double* __restrict__ rec_scal,
                              const float* __restrict__ rec_bins) {
    __shared__ double part[kThreads];
    const DevTensor& D = dts[blockIdx.y];
    const int64_t rm = hdr->rm, tb = hdr->tb;
    const int64_t ns = pass == 1 ? 1 : (pass == 4 ? kGram : 2 + 2 * rm);
    const int64_t na = red_scal_len(pass, rm, tb);                      // scalar + bin outputs
    const int64_t nc = red_len(pass, rm, tb, D.cols, D.ndim) - na;      // column outputs
    const bool kind_a = (int)blockIdx.x < blocks_a;
    // column outputs of a tensor with per-run partials (col_runs): a thread per output,
    // each adding its column's one or two block runs, so every thread of the block works
    const bool runs = !kind_a && D.col_runs;
    const int outs = kind_a ? kRedOutA : (runs ? kThreads : kRedOutB);
    const int grps = kind_a ? kRedGrpA : (runs ? 1 : kRedGrpB);
    const int64_t first = kind_a ? (int64_t)blockIdx.x * kRedOutA : na + (int64_t)(blockIdx.x - blocks_a) * outs;
    const int64_t last = kind_a ? na : na + nc;
    if (first >= last) return;  // block-uniform
    const int j = threadIdx.x % outs, g = threadIdx.x / outs;
    const int64_t o = first + j;
    double s = 0.0;
    if (o < last) {
        const int r0 = D.recbase[pass], nr = D.nrec[pass];
        if (o < ns) {
            for (int r = g; r < nr; r += grps) s += rec_scal[(int64_t)(r0 + r) * kNSRec + o];
        } else if (o < na) {
            if (D.flags & F_HASH)
                for (int r = g; r < nr; r += grps) s += (double)rec_bins[(int64_t)(r0 + r) * tb + (o - ns)];
        } else {
            const int64_t c = o - na;
            if (D.col_runs) {
                // the records of the blocks whose items cover column tile c / TC: block b of
                // the launch owns items [b ci / g, (b + 1) ci / g), so item x lies in block
                // ((x + 1) g - 1) / ci
                if (g == 0) {
                    const int64_t ci = hdr->cls_items[0], gg = hdr->grid[0][2];
                    const int64_t first = D.item_base + (c / D.TC) * D.n_bands, last = first + D.n_bands - 1;
                    const int64_t b0 = ((first + 1) * gg - 1) / ci, b1 = ((last + 1) * gg - 1) / ci;
                    const double* cp = reinterpret_cast<const double*>(D.colpart);
                    for (int64_t b = b0; b <= b1; ++b) s += cp[(b - D.cfirst[2]) * D.cols + c];
                }
            } else {
                for (int b = g; b < D.n_bands; b += grps) s += (double)D.colpart[(int64_t)b * D.cols + c];
            }
        }
    }
    part[g * outs + j] = s;
    __syncthreads();
    if (g == 0 && o < last) {
        double t = part[j];
        for (int q = 1; q < grps; ++q) t += part[q * outs + j];
        D.red[pass][o] = t;
    }
}

// ---------------------------------------------------------------------------
// Finalize kernels (one block per tensor)
// ---------------------------------------------------------------------------

// Folds (alpha, beta) on the normalised carriers into inv-scaled coefficients
// and the constant term; threads k < RM, result K valid for all threads.
template <int RM>
__device__ void fold_recon(const ModeStats* stats, int R, double alpha, double beta, float* al, float* be, float* K,
                           double* s_red) {
    const int k = threadIdx.x;
    double kpart = 0.0;
    if (k < RM) {
        double a = 0.0, b = 0.0;
        if (k < R) {
            a = alpha * stats[k].inv_c;
            b = beta * stats[k].inv_s;
            kpart = -(a * stats[k].mu_c + b * stats[k].mu_s);
        }
        al[k] = (float)a;
        be[k] = (float)b;
    }
    // mode 0 is the zero-frequency carrier (1, 0): fold its constant term into K
    if (k == 0) kpart += alpha * stats[0].inv_c;
    const double tot = block_sum(kpart, s_red);
    if (threadIdx.x == 0) *K = (float)tot;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

template <int RM>
__global__ void finalize1_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts) {
    const DevTensor& D = dts[blockIdx.x];
    if (threadIdx.x != 0) return;
    const double* hp = hdr->hp;
    const float eps = (float)hp[H_EPS];
    const float frn = sqrtf((float)(D.red[1][0] / (double)D.N) + eps);
    const float fr = reservoir(*D.force_rms, frn, hp[H_RD], D.step);
    *D.force_rms = fr;
    const float scale = fmaxf(fr, eps);
    D.cst->scale = scale;
    D.cst->inv_scale = 1.0f / scale;
}

template <int RM>
__global__ void finalize2_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts) {
    __shared__ double s_red[kWarps + 1];
    __shared__ float s_meanE[64];
    const DevTensor& D = dts[blockIdx.x];
    TensorConsts& C = *D.cst;
    const double* hp = hdr->hp;
    const float eps = (float)hp[H_EPS];
    const int tid = threadIdx.x;
    const int R = D.R, B = (int)hdr->bins, T = (int)hdr->tables, TB = (int)hdr->tb;
    const double N = (double)D.N;
    const double* red = D.red[2];
    const double sumL = red[0], sumd = red[1];
    const int64_t rm = hdr->rm;
    if (blockIdx.y > 0) {
        // blocks 1..gridDim.y-1 of a 2-D tensor: the instant axial metric factors of its
        // rows and columns (cresso_v5.py:243-262), exp(c / (2 p) (log(max(axis mean / mean,
        // eps)))); a row's sum adds its column-tile partials in order
        if (!(D.flags & F_INST2D) || D.ndim != 2) return;
        const float pw = fmaxf((float)hp[H_IP], 0.25f);
        const float gmc = fmaxf((float)(sumd / N), eps);
        const float kk = (float)(hp[H_IC] / ((double)D.ndim * (double)pw));
        const int64_t grows = D.N / D.gcols;
        const int64_t step = (int64_t)(gridDim.y - 1) * kThreads;
        for (int64_t r = (int64_t)(blockIdx.y - 1) * kThreads + tid; r < D.rows; r += step) {
            double s = 0.0;
            for (int c = 0; c < D.n_ct; ++c) s += (double)D.rowpart[(int64_t)c * D.rows + r];
            const float rmean = (float)(s / (double)D.gcols);
            D.rowf[r] = expf(kk * logf(fmaxf(rmean / gmc, eps)));
        }
        const double* cols = red + 2 + 2 * rm + TB;
        for (int64_t c = (int64_t)(blockIdx.y - 1) * kThreads + tid; c < D.cols; c += step) {
            const float cmean = (float)(cols[c] / (double)grows);
            D.colf[c] = expf(kk * logf(fmaxf(cmean / gmc, eps)));
        }
        return;
    }

    // ---- hash metric (cresso_v5.py:1013-1056)
    if (D.flags & F_HASH) {
        const double* bins = red + 2 + 2 * rm;
        for (int tb = tid; tb < TB; tb += kThreads) {
            const float cell = (float)bins[tb] / fmaxf(D.counts[tb], 1.0f);
            D.h_energy[tb] = reservoir(D.h_energy[tb], cell, hp[H_HD], D.step);
        }
        __syncthreads();
        for (int t = 0; t < T; ++t) {
            double s = 0.0;
            for (int b = tid; b < B; b += kThreads) s += (double)D.h_energy[t * B + b];
            s = block_sum(s, s_red);
            if (tid == 0) s_meanE[t & 63] = (float)(s / (double)B);
            __syncthreads();
            const float meanE = fmaxf(s_meanE[t & 63], eps);
            const float ex = (float)(hp[H_HMC] / fmax(0.25, hp[H_EP]));
            for (int b = tid; b < B; b += kThreads) {
                const float hm = fmaxf(D.h_energy[t * B + b] / meanE, eps);
                const float v = clampf(powf(hm, ex), 0.08f, 12.0f);
                // per-bin root m^(1/T); the per-element metric is the product over tables
                D.htab[t * B + b] = (float)exp(log((double)fmaxf(v, eps)) / (double)T);
            }
            __syncthreads();
        }
    }

    // ---- spectral metric oscillator (cresso_v5.py:1057-1088)
    const double shrink = recon_shrink(R);
    const float M = fmaxf((float)(sumL / N), eps);
    double m_alpha = 0.0, m_beta = 0.0, p_alpha = 0.0, p_beta = 0.0;
    if (tid < R) {
        const int k = tid;
        const ModeStats st = D.stats[k];
        // P2 accumulated sum (log1p(ds) - 1/2) * raw; restore sum log1p(ds) * raw exactly
        const double Cc = red[2 + k] + 0.5 * N * st.rawmean_c;
        const double Cs = red[2 + rm + k] + 0.5 * N * st.rawmean_s;
        const float pc = (float)((st.inv_c * (Cc - st.mu_c * sumL) / N) / (double)M - st.mhat_c);
        const float ps = (float)((st.inv_s * (Cs - st.mu_s * sumL) / N) / (double)M - st.mhat_s);
        const float mdt = (float)hp[H_MDT];
        const float damp = (float)fmax(0.0, 1.0 - hp[H_MDT] * hp[H_MF]);
        const float om = D.omega[k];
        const float om2 = om * om;
        float mp = D.mp_cos[k] * damp;
        float mq = D.m_cos[k];
        mp = mp + mdt * (pc - om2 * mq);
        mq = clampf(mq + mdt * mp, -3.0f, 3.0f);
        D.mp_cos[k] = mp;
        D.m_cos[k] = mq;
        float mps = D.mp_sin[k] * damp;
        float mqs = D.m_sin[k];
        mps = mps + mdt * (ps - om2 * mqs);
        mqs = clampf(mqs + mdt * mps, -3.0f, 3.0f);
        D.mp_sin[k] = mps;
        D.m_sin[k] = mqs;
        m_alpha = (double)mq * shrink;
        m_beta = (double)mqs * shrink;
        // prediction from the old oscillators (cresso_v5.py:1128-1129)
        const float gate = sigmoidf_((float)hp[H_CONFG] * D.conf[k]);
        p_alpha = (double)D.q_cos[k] * shrink * (double)gate;
        p_beta = (double)D.q_sin[k] * shrink * (double)gate;
    }
    if (tid < 2 * kMaxRank) C.pv[tid] = 0.0;
    __syncthreads();
    if (tid < R) {
        C.pv[2 * tid] = p_alpha;
        C.pv[2 * tid + 1] = p_beta;
    }
    fold_recon<RM>(D.stats, R, m_alpha, m_beta, C.m_al, C.m_be, &C.m_K, s_red);
    fold_recon<RM>(D.stats, R, p_alpha, p_beta, C.p0_al, C.p0_be, &C.p0_K, s_red);

    // ---- instant axial metric factors (cresso_v5.py:243-262, 1102-1122)
    const float pw = fmaxf((float)hp[H_IP], 0.25f);
    const float gmc = fmaxf((float)(sumd / N), eps);
    if (D.flags & F_INST2D) {
        // exp(c / (ndim * p) * sum over axes of log(max(axis mean / mean, eps)))
        const float kk = (float)(hp[H_IC] / ((double)D.ndim * (double)pw));
        const int64_t grows = D.N / D.gcols;
        if (D.ndim == 2) {
            // rows and columns: the blocks with blockIdx.y > 0 (above)
        } else {
            // rank >= 3 (never sharded): the row index is the flattened leading axes.  Row
            // sums into rowf, then per leading axis a and coordinate c the marginal mean
            // (a fixed-order float64 sum over the rows with that coordinate), whose log
            // goes to s_lax; a row's factor is the exponential of its axes' logs.
            __shared__ float s_lax[kMaxLeadSum];
            for (int64_t r = tid; r < D.rows; r += kThreads) {
                double s = 0.0;
                for (int c = 0; c < D.n_ct; ++c) s += (double)D.rowpart[(int64_t)c * D.rows + r];
                D.rowf[r] = (float)s;
            }
            __syncthreads();
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
                const int64_t outer = grows / (D.dims[a] * inner);
                double m = 0.0;
                for (int64_t o = 0; o < outer; ++o)
                    for (int64_t i = 0; i < inner; ++i) m += (double)D.rowf[(o * D.dims[a] + c) * inner + i];
                const double per = (double)D.N / (double)D.dims[a];
                s_lax[j] = logf(fmaxf((float)(m / per) / gmc, eps));
            }
            __syncthreads();
            for (int64_t r = tid; r < D.rows; r += kThreads) {
                float lsum = 0.0f;
                int64_t rem = r;
                int off = lead_sum;
                for (int a = nl - 1; a >= 0; --a) {
                    off -= (int)D.dims[a];
                    lsum += s_lax[off + (int)(rem % D.dims[a])];
                    rem /= D.dims[a];
                }
                D.rowf[r] = expf(kk * lsum);
            }
        }
        if (D.ndim != 2) {
            const double* cols = red + 2 + 2 * rm + TB;
            for (int64_t c = tid; c < D.cols; c += kThreads) {
                const float cmean = (float)(cols[c] / (double)grows);
                D.colf[c] = expf(kk * logf(fmaxf(cmean / gmc, eps)));
            }
        }
    }
    if (tid == 0) {
        C.inst_k = (float)(hp[H_IC] / (double)pw);
        C.inst_gm = gmc;
    }
}

template <int RM>
__global__ void finalize3_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts) {
    __shared__ double s_red[kWarps + 1];
    __shared__ float s_S;
    __shared__ float s_pc[kMaxRank], s_ps[kMaxRank];
    const DevTensor& D = dts[blockIdx.x];
    TensorConsts& C = *D.cst;
    const double* hp = hdr->hp;
    const float eps = (float)hp[H_EPS];
    const int tid = threadIdx.x, lane = tid & 31;
    const int R = D.R, TB = (int)hdr->tb;
    const int64_t rm = hdr->rm;
    const double N = (double)D.N;
    const double* red = D.red[3];

    // surprise (cresso_v5.py:1131-1133)
    if (tid == 0) {
        const float sn = sqrtf((float)(red[0] / N) + eps);
        const float S = reservoir(*D.surprise, sn, hp[H_SD], D.step);
        *D.surprise = S;
        s_S = S;
    }
    __syncthreads();
    const float S = s_S;
    const double sumt = red[1];

    // projections of t and of the port  (cresso_v5.py:1135-1138; port = (1+tm) t - pred)
    double Pc = 0.0, Ps = 0.0;
    if (tid < R) {
        const int k = tid;
        const ModeStats st = D.stats[k];
        Pc = st.inv_c * (red[2 + k] - st.mu_c * sumt) / N;
        Ps = st.inv_s * (red[2 + rm + k] - st.mu_s * sumt) / N;
        double gvc = 0.0, gvs = 0.0;
        const int P = 2 * (int)rm;
        for (int y = 0; y < 2 * R; ++y) {
            gvc += D.gram[(2 * k) * P + y] * C.pv[y];
            gvs += D.gram[(2 * k + 1) * P + y] * C.pv[y];
        }
        const double tm1 = 1.0 + hp[H_TM];
        s_pc[k] = (float)(tm1 * Pc - gvc);
        s_ps[k] = (float)(tm1 * Ps - gvs);
    }

    // hash impulse reservoirs (cresso_v5.py:1140-1184)
    if (D.flags & F_HASH) {
        const double* bins = red + 2 + 2 * rm;
        const float hd = (float)hp[H_HD], hd1 = (float)(1.0 - hp[H_HD]);
        const float hid = (float)hp[H_HID], hid1 = (float)(1.0 - hp[H_HID]);
        const float rg = (float)hp[H_RG];
        for (int tb = tid; tb < TB; tb += kThreads) {
            const float cell = (float)bins[tb] / fmaxf(D.counts[tb], 1.0f);
            const float ref = D.h_refractory[tb] * hd + fabsf(cell) * hd1;
            const float gate = 1.0f / (1.0f + rg * ref);
            const float imp = D.h_impulse[tb] * hid + (cell * gate) * hid1;
            D.h_refractory[tb] = ref;
            D.h_impulse[tb] = imp;
            D.htab[tb] = imp;
        }
    }
    __syncthreads();

    // confidence and the two contact half-updates run in warp 0, lane = mode
    if (tid < 32) {
        const bool act = lane < R;
        const int k = act ? lane : 0;
        const float pc = act ? s_pc[k] : 0.0f, ps = act ? s_ps[k] : 0.0f;
        float qc = act ? D.q_cos[k] : 0.0f, qs = act ? D.q_sin[k] : 0.0f;
        // confidence (cresso_v5.py:1199-1202), with the old q
        if (act) {
            const float pe = sqrtf(pc * pc + ps * ps + eps);
            const float sup = (pc * qc + ps * qs) / (pe * sqrtf(qc * qc + qs * qs + eps) + eps);
            const float cd = (float)hp[H_CD];
            float cf = D.conf[k] * cd + clampf(sup, -1.0f, 1.0f) * (float)(1.0 - hp[H_CD]);
            D.conf[k] = clampf(cf, -4.0f, 4.0f);
        }
        // contact oscillators (cresso_v5.py:914-943, 1204-1250)
        const float dt = (float)hp[H_DT];
        const float rd = (float)hp[H_REFD], rd1 = (float)(1.0 - hp[H_REFD]);
        const float plast = 1.0f + (float)hp[H_SG] * S / (1.0f + S);
        const float brake = 1.0f / (1.0f + (float)hp[H_SB] * S);
        const float om = act ? D.omega[k] : 0.0f;
        float action = *D.action;
        for (int half = 0; half < 2; ++half) {
            float* qp = half == 0 ? D.q_cos : D.q_sin;
            float* pp = half == 0 ? D.p_cos : D.p_sin;
            float* cp = half == 0 ? D.ca_cos : D.ca_sin;
            const float port = half == 0 ? pc : ps;
            float q = act ? qp[k] : 0.0f, p = act ? pp[k] : 0.0f, ca = act ? cp[k] : 0.0f;
            ca = ca * rd + fabsf(port) * rd1;
            const float rgate = 1.0f / (1.0f + (float)hp[H_RG] * ca);
            const float gp = port * rgate * plast * brake;
            const float omq = om * q;
            const float e2 = warp_sum(act ? p * p : 0.0f) / (float)R;
            const float w2 = warp_sum(act ? omq * omq : 0.0f) / (float)R;
            const float energy = 0.5f * (e2 + w2);
            const float ppow = warp_sum(act ? gp * p : 0.0f) / (float)R;
            action = action * 0.985f + (ppow - energy) * dt;
            const float fr = (float)hp[H_IF] + (float)hp[H_CG] * tanhf(fabsf(action));
            p = p * fmaxf(1.0f - dt * fr, 0.0f);
            p = p + dt * (gp - (float)hp[H_REST] * (om * om) * q - (float)hp[H_CUBIC] * (q * q * q));
            q = clampf(q + dt * p, -8.0f, 8.0f);
            if (act) {
                qp[k] = q;
                pp[k] = p;
                cp[k] = ca;
            }
        }
        if (lane == 0) *D.action = action;
    }
    __syncthreads();

    // new prediction and echo coefficients (cresso_v5.py:1252-1258)
    const double shrink = recon_shrink(R);
    double pa = 0.0, pb = 0.0, ea = 0.0, eb = 0.0;
    if (tid < R) {
        const float gate = sigmoidf_((float)hp[H_CONFG] * D.conf[tid]);
        pa = (double)D.q_cos[tid] * shrink * (double)gate;
        pb = (double)D.q_sin[tid] * shrink * (double)gate;
        ea = (double)(float)Pc * shrink;
        eb = (double)(float)Ps * shrink;
    }
    fold_recon<RM>(D.stats, R, pa, pb, C.pr_al, C.pr_be, &C.pr_K, s_red);
    fold_recon<RM>(D.stats, R, ea, eb, C.ec_al, C.ec_be, &C.ec_K, s_red);
    if (tid == 0) {
        const float clip = (float)hp[H_CLIP];
        C.S = S;
        C.sp = (float)hp[H_SPIKE] / (1.0f + S);
        C.invD = 1.0f / (clip * (1.0f + S));
        C.clip = clip;
        C.inv_clip = 1.0f / clip;
        C.clip2 = (float)(hp[H_CLIP] * hp[H_CLIP]);
    }
}

template <int RM>
__global__ void finalize4_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts) {
    __shared__ float s_cp, s_ce;
    const DevTensor& D = dts[blockIdx.x];
    TensorConsts& C = *D.cst;
    const double* hp = hdr->hp;
    if (threadIdx.x == 0) {
        const float eps = (float)hp[H_EPS];
        const double N = (double)D.N;
        const double* g = D.red[4];
        auto Gm = [&](int a, int b) { return a <= b ? g[gram_idx(a, b)] : g[gram_idx(b, a)]; };
        enum { U = 0, RT = 1, TT = 2, PR = 3, NV = 4, EC = 5, HP = 6 };
        const bool hard = (D.flags & F_HARD) != 0;
        const float S = C.S;
        // cresso_v5.py:1303-1346
        const float frms = sqrtf((float)(Gm(TT, TT) / N) + eps);
        const float prms = sqrtf((float)(Gm(PR, PR) / N) + eps);
        const float align = clampf((float)(Gm(TT, PR) / N) / (frms * prms + eps), -1.0f, 1.0f);
        const float align_gate = prms > (float)sqrt(hp[H_EPS]) ? clampf((align + 1.0f) * 0.5f, 0.0f, 1.0f) : 0.0f;
        const int ws = (int)hp[H_WS];
        const double warm = ws == 0 ? 1.0 : (1.0 - exp(-(double)D.step / (double)(ws > 1 ? ws : 1)));
        const float mix = (float)(hp[H_PM] * warm) * align_gate * (1.0f / (1.0f + S));
        const float rat_rms = sqrtf((float)(g[28] / N) + eps);
        const float root_rms = sqrtf((float)(Gm(RT, RT) / N) + eps);
        const float k_root = rat_rms / fmaxf(root_rms, eps);
        const float root_mix = (hard ? (float)hp[H_RCM] : 0.0f) / (1.0f + 0.5f * S);
        const double a = 1.0 - (double)root_mix, b = (double)root_mix * (double)k_root;
        const double sh2 = a * a * Gm(U, U) + 2.0 * a * b * Gm(U, RT) + b * b * Gm(RT, RT);
        const float shaped_rms = sqrtf((float)(sh2 / N) + eps);
        const bool echo_on = (D.flags & F_ECHO) != 0, hash_on = (D.flags & F_HASH) != 0;
        const float k_e = echo_on ? shaped_rms / fmaxf(sqrtf((float)(Gm(EC, EC) / N) + eps), eps) : 0.0f;
        const float k_h = hash_on ? shaped_rms / fmaxf(sqrtf((float)(Gm(HP, HP) / N) + eps), eps) : 0.0f;
        const float dm = (float)hp[H_DFM] / (1.0f + 0.35f * S);
        const float k_d = shaped_rms / fmaxf(frms, eps);
        const double cu = (1.0 - dm) * a, cr = (1.0 - dm) * b, ctt = (double)dm * k_d;
        const double core2 = cu * cu * Gm(U, U) + cr * cr * Gm(RT, RT) + ctt * ctt * Gm(TT, TT) +
                             2.0 * (cu * cr * Gm(U, RT) + cu * ctt * Gm(U, TT) + cr * ctt * Gm(RT, TT));
        const float core_rms = sqrtf((float)(core2 / N) + eps);
        const float resm = (float)hp[H_RFM] / (1.0f + S);
        const double err2 = Gm(TT, TT) - 2.0 * Gm(TT, PR) + Gm(PR, PR);
        const float k_r = core_rms / fmaxf(sqrtf((float)(fmax(err2, 0.0) / N) + eps), eps);
        double c[7];
        c[U] = (1.0 - mix) * cu;
        c[RT] = (1.0 - mix) * cr;
        c[TT] = (1.0 - mix) * ctt + (double)resm * k_r;
        c[PR] = (double)mix - (double)resm * k_r;
        c[NV] = hp[H_NM];
        c[EC] = (hard ? hp[H_EM] : 0.0) * (double)k_e;
        c[HP] = (hard ? hp[H_HDM] : 0.0) * (double)k_h;
        double d2 = 0.0;
        for (int i = 0; i < 7; ++i)
            for (int j = 0; j < 7; ++j) d2 += c[i] * c[j] * Gm(i, j);
        const float den = (float)(fmax(d2, 0.0) / N);
        const float DE = reservoir(*D.drive_energy, den, hp[H_RD], D.step);
        *D.drive_energy = DE;
        const float gain = clampf((float)hp[H_TGT] / sqrtf(DE + eps), (float)hp[H_MING], (float)hp[H_MAXG]);
        C.c_u = (float)c[U];
        C.c_root = (float)c[RT];
        C.c_t = (float)c[TT];
        C.c_nov = (float)c[NV];
        C.c_hp = (float)c[HP];
        C.gain = gain;
        C.neg_lr = (float)(-hp[H_LR]);
        s_cp = (float)c[PR];
        s_ce = (float)c[EC];
    }
    __syncthreads();
    if (threadIdx.x < RM) {
        const int k = threadIdx.x;
        C.cb_al[k] = s_cp * C.pr_al[k] + s_ce * C.ec_al[k];
        C.cb_be[k] = s_cp * C.pr_be[k] + s_ce * C.ec_be[k];
    }
    if (threadIdx.x == 0) C.cb_K = s_cp * C.pr_K + s_ce * C.ec_K;
}

// ---------------------------------------------------------------------------
// Host plan
// ---------------------------------------------------------------------------
// Floats of a tensor's pass-2 column partials (a multiple of 64, so every tensor's
// region starts on a 256-byte boundary).
static int64_t colpart_floats(const DevTensor& D) {
    const int64_t n = D.col_runs ? 2 * (int64_t)D.nrec[2] * D.cols : (int64_t)D.n_bands * D.cols;
    return align_up(n, 64);
}

struct Plan {
    GroupHdr hdr;
    std::vector<DevTensor> dts;
    std::vector<int64_t> item_lists;   // class 0 item prefix sums (n0 + 1), then class 1 (n1 + 1)
    std::vector<int32_t> tensor_lists; // class 0 tensor indices, then class 1
    int64_t off_status;
    int64_t off_hdr, off_dts, off_items, off_tmap, off_cst, off_htab, off_rowf, off_colf, off_rowpart, off_colpart;
    int64_t off_recs, off_recb, off_red[5], len_red[5], off_tbuf, bytes;
    int64_t n_rec_max;
    int64_t off_p32, half_elems;  // float32 copies of the 16-bit parameters
    int rm;
    bool fast;  // class 0 runs P2-P5 on fast_pass_kernel
};

static size_t pass_smem(int pass, const GroupHdr& H, int64_t iters, bool tc = false);

static int64_t take(int64_t& off, int64_t bytes) {
    const int64_t o = off;
    off = align_up(off + bytes, 256);
    return o;
}

// A tensor of rank n >= 2 is (product of the n - 1 leading axes) x (last axis);
// rank 1 is one row.
static int64_t g_rows(const cresso_tensor_desc& d) {
    int64_t r = 1;
    for (int64_t a = 0; a + 1 < d.ndim; ++a) r *= d.shape[a];
    return r;
}
static int64_t g_cols(const cresso_tensor_desc& d) { return d.shape[d.ndim - 1]; }

static int hp_flags_hard(const cresso_tensor_desc& d, const cresso_hparams& hp, int64_t N) {
    const int64_t cutoff = (int64_t)hp.thin_matrix_hard_cutoff;
    bool thin = false;
    if (d.ndim == 2 && cutoff > 0) thin = std::min(d.shape[0], d.shape[1]) <= cutoff;
    return N >= (int64_t)hp.hard_channel_min_size && !thin;
}

static int build_plan(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, int64_t num_sms, Plan& P) {
    CRESSO_REQUIRE(descs != nullptr && hp != nullptr, CRESSO_EINVAL, "spectral: NULL descriptors or hparams");
    CRESSO_REQUIRE(n >= 1, CRESSO_EINVAL, "spectral: need at least one tensor");
    CRESSO_REQUIRE(num_sms >= 1, CRESSO_EINVAL, "spectral: num_sms must be >= 1");
    const int64_t rank = (int64_t)hp->rank, bins = (int64_t)hp->hash_bins, tables = (int64_t)hp->hash_tables;
    CRESSO_REQUIRE(rank >= 1 && rank <= kMaxRank, CRESSO_EUNSUPPORTED,
                   "rank must be in [1, %d] on the CUDA spectral path (got %lld)", kMaxRank, (long long)rank);
    CRESSO_REQUIRE(tables >= 1 && bins >= 0, CRESSO_EINVAL, "hash_tables must be >= 1, hash_bins >= 0");
    CRESSO_REQUIRE(bins <= kMaxBins && bins * tables <= kMaxTB, CRESSO_EUNSUPPORTED,
                   "hash_bins <= %d and hash_bins * hash_tables <= %d on the CUDA path", kMaxBins, kMaxTB);
    const int rm = rank_pad(rank);
    P.rm = rm;
    memset(&P.hdr, 0, sizeof(P.hdr));
    GroupHdr& H = P.hdr;
    H.n_tensors = n;
    H.rm = rm;
    H.bins = bins;
    H.tables = tables;
    H.tb = bins * tables;
    H.idx_bytes = bins <= 256 ? 1 : 2;
    memcpy(H.hp, hp, sizeof(cresso_hparams));
    P.dts.assign(n, DevTensor{});
    std::vector<char> full(n, 0);

    // geometry and item counts; ITERS chosen so that the busiest pass has >= ~8 items per block
    int64_t total_rows_work = 0;
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        CRESSO_REQUIRE(d.ndim >= 1 && d.ndim <= CRESSO_MAX_NDIM, CRESSO_EUNSUPPORTED,
                       "tensor %lld: spectral route supports tensors of rank 1 to %d (ndim=%lld)", (long long)i,
                       CRESSO_MAX_NDIM, (long long)d.ndim);
        CRESSO_REQUIRE(d.dtype == CRESSO_DTYPE_F32 || d.dtype == CRESSO_DTYPE_F16 || d.dtype == CRESSO_DTYPE_BF16,
                       CRESSO_EUNSUPPORTED, "tensor %lld: dtype code %lld (float32, float16 and bfloat16 are supported)",
                       (long long)i, (long long)d.dtype);
        CRESSO_REQUIRE(d.param && d.grad && d.shape_ws, CRESSO_EINVAL, "tensor %lld: NULL param / grad / workspace",
                       (long long)i);
        CRESSO_REQUIRE(d.rows >= 1 && d.cols >= 1 && d.row0 >= 0 && d.col0 >= 0, CRESSO_EINVAL,
                       "tensor %lld: bad local block", (long long)i);
        const int64_t grows = g_rows(d);
        const int64_t gcols = g_cols(d);
        CRESSO_REQUIRE(d.row0 + d.rows <= grows && d.col0 + d.cols <= gcols, CRESSO_EINVAL,
                       "tensor %lld: local block outside the global shape", (long long)i);
        CRESSO_REQUIRE(d.ndim == 1 || (d.col0 == 0 && d.cols == gcols), CRESSO_EUNSUPPORTED,
                       "tensor %lld: 2-D tensors are sharded by rows only", (long long)i);
        CRESSO_REQUIRE(d.ndim <= 2 || (d.row0 == 0 && d.rows == grows), CRESSO_EUNSUPPORTED,
                       "tensor %lld: tensors of rank >= 3 are not sharded", (long long)i);
        if (d.ndim >= 3) {
            int64_t lead_sum = 0;
            for (int64_t a = 0; a + 1 < d.ndim; ++a) lead_sum += d.shape[a];
            CRESSO_REQUIRE(lead_sum <= kMaxLeadSum, CRESSO_EUNSUPPORTED,
                           "tensor %lld: leading axes of a rank-%lld tensor sum to %lld (at most %d)", (long long)i,
                           (long long)d.ndim, (long long)lead_sum, kMaxLeadSum);
        }
        CRESSO_REQUIRE(d.step >= 1, CRESSO_EINVAL, "tensor %lld: step must be >= 1", (long long)i);
        CRESSO_REQUIRE(grows * gcols < (1LL << 31), CRESSO_EUNSUPPORTED,
                       "tensor %lld: more than 2^31 - 1 elements per tensor", (long long)i);
        total_rows_work += d.rows * ceil_div(d.cols, 256);
    }
    // Rows per thread and item: large enough to amortise the per-item set-up,
    // small enough for >= ~8 items per block and for the staging buffers of
    // every pass to leave room for two blocks per SM.
    std::vector<char> vec(n, 0);
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        const int64_t gcols = g_cols(d);
        const int64_t ib = bins <= 256 ? 1 : 2;
        bool ok = d.cols >= 16 && d.cols % 16 == 0 && d.col0 % 16 == 0 && (d.ndim == 1 || gcols % 16 == 0);
        // 16-bit tensors are read through 256-byte aligned float32 copies in the scratch
        // (16-bit tensors: the gradient is read through an aligned float32 copy, the
        // parameter staged in its own type by P5)
        ok = ok && d.param % 16 == 0 && (d.dtype != CRESSO_DTYPE_F32 || d.grad % 16 == 0);
        if (d.hash_cache) ok = ok && d.hash_cache % 16 == 0 && (d.hash_cache_n * ib) % 16 == 0;
        vec[i] = ok;
    }
    int iters = 32;
    const int64_t target_blocks = num_sms * 2;
    while (iters > 4 && total_rows_work / iters < target_blocks * 8) iters >>= 1;
    const size_t budget = rm > 8 ? 200 * 1024 : 110 * 1024;
    for (;; iters >>= 1) {
        int64_t rb_max = 0;
        for (int64_t i = 0; i < n; ++i)
            if (vec[i]) rb_max = std::max<int64_t>(rb_max, (int64_t)(256 / std::min(256, pow2_ceil(descs[i].cols))) * iters);
        H.rb_max = rb_max;
        size_t need = 0;
        for (int p = 1; p <= 5; ++p) need = std::max(need, pass_smem(p, H, iters, p >= 3 && rm == 8 && iters == 16));
        if (need <= budget || iters <= 4) break;
    }
    H.iters = iters;

    int64_t items = 0;
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        DevTensor& D = P.dts[i];
        D.ndim = (int32_t)d.ndim;
        D.rows = d.rows;
        D.cols = d.cols;
        D.row0 = d.row0;
        D.col0 = d.col0;
        D.gcols = g_cols(d);
        D.N = g_rows(d) * D.gcols;
        for (int64_t a = 0; a < CRESSO_MAX_NDIM; ++a) D.dims[a] = a < d.ndim ? d.shape[a] : 0;
        D.step = d.step;
        D.R = (int32_t)rank;
        D.TC = std::min(256, pow2_ceil(d.cols));
        D.RPI = 256 / D.TC;
        D.RB = D.RPI * iters;
        D.n_ct = (int32_t)ceil_div(d.cols, D.TC);
        D.n_bands = (int32_t)ceil_div(d.rows, D.RB);
        D.n_items = (int64_t)D.n_ct * D.n_bands;
        items += D.n_items;
        const bool hard = hp_flags_hard(d, *hp, D.N);
        int fl = 0;
        if (hp->maximize != 0.0) fl |= F_MAXIMIZE;
        if (hp->weight_decay != 0.0) fl |= F_WD;
        if (hard) fl |= F_HARD;
        const bool hash_on = hard && bins > 0 && d.hash_energy && d.hash_impulse && d.hash_refractory;
        if (hash_on) {
            fl |= F_HASH;
            CRESSO_REQUIRE(d.hash_cache != 0 && d.hash_cache_n >= D.N, CRESSO_EINVAL,
                           "tensor %lld: hash cache missing or smaller than the tensor", (long long)i);
        }
        if (hp->local_sharpness != 0.0) fl |= F_LOCAL;
        if (hard && hp->echo_mix != 0.0) fl |= F_ECHO;
        const double ic = hard ? hp->instant_metric_coupling : 0.0;
        if (ic != 0.0 && D.N > 1) fl |= (d.ndim >= 2 ? F_INST2D : F_INST1D);  // rank >= 3: leading-axis factors
        if (fmax(hp->instant_metric_power, 0.25) == 1.0) fl |= F_IPOW1;
        if (vec[i]) fl |= F_VEC;
        full[i] = vec[i] && D.TC == 256 && d.cols % 256 == 0 && d.rows % D.RB == 0 && bins <= 256;
        D.flags = fl;
        // pointers into the caller's objects
        const char* ws = (const char*)d.shape_ws;
        ShapeWsHeader wh = shape_ws_layout(d.ndim, g_rows(d), D.gcols, rank, rm, bins,
                                           hash_on || bins > 0 ? tables : 0);
        if (bins == 0) wh = shape_ws_layout(d.ndim, g_rows(d), D.gcols, rank, rm, 0, 0);
        D.rowtab = (const float*)(ws + wh.off_rowtab);
        D.coltab = (const float*)(ws + wh.off_coltab);
        D.stats = (const ModeStats*)(ws + wh.off_stats);
        D.gram = (const double*)(ws + wh.off_gram);
        D.counts = (const float*)(ws + wh.off_counts);
        D.hidx = (const void*)d.hash_cache;
        D.hidx_n = d.hash_cache_n;
        D.param = (float*)d.param;
        D.grad = (const float*)d.grad;
        D.param_h = nullptr;
        D.grad_h = nullptr;
        if (d.dtype != CRESSO_DTYPE_F32) {  // rebound to the float32 copies by bind_scratch
            D.param_h = (void*)d.param;
            D.grad_h = (const void*)d.grad;
            D.flags |= d.dtype == CRESSO_DTYPE_F16 ? F_F16 : F_BF16;
        }
        D.omega = (float*)d.omega;
        D.q_cos = (float*)d.q_cos;
        D.q_sin = (float*)d.q_sin;
        D.p_cos = (float*)d.p_cos;
        D.p_sin = (float*)d.p_sin;
        D.m_cos = (float*)d.metric_cos;
        D.m_sin = (float*)d.metric_sin;
        D.mp_cos = (float*)d.metric_p_cos;
        D.mp_sin = (float*)d.metric_p_sin;
        D.ca_cos = (float*)d.calcium_cos;
        D.ca_sin = (float*)d.calcium_sin;
        D.conf = (float*)d.mode_confidence;
        D.h_energy = (float*)d.hash_energy;
        D.h_impulse = (float*)d.hash_impulse;
        D.h_refractory = (float*)d.hash_refractory;
        D.force_rms = (float*)d.force_rms;
        D.drive_energy = (float*)d.drive_energy;
        D.surprise = (float*)d.surprise;
        D.action = (float*)d.action;
        CRESSO_REQUIRE(D.omega && D.q_cos && D.q_sin && D.p_cos && D.p_sin && D.m_cos && D.m_sin && D.mp_cos &&
                           D.mp_sin && D.ca_cos && D.ca_sin && D.conf && D.force_rms && D.drive_energy &&
                           D.surprise && D.action,
                       CRESSO_EINVAL, "tensor %lld: NULL state pointer", (long long)i);
    }
    H.n_items = items;
    // the lean kernels of the full-tile class (spectral_fast.cuh): default hyper-parameters,
    // two tables of <= 64 bins (joint cache section), rank pad 8, 16-row items, and every
    // class-0 tensor with the hash and the axial instant metric on
    P.fast = rm == 8 && tables == 2 && bins >= 1 && bins <= 64 && iters == 16 && hp->weight_decay == 0.0 &&
             hp->local_sharpness == 0.0 && fmax(hp->instant_metric_power, 0.25) == 1.0;
    for (int64_t i = 0; i < n; ++i)
        if (full[i] && !(P.dts[i].flags & (F_F16 | F_BF16)))
            P.fast = P.fast && (P.dts[i].flags & F_HASH) && (P.dts[i].flags & F_INST2D);
    // the three launch classes: item lists in tensor order within each class
    P.item_lists.clear();
    P.tensor_lists.clear();
    for (int c = 0; c < 3; ++c) {
        int64_t ci = 0, cn = 0;
        for (int64_t i = 0; i < n; ++i) {
            const int ci_cls = !full[i] ? 1 : ((P.dts[i].flags & (F_F16 | F_BF16)) ? 2 : 0);
            if (ci_cls != c) continue;
            P.item_lists.push_back(ci);
            P.tensor_lists.push_back((int32_t)i);
            P.dts[i].item_base = ci;
            ci += P.dts[i].n_items;
            ++cn;
        }
        P.item_lists.push_back(ci);
        H.cls_items[c] = ci;
        H.cls_nt[c] = cn;
    }
    // blocks per pass and class, and record placement (a record per (block, tensor) pair)
    const int occ[6] = {0, 4, 2, 2, 2, 2};
    P.n_rec_max = 0;
    for (int p = 1; p <= 5; ++p) {
        int64_t rb = 0;
        int64_t tl_off = 0;
        for (int c = 0; c < 3; ++c) {
            const int64_t ci = H.cls_items[c];
            const int64_t g = ci == 0 ? 0 : std::max<int64_t>(1, std::min<int64_t>(ci, num_sms * (rm > 8 ? 1 : occ[p])));
            H.grid[c][p] = g;
            int64_t b = 0;
            const int32_t* tl = P.tensor_lists.data() + tl_off;
            tl_off += H.cls_nt[c];
            for (int64_t j = 0; j < H.cls_nt[c]; ++j) {
                DevTensor& D = P.dts[tl[j]];
                const int64_t first = D.item_base, last = D.item_base + D.n_items - 1;
                // block b of the class's launch owns items [b*ci/g, (b+1)*ci/g)
                while ((b + 1) * ci / g <= first) ++b;
                int64_t b_last = b;
                while ((b_last + 1) * ci / g <= last) ++b_last;
                D.cfirst[p] = (int32_t)b;
                D.recbase[p] = (int32_t)rb;
                D.nrec[p] = (int32_t)(b_last - b + 1);
                rb += D.nrec[p];
            }
        }
        P.n_rec_max = std::max(P.n_rec_max, rb);
    }
    for (int64_t i = 0; i < n; ++i) {
        const bool cls0 = full[i] && !(P.dts[i].flags & (F_F16 | F_BF16));
        P.dts[i].col_runs = (P.fast && cls0 && (P.dts[i].flags & F_INST2D)) ? 1 : 0;
    }

    // scratch layout
    int64_t off = 0;
    P.off_hdr = take(off, sizeof(GroupHdr));
    P.off_dts = take(off, sizeof(DevTensor) * n);
    P.off_items = take(off, sizeof(int64_t) * (n + 3));
    P.off_tmap = take(off, sizeof(int32_t) * n);
    P.off_status = take(off, sizeof(int32_t));
    P.off_cst = take(off, sizeof(TensorConsts) * n);
    int64_t rows_tot = 0, cols_tot = 0, rowpart_tot = 0, colpart_tot = 0, elems = 0;
    for (auto& D : P.dts) {
        rows_tot += D.rows;
        cols_tot += D.cols;
        rowpart_tot += (int64_t)D.n_ct * D.rows;
        colpart_tot += colpart_floats(D);
        elems += align_up(D.rows * D.cols, 64);
    }
    P.off_htab = take(off, 4 * std::max<int64_t>(H.tb, 1) * n);
    P.off_rowf = take(off, 4 * rows_tot);
    P.off_colf = take(off, 4 * cols_tot);
    P.off_rowpart = take(off, 4 * rowpart_tot);
    P.off_colpart = take(off, 4 * colpart_tot);
    P.off_recs = take(off, 8 * kNSRec * P.n_rec_max);
    P.off_recb = take(off, 4 * std::max<int64_t>(H.tb, 1) * P.n_rec_max);
    for (int p = 1; p <= 4; ++p) {
        int64_t len = 0;
        for (auto& D : P.dts) len += red_len(p, rm, H.tb, D.cols, D.ndim);
        P.len_red[p] = len;
        P.off_red[p] = take(off, 8 * len);
    }
    P.off_tbuf = take(off, 4 * elems);
    P.half_elems = 0;
    for (auto& D : P.dts)
        if (D.flags & (F_F16 | F_BF16)) P.half_elems += align_up(D.rows * D.cols, 64);
    // float32 parameter copies only when weight decay reads the parameter in P1-P3
    P.off_p32 = take(off, 4 * std::max<int64_t>(hp->weight_decay != 0.0 ? P.half_elems : 0, 1));
    P.bytes = off;
    return CRESSO_OK;
}

static void bind_scratch(Plan& P, char* base) {
    int64_t rows_o = 0, cols_o = 0, rowpart_o = 0, colpart_o = 0, elem_o = 0, red_o[5] = {0, 0, 0, 0, 0}, p32_o = 0;
    const int64_t tbs = std::max<int64_t>(P.hdr.tb, 1);
    for (size_t i = 0; i < P.dts.size(); ++i) {
        DevTensor& D = P.dts[i];
        D.cst = reinterpret_cast<TensorConsts*>(base + P.off_cst) + i;
        D.htab = reinterpret_cast<float*>(base + P.off_htab) + i * tbs;
        D.rowf = reinterpret_cast<float*>(base + P.off_rowf) + rows_o;
        D.colf = reinterpret_cast<float*>(base + P.off_colf) + cols_o;
        D.rowpart = reinterpret_cast<float*>(base + P.off_rowpart) + rowpart_o;
        D.colpart = reinterpret_cast<float*>(base + P.off_colpart) + colpart_o;
        D.tbuf = reinterpret_cast<float*>(base + P.off_tbuf) + elem_o;
        if (D.flags & (F_F16 | F_BF16)) {
            // the float32 parameter copy exists with weight decay only; without it no pass reads D.param
            D.param = P.hdr.hp[H_WD] != 0.0 ? reinterpret_cast<float*>(base + P.off_p32) + p32_o : nullptr;
            D.grad = D.tbuf;
            p32_o += align_up(D.rows * D.cols, 64);
        }
        for (int p = 1; p <= 4; ++p) {
            D.red[p] = reinterpret_cast<double*>(base + P.off_red[p]) + red_o[p];
            red_o[p] += red_len(p, P.rm, P.hdr.tb, D.cols, D.ndim);
        }
        D.red[0] = nullptr;
        rows_o += D.rows;
        cols_o += D.cols;
        rowpart_o += (int64_t)D.n_ct * D.rows;
        colpart_o += colpart_floats(D);
        elem_o += align_up(D.rows * D.cols, 64);
    }
}

static size_t pass_smem(int pass, const GroupHdr& H, int64_t iters, bool tc) {
    const int tb = (int)H.tb;
    const int rm = (int)H.rm;
    const int nacc = pass == 4 ? kWarps * 32 : (pass == 2 || pass == 3 ? 2 * rm * kThreads : 0);
    const int T2 = H.tables < 2 ? (int)H.tables : 2;
    const bool with_p = pass == 5 || (pass <= 3 && H.hp[H_WD] != 0.0);
    size_t b = 2 * (size_t)stage_bytes((int)iters, rm, pass >= 2 ? T2 : 0, (int)H.idx_bytes, with_p, (int)H.rb_max);
    b += (size_t)(kNSRec * kWarps + kNSRec + nacc) * sizeof(double);
    b += (size_t)(4 * rm + 4) * 4;
    if (pass == 2 || pass == 3) {
        b += (size_t)tb * (8 + 4) + (size_t)bin_copies(tb) * (tb + 1) * 4;
    }
    if (pass >= 3) b += (size_t)tb * 4;
    if (pass == 2) b += (size_t)(8 * iters + kThreads) * 4;
    if (tc) {
        // B tiles (128-byte aligned), mbarrier, TMEM slot, wait flag; and at least 78 KB so
        // that at most two blocks (2 x 256 TMEM columns) share an SM
        b += 128 + 4 * kTcTileBytes + 16;
        b = std::max<size_t>(b, 78 * 1024);
    }
    return b;
}

// 16-bit tensors: before P1, float32 copies of the gradient (into the tangent
// buffer, which P3 overwrites element by element after reading it) and, when
// weight decay reads it in P1-P3, of the parameter.  P5 updates the 16-bit
// parameter in place.  Eight elements per thread and step where the tensor
// allows 16-byte loads.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ void widen(const void* src_v, float* dst, int64_t N) {
    const T* src = reinterpret_cast<const T*>(src_v);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (((uintptr_t)src & 15) == 0 && (N & 7) == 0) {
        for (int64_t c = t0; c < N / 8; c += stride) {
            const uint4 raw = reinterpret_cast<const uint4*>(src)[c];
            const T* h = reinterpret_cast<const T*>(&raw);
            float4 a = make_float4(to_f32(h[0]), to_f32(h[1]), to_f32(h[2]), to_f32(h[3]));
            float4 b = make_float4(to_f32(h[4]), to_f32(h[5]), to_f32(h[6]), to_f32(h[7]));
            reinterpret_cast<float4*>(dst)[2 * c] = a;
            reinterpret_cast<float4*>(dst)[2 * c + 1] = b;
        }
    } else {
        for (int64_t e = t0; e < N; e += stride) dst[e] = to_f32(src[e]);
    }
}

__global__ void half_widen_kernel(const DevTensor* __restrict__ dts, int n, int with_param) {
    for (int k = blockIdx.y; k < n; k += gridDim.y) {
        const DevTensor& D = dts[k];
        const int fl = D.flags;
        if (!(fl & (F_F16 | F_BF16))) continue;
        const int64_t N = D.rows * D.cols;
        if (fl & F_BF16) {
            widen<__nv_bfloat16>(D.grad_h, D.tbuf, N);
            if (with_param) widen<__nv_bfloat16>(D.param_h, D.param, N);
        } else {
            widen<__half>(D.grad_h, D.tbuf, N);
            if (with_param) widen<__half>(D.param_h, D.param, N);
        }
    }
}

static int launch_half_widen(const Plan& P, char* base, cudaStream_t s) {
    if (P.half_elems == 0) return CRESSO_OK;
    const DevTensor* dts = reinterpret_cast<const DevTensor*>(base + P.off_dts);
    const int n = (int)P.hdr.n_tensors;
    dim3 grid(148, (unsigned)std::min(n, 65535));
    half_widen_kernel<<<grid, kThreads, 0, s>>>(dts, n, P.hdr.hp[H_WD] != 0.0 ? 1 : 0);
    CRESSO_LAUNCHED("half_widen_kernel");
    return CRESSO_OK;
}

// The bounded mbarrier wait of the tensor-core passes, on an mbarrier that
// completes only when `arrive` is set (one arrival by lane 0 before the wait):
// without it nothing ever arrives, the wait runs out after limit_ns and the
// kernel stores 1 in *status (0 when the phase completed).  No tensor-core
// work and no TMEM are involved, so running out leaves nothing in flight.
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, bool arrive, int32_t* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) {
            uint64_t token;
            asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];" : "=l"(token) : "r"(smem_u32(&bar)) : "memory");
            (void)token;
        }
        const bool ok = mbar_wait_bounded(smem_u32(&bar), 0, limit_ns);
        *status = ok ? 0 : 1;
    }
}

template <int RM, int NT>
static int launch_stage(int stage, const Plan& P, char* base, cudaStream_t s) {
    const GroupHdr* hdr = reinterpret_cast<const GroupHdr*>(base + P.off_hdr);
    const DevTensor* dts = reinterpret_cast<const DevTensor*>(base + P.off_dts);
    const int64_t* items = reinterpret_cast<const int64_t*>(base + P.off_items);
    const int32_t* tmap = reinterpret_cast<const int32_t*>(base + P.off_tmap);
    double* recs = reinterpret_cast<double*>(base + P.off_recs);
    float* recb = reinterpret_cast<float*>(base + P.off_recb);
    const int n = (int)P.hdr.n_tensors;
    // classes 0 and 2 of P3-P5 at rank pad 8 with 16-row items: the tensor-core kernels;
    // class 2 uses the 16-bit forms (which differ from class 0's in P5 only)
    auto run_pass = [&](auto kern_tc, auto kern_full, auto kern_gen, auto kern_tc16, auto kern_full16,
                        int pass) -> int {
        for (int c = 0; c < 3; ++c) {
            if (P.hdr.grid[c][pass] == 0) continue;
            if (c == 0 && P.fast && pass >= 2 && RM == 8 && NT == 2) {
                size_t off[13];
                size_t smem = fast_smem_layout(pass, (int)P.hdr.tb, off);
                if (pass >= 3) smem = std::max<size_t>(smem, 78 * 1024);  // two blocks per SM at most (TMEM)
                auto fk = pass == 2 ? fast_pass_kernel<2> : pass == 3 ? fast_pass_kernel<3>
                                                          : pass == 4 ? fast_pass_kernel<4> : fast_pass_kernel<5>;
                CRESSO_CUDA(cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                fk<<<(unsigned)P.hdr.grid[0][pass], kThreads, smem, s>>>(hdr, dts, items, tmap, recs, recb);
                CRESSO_LAUNCHED("fast_pass_kernel");
                continue;
            }
            const bool tc = c != 1 && pass >= 3 && RM == 8 && P.hdr.iters == 16;
            const size_t smem = pass_smem(pass, P.hdr, P.hdr.iters, tc);
            auto kern = c == 1 ? kern_gen : (c == 0 ? (tc ? kern_tc : kern_full) : (tc ? kern_tc16 : kern_full16));
            if (smem > 48 * 1024)
                CRESSO_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            int64_t lo = 0, to = 0;  // this class's item and tensor lists
            for (int k = 0; k < c; ++k) {
                lo += P.hdr.cls_nt[k] + 1;
                to += P.hdr.cls_nt[k];
            }
            kern<<<(unsigned)P.hdr.grid[c][pass], kThreads, smem, s>>>(hdr, dts, items + lo, tmap + to, recs, recb, c);
            CRESSO_LAUNCHED("spectral_pass_kernel");
        }
        return CRESSO_OK;
    };
    auto run_reduce = [&](int pass) -> int {
        const int64_t na = red_scal_len(pass, P.rm, P.hdr.tb);
        int64_t maxb = 0;  // column blocks of the tensor that needs the most
        for (auto& D : P.dts)
            maxb = std::max(maxb, ceil_div(red_len(pass, P.rm, P.hdr.tb, D.cols, D.ndim) - na,
                                           D.col_runs ? kThreads : kRedOutB));
        const int blocks_a = (int)ceil_div(na, kRedOutA);
        dim3 grid((unsigned)(blocks_a + maxb), (unsigned)n);
        reduce_kernel<<<grid, kThreads, 0, s>>>(pass, blocks_a, hdr, dts, recs, recb);
        CRESSO_LAUNCHED("reduce_kernel");
        return CRESSO_OK;
    };
    switch (stage) {
        case 1: return run_pass(spectral_pass_kernel<1, RM, NT, true, false>, spectral_pass_kernel<1, RM, NT, true, false>,
                            spectral_pass_kernel<1, RM, NT, false, false>, spectral_pass_kernel<1, RM, NT, true, false>,
                            spectral_pass_kernel<1, RM, NT, true, false>, 1);
        case 2: return run_reduce(1);
        case 3:
            finalize1_kernel<RM><<<n, kThreads, 0, s>>>(hdr, dts);
            CRESSO_LAUNCHED("finalize1_kernel");
            return CRESSO_OK;
        case 4: return run_pass(spectral_pass_kernel<2, RM, NT, true, false>, spectral_pass_kernel<2, RM, NT, true, false>,
                            spectral_pass_kernel<2, RM, NT, false, false>, spectral_pass_kernel<2, RM, NT, true, false>,
                            spectral_pass_kernel<2, RM, NT, true, false>, 2);
        case 5: return run_reduce(2);
        case 6: {
            // blocks 1.. of grid.y: the row / column factors of the 2-D tensors
            int64_t axis = 0;
            for (auto& D : P.dts)
                if ((D.flags & F_INST2D) && D.ndim == 2) axis = std::max<int64_t>(axis, std::max<int64_t>(D.rows, D.cols));
            const unsigned gy = 1 + (unsigned)std::min<int64_t>(ceil_div(axis, kThreads), 32);
            finalize2_kernel<RM><<<dim3((unsigned)n, gy), kThreads, 0, s>>>(hdr, dts);
            CRESSO_LAUNCHED("finalize2_kernel");
            return CRESSO_OK;
        }
        case 7: return run_pass(spectral_pass_kernel<3, RM, NT, true, RM == 8>, spectral_pass_kernel<3, RM, NT, true, false>,
                            spectral_pass_kernel<3, RM, NT, false, false>, spectral_pass_kernel<3, RM, NT, true, RM == 8>,
                            spectral_pass_kernel<3, RM, NT, true, false>, 3);
        case 8: return run_reduce(3);
        case 9:
            finalize3_kernel<RM><<<n, kThreads, 0, s>>>(hdr, dts);
            CRESSO_LAUNCHED("finalize3_kernel");
            return CRESSO_OK;
        case 10: return run_pass(spectral_pass_kernel<4, RM, NT, true, RM == 8>, spectral_pass_kernel<4, RM, NT, true, false>,
                            spectral_pass_kernel<4, RM, NT, false, false>, spectral_pass_kernel<4, RM, NT, true, RM == 8>,
                            spectral_pass_kernel<4, RM, NT, true, false>, 4);
        case 11: return run_reduce(4);
        case 12:
            finalize4_kernel<RM><<<n, kThreads, 0, s>>>(hdr, dts);
            CRESSO_LAUNCHED("finalize4_kernel");
            return CRESSO_OK;
        case 13: return run_pass(spectral_pass_kernel<5, RM, NT, true, RM == 8>, spectral_pass_kernel<5, RM, NT, true, false>,
                            spectral_pass_kernel<5, RM, NT, false, false>, spectral_pass_kernel<5, RM, NT, true, RM == 8, true>,
                            spectral_pass_kernel<5, RM, NT, true, false, true>, 5);
        default: return CRESSO_OK;
    }
}

}  // namespace cresso

using namespace cresso;

extern "C" {

int cresso_spectral_layout(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, int64_t num_sms,
                           int64_t* layout, int64_t layout_len) {
    CRESSO_REQUIRE(layout != nullptr && layout_len >= 9, CRESSO_EINVAL, "spectral_layout: need a layout array of >= 9");
    Plan P;
    int st = build_plan(descs, n, hp, num_sms, P);
    if (st) return st;
    layout[0] = P.bytes;
    for (int p = 1; p <= 4; ++p) {
        layout[2 * p - 1] = P.off_red[p];
        layout[2 * p] = P.len_red[p];
    }
    if (layout_len >= 10) layout[9] = P.off_status;
    if (layout_len >= 12) {
        layout[10] = P.hdr.iters;
        layout[11] = (P.hdr.cls_items[0] + P.hdr.cls_items[2] > 0 && P.rm == 8 && P.hdr.iters == 16) ? ((1 << 3) | (1 << 4) | (1 << 5)) : 0;
    }
    return CRESSO_OK;
}

int cresso_selftest_bounded_wait(int64_t limit_ns, int64_t arrive, void* status_word, cresso_stream_t stream) {
    CRESSO_REQUIRE(status_word != nullptr, CRESSO_EINVAL, "selftest_bounded_wait: NULL status word");
    CRESSO_REQUIRE(limit_ns >= 0 && limit_ns <= 2000000000LL, CRESSO_EINVAL,
                   "selftest_bounded_wait: limit must be in [0, 2 s]");
    bounded_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((uint64_t)limit_ns, arrive != 0,
                                                                      reinterpret_cast<int32_t*>(status_word));
    CRESSO_LAUNCHED("bounded_wait_selftest_kernel");
    return CRESSO_OK;
}

int cresso_spectral_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                        int64_t scratch_bytes, int64_t stage_begin, int64_t stage_end, int64_t num_sms,
                        cresso_stream_t stream) {
    return cresso_spectral_run_status(descs, n, hp, scratch, scratch_bytes, stage_begin, stage_end, num_sms, nullptr,
                                      stream);
}

int cresso_spectral_run_status(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                               int64_t scratch_bytes, int64_t stage_begin, int64_t stage_end, int64_t num_sms,
                               void* status_word, cresso_stream_t stream) {
    CRESSO_REQUIRE(status_word == nullptr || ((uintptr_t)status_word & 3) == 0, CRESSO_EINVAL,
                   "spectral_run: status word not 4-byte aligned");
    Plan P;
    int st = build_plan(descs, n, hp, num_sms, P);
    if (st) return st;
    CRESSO_REQUIRE(scratch != nullptr, CRESSO_EINVAL, "spectral_run: NULL scratch");
    CRESSO_REQUIRE(scratch_bytes >= P.bytes, CRESSO_ESCRATCH, "spectral_run: scratch of %lld bytes, need %lld",
                   (long long)scratch_bytes, (long long)P.bytes);
    CRESSO_REQUIRE(stage_begin >= 0 && stage_end <= kStages && stage_begin <= stage_end, CRESSO_EINVAL,
                   "spectral_run: stages must satisfy 0 <= begin <= end <= %d", kStages);
    char* base = (char*)scratch;
    cudaStream_t s = (cudaStream_t)stream;
    NvtxRange range("cresso_spectral_run %lld tensors, stages [%lld, %lld)", (long long)n, (long long)stage_begin,
                    (long long)stage_end);
    bind_scratch(P, base);
    // failure bits go to the caller's word (never cleared here) or to the scratch word,
    // which stage 0 clears
    P.hdr.status = status_word ? reinterpret_cast<int32_t*>(status_word) : reinterpret_cast<int32_t*>(base + P.off_status);
    if (stage_begin == 0) {
        // header, descriptors, item and tensor lists and the cleared scratch status word
        // lie back to back in the scratch: one upload of the whole range
        static thread_local std::vector<unsigned char> blob;
        const int64_t lo = P.off_hdr, hi = P.off_status + (int64_t)sizeof(int32_t);
        blob.assign((size_t)(hi - lo), 0);
        memcpy(blob.data() + (P.off_hdr - lo), &P.hdr, sizeof(GroupHdr));
        memcpy(blob.data() + (P.off_dts - lo), P.dts.data(), sizeof(DevTensor) * n);
        memcpy(blob.data() + (P.off_items - lo), P.item_lists.data(), sizeof(int64_t) * (n + 3));
        memcpy(blob.data() + (P.off_tmap - lo), P.tensor_lists.data(), sizeof(int32_t) * n);
        const int ust = upload_async(base + lo, blob.data(), blob.size(), s);
        if (ust) return ust;
        const int hs = launch_half_widen(P, base, s);
        if (hs) return hs;
    }
    static const char* const kStageName[kStages] = {
        "upload",     "P1 force energy", "reduce 1", "finalize 1", "P2 density / bins / projection",
        "reduce 2",   "finalize 2",      "P3 tangent / port", "reduce 3", "finalize 3",
        "P4 drive Gram", "reduce 4",     "finalize 4", "P5 update"};
    for (int64_t stage = std::max<int64_t>(stage_begin, 1); stage < stage_end; ++stage) {
        NvtxRange stage_range("cresso stage %lld: %s", (long long)stage, kStageName[stage]);
        const int nt = P.hdr.tables == 1 ? 1 : (P.hdr.tables == 2 ? 2 : 0);
        switch (P.rm * 4 + nt) {
            case 16: st = launch_stage<4, 0>((int)stage, P, base, s); break;
            case 17: st = launch_stage<4, 1>((int)stage, P, base, s); break;
            case 18: st = launch_stage<4, 2>((int)stage, P, base, s); break;
            case 32: st = launch_stage<8, 0>((int)stage, P, base, s); break;
            case 33: st = launch_stage<8, 1>((int)stage, P, base, s); break;
            case 34: st = launch_stage<8, 2>((int)stage, P, base, s); break;
            case 64: st = launch_stage<16, 0>((int)stage, P, base, s); break;
            case 65: st = launch_stage<16, 1>((int)stage, P, base, s); break;
            default: st = launch_stage<16, 2>((int)stage, P, base, s); break;
        }
        if (st) return st;
    }
    // The upload carried the plan in kernel parameters, copied at launch, so the
    // plan's host vectors may be released here.
    return CRESSO_OK;
}

}  // extern "C"
