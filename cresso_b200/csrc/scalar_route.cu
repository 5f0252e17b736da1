// Scalar-route CRESSO5 step (cresso_v5.py:1434-1582): LoRA-thin matrices and
// tensors below min_spectral_size.  All tensors of a group go in one launch
// per form (the reference needs 13 launches + 2 memsets per tensor,
// scalar_update_2d_cuda, cresso_cuda_kernel.cu:3225-3605, and covers only 2-D
// tensors; this file covers 0-d to 8-d):
//  * scalar_cluster_kernel (tensors of rank <= 2 whose slices fit): a
//    thread-block cluster per tensor keeps the tensor in shared memory across
//    the five stages and sums over the cluster through distributed shared
//    memory;
//  * scalar_route_kernel (the rest, e.g. N-d tensors): one 256-thread block
//    per tensor, re-reading the gradient between the stages.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <cooperative_groups.h>

#include <algorithm>
#include <vector>

#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

struct ScalTensor {
    int64_t ndim, N, rows, cols, step;
    int64_t dims[CRESSO_MAX_NDIM];
    int32_t TC, RPI, n_ct, nw;
    float* param;       // element type `dtype` (CRESSO_DTYPE_*)
    const float* grad;  // element type `dtype`
    float *q, *impulse, *metric_q, *metric_impulse, *force_rms, *drive_energy, *surprise, *action;
    float* work;  // per-tensor float scratch (row partials, row / column factors, N-d marginals)
    // cluster form: slices are row ranges (split_rows) or column ranges of `chunk` rows /
    // columns; ctc / crpi are the thread mapping of one slice
    int64_t chunk;
    int32_t split_rows, ctc, crpi, dtype;
};

struct ScalHdr {
    int64_t n;
    double hp[64];
};

// hparams indices (same field order as cresso_hparams)
enum {
    S_LR, S_WD, S_EP, S_DT, S_IF, S_CG, S_REST, S_CUBIC, S_MDT, S_MF, S_MC, S_LS, S_IC, S_IP, S_RCM, S_EM, S_TM,
    S_HD, S_HID, S_HMC, S_HDM, S_DFM, S_RFM, S_RD, S_REFD, S_RG, S_CD, S_CONFG, S_SG, S_SD, S_PM, S_NM, S_WS, S_SB,
    S_TGT, S_MING, S_MAXG, S_CLIP, S_SPIKE, S_EPS, S_MAX
};

template <typename W>
struct ScalShared {
    double red[16 * kWarps];
    double tot[16];
    W scale, inv_scale, metric, q_old, q_new, S, gm, inst_k;
    W c_u, c_root, c_t, c_pred, c_nov, gain, sp, invD;
    int inst_mode;  // 0 none, 1 one axis (per element), 2 rows x cols, 3 N-d marginals
};

__device__ __forceinline__ float sgnf_s(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }

// Walks the elements of a (rows, cols) view: the thread owns column lc of
// column tile ct and rows rs, rs + RPI, ...; `fn(e, r, c, ct, valid)` runs for
// every (thread, row slot), the same number of times in every thread, so it
// may contain warp shuffles and block barriers.  N-d tensors (ndim >= 3) are
// walked flat.

template <typename Fn>
__device__ __forceinline__ void walk_elems(const ScalTensor& D, Fn fn) {
    const int tid = threadIdx.x;
    if (D.ndim <= 2) {
        const int lc = tid & (D.TC - 1), rs = tid / D.TC;
        for (int ct = 0; ct < D.n_ct; ++ct) {
            const int64_t c = (int64_t)ct * D.TC + lc;
            for (int64_t r0 = 0; r0 < D.rows; r0 += D.RPI) {
                const int64_t r = r0 + rs;
                const bool valid = c < D.cols && r < D.rows;
                fn(valid ? r * D.cols + c : 0, r, c, ct, valid);
            }
        }
    } else {
        for (int64_t e0 = 0; e0 < D.N; e0 += kThreads) {
            const int64_t e = e0 + tid;
            fn(e < D.N ? e : 0, 0, 0, 0, e < D.N);
        }
    }
}

// Product of the per-axis instant factors of element e of an N-d tensor;
// work holds the factors of axis a at [sum(dims[:a]), sum(dims[:a+1])).
template <typename W>
__device__ __forceinline__ W nd_factor(const ScalTensor& D, int64_t e) {
    const W* work = reinterpret_cast<const W*>(D.work);
    W prod = W(1.0);
    int64_t rem = e;
    int64_t base = 0;
    for (int64_t a = 0; a < D.ndim; ++a) base += D.dims[a];
    for (int64_t a = D.ndim - 1; a >= 0; --a) {
        base -= D.dims[a];
        const int64_t coord = rem % D.dims[a];
        rem /= D.dims[a];
        prod *= work[base + coord];
    }
    return prod;
}

template <typename W>
__global__ void __launch_bounds__(kThreads) scalar_route_kernel(const ScalHdr* __restrict__ hdr,
                                                                 const ScalTensor* __restrict__ dts) {
    __shared__ ScalShared<W> sh;
    const ScalTensor& D = dts[blockIdx.x];
    W* work = reinterpret_cast<W*>(D.work);
    auto st = [](float* ptr) { return reinterpret_cast<W*>(ptr); };  // 0-d state of the work type
    const double* hp = hdr->hp;
    const int tid = threadIdx.x, lane = tid & 31;
    const W eps = (W)hp[S_EPS];
    const W sgn = hp[S_MAX] != 0.0 ? -W(1.0) : W(1.0);
    const W wd = (W)hp[S_WD];
    const bool wd_on = hp[S_WD] != 0.0;
    const double N = (double)D.N;
    auto force = [&](int64_t e) {
        W f = sgn * load_w<W>(D.grad, e, D.dtype);
        if (wd_on) f = f + wd * load_w<W>(D.param, e, D.dtype);
        return f;
    };

    // ---- stage 1: force energy -> force_rms, scale  (cresso_v5.py:1505-1508)
    {
        double s = 0.0;
        walk_elems(D, [&](int64_t e, int64_t, int64_t, int, bool valid) {
            if (valid) {
                const W f = force(e);
                s += (double)(f * f);
            }
        });
        double v[1] = {s};
        block_sum_to<1>(v, sh.red, sh.tot);
        if (tid == 0) {
            const W frn = w_sqrt((W)(sh.tot[0] / N) + eps);
            const W fr = reservoir(*st(D.force_rms), frn, hp[S_RD], D.step);
            *st(D.force_rms) = fr;
            sh.scale = w_max(fr, eps);
            sh.inv_scale = W(1.0) / sh.scale;
        }
        __syncthreads();
    }
    const W scale = sh.scale, inv_scale = sh.inv_scale;
    const W ep = (W)hp[S_EP];
    const W pw = w_max((W)hp[S_IP], W(0.25));
    const bool ipow1 = pw == W(1.0);
    const W ic = (W)hp[S_IC];
    int inst_mode = 0;
    if (ic != W(0.0) && D.ndim > 0 && D.N > 1) inst_mode = D.ndim == 1 ? 1 : (D.ndim == 2 ? 2 : 3);
    auto dens = [&](W rel) { return ipow1 ? rel : w_min(w_pow(w_max(rel, eps), pw), W(1.0e6)); };

    // ---- stage 2: density metric and the instant-metric axis sums  (cresso_v5.py:1510-1525)
    {
        W* rowpart = work;  // [n_ct * nw][rows]
        const int nw = D.nw;
        W* colsum = work + (int64_t)D.n_ct * nw * D.rows + D.rows;  // [cols]
        __syncthreads();
        double sL = 0.0, sd = 0.0;
        W colacc = W(0.0);
        __shared__ W s_col[kThreads];
        const int lc = tid & (D.TC - 1), rs = tid / D.TC;
        int cur_ct = -1;
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int ct, bool valid) {
            if (D.ndim <= 2 && ct != cur_ct) {
                if (cur_ct >= 0) {  // flush column sums of the previous tile
                    s_col[tid] = colacc;
                    __syncthreads();
                    const int64_t cc = (int64_t)cur_ct * D.TC + lc;
                    if (rs == 0 && cc < D.cols) {
                        W s = W(0.0);
                        for (int q = 0; q < D.RPI; ++q) s += s_col[q * D.TC + lc];
                        colsum[cc] = s;
                    }
                    __syncthreads();
                }
                colacc = W(0.0);
                cur_ct = ct;
            }
            W d = W(0.0);
            if (valid) {
                const W f = force(e);
                const W rel0 = w_abs(f) * inv_scale + eps;
                sL += (double)w_log1p(w_pow(rel0, ep));
                const W rel = w_min(rel0, W(1.0e4));
                d = dens(rel);
                sd += (double)d;
                colacc += d;
            }
            if (inst_mode == 2) {
                W v = d;
                const int w = min(D.TC, 32);
                for (int o = w >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const bool leader = D.TC <= 32 ? (lc == 0) : (lane == 0);
                const int wi = D.TC <= 32 ? 0 : (lc >> 5);
                if (leader && r < D.rows) rowpart[((int64_t)ct * nw + wi) * D.rows + r] = v;
            }
        });
        if (D.ndim <= 2 && cur_ct >= 0) {
            s_col[tid] = colacc;
            __syncthreads();
            const int64_t cc = (int64_t)cur_ct * D.TC + lc;
            if (rs == 0 && cc < D.cols) {
                W s = W(0.0);
                for (int q = 0; q < D.RPI; ++q) s += s_col[q * D.TC + lc];
                colsum[cc] = s;
            }
        }
        double v[2] = {sL, sd};
        block_sum_to<2>(v, sh.red, sh.tot);  // includes __syncthreads
        if (tid == 0) {
            // metric oscillator on the scalar density  (cresso_v5.py:1510-1519)
            const W density = (W)(sh.tot[0] / N);
            const W mq0 = *st(D.metric_q);
            const W port = density - w_tanh(mq0);
            const W mdt = (W)hp[S_MDT];
            W mp = *st(D.metric_impulse) * (W)fmax(0.0, 1.0 - hp[S_MDT] * hp[S_MF]);
            mp = mp + mdt * (port - mq0);
            const W mq = clampw(mq0 + mdt * mp, -W(3.0), W(3.0));
            *st(D.metric_impulse) = mp;
            *st(D.metric_q) = mq;
            sh.metric = clampw(w_exp((W)hp[S_MC] * mq), W(0.06), W(16.0));
            sh.gm = w_max((W)(sh.tot[1] / N), eps);
            sh.inst_k = ic / ((W)(D.ndim > 1 ? D.ndim : 1) * pw);
            sh.q_old = *st(D.q);
        }
        __syncthreads();
        // per-axis factors exp(k * log(max(mean / gmean, eps)))  (cresso_v5.py:243-262)
        const W gm = sh.gm, kk = sh.inst_k;
        if (inst_mode == 2) {
            W* rowf = work + (int64_t)D.n_ct * nw * D.rows;
            for (int64_t r = tid; r < D.rows; r += kThreads) {
                double s = 0.0;
                for (int64_t j = 0; j < (int64_t)D.n_ct * nw; ++j) s += (double)rowpart[j * D.rows + r];
                rowf[r] = w_exp(kk * w_log(w_max((W)(s / (double)D.cols) / gm, eps)));
            }
            for (int64_t c = tid; c < D.cols; c += kThreads)
                colsum[c] = w_exp(kk * w_log(w_max((W)((double)colsum[c] / (double)D.rows) / gm, eps)));
        } else if (inst_mode == 3) {
            // N-d marginals: one thread per (axis, coordinate) sums its slab in a fixed
            // order (deterministic), then turns the mean into the axis factor.
            int64_t tot = 0;
            for (int64_t a = 0; a < D.ndim; ++a) tot += D.dims[a];
            for (int64_t j = tid; j < tot; j += kThreads) {
                int64_t a = 0, c = j;
                while (c >= D.dims[a]) {
                    c -= D.dims[a];
                    ++a;
                }
                int64_t inner = 1;
                for (int64_t b = a + 1; b < D.ndim; ++b) inner *= D.dims[b];
                const int64_t outer = D.N / (D.dims[a] * inner);
                double m = 0.0;
                for (int64_t o = 0; o < outer; ++o)
                    for (int64_t i = 0; i < inner; ++i) {
                        const int64_t e = (o * D.dims[a] + c) * inner + i;
                        const W f = force(e);
                        m += (double)dens(w_min(w_abs(f) * inv_scale + eps, W(1.0e4)));
                    }
                const double per = N / (double)D.dims[a];
                work[j] = w_exp(kk * w_log(w_max((W)(m / per) / gm, eps)));
            }
        }
        __syncthreads();
    }

    const W metric = sh.metric, gm = sh.gm, kk = sh.inst_k;
    const W ls = (W)hp[S_LS];
    const bool local_on = hp[S_LS] != 0.0;
    const W* rowf = work + (int64_t)D.n_ct * D.nw * D.rows;
    const W* colf = rowf + D.rows;
    auto tangent = [&](int64_t e, int64_t r, int64_t c) {
        const W f = force(e);
        const W rel = w_min(w_abs(f) * inv_scale + eps, W(1.0e4));
        W den = scale * metric;
        if (local_on) den = den * clampw(W(1.0) + ls * w_sqrt(w_min(rel, W(100.0))), W(1.0), W(8.0));
        if (inst_mode == 1) {
            den = den * clampw(w_exp(kk * w_log(w_max(dens(rel) / gm, eps))), W(0.08), W(12.0));
        } else if (inst_mode == 2) {
            den = den * clampw(rowf[r] * colf[c], W(0.08), W(12.0));
        } else if (inst_mode == 3) {
            den = den * clampw(nd_factor<W>(D, e), W(0.08), W(12.0));
        }
        return clampw(w_div(f, den + eps), -W(1.0e4), W(1.0e4));
    };

    // ---- stage 3: prediction error, surprise, scalar contact  (cresso_v5.py:1526-1546)
    {
        const W q0 = sh.q_old;
        double se = 0.0, se2 = 0.0;
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int, bool valid) {
            if (valid) {
                const W err = tangent(e, r, c) - q0;
                se += (double)err;
                se2 += (double)(err * err);
            }
        });
        double v[2] = {se, se2};
        block_sum_to<2>(v, sh.red, sh.tot);
        if (tid == 0) {
            const W sn = w_sqrt((W)(sh.tot[1] / N) + eps);
            const W S = reservoir(*st(D.surprise), sn, hp[S_SD], D.step);
            *st(D.surprise) = S;
            const W port = (W)(sh.tot[0] / N);
            const W dt = (W)hp[S_DT];
            const W plast = W(1.0) + (W)hp[S_SG] * S / (W(1.0) + S);
            const W brake = W(1.0) / (W(1.0) + (W)hp[S_SB] * S);
            W imp = *st(D.impulse), q = q0, action = *st(D.action);
            const W energy = W(0.5) * (imp * imp + q * q);
            action = action * W(0.985) + (port * imp - energy) * dt;
            const W fr = (W)hp[S_IF] + (W)hp[S_CG] * w_tanh(w_abs(action));
            imp = imp * w_max(W(1.0) - dt * fr, W(0.0));
            imp = imp + dt * (plast * brake * port - (W)hp[S_REST] * q - (W)hp[S_CUBIC] * (q * q * q));
            q = clampw(q + dt * imp, -W(8.0), W(8.0));
            *st(D.impulse) = imp;
            *st(D.action) = action;
            *st(D.q) = q;
            sh.q_new = q;
            sh.S = S;
            const W clip = (W)hp[S_CLIP];
            sh.sp = (W)hp[S_SPIKE] / (W(1.0) + S);
            sh.invD = W(1.0) / (clip * (W(1.0) + S));
        }
        __syncthreads();
    }

    const W qn = sh.q_new, S = sh.S, sp = sh.sp, invD = sh.invD;
    const W clip = (W)hp[S_CLIP], inv_clip = W(1.0) / clip, clip2 = (W)(hp[S_CLIP] * hp[S_CLIP]);
    struct Parts {
        W u, root, t, nov, rat;
    };
    auto parts = [&](int64_t e, int64_t r, int64_t c) {
        Parts P;
        P.t = tangent(e, r, c);
        const W at = w_abs(P.t);
        P.rat = P.t / (W(1.0) + at * inv_clip);
        const W bnd = w_tanh(P.t * inv_clip) * clip;
        P.root = w_sgn(P.t) * w_sqrt(w_min(at, clip2) + eps);
        P.u = (W(1.0) - sp) * P.rat + sp * bnd;
        P.nov = w_tanh((P.t - qn) * invD) * clip;
        return P;
    };

    // ---- stage 4: drive statistics as a Gram of (u, root, t, pred, nov)  (cresso_v5.py:1548-1581)
    {
        double g[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) g[j] = 0.0;
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int, bool valid) {
            if (valid) {
                const Parts P = parts(e, r, c);
                const W v[5] = {P.u, P.root, P.t, qn, P.nov};
                int j = 0;
#pragma unroll
                for (int a = 0; a < 5; ++a)
#pragma unroll
                    for (int b = a; b < 5; ++b) g[j++] += (double)(v[a] * v[b]);
                g[15] += (double)(P.rat * P.rat);
            }
        });
        block_sum_to<16>(g, sh.red, sh.tot);
        if (tid == 0) {
            const double* G = sh.tot;
            auto Gm = [&](int a, int b) {
                if (a > b) { const int t = a; a = b; b = t; }
                return G[a * 5 - (a * (a - 1)) / 2 + (b - a)];
            };
            enum { U = 0, RT = 1, TT = 2, PR = 3, NV = 4 };
            const W frms = w_sqrt((W)(Gm(TT, TT) / N) + eps);
            const W prms = w_sqrt((W)(Gm(PR, PR) / N) + eps);
            const W align = clampw((W)(Gm(TT, PR) / N) / (frms * prms + eps), -W(1.0), W(1.0));
            const W align_gate = prms > (W)sqrt(hp[S_EPS]) ? clampw((align + W(1.0)) * W(0.5), W(0.0), W(1.0)) : W(0.0);
            const int ws = (int)hp[S_WS];
            const double warm = ws == 0 ? 1.0 : (1.0 - exp(-(double)D.step / (double)(ws > 1 ? ws : 1)));
            const W mix = (W)(hp[S_PM] * warm) * align_gate / (W(1.0) + S);
            const W rat_rms = w_sqrt((W)(G[15] / N) + eps);
            const W root_rms = w_sqrt((W)(Gm(RT, RT) / N) + eps);
            const W k_root = rat_rms / w_max(root_rms, eps);
            const W root_mix = (W)hp[S_RCM] / (W(1.0) + W(0.5) * S);
            const double a = 1.0 - (double)root_mix, b = (double)root_mix * (double)k_root;
            const double sh2 = a * a * Gm(U, U) + 2.0 * a * b * Gm(U, RT) + b * b * Gm(RT, RT);
            const W shaped_rms = w_sqrt((W)(sh2 / N) + eps);
            const W dm = (W)hp[S_DFM] / (W(1.0) + W(0.35) * S);
            const W k_d = shaped_rms / w_max(frms, eps);
            const double cu = (1.0 - dm) * a, cr = (1.0 - dm) * b, ctt = (double)dm * k_d;
            const double core2 = cu * cu * Gm(U, U) + cr * cr * Gm(RT, RT) + ctt * ctt * Gm(TT, TT) +
                                 2.0 * (cu * cr * Gm(U, RT) + cu * ctt * Gm(U, TT) + cr * ctt * Gm(RT, TT));
            const W core_rms = w_sqrt((W)(core2 / N) + eps);
            const W resm = (W)hp[S_RFM] / (W(1.0) + S);
            const double err2 = Gm(TT, TT) - 2.0 * Gm(TT, PR) + Gm(PR, PR);
            const W k_r = core_rms / w_max(w_sqrt((W)(fmax(err2, 0.0) / N) + eps), eps);
            double c[5];
            c[U] = (1.0 - mix) * cu;
            c[RT] = (1.0 - mix) * cr;
            c[TT] = (1.0 - mix) * ctt + (double)resm * k_r;
            c[PR] = (double)mix - (double)resm * k_r;
            c[NV] = hp[S_NM];
            double d2 = 0.0;
            for (int i = 0; i < 5; ++i)
                for (int j = 0; j < 5; ++j) d2 += c[i] * c[j] * Gm(i, j);
            const W den = (W)(fmax(d2, 0.0) / N);
            const W DE = reservoir(*st(D.drive_energy), den, hp[S_RD], D.step);
            *st(D.drive_energy) = DE;
            sh.gain = clampw((W)hp[S_TGT] / w_sqrt(DE + eps), (W)hp[S_MING], (W)hp[S_MAXG]);
            sh.c_u = (W)c[U];
            sh.c_root = (W)c[RT];
            sh.c_t = (W)c[TT];
            sh.c_pred = (W)c[PR];
            sh.c_nov = (W)c[NV];
        }
        __syncthreads();
    }

    // ---- stage 5: parameter update  (cresso_v5.py:1582)
    {
        const W cu = sh.c_u, cr = sh.c_root, ctt = sh.c_t, cp = sh.c_pred, cn = sh.c_nov, gain = sh.gain;
        const W neg_lr = (W)(-hp[S_LR]);
        const W neg_lr16 = neg_lr_w<W>(hp[S_LR], D.dtype);
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int, bool valid) {
            if (valid) {
                const Parts P = parts(e, r, c);
                const W drive = cu * P.u + cr * P.root + ctt * P.t + cp * qn + cn * P.nov;
                apply_update_w<W>(D.param, e, D.dtype, neg_lr, neg_lr16, drive * gain);
            }
        });
    }
}

// ---------------------------------------------------------------------------
// Cluster form of the scalar route (tensors of rank <= 2 that fit).
//
// A cluster of CS CTAs steps one tensor.  The tensor is cut along its longer
// axis into CS slices; CTA k keeps the force field of slice k in shared memory
// for the whole step, so the gradient is read from HBM once and the parameter
// once (plus once more when weight decay is on) and written once.  The five
// stages are those of scalar_route_kernel; each global sum is a block sum in
// every CTA, published in that CTA's shared memory, and added up over the
// cluster's CTAs in rank order through distributed shared memory, so every
// CTA obtains the same totals and runs the same scalar arithmetic.  The axis
// sums of the instant metric are complete inside a CTA along the split axis;
// the other axis's partial sums are added up over the cluster the same way.
// CTA 0 alone writes the scalar state, and every CTA reads the old state
// before the first cluster barrier.
// ---------------------------------------------------------------------------
namespace cg = cooperative_groups;

constexpr int kClMax = 8;         // CTAs per cluster (portable maximum)
constexpr int kClSlice = 16384;   // slice elements held in shared memory (with the row pad)
constexpr int kClShort = 1024;    // longest unsplit axis
constexpr int kClLocal = 4096;    // longest slice along the split axis

struct ClShared {
    double red[16 * kWarps];
    double tot[16];
    double slot1[1], slot2[2], slot3[2], slot4[16];  // this CTA's block totals, read by the cluster
    double all[16];                                  // cluster totals
    float scale, inv_scale, metric, gm, inst_k, q_new, S, sp, invD;
    float c_u, c_root, c_t, c_pred, c_nov, gain;
};

// Sums the K block totals of every CTA of the cluster in rank order into sh.all.
template <int K>
__device__ __forceinline__ void cluster_sum(cg::cluster_group& cl, double (&v)[K], double* slot, ClShared& sh) {
    block_sum_to<K>(v, sh.red, sh.tot);
    if (threadIdx.x < K) slot[threadIdx.x] = sh.tot[threadIdx.x];
    cl.sync();
    if (threadIdx.x < K) {
        double s = 0.0;
        for (unsigned r = 0; r < cl.num_blocks(); ++r) s += cl.map_shared_rank(slot, r)[threadIdx.x];
        sh.all[threadIdx.x] = s;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 4) scalar_cluster_kernel(const ScalHdr* __restrict__ hdr,
                                                                   const ScalTensor* __restrict__ dts,
                                                                   int slice_cap, int loc_cap, int short_cap) {
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank(), cs = (int)cl.num_blocks();
    const ScalTensor& D = dts[blockIdx.x / cs];
    extern __shared__ __align__(16) float smf[];
    float* F = smf;                       // slice: force, then tangent   [slice_cap]
    float* loc_sum = F + slice_cap;       // split-axis sums, then factors [loc_cap]
    float* sh_part = loc_sum + loc_cap;   // this CTA's partial sums of the other axis [short_cap]
    float* sh_fac = sh_part + short_cap;  // the other axis's factors [short_cap]
    __shared__ ClShared sh;
    const double* hp = hdr->hp;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float eps = (float)hp[S_EPS];
    const float sgn = hp[S_MAX] != 0.0 ? -1.0f : 1.0f;
    const float wd = (float)hp[S_WD];
    const bool wd_on = hp[S_WD] != 0.0;
    const double N = (double)D.N;
    const int64_t cols = D.cols;
    const float* __restrict__ grad = D.grad;
    float* __restrict__ param = D.param;
    const int dt = D.dtype;

    // slice geometry
    const bool sr = D.split_rows != 0;
    const int64_t long_len = sr ? D.rows : D.cols;
    const int64_t lo = (int64_t)rank * D.chunk;
    const int64_t nloc = lo < long_len ? min(D.chunk, long_len - lo) : 0;
    const int64_t lrows = sr ? nloc : D.rows, lcols = sr ? D.cols : nloc;
    const int64_t r_off = sr ? lo : 0, c_off = sr ? 0 : lo;
    const int64_t ld = (lcols & 1) ? lcols : lcols + 1;  // odd row pitch: conflict-free column sweeps
    const int TC = D.ctc, RPI = D.crpi;
    const int lc = tid & (TC - 1), rs = tid / TC;
    auto for_slice = [&](auto fn) {  // fn(i, j, shared index, global index); no barriers inside
        for (int64_t j0 = 0; j0 < lcols; j0 += TC) {
            const int64_t j = j0 + lc;
            if (j < lcols) {
                int64_t i = rs;
                for (; i + 3 * RPI < lrows; i += 4 * RPI) {
                    fn(i, j, i * ld + j, (i + r_off) * cols + j + c_off);
                    fn(i + RPI, j, (i + RPI) * ld + j, (i + RPI + r_off) * cols + j + c_off);
                    fn(i + 2 * RPI, j, (i + 2 * RPI) * ld + j, (i + 2 * RPI + r_off) * cols + j + c_off);
                    fn(i + 3 * RPI, j, (i + 3 * RPI) * ld + j, (i + 3 * RPI + r_off) * cols + j + c_off);
                }
                for (; i < lrows; i += RPI) fn(i, j, i * ld + j, (i + r_off) * cols + j + c_off);
            }
        }
    };

    // the old scalar state, read before any CTA of the cluster writes it
    float st_fr = 0.f, st_mq = 0.f, st_mp = 0.f, st_q = 0.f, st_S = 0.f, st_imp = 0.f, st_act = 0.f, st_de = 0.f;
    if (tid == 0) {
        st_fr = *D.force_rms;
        st_mq = *D.metric_q;
        st_mp = *D.metric_impulse;
        st_q = *D.q;
        st_S = *D.surprise;
        st_imp = *D.impulse;
        st_act = *D.action;
        st_de = *D.drive_energy;
    }
    const bool writer = rank == 0 && tid == 0;

    // ---- stage 1: force field into shared memory, force energy -> force_rms, scale
    {
        // float partials over this thread's elements (at most kClSlice / kThreads), float64 above
        float a0 = 0.0f;
        for_slice([&](int64_t, int64_t, int64_t q, int64_t e) {
            float f = sgn * (dt == CRESSO_DTYPE_F32 ? __ldg(grad + e) : load_elem(grad, e, dt));
            if (wd_on) f = f + wd * (dt == CRESSO_DTYPE_F32 ? param[e] : load_elem(param, e, dt));
            F[q] = f;
            a0 = fmaf(f, f, a0);
        });
        double v[1] = {(double)a0};
        cluster_sum<1>(cl, v, sh.slot1, sh);
        if (tid == 0) {
            const float frn = sqrtf((float)(sh.all[0] / N) + eps);
            const float fr = reservoir(st_fr, frn, hp[S_RD], D.step);
            if (writer) *D.force_rms = fr;
            sh.scale = fmaxf(fr, eps);
            sh.inv_scale = 1.0f / sh.scale;
        }
        __syncthreads();
    }
    const float scale = sh.scale, inv_scale = sh.inv_scale;
    const float ep = (float)hp[S_EP];
    const float pw = fmaxf((float)hp[S_IP], 0.25f);
    const bool ipow1 = pw == 1.0f;
    const float ic = (float)hp[S_IC];
    int inst_mode = 0;
    if (ic != 0.0f && D.ndim > 0 && D.N > 1) inst_mode = D.ndim == 1 ? 1 : 2;
    auto dens = [&](float rel) { return ipow1 ? rel : fminf(powf(fmaxf(rel, eps), pw), 1.0e6f); };
    auto dens_of = [&](float f) { return dens(fminf(fabsf(f) * inv_scale + eps, 1.0e4f)); };

    // ---- stage 2: density metric and the instant-metric axis sums
    {
        float a0 = 0.0f, a1 = 0.0f;
        for_slice([&](int64_t, int64_t, int64_t q, int64_t) {
            const float rel0 = fabsf(F[q]) * inv_scale + eps;  // >= eps > 0 (normal)
            a0 += log1p_pos(exp2f(ep * __log2f(rel0)));
            a1 += dens(fminf(rel0, 1.0e4f));
        });
        double v[2] = {(double)a0, (double)a1};
        if (inst_mode == 2) {
            // split-axis sums (complete here) and this CTA's part of the other axis's sums:
            // one warp per line, lanes along it, float partials added in a fixed order
            const int64_t n_loc = sr ? lrows : lcols, n_sh = sr ? lcols : lrows;
            for (int64_t a = warp; a < n_loc + n_sh; a += kWarps) {
                const bool is_loc = a < n_loc;
                const int64_t idx = is_loc ? a : a - n_loc;
                const bool is_row = is_loc == sr;  // a row of the slice
                const int64_t len = is_row ? lcols : lrows;
                float s = 0.0f;
                for (int64_t b = lane; b < len; b += 32) s += dens_of(F[is_row ? idx * ld + b : b * ld + idx]);
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) (is_loc ? loc_sum : sh_part)[idx] = s;
            }
        }
        cluster_sum<2>(cl, v, sh.slot2, sh);  // its cluster barrier also publishes sh_part
        if (tid == 0) {
            // metric oscillator on the scalar density  (cresso_v5.py:1510-1519)
            const float density = (float)(sh.all[0] / N);
            const float port = density - tanhf(st_mq);
            const float mdt = (float)hp[S_MDT];
            float mp = st_mp * (float)fmax(0.0, 1.0 - hp[S_MDT] * hp[S_MF]);
            mp = mp + mdt * (port - st_mq);
            const float mq = clampf(st_mq + mdt * mp, -3.0f, 3.0f);
            if (writer) {
                *D.metric_impulse = mp;
                *D.metric_q = mq;
            }
            sh.metric = clampf(expf((float)hp[S_MC] * mq), 0.06f, 16.0f);
            sh.gm = fmaxf((float)(sh.all[1] / N), eps);
            sh.inst_k = ic / ((float)(D.ndim > 1 ? D.ndim : 1) * pw);
        }
        __syncthreads();
        if (inst_mode == 2) {
            // per-axis factors exp(k * log(max(mean / gmean, eps)))  (cresso_v5.py:243-262)
            const float gm = sh.gm, kk = sh.inst_k;
            const int64_t n_loc = sr ? lrows : lcols, n_sh = sr ? lcols : lrows;
            const double len_loc = (double)(sr ? D.cols : D.rows), len_sh = (double)(sr ? D.rows : D.cols);
            for (int64_t a = tid; a < n_loc; a += kThreads)
                loc_sum[a] = expf(kk * logf(fmaxf((float)((double)loc_sum[a] / len_loc) / gm, eps)));
            for (int64_t a = tid; a < n_sh; a += kThreads) {
                double t = 0.0;
                for (int r = 0; r < cs; ++r) t += (double)cl.map_shared_rank(sh_part, r)[a];
                sh_fac[a] = expf(kk * logf(fmaxf((float)(t / len_sh) / gm, eps)));
            }
            __syncthreads();
        }
    }

    const float metric = sh.metric, gm = sh.gm, kk = sh.inst_k;
    const float ls = (float)hp[S_LS];
    const bool local_on = hp[S_LS] != 0.0;
    const float* rowf = sr ? loc_sum : sh_fac;  // indexed by local row
    const float* colf = sr ? sh_fac : loc_sum;  // indexed by local column
    auto tangent = [&](float f, int64_t i, int64_t j) {
        const float rel = fminf(fabsf(f) * inv_scale + eps, 1.0e4f);
        float den = scale * metric;
        if (local_on) den = den * clampf(1.0f + ls * sqrt_sfu(fminf(rel, 100.0f)), 1.0f, 8.0f);
        if (inst_mode == 1) {
            den = den * clampf(expf(kk * logf(fmaxf(dens(rel) / gm, eps))), 0.08f, 12.0f);
        } else if (inst_mode == 2) {
            den = den * clampf(rowf[i] * colf[j], 0.08f, 12.0f);
        }
        return clampf(__fdividef(f, den + eps), -1.0e4f, 1.0e4f);
    };

    // ---- stage 3: tangent (kept in place of the force), prediction error, surprise, contact
    {
        const float q0 = st_q;
        float q0b;
        if (tid == 0) sh.q_new = q0;  // broadcast of the old q (only thread 0 read it)
        __syncthreads();
        q0b = sh.q_new;
        float a0 = 0.0f, a1 = 0.0f;
        for_slice([&](int64_t i, int64_t j, int64_t q, int64_t) {
            const float t = tangent(F[q], i, j);
            F[q] = t;
            const float err = t - q0b;
            a0 += err;
            a1 = fmaf(err, err, a1);
        });
        double v[2] = {(double)a0, (double)a1};
        cluster_sum<2>(cl, v, sh.slot3, sh);
        if (tid == 0) {
            const float sn = sqrtf((float)(sh.all[1] / N) + eps);
            const float S = reservoir(st_S, sn, hp[S_SD], D.step);
            const float port = (float)(sh.all[0] / N);
            const float dt = (float)hp[S_DT];
            const float plast = 1.0f + (float)hp[S_SG] * S / (1.0f + S);
            const float brake = 1.0f / (1.0f + (float)hp[S_SB] * S);
            float imp = st_imp, q = q0, action = st_act;
            const float energy = 0.5f * (imp * imp + q * q);
            action = action * 0.985f + (port * imp - energy) * dt;
            const float fr = (float)hp[S_IF] + (float)hp[S_CG] * tanhf(fabsf(action));
            imp = imp * fmaxf(1.0f - dt * fr, 0.0f);
            imp = imp + dt * (plast * brake * port - (float)hp[S_REST] * q - (float)hp[S_CUBIC] * (q * q * q));
            q = clampf(q + dt * imp, -8.0f, 8.0f);
            if (writer) {
                *D.surprise = S;
                *D.impulse = imp;
                *D.action = action;
                *D.q = q;
            }
            sh.q_new = q;
            sh.S = S;
            sh.sp = (float)hp[S_SPIKE] / (1.0f + S);
            sh.invD = 1.0f / ((float)hp[S_CLIP] * (1.0f + S));
        }
        __syncthreads();
    }

    const float qn = sh.q_new, S = sh.S, sp = sh.sp, invD = sh.invD;
    const float clip = (float)hp[S_CLIP], inv_clip = 1.0f / clip, clip2 = (float)(hp[S_CLIP] * hp[S_CLIP]);
    struct Parts {
        float u, root, t, nov, rat;
    };
    auto parts = [&](float t) {
        Parts P;
        P.t = t;
        const float at = fabsf(t);
        P.rat = __fdividef(t, 1.0f + at * inv_clip);  // denominator in [1, 1 + 1e4 / clip]
        const float bnd = tanhf(t * inv_clip) * clip;
        P.root = sgnf_s(t) * sqrt_sfu(fminf(at, clip2) + eps);
        P.u = (1.0f - sp) * P.rat + sp * bnd;
        P.nov = tanhf((t - qn) * invD) * clip;
        return P;
    };

    // ---- stage 4: drive statistics as a Gram of (u, root, t, pred, nov)
    {
        float g32[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) g32[j] = 0.0f;
        for_slice([&](int64_t, int64_t, int64_t q, int64_t) {
            const Parts P = parts(F[q]);
            const float v[5] = {P.u, P.root, P.t, qn, P.nov};
            int j = 0;
#pragma unroll
            for (int a = 0; a < 5; ++a)
#pragma unroll
                for (int b = a; b < 5; ++b, ++j) g32[j] = fmaf(v[a], v[b], g32[j]);
            g32[15] = fmaf(P.rat, P.rat, g32[15]);
        });
        double g[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) g[j] = (double)g32[j];
        cluster_sum<16>(cl, g, sh.slot4, sh);
        if (tid == 0) {
            const double* G = sh.all;
            auto Gm = [&](int a, int b) {
                if (a > b) {
                    const int t = a;
                    a = b;
                    b = t;
                }
                return G[a * 5 - (a * (a - 1)) / 2 + (b - a)];
            };
            enum { U = 0, RT = 1, TT = 2, PR = 3, NV = 4 };
            const float frms = sqrtf((float)(Gm(TT, TT) / N) + eps);
            const float prms = sqrtf((float)(Gm(PR, PR) / N) + eps);
            const float align = clampf((float)(Gm(TT, PR) / N) / (frms * prms + eps), -1.0f, 1.0f);
            const float align_gate = prms > (float)sqrt(hp[S_EPS]) ? clampf((align + 1.0f) * 0.5f, 0.0f, 1.0f) : 0.0f;
            const int ws = (int)hp[S_WS];
            const double warm = ws == 0 ? 1.0 : (1.0 - exp(-(double)D.step / (double)(ws > 1 ? ws : 1)));
            const float mix = (float)(hp[S_PM] * warm) * align_gate / (1.0f + S);
            const float rat_rms = sqrtf((float)(G[15] / N) + eps);
            const float root_rms = sqrtf((float)(Gm(RT, RT) / N) + eps);
            const float k_root = rat_rms / fmaxf(root_rms, eps);
            const float root_mix = (float)hp[S_RCM] / (1.0f + 0.5f * S);
            const double a = 1.0 - (double)root_mix, b = (double)root_mix * (double)k_root;
            const double sh2 = a * a * Gm(U, U) + 2.0 * a * b * Gm(U, RT) + b * b * Gm(RT, RT);
            const float shaped_rms = sqrtf((float)(sh2 / N) + eps);
            const float dm = (float)hp[S_DFM] / (1.0f + 0.35f * S);
            const float k_d = shaped_rms / fmaxf(frms, eps);
            const double cu = (1.0 - dm) * a, cr = (1.0 - dm) * b, ctt = (double)dm * k_d;
            const double core2 = cu * cu * Gm(U, U) + cr * cr * Gm(RT, RT) + ctt * ctt * Gm(TT, TT) +
                                 2.0 * (cu * cr * Gm(U, RT) + cu * ctt * Gm(U, TT) + cr * ctt * Gm(RT, TT));
            const float core_rms = sqrtf((float)(core2 / N) + eps);
            const float resm = (float)hp[S_RFM] / (1.0f + S);
            const double err2 = Gm(TT, TT) - 2.0 * Gm(TT, PR) + Gm(PR, PR);
            const float k_r = core_rms / fmaxf(sqrtf((float)(fmax(err2, 0.0) / N) + eps), eps);
            double c[5];
            c[U] = (1.0 - mix) * cu;
            c[RT] = (1.0 - mix) * cr;
            c[TT] = (1.0 - mix) * ctt + (double)resm * k_r;
            c[PR] = (double)mix - (double)resm * k_r;
            c[NV] = hp[S_NM];
            double d2 = 0.0;
            for (int i = 0; i < 5; ++i)
                for (int j = 0; j < 5; ++j) d2 += c[i] * c[j] * Gm(i, j);
            const float den = (float)(fmax(d2, 0.0) / N);
            const float DE = reservoir(st_de, den, hp[S_RD], D.step);
            if (writer) *D.drive_energy = DE;
            sh.gain = clampf((float)hp[S_TGT] / sqrtf(DE + eps), (float)hp[S_MING], (float)hp[S_MAXG]);
            sh.c_u = (float)c[U];
            sh.c_root = (float)c[RT];
            sh.c_t = (float)c[TT];
            sh.c_pred = (float)c[PR];
            sh.c_nov = (float)c[NV];
        }
        // no CTA leaves (or reuses) shared memory another CTA may still read
        cl.sync();
    }

    // ---- stage 5: parameter update
    {
        const float cu = sh.c_u, cr = sh.c_root, ctt = sh.c_t, cp = sh.c_pred, cn = sh.c_nov, gain = sh.gain;
        const float neg_lr = (float)(-hp[S_LR]);
        const float neg_lr16 = neg_lr_in(hp[S_LR], D.dtype);
        for_slice([&](int64_t, int64_t, int64_t q, int64_t e) {
            const Parts P = parts(F[q]);
            const float drive = cu * P.u + cr * P.root + ctt * P.t + cp * qn + cn * P.nov;
            if (dt == CRESSO_DTYPE_F32)
                param[e] = param[e] + neg_lr * (drive * gain);
            else
                apply_update(param, e, dt, neg_lr, neg_lr16, drive * gain);
        });
    }
}

static int64_t scal_work_floats(const cresso_tensor_desc& d, int* TC, int* RPI, int* n_ct, int* nw, int64_t* rows,
                                int64_t* cols) {
    int64_t N = 1;
    for (int64_t a = 0; a < d.ndim; ++a) N *= d.shape[a];
    if (d.ndim <= 2) {
        *rows = d.ndim == 2 ? d.shape[0] : 1;
        *cols = d.ndim == 2 ? d.shape[1] : (d.ndim == 1 ? d.shape[0] : 1);
        *TC = std::min(256, pow2_ceil(*cols));
        *RPI = 256 / *TC;
        *n_ct = (int)ceil_div(*cols, *TC);
        *nw = std::max(1, *TC / 32);
        return (int64_t)(*n_ct) * (*nw) * (*rows) + *rows + *cols;
    }
    *rows = 1;
    *cols = N;
    *TC = 256;
    *RPI = 1;
    *n_ct = 1;
    *nw = 1;
    int64_t s = 0;
    for (int64_t a = 0; a < d.ndim; ++a) s += d.shape[a];
    return s;
}

static int scal_layout(const cresso_tensor_desc* descs, int64_t n, std::vector<ScalTensor>* out, int64_t* bytes) {
    CRESSO_REQUIRE(descs != nullptr && n >= 1, CRESSO_EINVAL, "scalar route: need at least one tensor");
    int64_t off = align_up((int64_t)sizeof(ScalHdr), 256);
    const int64_t off_dts = off;
    off = align_up(off + (int64_t)sizeof(ScalTensor) * n, 256);
    if (out) out->assign(n, ScalTensor{});
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        CRESSO_REQUIRE(d.dtype == CRESSO_DTYPE_F32 || d.dtype == CRESSO_DTYPE_F16 || d.dtype == CRESSO_DTYPE_BF16 ||
                           d.dtype == CRESSO_DTYPE_F64,
                       CRESSO_EUNSUPPORTED,
                       "tensor %lld: dtype code %lld (float32, float16, bfloat16 and float64 are supported)",
                       (long long)i, (long long)d.dtype);
        CRESSO_REQUIRE(d.ndim >= 0 && d.ndim <= CRESSO_MAX_NDIM, CRESSO_EUNSUPPORTED,
                       "tensor %lld: ndim %lld outside [0, %d]", (long long)i, (long long)d.ndim, CRESSO_MAX_NDIM);
        for (int64_t a = 0; a < d.ndim; ++a)
            CRESSO_REQUIRE(d.shape[a] >= 1, CRESSO_EINVAL, "tensor %lld: empty dimension", (long long)i);
        int TC, RPI, n_ct, nw;
        int64_t rows, cols;
        // float64 tensors keep their work values in float64: two float slots each
        const int64_t wf = scal_work_floats(d, &TC, &RPI, &n_ct, &nw, &rows, &cols) * (d.dtype == CRESSO_DTYPE_F64 ? 2 : 1);
        if (out) {
            ScalTensor& S = (*out)[i];
            S.ndim = d.ndim;
            S.N = 1;
            for (int64_t a = 0; a < d.ndim; ++a) {
                S.N *= d.shape[a];
                S.dims[a] = d.shape[a];
            }
            for (int64_t a = d.ndim; a < CRESSO_MAX_NDIM; ++a) S.dims[a] = 0;
            S.rows = rows;
            S.cols = cols;
            S.step = d.step;
            S.TC = TC;
            S.RPI = RPI;
            S.n_ct = n_ct;
            S.nw = nw;
            S.param = (float*)d.param;
            S.grad = (const float*)d.grad;
            S.dtype = (int32_t)d.dtype;
            S.q = (float*)d.q;
            S.impulse = (float*)d.impulse;
            S.metric_q = (float*)d.metric_q;
            S.metric_impulse = (float*)d.metric_impulse;
            S.force_rms = (float*)d.force_rms;
            S.drive_energy = (float*)d.drive_energy;
            S.surprise = (float*)d.surprise;
            S.action = (float*)d.action;
            S.work = (float*)(intptr_t)off;  // offset, rebased on the scratch pointer by the caller
            CRESSO_REQUIRE(S.param && S.grad && S.q && S.impulse && S.metric_q && S.metric_impulse && S.force_rms &&
                               S.drive_energy && S.surprise && S.action,
                           CRESSO_EINVAL, "tensor %lld: NULL param / grad / state pointer", (long long)i);
            CRESSO_REQUIRE(d.step >= 1, CRESSO_EINVAL, "tensor %lld: step must be >= 1", (long long)i);
        }
        off = align_up(off + 4 * wf, 256);
    }
    (void)off_dts;
    *bytes = off;
    return CRESSO_OK;
}


// Slice geometry of a tensor of rank <= 2 cut into cs slices along its longer
// axis; false when a slice does not fit the cluster form's shared memory.
struct ClGeom {
    bool sr;
    int64_t chunk, lrows, lcols, ld, shortlen;
};
static bool cl_geometry(const ScalTensor& S, int cs, ClGeom* g) {
    if (S.ndim > 2 || S.dtype == CRESSO_DTYPE_F64) return false;  // the cluster form works in float32
    g->sr = S.ndim == 2 && S.rows >= S.cols;
    const int64_t longlen = g->sr ? S.rows : S.cols;
    g->shortlen = g->sr ? S.cols : S.rows;
    g->chunk = ceil_div(longlen, cs);
    g->lrows = g->sr ? g->chunk : S.rows;
    g->lcols = g->sr ? S.cols : g->chunk;
    g->ld = (g->lcols & 1) ? g->lcols : g->lcols + 1;
    return g->lrows * g->ld <= kClSlice && g->shortlen <= kClShort && g->chunk <= kClLocal;
}

// Uploads the header and descriptors into the scratch at `base` and launches
// the group: the tensors that fit go to the cluster form (listed first), the
// rest to scalar_route_kernel.
static int scal_launch(std::vector<ScalTensor>& dts, const cresso_hparams* hp, char* base, cudaStream_t s) {
    const int64_t n = (int64_t)dts.size();
    int dev = 0, sms = 148;
    CRESSO_CUDA(cudaGetDevice(&dev));
    CRESSO_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // smallest cluster size that holds every tensor that fits at all, then more CTAs per
    // tensor while the grid is below two CTAs per SM
    std::vector<char> fits(n, 0);
    int cs = 1;
    int64_t n_cl = 0;
    for (int64_t i = 0; i < n; ++i) {
        ClGeom g;
        for (int c = 1; c <= kClMax; c *= 2)
            if (cl_geometry(dts[i], c, &g)) {
                fits[i] = 1;
                cs = std::max(cs, c);
                ++n_cl;
                break;
            }
    }
    while (cs < kClMax && n_cl * cs < 2 * (int64_t)sms) cs *= 2;
    std::vector<ScalTensor> ord;
    ord.reserve(n);
    int64_t slice_cap = 1, loc_cap = 1, short_cap = 1;
    for (int64_t i = 0; i < n; ++i) {
        if (!fits[i]) continue;
        ScalTensor S = dts[i];
        ClGeom g;
        cl_geometry(S, cs, &g);
        S.chunk = g.chunk;
        S.split_rows = g.sr ? 1 : 0;
        S.ctc = std::min(256, pow2_ceil(std::max<int64_t>(g.lcols, 1)));
        S.crpi = 256 / S.ctc;
        slice_cap = std::max(slice_cap, g.lrows * g.ld);
        loc_cap = std::max(loc_cap, g.chunk);
        short_cap = std::max(short_cap, g.shortlen);
        ord.push_back(S);
    }
    int64_t n_f32 = 0;  // general-form tensors of float32 work, then the float64 ones
    for (int64_t i = 0; i < n; ++i)
        if (!fits[i] && dts[i].dtype != CRESSO_DTYPE_F64) {
            ord.push_back(dts[i]);
            ++n_f32;
        }
    for (int64_t i = 0; i < n; ++i)
        if (!fits[i] && dts[i].dtype == CRESSO_DTYPE_F64) ord.push_back(dts[i]);
    ScalHdr h{};
    h.n = n;
    memcpy(h.hp, hp, sizeof(cresso_hparams));
    const int64_t off_dts = align_up((int64_t)sizeof(ScalHdr), 256);
    // header and descriptors in one upload
    static thread_local std::vector<unsigned char> blob;
    blob.assign((size_t)(off_dts + (int64_t)sizeof(ScalTensor) * n), 0);
    memcpy(blob.data(), &h, sizeof(h));
    memcpy(blob.data() + off_dts, ord.data(), sizeof(ScalTensor) * n);
    int ust = upload_async(base, blob.data(), blob.size(), s);
    if (ust) return ust;
    const ScalHdr* dh = reinterpret_cast<const ScalHdr*>(base);
    const ScalTensor* dd = reinterpret_cast<const ScalTensor*>(base + off_dts);
    if (n_cl > 0) {
        const size_t smem = 4 * (size_t)(slice_cap + loc_cap + 2 * short_cap);
        if (smem > 48 * 1024)
            CRESSO_CUDA(cudaFuncSetAttribute(scalar_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(n_cl * cs));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)cs;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CRESSO_CUDA(cudaLaunchKernelEx(&cfg, scalar_cluster_kernel, dh, dd, (int)slice_cap, (int)loc_cap, (int)short_cap));
        CRESSO_LAUNCHED("scalar_cluster_kernel");
    }
    if (n_f32 > 0) {
        scalar_route_kernel<float><<<(unsigned)n_f32, kThreads, 0, s>>>(dh, dd + n_cl);
        CRESSO_LAUNCHED("scalar_route_kernel<float>");
    }
    if (n_cl + n_f32 < n) {
        scalar_route_kernel<double><<<(unsigned)(n - n_cl - n_f32), kThreads, 0, s>>>(dh, dd + n_cl + n_f32);
        CRESSO_LAUNCHED("scalar_route_kernel<double>");
    }
    return CRESSO_OK;
}

}  // namespace cresso

using namespace cresso;

extern "C" {

int cresso_scalar_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, int64_t* bytes) {
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "scalar_scratch_bytes: NULL output");
    return scal_layout(descs, n, nullptr, bytes);
}

int cresso_scalar_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                      int64_t scratch_bytes, cresso_stream_t stream) {
    CRESSO_REQUIRE(hp != nullptr, CRESSO_EINVAL, "scalar_run: NULL hparams");
    std::vector<ScalTensor> dts;
    int64_t bytes = 0;
    int st = scal_layout(descs, n, &dts, &bytes);
    if (st) return st;
    CRESSO_REQUIRE(scratch != nullptr, CRESSO_EINVAL, "scalar_run: NULL scratch");
    CRESSO_REQUIRE(scratch_bytes >= bytes, CRESSO_ESCRATCH, "scalar_run: scratch of %lld bytes, need %lld",
                   (long long)scratch_bytes, (long long)bytes);
    char* base = (char*)scratch;
    for (auto& S : dts) S.work = (float*)(base + (intptr_t)S.work);
    NvtxRange range("cresso_scalar_run %lld tensors", (long long)n);
    return scal_launch(dts, hp, base, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the scalar-route step.
//
// Its scratch (the launch header, the tensor descriptors and the per-tensor
// work floats) lives in this file-scope device array instead of caller memory.
// Every GPU that loads the library keeps the array until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[CRESSO_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch in the current device's current context.
// In host code the array's name is only a host-side stand-in, so the address is
// asked of the runtime (cudaGetSymbolAddress, with the target device current)
// on every call: a cached address would go stale after cudaDeviceReset or when
// an FFI host drives the device through a context of its own, and the lookup is
// cheap next to the launch.  The first lookup on a device loads the library's
// module there.
static int noalloc_scratch_address(void** out) {
    void* ptr = nullptr;
    CRESSO_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    CRESSO_REQUIRE(ptr != nullptr, CRESSO_ECUDA, "scalar_run_noalloc: cudaGetSymbolAddress returned NULL");
    *out = ptr;
    return CRESSO_OK;
}

}  // extern "C"

extern "C" int cresso_scalar_run_noalloc(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                         cresso_stream_t stream) {
    CRESSO_REQUIRE(hp != nullptr, CRESSO_EINVAL, "scalar_run_noalloc: NULL hparams");
    std::vector<ScalTensor> dts;
    int64_t bytes = 0;
    int st = scal_layout(descs, n, &dts, &bytes);
    if (st) return st;
    CRESSO_REQUIRE(bytes <= (int64_t)CRESSO_NOALLOC_SCRATCH_BYTES, CRESSO_ESCRATCH,
                   "scalar_run_noalloc: these %lld tensors need %lld bytes of scratch, more than the %lld-byte "
                   "built-in array; split them over several calls or use cresso_scalar_run",
                   (long long)n, (long long)bytes, (long long)CRESSO_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    st = noalloc_scratch_address(&scratch);
    if (st) return st;
    // Same launch as cresso_scalar_run, on the built-in array.  Nothing in the
    // array has to start at zero: the header and descriptors are uploaded here
    // and the kernel writes every work float before reading it.
    char* base = (char*)scratch;
    for (auto& S : dts) S.work = (float*)(base + (intptr_t)S.work);
    return scal_launch(dts, hp, base, (cudaStream_t)stream);
}
