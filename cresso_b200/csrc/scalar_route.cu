// Scalar-route CRESSO5 step (cresso_v5.py:1434-1582): LoRA-thin matrices and
// tensors below min_spectral_size.  One 256-thread block runs the whole step
// of one tensor, re-reading the gradient between its five stages (the
// tensors are small, so the re-reads hit L2); all tensors of a group go in
// one launch.  The reference needs 13 launches + 2 memsets per tensor
// (scalar_update_2d_cuda, cresso_cuda_kernel.cu:3225-3605) and covers only
// 2-D tensors; this kernel covers 0-d to 8-d.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

struct ScalTensor {
    int64_t ndim, N, rows, cols, step;
    int64_t dims[CRESSO_MAX_NDIM];
    int32_t TC, RPI, n_ct, nw;
    float* param;
    const float* grad;
    float *q, *impulse, *metric_q, *metric_impulse, *force_rms, *drive_energy, *surprise, *action;
    float* work;  // per-tensor float scratch (row partials, row / column factors, N-d marginals)
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

struct ScalShared {
    double red[16 * kWarps];
    double tot[16];
    float scale, inv_scale, metric, q_old, q_new, S, gm, inst_k;
    float c_u, c_root, c_t, c_pred, c_nov, gain, sp, invD;
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
__device__ __forceinline__ float nd_factor(const ScalTensor& D, int64_t e) {
    float prod = 1.0f;
    int64_t rem = e;
    int64_t base = 0;
    for (int64_t a = 0; a < D.ndim; ++a) base += D.dims[a];
    for (int64_t a = D.ndim - 1; a >= 0; --a) {
        base -= D.dims[a];
        const int64_t coord = rem % D.dims[a];
        rem /= D.dims[a];
        prod *= D.work[base + coord];
    }
    return prod;
}

__global__ void __launch_bounds__(kThreads) scalar_route_kernel(const ScalHdr* __restrict__ hdr,
                                                                 const ScalTensor* __restrict__ dts) {
    __shared__ ScalShared sh;
    const ScalTensor& D = dts[blockIdx.x];
    const double* hp = hdr->hp;
    const int tid = threadIdx.x, lane = tid & 31;
    const float eps = (float)hp[S_EPS];
    const float sgn = hp[S_MAX] != 0.0 ? -1.0f : 1.0f;
    const float wd = (float)hp[S_WD];
    const bool wd_on = hp[S_WD] != 0.0;
    const double N = (double)D.N;
    auto force = [&](int64_t e) {
        float f = sgn * __ldg(D.grad + e);
        if (wd_on) f = f + wd * D.param[e];
        return f;
    };

    // ---- stage 1: force energy -> force_rms, scale  (cresso_v5.py:1505-1508)
    {
        double s = 0.0;
        walk_elems(D, [&](int64_t e, int64_t, int64_t, int, bool valid) {
            if (valid) {
                const float f = force(e);
                s += (double)(f * f);
            }
        });
        double v[1] = {s};
        block_sum_to<1>(v, sh.red, sh.tot);
        if (tid == 0) {
            const float frn = sqrtf((float)(sh.tot[0] / N) + eps);
            const float fr = reservoir(*D.force_rms, frn, hp[S_RD], D.step);
            *D.force_rms = fr;
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
    if (ic != 0.0f && D.ndim > 0 && D.N > 1) inst_mode = D.ndim == 1 ? 1 : (D.ndim == 2 ? 2 : 3);
    auto dens = [&](float rel) { return ipow1 ? rel : fminf(powf(fmaxf(rel, eps), pw), 1.0e6f); };

    // ---- stage 2: density metric and the instant-metric axis sums  (cresso_v5.py:1510-1525)
    {
        float* rowpart = D.work;  // [n_ct * nw][rows]
        const int nw = D.nw;
        float* colsum = D.work + (int64_t)D.n_ct * nw * D.rows + D.rows;  // [cols]
        __syncthreads();
        double sL = 0.0, sd = 0.0;
        float colacc = 0.0f;
        __shared__ float s_col[kThreads];
        const int lc = tid & (D.TC - 1), rs = tid / D.TC;
        int cur_ct = -1;
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int ct, bool valid) {
            if (D.ndim <= 2 && ct != cur_ct) {
                if (cur_ct >= 0) {  // flush column sums of the previous tile
                    s_col[tid] = colacc;
                    __syncthreads();
                    const int64_t cc = (int64_t)cur_ct * D.TC + lc;
                    if (rs == 0 && cc < D.cols) {
                        float s = 0.0f;
                        for (int q = 0; q < D.RPI; ++q) s += s_col[q * D.TC + lc];
                        colsum[cc] = s;
                    }
                    __syncthreads();
                }
                colacc = 0.0f;
                cur_ct = ct;
            }
            float d = 0.0f;
            if (valid) {
                const float f = force(e);
                const float rel0 = fabsf(f) * inv_scale + eps;
                sL += (double)log1pf(powf(rel0, ep));
                const float rel = fminf(rel0, 1.0e4f);
                d = dens(rel);
                sd += (double)d;
                colacc += d;
            }
            if (inst_mode == 2) {
                float v = d;
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
                float s = 0.0f;
                for (int q = 0; q < D.RPI; ++q) s += s_col[q * D.TC + lc];
                colsum[cc] = s;
            }
        }
        double v[2] = {sL, sd};
        block_sum_to<2>(v, sh.red, sh.tot);  // includes __syncthreads
        if (tid == 0) {
            // metric oscillator on the scalar density  (cresso_v5.py:1510-1519)
            const float density = (float)(sh.tot[0] / N);
            const float mq0 = *D.metric_q;
            const float port = density - tanhf(mq0);
            const float mdt = (float)hp[S_MDT];
            float mp = *D.metric_impulse * (float)fmax(0.0, 1.0 - hp[S_MDT] * hp[S_MF]);
            mp = mp + mdt * (port - mq0);
            const float mq = clampf(mq0 + mdt * mp, -3.0f, 3.0f);
            *D.metric_impulse = mp;
            *D.metric_q = mq;
            sh.metric = clampf(expf((float)hp[S_MC] * mq), 0.06f, 16.0f);
            sh.gm = fmaxf((float)(sh.tot[1] / N), eps);
            sh.inst_k = ic / ((float)(D.ndim > 1 ? D.ndim : 1) * pw);
            sh.q_old = *D.q;
        }
        __syncthreads();
        // per-axis factors exp(k * log(max(mean / gmean, eps)))  (cresso_v5.py:243-262)
        const float gm = sh.gm, kk = sh.inst_k;
        if (inst_mode == 2) {
            float* rowf = D.work + (int64_t)D.n_ct * nw * D.rows;
            for (int64_t r = tid; r < D.rows; r += kThreads) {
                double s = 0.0;
                for (int64_t j = 0; j < (int64_t)D.n_ct * nw; ++j) s += (double)rowpart[j * D.rows + r];
                rowf[r] = expf(kk * logf(fmaxf((float)(s / (double)D.cols) / gm, eps)));
            }
            for (int64_t c = tid; c < D.cols; c += kThreads)
                colsum[c] = expf(kk * logf(fmaxf((float)((double)colsum[c] / (double)D.rows) / gm, eps)));
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
                        const float f = force(e);
                        m += (double)dens(fminf(fabsf(f) * inv_scale + eps, 1.0e4f));
                    }
                const double per = N / (double)D.dims[a];
                D.work[j] = expf(kk * logf(fmaxf((float)(m / per) / gm, eps)));
            }
        }
        __syncthreads();
    }

    const float metric = sh.metric, gm = sh.gm, kk = sh.inst_k;
    const float ls = (float)hp[S_LS];
    const bool local_on = hp[S_LS] != 0.0;
    const float* rowf = D.work + (int64_t)D.n_ct * D.nw * D.rows;
    const float* colf = rowf + D.rows;
    auto tangent = [&](int64_t e, int64_t r, int64_t c) {
        const float f = force(e);
        const float rel = fminf(fabsf(f) * inv_scale + eps, 1.0e4f);
        float den = scale * metric;
        if (local_on) den = den * clampf(1.0f + ls * sqrtf(fminf(rel, 100.0f)), 1.0f, 8.0f);
        if (inst_mode == 1) {
            den = den * clampf(expf(kk * logf(fmaxf(dens(rel) / gm, eps))), 0.08f, 12.0f);
        } else if (inst_mode == 2) {
            den = den * clampf(rowf[r] * colf[c], 0.08f, 12.0f);
        } else if (inst_mode == 3) {
            den = den * clampf(nd_factor(D, e), 0.08f, 12.0f);
        }
        return clampf(__fdiv_rn(f, den + eps), -1.0e4f, 1.0e4f);
    };

    // ---- stage 3: prediction error, surprise, scalar contact  (cresso_v5.py:1526-1546)
    {
        const float q0 = sh.q_old;
        double se = 0.0, se2 = 0.0;
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int, bool valid) {
            if (valid) {
                const float err = tangent(e, r, c) - q0;
                se += (double)err;
                se2 += (double)(err * err);
            }
        });
        double v[2] = {se, se2};
        block_sum_to<2>(v, sh.red, sh.tot);
        if (tid == 0) {
            const float sn = sqrtf((float)(sh.tot[1] / N) + eps);
            const float S = reservoir(*D.surprise, sn, hp[S_SD], D.step);
            *D.surprise = S;
            const float port = (float)(sh.tot[0] / N);
            const float dt = (float)hp[S_DT];
            const float plast = 1.0f + (float)hp[S_SG] * S / (1.0f + S);
            const float brake = 1.0f / (1.0f + (float)hp[S_SB] * S);
            float imp = *D.impulse, q = q0, action = *D.action;
            const float energy = 0.5f * (imp * imp + q * q);
            action = action * 0.985f + (port * imp - energy) * dt;
            const float fr = (float)hp[S_IF] + (float)hp[S_CG] * tanhf(fabsf(action));
            imp = imp * fmaxf(1.0f - dt * fr, 0.0f);
            imp = imp + dt * (plast * brake * port - (float)hp[S_REST] * q - (float)hp[S_CUBIC] * (q * q * q));
            q = clampf(q + dt * imp, -8.0f, 8.0f);
            *D.impulse = imp;
            *D.action = action;
            *D.q = q;
            sh.q_new = q;
            sh.S = S;
            const float clip = (float)hp[S_CLIP];
            sh.sp = (float)hp[S_SPIKE] / (1.0f + S);
            sh.invD = 1.0f / (clip * (1.0f + S));
        }
        __syncthreads();
    }

    const float qn = sh.q_new, S = sh.S, sp = sh.sp, invD = sh.invD;
    const float clip = (float)hp[S_CLIP], inv_clip = 1.0f / clip, clip2 = (float)(hp[S_CLIP] * hp[S_CLIP]);
    struct Parts {
        float u, root, t, nov, rat;
    };
    auto parts = [&](int64_t e, int64_t r, int64_t c) {
        Parts P;
        P.t = tangent(e, r, c);
        const float at = fabsf(P.t);
        P.rat = P.t / (1.0f + at * inv_clip);
        const float bnd = tanhf(P.t * inv_clip) * clip;
        P.root = sgnf_s(P.t) * sqrtf(fminf(at, clip2) + eps);
        P.u = (1.0f - sp) * P.rat + sp * bnd;
        P.nov = tanhf((P.t - qn) * invD) * clip;
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
                const float v[5] = {P.u, P.root, P.t, qn, P.nov};
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
            const float DE = reservoir(*D.drive_energy, den, hp[S_RD], D.step);
            *D.drive_energy = DE;
            sh.gain = clampf((float)hp[S_TGT] / sqrtf(DE + eps), (float)hp[S_MING], (float)hp[S_MAXG]);
            sh.c_u = (float)c[U];
            sh.c_root = (float)c[RT];
            sh.c_t = (float)c[TT];
            sh.c_pred = (float)c[PR];
            sh.c_nov = (float)c[NV];
        }
        __syncthreads();
    }

    // ---- stage 5: parameter update  (cresso_v5.py:1582)
    {
        const float cu = sh.c_u, cr = sh.c_root, ctt = sh.c_t, cp = sh.c_pred, cn = sh.c_nov, gain = sh.gain;
        const float neg_lr = (float)(-hp[S_LR]);
        walk_elems(D, [&](int64_t e, int64_t r, int64_t c, int, bool valid) {
            if (valid) {
                const Parts P = parts(e, r, c);
                const float drive = cu * P.u + cr * P.root + ctt * P.t + cp * qn + cn * P.nov;
                D.param[e] = D.param[e] + neg_lr * (drive * gain);
            }
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
        CRESSO_REQUIRE(d.ndim >= 0 && d.ndim <= CRESSO_MAX_NDIM, CRESSO_EUNSUPPORTED,
                       "tensor %lld: ndim %lld outside [0, %d]", (long long)i, (long long)d.ndim, CRESSO_MAX_NDIM);
        for (int64_t a = 0; a < d.ndim; ++a)
            CRESSO_REQUIRE(d.shape[a] >= 1, CRESSO_EINVAL, "tensor %lld: empty dimension", (long long)i);
        int TC, RPI, n_ct, nw;
        int64_t rows, cols;
        const int64_t wf = scal_work_floats(d, &TC, &RPI, &n_ct, &nw, &rows, &cols);
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
    ScalHdr h{};
    h.n = n;
    memcpy(h.hp, hp, sizeof(cresso_hparams));
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t off_dts = align_up((int64_t)sizeof(ScalHdr), 256);
    CRESSO_CUDA(cudaMemcpyAsync(base, &h, sizeof(h), cudaMemcpyHostToDevice, s));
    CRESSO_CUDA(cudaMemcpyAsync(base + off_dts, dts.data(), sizeof(ScalTensor) * n, cudaMemcpyHostToDevice, s));
    scalar_route_kernel<<<(unsigned)n, kThreads, 0, s>>>(reinterpret_cast<const ScalHdr*>(base),
                                                         reinterpret_cast<const ScalTensor*>(base + off_dts));
    CRESSO_LAUNCHED("scalar_route_kernel");
    return CRESSO_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the scalar-route step.
//
// Its scratch (the launch header, the tensor descriptors and the per-tensor
// work floats) lives in this file-scope device array instead of caller memory.
// Every GPU that loads the library keeps the array until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[CRESSO_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_addr[256] = {nullptr};  // device address of the array, per device ordinal

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device with cudaGetSymbolAddress (with that device current) and cached.
static int noalloc_scratch_address(void** out) {
    int dev = -1;
    CRESSO_CUDA(cudaGetDevice(&dev));
    CRESSO_REQUIRE(dev >= 0 && dev < 256, CRESSO_EUNSUPPORTED, "scalar_run_noalloc: device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
        void* ptr = nullptr;
        CRESSO_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        CRESSO_REQUIRE(ptr != nullptr, CRESSO_ECUDA, "scalar_run_noalloc: cudaGetSymbolAddress returned NULL");
        g_noalloc_addr[dev] = ptr;
    }
    *out = g_noalloc_addr[dev];
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
    ScalHdr h{};
    h.n = n;
    memcpy(h.hp, hp, sizeof(cresso_hparams));
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t off_dts = align_up((int64_t)sizeof(ScalHdr), 256);
    CRESSO_CUDA(cudaMemcpyAsync(base, &h, sizeof(h), cudaMemcpyHostToDevice, s));
    CRESSO_CUDA(cudaMemcpyAsync(base + off_dts, dts.data(), sizeof(ScalTensor) * n, cudaMemcpyHostToDevice, s));
    scalar_route_kernel<<<(unsigned)n, kThreads, 0, s>>>(reinterpret_cast<const ScalHdr*>(base),
                                                         reinterpret_cast<const ScalTensor*>(base + off_dts));
    CRESSO_LAUNCHED("scalar_route_kernel");
    return CRESSO_OK;
}
