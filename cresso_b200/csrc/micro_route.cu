// Micro-field CRESSO5 step (cresso_v5.py:1355-1432): every tensor with
// 0 < numel <= micro_field_max_size keeps float32 per-element energy, impulse
// and refractory fields.  The reference runs this route on its PyTorch path
// only (about 40 tensor operations per tensor and step); here one 256-thread
// block steps one tensor and all tensors of a group go in one launch.
//
// Four sweeps over the tensor with a block reduction after each of the first
// three (float64 sums in a fixed order, so a step is deterministic):
//   1  force energy                      -> force_rms, scale
//   2  energy field update, instant-metric density  -> energy mean, density mean
//      (rank >= 2 with the instant metric on: per-axis marginal means)
//   3  tangent, refractory and impulse fields, a Gram of
//      (rational, bounded, tangent, prediction, error)  -> surprise, drive
//      coefficients, drive energy, gain
//   4  drive from the Gram coefficients, parameter update
// Per-element values the later sweeps need (force, tangent) are recomputed
// from the gradient, the parameter and the updated fields with the same
// arithmetic, so they are identical in every sweep.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

struct MicroTensor {
    int64_t ndim, N, step;
    int64_t dims[CRESSO_MAX_NDIM];
    void* param;       // element type `dtype` (CRESSO_DTYPE_*)
    const void* grad;  // element type `dtype`
    float *energy, *impulse, *refractory, *force_rms, *drive_energy, *surprise;
    float* work;  // rank >= 2: per-axis log marginal terms, sum(dims) floats
    int32_t dtype, pad;
};

struct MicroHdr {
    int64_t n;
    double hp[64];
};

// hparams indices (field order of cresso_hparams)
enum {
    M_LR, M_WD, M_EP, M_DT, M_IF, M_CG, M_REST, M_CUBIC, M_MDT, M_MF, M_MC, M_LS, M_IC, M_IP, M_RCM, M_EM, M_TM,
    M_HD, M_HID, M_HMC, M_HDM, M_DFM, M_RFM, M_RD, M_REFD, M_RG, M_CD, M_CONFG, M_SG, M_SD, M_PM, M_NM, M_WS, M_SB,
    M_TGT, M_MING, M_MAXG, M_CLIP, M_SPIKE, M_EPS, M_MAX, M_RANK, M_MAXF, M_BINS, M_TABLES, M_HARDMIN, M_THINCUT,
    M_MD, M_MID, M_MDM, M_COUNT
};
static_assert(sizeof(cresso_hparams) == M_COUNT * sizeof(double), "cresso_hparams field order");

template <typename W>
struct MicroShared {
    double red[16 * kWarps];
    double tot[16];
    W scale, emean, gm, kk;
    W c_rat, c_bnd, c_t, c_pred, c_err, gain;
};

// Gram index of the pair (a, b), a <= b, of five vectors.
__host__ __device__ constexpr int g5(int a, int b) { return a * 5 - (a * (a - 1)) / 2 + (b - a); }

template <typename W>
__global__ void __launch_bounds__(kThreads) micro_route_kernel(const MicroHdr* __restrict__ hdr,
                                                                const MicroTensor* __restrict__ dts) {
    __shared__ MicroShared<W> sh;
    const MicroTensor& D = dts[blockIdx.x];
    // fields and 0-d state in the work type
    W* energy = reinterpret_cast<W*>(D.energy);
    W* impulse = reinterpret_cast<W*>(D.impulse);
    W* refractory = reinterpret_cast<W*>(D.refractory);
    W* work = reinterpret_cast<W*>(D.work);
    auto st = [](float* ptr) { return reinterpret_cast<W*>(ptr); };
    const double* hp = hdr->hp;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dt = D.dtype;
    const int64_t N = D.N;
    const double Nd = (double)N;
    const W eps = (W)hp[M_EPS];
    const W sgn = hp[M_MAX] != 0.0 ? -W(1.0) : W(1.0);
    const W wd = (W)hp[M_WD];
    const bool wd_on = hp[M_WD] != 0.0;
    // f = g (+ wd p), with g negated under maximize (cresso_v5.py:833-834, 907-912)
    auto force = [&](int64_t e) {
        W f = sgn * load_w<W>(D.grad, e, dt);
        if (wd_on) f = f + wd * load_w<W>(D.param, e, dt);
        return f;
    };

    // ---- sweep 1: force energy -> force_rms, scale  (cresso_v5.py:1375-1378)
    {
        double s = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const W f = force(e);
            s += (double)(f * f);
        }
        double v[1] = {s};
        block_sum_to<1>(v, sh.red, sh.tot);
        if (tid == 0) {
            const W frn = w_sqrt((W)(sh.tot[0] / Nd) + eps);
            const W fr = reservoir(*st(D.force_rms), frn, hp[M_RD], D.step);
            *st(D.force_rms) = fr;
            sh.scale = w_max(fr, eps);
        }
        __syncthreads();
    }
    const W scale = sh.scale;
    auto rel_of = [&](W f) { return w_min(w_abs(f) / scale + eps, W(1.0e4)); };

    // instant metric of the micro route: coupling min(0.35, c), every axis (cresso_v5.py:1390-1392, 243-262)
    const double ic = fmin(0.35, hp[M_IC]);
    const W pw = w_max((W)hp[M_IP], W(0.25));
    const bool inst_on = ic != 0.0 && N > 1;
    const bool marg = inst_on && D.ndim >= 2;
    auto idens = [&](W rel) { return pw == W(1.0) ? w_max(rel, eps) : w_min(w_pow(w_max(rel, eps), pw), W(1.0e6)); };

    // ---- sweep 2: energy field and the instant-metric density  (cresso_v5.py:1380-1392)
    {
        const W ep = (W)hp[M_EP];
        const W md = (W)hp[M_MD], omd = (W)(1.0 - hp[M_MD]);
        const bool first = D.step <= 1;
        double se = 0.0, sd = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const W rel = rel_of(force(e));
            const W dens = w_pow(rel, ep);
            const W en = first ? dens : energy[e] * md + omd * dens;
            energy[e] = en;
            se += (double)en;
            if (inst_on) sd += (double)idens(rel);
        }
        double v[2] = {se, sd};
        block_sum_to<2>(v, sh.red, sh.tot);
        if (tid == 0) {
            sh.emean = w_max((W)(sh.tot[0] / Nd), eps);
            sh.gm = w_max((W)(sh.tot[1] / Nd), eps);
            sh.kk = (W)(ic / ((double)D.ndim * (double)pw));
        }
        __syncthreads();
        if (marg) {
            // log(max(axis mean / mean, eps)) per axis and coordinate: the elements of one
            // coordinate (a slab of N / dims[a]) are summed by one thread when the slab is
            // short, else by one warp (lane-strided, then a shuffle tree); fixed order both ways
            const W gm = sh.gm;
            uint32_t off = 0;
            for (int a = 0; a < (int)D.ndim; ++a) {
                const uint32_t da = (uint32_t)D.dims[a];
                uint32_t inner = 1;
                for (int b = a + 1; b < (int)D.ndim; ++b) inner *= (uint32_t)D.dims[b];
                const uint32_t slab = (uint32_t)N / da;
                const double inv_slab = 1.0 / (double)slab;
                auto elem = [&](uint32_t c, uint32_t s) {  // s-th element of coordinate c along axis a
                    const uint32_t o = s / inner, i = s - o * inner;
                    return (int64_t)((o * da + c) * inner + i);
                };
                if (slab < 32) {
                    for (uint32_t c = tid; c < da; c += kThreads) {
                        double m = 0.0;
                        for (uint32_t s = 0; s < slab; ++s) m += (double)idens(rel_of(force(elem(c, s))));
                        work[off + c] = w_log(w_max((W)(m * inv_slab) / gm, eps));
                    }
                } else {
                    for (uint32_t c = warp; c < da; c += kWarps) {
                        double m = 0.0;
                        for (uint32_t s = lane; s < slab; s += 32) m += (double)idens(rel_of(force(elem(c, s))));
                        m = warp_sum(m);
                        if (lane == 0) work[off + c] = w_log(w_max((W)(m * inv_slab) / gm, eps));
                    }
                }
                off += da;
            }
            __syncthreads();
        }
    }
    const W emean = sh.emean, gm = sh.gm, kk = sh.kk;
    const W xm = (W)(hp[M_HMC] / fmax(0.25, hp[M_EP]));
    auto tangent = [&](int64_t e, W f) {
        const W rel = rel_of(f);
        const W metric = clampw(w_pow(energy[e] / emean, xm), W(0.08), W(12.0));
        W inst = W(1.0);
        if (marg) {
            // 32-bit index arithmetic (N < 2^31): 64-bit division is a subroutine call
            W lsum = W(0.0);
            uint32_t rem = (uint32_t)e, off = 0;
            for (int a = 0; a < (int)D.ndim; ++a) off += (uint32_t)D.dims[a];
            for (int a = (int)D.ndim - 1; a >= 0; --a) {
                const uint32_t da = (uint32_t)D.dims[a];
                off -= da;
                lsum += work[off + rem % da];
                rem /= da;
            }
            inst = clampw(w_exp(kk * lsum), W(0.08), W(12.0));
        } else if (inst_on) {
            inst = clampw(w_exp(kk * w_log(w_max(idens(rel) / gm, eps))), W(0.08), W(12.0));
        }
        return clampw(f / (scale * metric * inst + eps), -W(1.0e4), W(1.0e4));
    };
    const W clip = (W)hp[M_CLIP];

    // ---- sweep 3: refractory-gated impulse, prediction error, drive statistics  (cresso_v5.py:1394-1431)
    {
        const W rd = (W)hp[M_REFD], ord = (W)(1.0 - hp[M_REFD]);
        const W rg = (W)hp[M_RG];
        const W mid = (W)hp[M_MID], omid = (W)(1.0 - hp[M_MID]);
        double g[15];
#pragma unroll
        for (int j = 0; j < 15; ++j) g[j] = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const W t = tangent(e, force(e));
            const W rf = refractory[e] * rd + ord * w_abs(t);
            refractory[e] = rf;
            const W gate = W(1.0) / (W(1.0) + rg * rf);
            const W im = impulse[e] * mid + omid * (t * gate);
            impulse[e] = im;
            const double v[5] = {(double)(t / (W(1.0) + w_abs(t) / clip)), (double)(w_tanh(t / clip) * clip), (double)t,
                                 (double)im, (double)(t - im)};
            int j = 0;
#pragma unroll
            for (int a = 0; a < 5; ++a)
#pragma unroll
                for (int b = a; b < 5; ++b) g[j++] += v[a] * v[b];
        }
        block_sum_to<15>(g, sh.red, sh.tot);
        if (tid == 0) {
            const double* G = sh.tot;
            enum { RAT = 0, BND = 1, TT = 2, PR = 3, ER = 4 };
            const W sn = w_sqrt((W)(G[g5(ER, ER)] / Nd) + eps);
            const W S = reservoir(*st(D.surprise), sn, hp[M_SD], D.step);
            *st(D.surprise) = S;
            const W sp = (W)hp[M_SPIKE] / (W(1.0) + S);
            const double a = (double)(W(1.0) - sp), b = (double)sp;
            const double sh2 = a * a * G[g5(RAT, RAT)] + 2.0 * a * b * G[g5(RAT, BND)] + b * b * G[g5(BND, BND)];
            const W target = w_sqrt((W)(sh2 / Nd) + eps);
            auto k_of = [&](int i) { return target / w_max(w_sqrt((W)(G[g5(i, i)] / Nd) + eps), eps); };
            const W dm = (W)hp[M_DFM] / (W(1.0) + W(0.35) * S);
            const W mm = (W)hp[M_MDM] / (W(1.0) + W(0.25) * S);
            const W rm = (W)hp[M_RFM] / (W(1.0) + S);
            const W core = clampw(W(1.0) - dm - W(0.5) * mm, W(0.0), W(1.0));
            double c[5];
            c[RAT] = (double)core * a;
            c[BND] = (double)core * b;
            c[TT] = (double)(dm * k_of(TT));
            c[PR] = (double)(mm * k_of(PR));
            c[ER] = (double)(rm * k_of(ER));
            double d2 = 0.0;
#pragma unroll
            for (int i = 0; i < 5; ++i)
#pragma unroll
                for (int j = 0; j < 5; ++j) d2 += c[i] * c[j] * G[i <= j ? g5(i, j) : g5(j, i)];
            const W DE = reservoir(*st(D.drive_energy), (W)(fmax(d2, 0.0) / Nd), hp[M_RD], D.step);
            *st(D.drive_energy) = DE;
            sh.gain = clampw((W)hp[M_TGT] / w_sqrt(DE + eps), (W)hp[M_MING], (W)hp[M_MAXG]);
            sh.c_rat = (W)c[RAT];
            sh.c_bnd = (W)c[BND];
            sh.c_t = (W)c[TT];
            sh.c_pred = (W)c[PR];
            sh.c_err = (W)c[ER];
        }
        __syncthreads();
    }

    // ---- sweep 4: parameter update  (cresso_v5.py:1432)
    {
        const W cr = sh.c_rat, cb = sh.c_bnd, ct = sh.c_t, cp = sh.c_pred, ce = sh.c_err, gain = sh.gain;
        const W neg_lr = (W)(-hp[M_LR]);
        const W neg_lr16 = neg_lr_w<W>(hp[M_LR], dt);
        for (int64_t e = tid; e < N; e += kThreads) {
            const W t = tangent(e, force(e));
            const W im = impulse[e];
            const W drive = cr * (t / (W(1.0) + w_abs(t) / clip)) + cb * (w_tanh(t / clip) * clip) + ct * t +
                                cp * im + ce * (t - im);
            apply_update_w<W>(D.param, e, dt, neg_lr, neg_lr16, drive * gain);
        }
    }
}

// Validates the descriptors and fills the device descriptors (work pointers as
// offsets into the scratch); *bytes = the scratch size.
static int micro_layout(const cresso_tensor_desc* descs, int64_t n, std::vector<MicroTensor>* out, int64_t* bytes) {
    CRESSO_REQUIRE(descs != nullptr || n == 0, CRESSO_EINVAL, "micro: NULL descriptors");
    CRESSO_REQUIRE(n >= 0 && n <= (1LL << 20), CRESSO_EINVAL, "micro: bad tensor count %lld", (long long)n);
    const int64_t off_dts = align_up((int64_t)sizeof(MicroHdr), 256);
    int64_t off = align_up(off_dts + (int64_t)sizeof(MicroTensor) * n, 256);
    if (out) out->resize(n);
    for (int64_t i = 0; i < n; ++i) {
        const cresso_tensor_desc& d = descs[i];
        CRESSO_REQUIRE(d.ndim >= 1 && d.ndim <= CRESSO_MAX_NDIM, CRESSO_EINVAL,
                       "tensor %lld: the micro route takes tensors of rank 1 to %d (ndim=%lld)", (long long)i,
                       CRESSO_MAX_NDIM, (long long)d.ndim);
        CRESSO_REQUIRE(d.dtype == CRESSO_DTYPE_F32 || d.dtype == CRESSO_DTYPE_F16 || d.dtype == CRESSO_DTYPE_BF16 ||
                           d.dtype == CRESSO_DTYPE_F64,
                       CRESSO_EUNSUPPORTED,
                       "tensor %lld: dtype code %lld (float32, float16, bfloat16 and float64 are supported)",
                       (long long)i, (long long)d.dtype);
        int64_t N = 1, lead_sum = 0;
        for (int64_t a = 0; a < d.ndim; ++a) {
            CRESSO_REQUIRE(d.shape[a] > 0, CRESSO_EINVAL, "tensor %lld: shape[%lld] must be > 0", (long long)i,
                           (long long)a);
            CRESSO_REQUIRE(N <= (1LL << 31) / d.shape[a], CRESSO_EUNSUPPORTED,
                           "tensor %lld: more than 2^31 elements on the micro route", (long long)i);
            N *= d.shape[a];
            lead_sum += d.shape[a];
        }
        CRESSO_REQUIRE(d.step >= 1, CRESSO_EINVAL, "tensor %lld: step must be >= 1", (long long)i);
        CRESSO_REQUIRE(d.param && d.grad && d.force_rms && d.drive_energy && d.surprise && d.micro_energy &&
                           d.micro_impulse && d.micro_refractory,
                       CRESSO_EINVAL, "tensor %lld: NULL param / grad / state pointer", (long long)i);
        if (out) {
            MicroTensor& M = (*out)[i];
            memset(&M, 0, sizeof(M));
            M.ndim = d.ndim;
            M.N = N;
            M.step = d.step;
            for (int64_t a = 0; a < d.ndim; ++a) M.dims[a] = d.shape[a];
            M.param = (void*)d.param;
            M.grad = (const void*)d.grad;
            M.energy = (float*)d.micro_energy;
            M.impulse = (float*)d.micro_impulse;
            M.refractory = (float*)d.micro_refractory;
            M.force_rms = (float*)d.force_rms;
            M.drive_energy = (float*)d.drive_energy;
            M.surprise = (float*)d.surprise;
            M.dtype = (int32_t)d.dtype;
            M.work = d.ndim >= 2 ? (float*)(intptr_t)off : nullptr;  // offset, rebased by the caller
        }
        if (d.ndim >= 2) off = align_up(off + (d.dtype == CRESSO_DTYPE_F64 ? 8 : 4) * lead_sum, 256);
    }
    *bytes = off;
    return CRESSO_OK;
}

}  // namespace cresso

using namespace cresso;

extern "C" {

int cresso_micro_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, int64_t* bytes) {
    CRESSO_REQUIRE(bytes != nullptr, CRESSO_EINVAL, "micro_scratch_bytes: NULL output");
    return micro_layout(descs, n, nullptr, bytes);
}

int cresso_micro_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                     int64_t scratch_bytes, cresso_stream_t stream) {
    CRESSO_REQUIRE(hp != nullptr, CRESSO_EINVAL, "micro_run: NULL hparams");
    std::vector<MicroTensor> dts;
    int64_t bytes = 0;
    int st = micro_layout(descs, n, &dts, &bytes);
    if (st) return st;
    if (n == 0) return CRESSO_OK;
    CRESSO_REQUIRE(scratch != nullptr, CRESSO_EINVAL, "micro_run: NULL scratch");
    CRESSO_REQUIRE(scratch_bytes >= bytes, CRESSO_ESCRATCH, "micro_run: scratch of %lld bytes, need %lld",
                   (long long)scratch_bytes, (long long)bytes);
    char* base = (char*)scratch;
    for (auto& M : dts)
        if (M.ndim >= 2) M.work = (float*)(base + (intptr_t)M.work);
    // float32-work tensors first, then the float64 ones (a kernel instantiation each)
    std::stable_partition(dts.begin(), dts.end(), [](const MicroTensor& M) { return M.dtype != CRESSO_DTYPE_F64; });
    int64_t n32 = 0;
    for (const auto& M : dts) n32 += M.dtype != CRESSO_DTYPE_F64;
    NvtxRange range("cresso_micro_run %lld tensors", (long long)n);
    MicroHdr h{};
    h.n = n;
    memcpy(h.hp, hp, sizeof(cresso_hparams));
    const int64_t off_dts = align_up((int64_t)sizeof(MicroHdr), 256);
    cudaStream_t s = (cudaStream_t)stream;
    // header and descriptors in one upload
    static thread_local std::vector<unsigned char> blob;
    blob.assign((size_t)(off_dts + (int64_t)sizeof(MicroTensor) * n), 0);
    memcpy(blob.data(), &h, sizeof(h));
    memcpy(blob.data() + off_dts, dts.data(), sizeof(MicroTensor) * n);
    int ust = upload_async(base, blob.data(), blob.size(), s);
    if (ust) return ust;
    const MicroHdr* dh = reinterpret_cast<const MicroHdr*>(base);
    const MicroTensor* dd = reinterpret_cast<const MicroTensor*>(base + off_dts);
    if (n32 > 0) {
        micro_route_kernel<float><<<(unsigned)n32, kThreads, 0, s>>>(dh, dd);
        CRESSO_LAUNCHED("micro_route_kernel<float>");
    }
    if (n32 < n) {
        micro_route_kernel<double><<<(unsigned)(n - n32), kThreads, 0, s>>>(dh, dd + n32);
        CRESSO_LAUNCHED("micro_route_kernel<double>");
    }
    return CRESSO_OK;
}

}  // extern "C"
