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

struct MicroShared {
    double red[16 * kWarps];
    double tot[16];
    float scale, emean, gm, kk;
    float c_rat, c_bnd, c_t, c_pred, c_err, gain;
};

// Gram index of the pair (a, b), a <= b, of five vectors.
__host__ __device__ constexpr int g5(int a, int b) { return a * 5 - (a * (a - 1)) / 2 + (b - a); }

__global__ void __launch_bounds__(kThreads) micro_route_kernel(const MicroHdr* __restrict__ hdr,
                                                                const MicroTensor* __restrict__ dts) {
    __shared__ MicroShared sh;
    const MicroTensor& D = dts[blockIdx.x];
    const double* hp = hdr->hp;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dt = D.dtype;
    const int64_t N = D.N;
    const double Nd = (double)N;
    const float eps = (float)hp[M_EPS];
    const float sgn = hp[M_MAX] != 0.0 ? -1.0f : 1.0f;
    const float wd = (float)hp[M_WD];
    const bool wd_on = hp[M_WD] != 0.0;
    // f = g (+ wd p), with g negated under maximize (cresso_v5.py:833-834, 907-912)
    auto force = [&](int64_t e) {
        float f = sgn * load_elem(D.grad, e, dt);
        if (wd_on) f = f + wd * load_elem(D.param, e, dt);
        return f;
    };

    // ---- sweep 1: force energy -> force_rms, scale  (cresso_v5.py:1375-1378)
    {
        double s = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const float f = force(e);
            s += (double)(f * f);
        }
        double v[1] = {s};
        block_sum_to<1>(v, sh.red, sh.tot);
        if (tid == 0) {
            const float frn = sqrtf((float)(sh.tot[0] / Nd) + eps);
            const float fr = reservoir(*D.force_rms, frn, hp[M_RD], D.step);
            *D.force_rms = fr;
            sh.scale = fmaxf(fr, eps);
        }
        __syncthreads();
    }
    const float scale = sh.scale;
    auto rel_of = [&](float f) { return fminf(fabsf(f) / scale + eps, 1.0e4f); };

    // instant metric of the micro route: coupling min(0.35, c), every axis (cresso_v5.py:1390-1392, 243-262)
    const double ic = fmin(0.35, hp[M_IC]);
    const float pw = fmaxf((float)hp[M_IP], 0.25f);
    const bool inst_on = ic != 0.0 && N > 1;
    const bool marg = inst_on && D.ndim >= 2;
    auto idens = [&](float rel) { return pw == 1.0f ? fmaxf(rel, eps) : fminf(powf(fmaxf(rel, eps), pw), 1.0e6f); };

    // ---- sweep 2: energy field and the instant-metric density  (cresso_v5.py:1380-1392)
    {
        const float ep = (float)hp[M_EP];
        const float md = (float)hp[M_MD], omd = (float)(1.0 - hp[M_MD]);
        const bool first = D.step <= 1;
        double se = 0.0, sd = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const float rel = rel_of(force(e));
            const float dens = powf(rel, ep);
            const float en = first ? dens : D.energy[e] * md + omd * dens;
            D.energy[e] = en;
            se += (double)en;
            if (inst_on) sd += (double)idens(rel);
        }
        double v[2] = {se, sd};
        block_sum_to<2>(v, sh.red, sh.tot);
        if (tid == 0) {
            sh.emean = fmaxf((float)(sh.tot[0] / Nd), eps);
            sh.gm = fmaxf((float)(sh.tot[1] / Nd), eps);
            sh.kk = (float)(ic / ((double)D.ndim * (double)pw));
        }
        __syncthreads();
        if (marg) {
            // log(max(axis mean / mean, eps)) per axis and coordinate: the elements of one
            // coordinate (a slab of N / dims[a]) are summed by one thread when the slab is
            // short, else by one warp (lane-strided, then a shuffle tree); fixed order both ways
            const float gm = sh.gm;
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
                        D.work[off + c] = logf(fmaxf((float)(m * inv_slab) / gm, eps));
                    }
                } else {
                    for (uint32_t c = warp; c < da; c += kWarps) {
                        double m = 0.0;
                        for (uint32_t s = lane; s < slab; s += 32) m += (double)idens(rel_of(force(elem(c, s))));
                        m = warp_sum(m);
                        if (lane == 0) D.work[off + c] = logf(fmaxf((float)(m * inv_slab) / gm, eps));
                    }
                }
                off += da;
            }
            __syncthreads();
        }
    }
    const float emean = sh.emean, gm = sh.gm, kk = sh.kk;
    const float xm = (float)(hp[M_HMC] / fmax(0.25, hp[M_EP]));
    auto tangent = [&](int64_t e, float f) {
        const float rel = rel_of(f);
        const float metric = clampf(powf(D.energy[e] / emean, xm), 0.08f, 12.0f);
        float inst = 1.0f;
        if (marg) {
            // 32-bit index arithmetic (N < 2^31): 64-bit division is a subroutine call
            float lsum = 0.0f;
            uint32_t rem = (uint32_t)e, off = 0;
            for (int a = 0; a < (int)D.ndim; ++a) off += (uint32_t)D.dims[a];
            for (int a = (int)D.ndim - 1; a >= 0; --a) {
                const uint32_t da = (uint32_t)D.dims[a];
                off -= da;
                lsum += D.work[off + rem % da];
                rem /= da;
            }
            inst = clampf(expf(kk * lsum), 0.08f, 12.0f);
        } else if (inst_on) {
            inst = clampf(expf(kk * logf(fmaxf(idens(rel) / gm, eps))), 0.08f, 12.0f);
        }
        return clampf(f / (scale * metric * inst + eps), -1.0e4f, 1.0e4f);
    };
    const float clip = (float)hp[M_CLIP];

    // ---- sweep 3: refractory-gated impulse, prediction error, drive statistics  (cresso_v5.py:1394-1431)
    {
        const float rd = (float)hp[M_REFD], ord = (float)(1.0 - hp[M_REFD]);
        const float rg = (float)hp[M_RG];
        const float mid = (float)hp[M_MID], omid = (float)(1.0 - hp[M_MID]);
        double g[15];
#pragma unroll
        for (int j = 0; j < 15; ++j) g[j] = 0.0;
        for (int64_t e = tid; e < N; e += kThreads) {
            const float t = tangent(e, force(e));
            const float rf = D.refractory[e] * rd + ord * fabsf(t);
            D.refractory[e] = rf;
            const float gate = 1.0f / (1.0f + rg * rf);
            const float im = D.impulse[e] * mid + omid * (t * gate);
            D.impulse[e] = im;
            const double v[5] = {(double)(t / (1.0f + fabsf(t) / clip)), (double)(tanhf(t / clip) * clip), (double)t,
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
            const float sn = sqrtf((float)(G[g5(ER, ER)] / Nd) + eps);
            const float S = reservoir(*D.surprise, sn, hp[M_SD], D.step);
            *D.surprise = S;
            const float sp = (float)hp[M_SPIKE] / (1.0f + S);
            const double a = (double)(1.0f - sp), b = (double)sp;
            const double sh2 = a * a * G[g5(RAT, RAT)] + 2.0 * a * b * G[g5(RAT, BND)] + b * b * G[g5(BND, BND)];
            const float target = sqrtf((float)(sh2 / Nd) + eps);
            auto k_of = [&](int i) { return target / fmaxf(sqrtf((float)(G[g5(i, i)] / Nd) + eps), eps); };
            const float dm = (float)hp[M_DFM] / (1.0f + 0.35f * S);
            const float mm = (float)hp[M_MDM] / (1.0f + 0.25f * S);
            const float rm = (float)hp[M_RFM] / (1.0f + S);
            const float core = clampf(1.0f - dm - 0.5f * mm, 0.0f, 1.0f);
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
            const float DE = reservoir(*D.drive_energy, (float)(fmax(d2, 0.0) / Nd), hp[M_RD], D.step);
            *D.drive_energy = DE;
            sh.gain = clampf((float)hp[M_TGT] / sqrtf(DE + eps), (float)hp[M_MING], (float)hp[M_MAXG]);
            sh.c_rat = (float)c[RAT];
            sh.c_bnd = (float)c[BND];
            sh.c_t = (float)c[TT];
            sh.c_pred = (float)c[PR];
            sh.c_err = (float)c[ER];
        }
        __syncthreads();
    }

    // ---- sweep 4: parameter update  (cresso_v5.py:1432)
    {
        const float cr = sh.c_rat, cb = sh.c_bnd, ct = sh.c_t, cp = sh.c_pred, ce = sh.c_err, gain = sh.gain;
        const float neg_lr = (float)(-hp[M_LR]);
        const float neg_lr16 = neg_lr_in(hp[M_LR], dt);
        for (int64_t e = tid; e < N; e += kThreads) {
            const float t = tangent(e, force(e));
            const float im = D.impulse[e];
            const float drive = cr * (t / (1.0f + fabsf(t) / clip)) + cb * (tanhf(t / clip) * clip) + ct * t +
                                cp * im + ce * (t - im);
            apply_update(D.param, e, dt, neg_lr, neg_lr16, drive * gain);
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
        CRESSO_REQUIRE(d.dtype == CRESSO_DTYPE_F32 || d.dtype == CRESSO_DTYPE_F16 || d.dtype == CRESSO_DTYPE_BF16,
                       CRESSO_EUNSUPPORTED, "tensor %lld: dtype code %lld (float32, float16 and bfloat16 are supported)",
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
        if (d.ndim >= 2) off = align_up(off + 4 * lead_sum, 256);
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
    MicroHdr h{};
    h.n = n;
    memcpy(h.hp, hp, sizeof(cresso_hparams));
    const int64_t off_dts = align_up((int64_t)sizeof(MicroHdr), 256);
    cudaStream_t s = (cudaStream_t)stream;
    CRESSO_CUDA(cudaMemcpyAsync(base, &h, sizeof(h), cudaMemcpyHostToDevice, s));
    CRESSO_CUDA(cudaMemcpyAsync(base + off_dts, dts.data(), sizeof(MicroTensor) * n, cudaMemcpyHostToDevice, s));
    micro_route_kernel<<<(unsigned)n, kThreads, 0, s>>>(reinterpret_cast<const MicroHdr*>(base),
                                                         reinterpret_cast<const MicroTensor*>(base + off_dts));
    CRESSO_LAUNCHED("micro_route_kernel");
    return CRESSO_OK;
}

}  // extern "C"
