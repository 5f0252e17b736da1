// Lean pass kernels P2-P5 for the dominant tensor class.
//
// The large 2-D weights of a transformer (every tensor of the 7B-shaped set
// but the norm vectors) are float32, made of full 256-column tiles, and
// stepped with the default hyper-parameters: two hash tables of <= 64 bins,
// rank padded to 8, no weight decay, no local sharpness, instant metric power
// 1.  For that class the general pass kernel (spectral_pass_kernel) is
// replaced by these kernels, which keep its item schedule, its per-(block,
// tensor) records and its reduction order (the reduce / finalize kernels are
// shared), and differ in how an item moves through the SM:
//
//  * staging by the TMA engine: the item's tiles (16 rows of 1 KB of the
//    gradient or tangent, 16 rows of the joint bin indices, the 16 carrier
//    rows, P5: the parameter rows) are 1-D bulk copies (cp.async.bulk) issued
//    by one warp and counted on an mbarrier, two stages deep, so no thread
//    computes a staging address per element;
//  * one 16-bit joint bin index per element, j = b0 + 64 b1 (a section of the
//    hash cache), and per-tensor joint tables in shared memory: P3 reads the
//    clamped hash metric of both tables, P4 / P5 the hash prediction, with a
//    single lookup; P2 / P3 split j for the two bin-sum atomics;
//  * P3 writes the tangent and P5 the updated parameter in place into the
//    staged tile, and the tile goes back to HBM as 16 bulk stores (the next
//    item's loads are issued half-way through the item, after the previous
//    store has finished reading its buffer);
//  * P4 / P5 evaluate the drive shaping on row pairs with the two-lane fp32
//    instructions of sm_100 (fma / mul / add .f32x2), including tanh, and P4
//    accumulates its 29-entry Gram on them;
//  * every wait is bounded: a stage that does not arrive within 1 s, or a
//    tensor-core product that does not complete, sets bit 1 of the status
//    word and stops the block after the copies and products in flight have
//    landed (bit 2 if those do not land within their own bound either).
//
// Arithmetic follows spectral_pass_kernel line for line except: tanh is the
// two-lane form below (within 5e-7 relative of tanhf), and the products of
// the joint tables are formed once per bin pair instead of per element (the
// same float operations, so the same values).
#pragma once

namespace cresso {

constexpr uint64_t kStageWaitNs = 1000000000ull;  // bound of one staging wait (1 s)

// 1-D bulk copy global -> this CTA's shared memory, its bytes counted on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// 1-D bulk copy shared -> global, tracked by this thread's bulk async-groups.
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every bulk store this thread issued has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until every bulk store this thread issued is complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// One non-blocking test of a phase (no loop).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait in two parts: one test inline (the common case: the phase is
// complete), the polling loop out of line so that it costs the streaming
// loop no registers.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    return mbar_wait_bounded(bar, parity, limit_ns);
}
__device__ __forceinline__ bool mbar_wait_quick(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    return mbar_test(bar, parity) || mbar_wait_slow(bar, parity, limit_ns);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// tanh of two values on the two-lane fp32 pipe: x P(x^2) / Q(x^2) with P and
// Q of degree 4, fitted here for minimum relative error of tanh on [0, 9]
// (4.6e-7 in float32 with the special-function reciprocal) and |x| clamped to
// 9, where tanh is 1 in float32 to within that bound.
__device__ __forceinline__ float2 tanh2(float2 x) {
    const float2 xc = f2(fminf(fmaxf(x.x, -9.0f), 9.0f), fminf(fmaxf(x.y, -9.0f), 9.0f));
    const float2 y = __fmul2_rn(xc, xc);
    float2 p = f2(1.3350115679600094e-08f);
    p = __ffma2_rn(p, y, f2(2.060582301055547e-05f));
    p = __ffma2_rn(p, y, f2(0.003495392156764865f));
    p = __ffma2_rn(p, y, f2(0.13380861282348633f));
    p = __ffma2_rn(p, y, f2(1.0f));
    float2 q = f2(7.774701771268155e-07f);
    q = __ffma2_rn(q, y, f2(0.0003285312559455633f));
    q = __ffma2_rn(q, y, f2(0.0258762389421463f));
    q = __ffma2_rn(q, y, f2(0.4671417772769928f));
    q = __ffma2_rn(q, y, f2(1.0f));
    return __fmul2_rn(__fmul2_rn(xc, p), f2(rcp_approx(q.x), rcp_approx(q.y)));
}

// log(1 + x), x >= 0, of two values: log1p_pos lane by lane, with its series on
// the two-lane pipe.
__device__ __forceinline__ float2 log1p_pos2(float2 x) {
    const float2 d = __fadd2_rn(x, f2(2.0f));  // in [2, 3] on the branch that uses it
    const float2 z = __fmul2_rn(x, f2(rcp_approx(d.x), rcp_approx(d.y)));
    const float2 w = __fmul2_rn(z, z);
    float2 p = f2(1.0f / 13.0f);
    p = __ffma2_rn(p, w, f2(1.0f / 11.0f));
    p = __ffma2_rn(p, w, f2(1.0f / 9.0f));
    p = __ffma2_rn(p, w, f2(1.0f / 7.0f));
    p = __ffma2_rn(p, w, f2(1.0f / 5.0f));
    p = __ffma2_rn(p, w, f2(1.0f / 3.0f));
    const float2 series = __fmul2_rn(f2(2.0f), __ffma2_rn(__fmul2_rn(z, w), p, z));
    const float2 u = __fadd2_rn(f2(1.0f), x);
    const float2 lg = __fmul2_rn(f2(0.693147180559945309f), f2(__log2f(u.x), __log2f(u.y)));
    return f2(x.x <= 1.0f ? series.x : lg.x, x.y <= 1.0f ? series.y : lg.y);
}

// Drive components of two elements (cresso_v5.py:1315-1326; drive_parts on a row pair).
// The bounded channel tanh(t / clip) clip enters only u, so its factor clip rides
// on the spike mix (DriveK2::sp_clip).  NOV_SCALED false returns the novelty
// without its factor clip, for a caller that folds clip into the novelty's
// coefficient (P5).
struct Drive2 {
    float2 u, root, nov, rat;
};
// Per-tensor constants of the drive shaping: omsp = 1 - sp and sp_clip = sp clip
// in place of the spike mix sp, and clip2e = clip^2 + eps: min(|t|, clip^2) + eps
// = min(|t| + eps, clip^2 + eps) exactly (rounding is monotone).
struct DriveK2 {
    float clip, inv_clip, clip2e, omsp, sp_clip, invD, eps;
};
template <bool NOV_SCALED = true>
__device__ __forceinline__ Drive2 drive_parts2(float2 t, float2 pred, const DriveK2& c) {
    Drive2 d;
    const float2 at = f2(fabsf(t.x), fabsf(t.y));
    const float2 den = __ffma2_rn(at, f2(c.inv_clip), f2(1.0f));  // in [1, 1 + 1e4 / clip]
    d.rat = __fmul2_rn(t, f2(rcp_approx(den.x), rcp_approx(den.y)));
    const float2 bnd1 = tanh2(__fmul2_rn(t, f2(c.inv_clip)));  // bounded channel over clip
    const float2 ae = __fadd2_rn(at, f2(c.eps));
    const float2 rr = f2(fminf(ae.x, c.clip2e), fminf(ae.y, c.clip2e));
    d.root = f2(t.x != 0.0f ? copysignf(sqrt_sfu(rr.x), t.x) : 0.0f, t.y != 0.0f ? copysignf(sqrt_sfu(rr.y), t.y) : 0.0f);
    d.u = __ffma2_rn(f2(c.sp_clip), bnd1, __fmul2_rn(f2(c.omsp), d.rat));
    d.nov = tanh2(__fmul2_rn(__fadd2_rn(t, f2(-pred.x, -pred.y)), f2(c.invD)));
    if constexpr (NOV_SCALED) d.nov = __fmul2_rn(d.nov, f2(c.clip));
    return d;
}

template <int PASS>
struct FastCfg {
    static constexpr int kRM = 8;
    static constexpr int kXB = 16 * 256 * 4;                             // gradient / tangent rows
    static constexpr int kJB = 16 * 256 * 2;                             // joint bin indices
    static constexpr int kRTB = PASS <= 3 ? 16 * 2 * kRM * 4 : 0;        // carrier rows (P2 / P3 projections)
    static constexpr int kPB = PASS == 5 ? kXB : 0;                      // parameter rows (P5)
    static constexpr int kStage = kXB + kJB + kRTB + kPB;
    static constexpr bool kTCR = PASS >= 3;
    static constexpr bool kBins = PASS == 2 || PASS == 3;
    static constexpr bool kJoint = PASS >= 3;                            // joint lookup table in shared memory
    static constexpr bool kStore = PASS == 3 || PASS == 5;               // the tile goes back to HBM
    // fixed-point bin copies per set (P3: two sets of 4 fit its shared memory, 113 KB)
    static constexpr int kCopies = PASS == 3 ? 4 : 16;
    // every pass waits on the stage and product barriers thread by thread and
    // synchronises the block once per item, at its end; the bin copies alternate by item
    static constexpr int kBinSets = kBins ? 2 : 1;
    static constexpr int kAcc = PASS == 4 ? kWarps * 32 : (kBins ? 2 * kRM * kThreads : 0);
};

// Shared-memory bytes of a fast pass kernel for tb = hash_bins * hash_tables.
__host__ __device__ inline size_t fast_smem_layout(int pass, int tb, size_t* off) {
    // off[0] stages, [1] barriers, [2] s_red, [3] s_tot, [4] s_acc, [5] s_coef, [6] s_ibin, [7] s_lbin,
    // [8] s_fbin, [9] s_joint, [10] s_rowred / s_rowf, [11] tc B tiles, [12] end
    const int xb = 16 * 256 * 4, jb = 16 * 256 * 2, rtb = pass <= 3 ? 16 * 16 * 4 : 0, pb = pass == 5 ? xb : 0;
    const size_t stage = (size_t)(xb + jb + rtb + pb);
    const bool bins = pass == 2 || pass == 3;
    const int copies = pass == 3 ? 4 : 16;
    const int sets = bins ? 2 : 1;
    const size_t acc = pass == 4 ? kWarps * 32 : (bins ? 2 * 8 * kThreads : 0);
    size_t o = 0;
    off[0] = o; o += 2 * stage;
    off[1] = o; o += 64;                                   // full[2], tc and drain barriers, TMEM slot, flags
    // s_red / s_tot: only the segment flush uses them; P3-P5 lay them over the joint table
    off[2] = o; o += pass >= 3 ? 0 : (size_t)kNSRec * kWarps * 8;
    off[3] = o; o += pass >= 3 ? 0 : (size_t)kNSRec * 8;
    off[4] = o; o += acc * 8;
    off[5] = o; o += (4 * 8 + 4) * 4;
    off[6] = o; o += bins ? (size_t)sets * copies * (tb + 1) * 4 : 0;
    o = (o + 7) & ~(size_t)7;
    off[7] = o; o += bins ? (size_t)tb * 8 : 0;
    off[8] = o; o += bins ? (size_t)tb * 4 : 0;
    off[9] = o; o += pass >= 3 ? 4096 * 4 : 0;
    off[10] = o; o += pass == 2 ? 2 * 16 * kWarps * 4 : (pass == 3 ? 2 * 16 * 4 : 0);
    o = (o + 127) & ~(size_t)127;
    off[11] = o; o += pass >= 3 ? 4 * kTcTileBytes + 128 : 0;  // + slack to align the tiles to 128 bytes
    off[12] = o;
    return o;
}

template <int PASS>
__global__ void __launch_bounds__(kThreads, 2)
fast_pass_kernel(const GroupHdr* __restrict__ hdr, const DevTensor* __restrict__ dts,
                 const int64_t* __restrict__ item_base, const int32_t* __restrict__ tmap,
                 double* __restrict__ rec_scal, float* __restrict__ rec_bins) {
    using Cfg = FastCfg<PASS>;
    constexpr int RM = Cfg::kRM;
    constexpr int ITERS = 16, UNR = 4;  // rows per TMEM read
    constexpr bool TCR = Cfg::kTCR;
    extern __shared__ __align__(128) unsigned char fast_smem[];
    unsigned char* smem_raw = fast_smem;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const int64_t n_items = hdr->cls_items[0];
    const int nt = (int)hdr->cls_nt[0];
    const int TB = (int)hdr->tb, B = (int)hdr->bins;
    const float eps = (float)hdr->hp[H_EPS];
    const float ep = (float)hdr->hp[H_EP];
    // P3's metric: exp(coupling * clamp(lm, -3, 3)) = 2^clamp(mc2 lm, -mhi, mhi), with the
    // factor mc2 folded into the reconstruction coefficients; clamping to [0.06, 16]
    // afterwards changes nothing when |3 mc2| <= 3.99 (2^3.99 < 16, 2^-3.99 > 0.06)
    const float mc2 = (float)hdr->hp[H_MC] * 1.4426950408889634f;
    const float mhi = fabsf(3.0f * mc2);
    const bool mclamp = !(mhi <= 3.99f);
    const float tmix = (float)hdr->hp[H_TM];
    const int64_t it0 = (int64_t)blockIdx.x * n_items / gridDim.x;
    const int64_t it1 = ((int64_t)blockIdx.x + 1) * n_items / gridDim.x;

    size_t off[13];
    fast_smem_layout(PASS, TB, off);
    unsigned char* s_stage = smem_raw + off[0];
    uint64_t* s_full = reinterpret_cast<uint64_t*>(smem_raw + off[1]);  // [0], [1]: stage barriers
    // one product barrier per D buffer: the products of item i + 1 (issued while slower
    // threads may still test item i's) complete the other buffer's barrier, so no barrier
    // runs two phases ahead of a thread that waits on it
    uint64_t* s_tcbar = s_full + 2;  // [2]
    uint64_t* s_drainbar = s_full + 4;
    uint32_t* s_tcslot = reinterpret_cast<uint32_t*>(s_full + 5);
    int* s_flag = reinterpret_cast<int*>(s_tcslot + 1);
    int* s_abort = s_flag + 1;
    double* s_red = reinterpret_cast<double*>(smem_raw + (PASS >= 3 ? off[9] : off[2]));
    double* s_tot = s_red + kNSRec * kWarps;
    double* s_acc = reinterpret_cast<double*>(smem_raw + off[4]);
    float* s_coef = reinterpret_cast<float*>(smem_raw + off[5]);
    int* s_ibin = reinterpret_cast<int*>(smem_raw + off[6]);
    long long* s_lbin = reinterpret_cast<long long*>(smem_raw + off[7]);
    float* s_fbin = reinterpret_cast<float*>(smem_raw + off[8]);
    float* s_joint = reinterpret_cast<float*>(smem_raw + off[9]);
    float* s_rows = reinterpret_cast<float*>(smem_raw + off[10]);
    unsigned char* s_tcb = smem_raw + off[11];
    s_tcb += ((smem_u32(s_tcb) + 127u) & ~127u) - smem_u32(s_tcb);  // 128-byte aligned operand tiles

    const uint32_t full0 = smem_u32(&s_full[0]);
    auto full_bar = [&](int b) -> uint32_t { return full0 + 8u * (uint32_t)b; };
    uint32_t tc_base = 0, tc_parity = 0;  // tc_parity bit b: parity of the next completion of s_tcbar[b]
    if (tid == 0) {
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        if constexpr (TCR) {
            mbar_init(&s_tcbar[0], 4);  // one arrival per issuing thread
            mbar_init(&s_tcbar[1], 4);
            mbar_init(s_drainbar, 4);   // the same four threads, once, after a give-up
        }
        *s_abort = 0;
    }
    if constexpr (TCR) {
        if (warp == 0) tc_alloc(s_tcslot, kTcCols);
        tc_fence_before();
    }
    __syncthreads();
    if constexpr (TCR) {
        tc_fence_after();
        tc_base = *s_tcslot;
    }

    constexpr int ncopies = Cfg::kCopies;
    const int cstride = TB + 1;
    const BinFix fix = bin_fix(ncopies, ITERS);
    int ip = 0;  // item parity: the bin copies and row sums of passes without a top barrier alternate

    uint32_t ph = 0u;        // bit b: parity of the next completion of stage barrier b
    uint32_t inflight = 0u;  // tid 0, bit b: loads issued into stage b and not yet consumed
    bool abort = false;
    int buf = 0;

    int k = find_tensor(item_base, nt, it0);
    int64_t it = it0;
    while (it < it1) {
        // ---- tensor descriptor and constants
        const DevTensor* __restrict__ Dp = dts + tmap[k];
        const int64_t rows = Dp->rows, cols = Dp->cols, row0 = Dp->row0, col0 = Dp->col0, gcols = Dp->gcols;
        const int64_t ibase = item_base[k];
        const int64_t seg_end = min(it1, item_base[k + 1]);
        const int flags = Dp->flags;
        const int n_bands = Dp->n_bands;
        const float* __restrict__ rowtab = Dp->rowtab;
        const float* __restrict__ coltab = Dp->coltab;
        const uint16_t* __restrict__ joint =
            reinterpret_cast<const uint16_t*>(reinterpret_cast<const unsigned char*>(Dp->hidx) +
                                              align_up(2 * Dp->hidx_n, 256));
        const float* __restrict__ xsrc = PASS <= 3 ? Dp->grad : Dp->tbuf;
        float* __restrict__ xdst = PASS == 3 ? Dp->tbuf : Dp->param;  // where the stored tile goes
        const TensorConsts* __restrict__ Cp = Dp->cst;
        const float sgn = (flags & F_MAXIMIZE) ? -1.0f : 1.0f;
        float scale = 0.f, inv_scale = 0.f, sscale = 0.f, seps = 0.f;
        DriveK2 dk{};
        float c_u = 0.f, c_root = 0.f, c_t = 0.f, c_nov = 0.f, c_hp = 0.f, gain = 0.f, neg_lr = 0.f;
        if constexpr (PASS == 2 || PASS == 3) {
            scale = Cp->scale;
            inv_scale = Cp->inv_scale;
            sscale = sgn * scale;
            seps = sgn * eps;
        }
        if constexpr (PASS >= 4)
            dk = DriveK2{Cp->clip, Cp->inv_clip, Cp->clip2 + eps, 1.0f - Cp->sp, Cp->sp * Cp->clip, Cp->invD, eps};
        if constexpr (PASS == 5) {
            c_u = Cp->c_u;
            c_root = Cp->c_root;
            c_t = Cp->c_t;
            c_nov = Cp->c_nov * Cp->clip;  // the novelty comes without its factor clip (drive_parts2<false>)
            c_hp = Cp->c_hp;
            gain = Cp->gain;
            neg_lr = Cp->neg_lr;
        }
        const bool echo_on = (flags & F_ECHO) != 0;
        __syncthreads();  // the previous segment is done with the shared tables
        if constexpr (PASS >= 3) {
            const float* al1 = PASS == 3 ? Cp->m_al : Cp->pr_al;
            const float* be1 = PASS == 3 ? Cp->m_be : Cp->pr_be;
            const float* al2 = PASS == 3 ? Cp->p0_al : (PASS == 4 ? Cp->ec_al : Cp->cb_al);
            const float* be2 = PASS == 3 ? Cp->p0_be : (PASS == 4 ? Cp->ec_be : Cp->cb_be);
            // P3: the log-metric coefficients scaled by mc2 = coupling * log2(e), so that the
            // product holds the exponent of the metric in base 2 directly
            const float c1 = PASS == 3 ? mc2 : 1.0f;
            if (tid < RM) {
                s_coef[tid] = al1[tid] * c1;
                s_coef[RM + tid] = be1[tid] * c1;
                s_coef[2 * RM + tid] = al2[tid];
                s_coef[3 * RM + tid] = be2[tid];
            }
            if (tid == 0) {
                s_coef[4 * RM] = PASS == 3 ? Cp->m_K * c1 : Cp->pr_K;
                s_coef[4 * RM + 1] = PASS == 3 ? Cp->p0_K : (PASS == 4 ? Cp->ec_K : Cp->cb_K);
            }
            // joint table over the bin pairs (b0, b1), j = b0 + 64 b1:
            //   P3: the clamped hash metric prod_t root_t(b_t); P4 / P5: mean_t impulse_t(b_t)
            const float* ht = Dp->htab;
            for (int j = tid; j < 4096; j += kThreads) {
                const int b0 = j & 63, b1 = j >> 6;
                float v = 0.0f;
                if (b0 < B && b1 < B) {
                    if constexpr (PASS == 3) {
                        float hm = 1.0f;
                        hm *= ht[b0];
                        hm *= ht[B + b1];
                        v = clampf(hm, 0.08f, 12.0f);
                    } else {
                        float hp = 0.0f;
                        hp += ht[b0];
                        hp += ht[B + b1];
                        v = hp * 0.5f;
                    }
                }
                s_joint[j] = v;
            }
        }
        if constexpr (Cfg::kBins) {
            for (int b = tid; b < Cfg::kBinSets * ncopies * cstride; b += kThreads) s_ibin[b] = 0;
            for (int b = tid; b < TB; b += kThreads) {
                s_lbin[b] = 0;
                s_fbin[b] = 0.0f;
            }
        }
        if constexpr (Cfg::kAcc > 0) {
            for (int j = tid; j < Cfg::kAcc; j += kThreads) s_acc[j] = 0.0;
        }
        // arm the stage barriers of the segment's first two items (the barrier below orders the
        // arming before their copies; every thread has consumed both barriers' earlier phases)
        auto arm_stage = [&](int b) {
            if (tid == 0) mbar_arrive_expect(full_bar(b), (uint32_t)Cfg::kStage);
        };
        arm_stage(buf);
        if (it + 1 < seg_end) arm_stage(buf ^ 1);
        __syncthreads();
        double acc0 = 0.0, acc1 = 0.0;
        const int lc = tid;  // this thread's column of the 256-column tile

        // Stage item (ct, band) into buffer b.  Every warp issues the copies of its two rows
        // (lanes 0-1: the tile that goes back to HBM in P3 / P5, or the gradient / tangent;
        // lanes 2-5: the other tiles), so no warp carries the whole item's copies.  The stage
        // barrier was armed with the item's bytes by thread 0 before a block barrier that
        // precedes every one of these copies (arm_stage).  Lanes 0-1 first wait until their
        // own stores of that buffer's previous rows have been read.
        auto stage = [&](int ct_, int band_, int b) {
            if constexpr (Cfg::kStore) {
                if (lane < 2) bulk_wait_read_all();
                __syncwarp();
            }
            if (tid == 0) inflight |= 1u << b;
            const uint32_t sb = smem_u32(s_stage + (size_t)b * Cfg::kStage);
            const int64_t rb = (int64_t)band_ * ITERS, cb = (int64_t)ct_ * 256;
            const int rr = 2 * warp + (lane & 1);  // this lane's row of the item
            const int64_t r = rb + rr;
            const int kind = lane >> 1;
            constexpr int kPOff = Cfg::kXB + Cfg::kJB + Cfg::kRTB;
            if (kind == 0) {
                if constexpr (Cfg::kPB > 0)
                    bulk_load(sb + kPOff + rr * 1024, Dp->param + r * cols + cb, 1024, full_bar(b));
                else
                    bulk_load(sb + rr * 1024, xsrc + r * cols + cb, 1024, full_bar(b));
            } else if (kind == 1) {
                if constexpr (Cfg::kPB > 0)
                    bulk_load(sb + rr * 1024, xsrc + r * cols + cb, 1024, full_bar(b));
                else
                    bulk_load(sb + Cfg::kXB + rr * 512, joint + (row0 + r) * gcols + col0 + cb, 512, full_bar(b));
            } else if (kind == 2) {
                if constexpr (Cfg::kPB > 0)
                    bulk_load(sb + Cfg::kXB + rr * 512, joint + (row0 + r) * gcols + col0 + cb, 512, full_bar(b));
                else if (Cfg::kRTB > 0 && warp == kWarps - 1 && lane == 4)
                    bulk_load(sb + Cfg::kXB + Cfg::kJB, rowtab + (row0 + rb) * 2 * RM, Cfg::kRTB, full_bar(b));
            }
        };

        float2 g2[PASS == 4 ? kGram : 1];
#pragma unroll
        for (int q = 0; q < (PASS == 4 ? kGram : 1); ++q) g2[q] = f2(0.0f);
        int ct = (int)((it - ibase) / n_bands);
        int band = (int)((it - ibase) - (int64_t)ct * n_bands);
        stage(ct, band, buf);
        if constexpr (PASS == 3) {  // the first item's instant-metric row factors (the prologue barrier follows)
            if (tid < ITERS) s_rows[ip * ITERS + tid] = Dp->rowf[band * ITERS + tid];
        }
        int items_since_flush = 0;
        float colf = 1.0f;
        int uv_ct = -1;
        int tcb = 0;
        int a_ct = -1;
        const int tc_h = tid >> 7;
        const uint32_t tc_lane = (uint32_t)(tid & 96) << 16;
        auto tc_build_a = [&](int c) {
            if constexpr (TCR) tc_column_factors<RM>(coltab, gcols, col0 + (int64_t)c * 256 + lc, s_coef, tc_base + tc_lane + 32 * tc_h);
        };
        auto tc_load_b = [&](int bnd) -> float {
            if constexpr (TCR) return __ldg(rowtab + (row0 + (int64_t)bnd * 16 + (tid >> 4)) * 16 + (tid & 15));
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
                tc_commit(smem_u32(&s_tcbar[bb]));
            }
        };
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
        float2 z12[RM];
        float zc = 0.0f;
        double colrun = 0.0;  // P2: this column's density over the current run of bands
#pragma unroll
        for (int q = 0; q < RM; ++q) z12[q] = f2(0.0f);

        for (; it < seg_end; ++it) {
            const int col = ct * 256 + lc;
            const int gc = (int)col0 + col;
            const int rbase = band * ITERS;
            const int nband = band + 1 == n_bands ? 0 : band + 1;
            const int nct = band + 1 == n_bands ? ct + 1 : ct;
            const bool has_next = it + 1 < seg_end;
            if (!Cfg::kStore && has_next) stage(nct, nband, buf ^ 1);
            // every thread waits for the stage and its products itself; a wait that gives
            // up marks the block, which stops at the end of this item (the item computes
            // on whatever the buffers hold; nothing is read or written out of bounds)
            bool ok = mbar_wait_quick(full_bar(buf), (ph >> buf) & 1u, kStageWaitNs);
            if (ok) {
                ph ^= 1u << buf;
                if (tid == 0) inflight &= ~(1u << buf);
            }
            if constexpr (TCR) {
                ok = mbar_wait_quick(smem_u32(&s_tcbar[tcb]), (tc_parity >> tcb) & 1u, kTcWaitNs) && ok;
                tc_parity ^= 1u << tcb;
            }
            if (!ok) {
                atomicOr(s_abort, 1);
                atomicOr(hdr->status, 1);
            }

            int* my_bins = s_ibin + (ip * ncopies + (tid & (ncopies - 1))) * cstride;
            float* rows_ip = s_rows + (PASS == 2 ? ip * ITERS * kWarps : 0);
            const unsigned char* sb = s_stage + (size_t)buf * Cfg::kStage;
            float* xb = reinterpret_cast<float*>(const_cast<unsigned char*>(sb));
            const uint16_t* jb = reinterpret_cast<const uint16_t*>(sb + Cfg::kXB);
            const float* rtb = reinterpret_cast<const float*>(sb + Cfg::kXB + Cfg::kJB);
            float* pb = reinterpret_cast<float*>(const_cast<unsigned char*>(sb + Cfg::kXB + Cfg::kJB + Cfg::kRTB));
            (void)rtb;
            (void)pb;

            if constexpr (PASS == 3) {
                if (ct != uv_ct) {
                    uv_ct = ct;
                    if (flags & F_INST2D) colf = Dp->colf[col];
                }
                // the next item's instant-metric row factors into the other buffer (read after
                // this item's end barrier); the first item's were loaded before the item loop
                if (has_next && tid < ITERS) s_rows[(ip ^ 1) * ITERS + tid] = Dp->rowf[nband * ITERS + tid];
            }
            if constexpr (TCR) {
                tc_fence_after();
                if (has_next) {
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
            const float* rowf_ip = s_rows + (PASS == 3 ? ip * ITERS : 0);
            float2 s02 = f2(0.0f), s12 = f2(0.0f), col2 = f2(0.0f);  // even / odd rows
            bool big = false;  // a bin value too large for the fixed-point sums (added after the rows)

#pragma unroll
            for (int m0 = 0; m0 < ITERS; m0 += UNR) {
                if (Cfg::kStore && m0 == ITERS / 2 && has_next) stage(nct, nband, buf ^ 1);
                float R1[UNR], R2[UNR];
                if constexpr (TCR) {
                    const uint32_t ta = tc_base + tc_lane + 128 + 64 * tcb + 16 * tc_h + m0;
                    tc_ld<UNR>(ta, R1);
                    tc_ld<UNR>(ta + 32, R2);
                    tc_wait_ld();
                }
                if constexpr (PASS == 2) {
                    float dv[UNR];
#pragma unroll
                    for (int u = 0; u < UNR; u += 2) {  // two rows on the two-lane pipe
                        const int m = m0 + u;
                        const int o = m * 256 + lc;
                        float2 rel = __ffma2_rn(f2(fabsf(xb[o]), fabsf(xb[o + 256])), f2(inv_scale), f2(eps));
                        rel = f2(fminf(rel.x, 1.0e4f), fminf(rel.y, 1.0e4f));  // |sgn x| = |x|
                        const float2 lg = __fmul2_rn(f2(ep), f2(__log2f(rel.x), __log2f(rel.y)));
                        const float2 ds = f2(ex2_approx(lg.x), ex2_approx(lg.y));
                        const float2 L = log1p_pos2(ds);
                        const float2 Lc = __fadd2_rn(L, f2(-0.5f));
                        dv[u] = rel.x;  // instant metric power 1: the axis density is rel
                        dv[u + 1] = rel.y;
                        s02 = __fadd2_rn(s02, L);
                        s12 = __fadd2_rn(s12, rel);
                        col2 = __fadd2_rn(col2, rel);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float a1[RM], a2[RM];
                            load_row<RM>(rtb, m + h, a1, a2);
                            const float lc_h = h ? Lc.y : Lc.x;
                            const float2 Lc2 = f2(lc_h);
#pragma unroll
                            for (int q = 1; q < RM; ++q) z12[q] = __ffma2_rn(f2(a1[q], a2[q]), Lc2, z12[q]);
                            zc += lc_h;
                            const float dsh = h ? ds.y : ds.x;
                            const int j = jb[o + 256 * h];
                            const bool fx = dsh < fix.vmax;
                            const int qv = fx ? __float2int_rn(dsh * fix.scale) : 0;
                            atomicAdd(&my_bins[j & 63], qv);
                            atomicAdd(&my_bins[B + (j >> 6)], qv);
                            big |= !fx;
                        }
                    }
                    // row sums over the 256 columns: a warp's 32 lanes here, the 8 warps after the item
                    const float x = group_sum4(dv, 32);
                    const int ur = 2 * ((lane & 16) != 0) + ((lane & 8) != 0);
                    if ((lane & 7) == 0) rows_ip[(m0 + ur) * kWarps + warp] = x;
                } else if constexpr (PASS == 3) {
#pragma unroll
                    for (int u = 0; u < UNR; u += 2) {  // two rows on the two-lane pipe
                        const int m = m0 + u;
                        const int o = m * 256 + lc;
                        // t = sgn x / (den + eps) = x / (sgn den + sgn eps): the sign rides on the
                        // scale and on eps (exact)
                        const float2 f = f2(xb[o], xb[o + 256]);
                        float2 metric = f2(ex2_approx(clampf(R1[u], -mhi, mhi)), ex2_approx(clampf(R1[u + 1], -mhi, mhi)));
                        if (mclamp) metric = f2(clampf(metric.x, 0.06f, 16.0f), clampf(metric.y, 0.06f, 16.0f));
                        float2 den = __fmul2_rn(f2(sscale), metric);
                        if (flags & F_INST2D)
                            den = __fmul2_rn(den, f2(clampf(rowf_ip[m] * colf, 0.08f, 12.0f),
                                                     clampf(rowf_ip[m + 1] * colf, 0.08f, 12.0f)));
                        const int j0 = jb[o], j1 = jb[o + 256];
                        den = __fmul2_rn(den, f2(s_joint[j0], s_joint[j1]));
                        const float2 de = __fadd2_rn(den, f2(seps));
                        float2 t = __fmul2_rn(f, f2(rcp_approx(de.x), rcp_approx(de.y)));
                        t = f2(clampf(t.x, -1.0e4f, 1.0e4f), clampf(t.y, -1.0e4f, 1.0e4f));
                        xb[o] = t.x;  // in place: the tile goes back to the tangent buffer
                        xb[o + 256] = t.y;
                        const float2 err = __fadd2_rn(t, f2(-R2[u], -R2[u + 1]));
                        s02 = __ffma2_rn(err, err, s02);
                        s12 = __fadd2_rn(s12, t);
                        const float2 port = __ffma2_rn(f2(tmix), t, err);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float a1[RM], a2[RM];
                            load_row<RM>(rtb, m + h, a1, a2);
                            const float th = h ? t.y : t.x;
                            const float2 t2 = f2(th);
#pragma unroll
                            for (int q = 1; q < RM; ++q) z12[q] = __ffma2_rn(f2(a1[q], a2[q]), t2, z12[q]);
                            zc += th;
                            const float ph_ = h ? port.y : port.x;
                            const int j = h ? j1 : j0;
                            const bool fx = fabsf(ph_) < fix.vmax;  // false for non-finite values
                            const int qv = fx ? __float2int_rn(ph_ * fix.scale) : 0;
                            atomicAdd(&my_bins[j & 63], qv);
                            atomicAdd(&my_bins[B + (j >> 6)], qv);
                            big |= !fx;
                        }
                    }
                } else if constexpr (PASS == 4) {
#pragma unroll
                    for (int u = 0; u < UNR; u += 2) {
                        const int o = (m0 + u) * 256 + lc;
                        const float2 t = f2(xb[o], xb[o + 256]);
                        const float2 pred = f2(R1[u], R1[u + 1]);
                        const float2 echo = echo_on ? f2(R2[u], R2[u + 1]) : f2(0.0f);
                        const float2 hp = f2(s_joint[jb[o]], s_joint[jb[o + 256]]);
                        const Drive2 dp = drive_parts2<true>(t, pred, dk);
                        const float2 v[7] = {dp.u, dp.root, t, pred, dp.nov, echo, hp};
#pragma unroll
                        for (int a = 0; a < 7; ++a)
#pragma unroll
                            for (int b = a; b < 7; ++b) g2[gram_idx(a, b)] = __ffma2_rn(v[a], v[b], g2[gram_idx(a, b)]);
                        g2[28] = __ffma2_rn(dp.rat, dp.rat, g2[28]);
                    }
                } else {  // PASS 5
#pragma unroll
                    for (int u = 0; u < UNR; u += 2) {
                        const int o = (m0 + u) * 256 + lc;
                        const float2 t = f2(xb[o], xb[o + 256]);
                        const float2 pred = f2(R1[u], R1[u + 1]);
                        const float2 comb = f2(R2[u], R2[u + 1]);
                        const float2 hp = f2(s_joint[jb[o]], s_joint[jb[o + 256]]);
                        const Drive2 dp = drive_parts2<false>(t, pred, dk);
                        float2 drive = __fmul2_rn(f2(c_u), dp.u);
                        drive = __ffma2_rn(f2(c_root), dp.root, drive);
                        drive = __ffma2_rn(f2(c_t), t, drive);
                        drive = __fadd2_rn(drive, comb);
                        drive = __ffma2_rn(f2(c_nov), dp.nov, drive);
                        drive = __ffma2_rn(f2(c_hp), hp, drive);
                        const float2 upd = __fmul2_rn(drive, f2(gain));
                        const float2 pn = __ffma2_rn(f2(neg_lr), upd, f2(pb[o], pb[o + 256]));
                        pb[o] = pn.x;
                        pb[o + 256] = pn.y;
                    }
                }
            }  // rows of the item

            if constexpr (PASS == 2 || PASS == 3) {
                // the rare values the fixed-point sums cannot hold go to the float bins here, off
                // the row loop: each is recomputed with the row loop's operations (so the same
                // elements fail its test); P3 reads its prediction from TMEM again (this item's
                // products stay there until the item after next is issued).  The condition is
                // warp-uniform, as the tensor-memory loads need.
                if (__any_sync(0xffffffffu, big)) {
#pragma unroll 1
                    for (int m0 = 0; m0 < ITERS; m0 += UNR) {
                        float R2[UNR];
                        if constexpr (TCR) {
                            const uint32_t ta = tc_base + tc_lane + 128 + 64 * tcb + 16 * tc_h + m0;
                            tc_ld<UNR>(ta + 32, R2);
                            tc_wait_ld();
                        }
#pragma unroll
                        for (int u = 0; u < UNR; ++u) {
                            const int o = (m0 + u) * 256 + lc;
                            float v;
                            bool fx;
                            if constexpr (PASS == 2) {
                                const float rel = fminf(__fmaf_rn(fabsf(xb[o]), inv_scale, eps), 1.0e4f);
                                v = ex2_approx(__fmul_rn(ep, __log2f(rel)));
                                fx = v < fix.vmax;
                            } else {
                                const float t = xb[o];
                                v = __fmaf_rn(tmix, t, __fadd_rn(t, -R2[u]));
                                fx = fabsf(v) < fix.vmax;
                            }
                            if (!fx) {
                                const int j = jb[o];
                                atomicAdd(&s_fbin[j & 63], v);
                                atomicAdd(&s_fbin[B + (j >> 6)], v);
                            }
                        }
                    }
                }
            }

            // ---- item epilogue
            if constexpr (PASS == 2 || PASS == 3) {
                acc0 += (double)(s02.x + s02.y);
                acc1 += (double)(s12.x + s12.y);
                if (nct != ct || it + 1 == seg_end || ++items_since_flush == 4) {
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
#pragma unroll
                    for (int q = 0; q < RM; ++q) z12[q] = f2(0.0f);
                    zc = 0.0f;
                    items_since_flush = 0;
                }
            } else if constexpr (PASS == 4) {
                if (++items_since_flush == 2 || it + 1 == seg_end) {
                    float v[32];
#pragma unroll
                    for (int q = 0; q < 32; ++q) v[q] = q < kGram ? g2[q < kGram ? q : 0].x + g2[q < kGram ? q : 0].y : 0.0f;
                    const float x = warp_transpose_sum32(v);
                    if (lane < kGram) s_acc[warp * 32 + lane] += (double)x;
#pragma unroll
                    for (int q = 0; q < kGram; ++q) g2[q] = f2(0.0f);
                    items_since_flush = 0;
                }
            }
            if constexpr (PASS == 2) {
                // column sums: one float64 per column over the block's run of bands of this
                // column tile, written when the run ends (reduce_kernel, col_runs)
                colrun += (double)(col2.x + col2.y);
                if (nct != ct || it + 1 == seg_end) {
                    reinterpret_cast<double*>(Dp->colpart)[(int64_t)((int)blockIdx.x - Dp->cfirst[2]) * cols + col] =
                        colrun;
                    colrun = 0.0;
                }
            }
            // the buffer of this item is next staged with item i + 2: arm its barrier now, before
            // the end barrier that precedes those copies (every thread consumed this item's phase)
            if (it + 2 < seg_end) arm_stage(buf);
            if constexpr (Cfg::kStore) tc_fence_smem();  // this thread's tile writes, before the bulk store
            if constexpr (TCR) {  // item i + 2's carrier rows into this item's B buffer (its products are done)
                if (it + 2 < seg_end) {
                    tc_store_b(tc_bnext, tcb);
                    tc_fence_smem();
                }
                tc_fence_before();
            }
            __syncthreads();  // the item's tiles and the reduction scratch are complete
            if (*s_abort) {  // a wait gave up in this item (uniform after the barrier)
                abort = true;
                break;
            }
            if constexpr (PASS == 2) {
                if (tid < ITERS) {
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) s += rows_ip[tid * kWarps + w];
                    Dp->rowpart[(int64_t)ct * rows + rbase + tid] = s;
                }
            }
            if constexpr (Cfg::kStore) {  // two rows per warp, each storing lane its own bulk group
                if (lane < 2) {  // this warp's two rows, by the lanes that load them
                    const int rr = 2 * warp + lane;
                    const uint32_t src = smem_u32(PASS == 3 ? (const void*)xb : (const void*)pb);
                    bulk_store(xdst + (int64_t)(rbase + rr) * cols + (int64_t)ct * 256, src + rr * 1024, 1024);
                    bulk_commit();
                }
            }
            if constexpr (TCR) tcb ^= 1;
            if constexpr (Cfg::kBins) {
                // empty this item's fixed-point copies into the exact block sums: before the next
                // item's atomics (P3: its top barrier) or before the item after it reuses them
                // (P2: the copies alternate, and this thread reaches the next end barrier first)
                int* cp = s_ibin + ip * ncopies * cstride;
                for (int b = tid; b < TB; b += kThreads) {
                    long long s = 0;
                    for (int c = 0; c < ncopies; ++c) {
                        s += cp[c * cstride + b];
                        cp[c * cstride + b] = 0;
                    }
                    s_lbin[b] += s;
                }
            }
            if constexpr (Cfg::kBinSets > 1) ip ^= 1;
            buf ^= 1;
            ct = nct;
            band = nband;
        }  // items of the segment
        if (abort) break;

        // ---- segment flush: one record per (block, tensor), as spectral_pass_kernel
        {
            const int rec = Dp->recbase[PASS] + ((int)blockIdx.x - Dp->cfirst[PASS]);
            double* out = rec_scal + (int64_t)rec * kNSRec;
            if constexpr (PASS == 4) {
                if (tid < kGram) {
                    double v = 0.0;
                    for (int w = 0; w < kWarps; ++w) v += s_acc[w * 32 + tid];
                    out[tid] = v;
                }
            } else if constexpr (PASS == 2 || PASS == 3) {
                constexpr int NS = 2 + 2 * RM;
                double v[NS];
                v[0] = acc0;
                v[1] = acc1;
#pragma unroll
                for (int q = 0; q < 2 * RM; ++q) v[2 + q] = s_acc[q * kThreads + tid];
                block_sum_to<NS>(v, s_red, s_tot);
                for (int j = tid; j < NS; j += kThreads) out[j] = s_tot[j];
                const double inv_fix = ldexp(1.0, -fix.s);
                for (int b = tid; b < TB; b += kThreads)
                    rec_bins[(int64_t)rec * TB + b] = (float)((double)s_lbin[b] * inv_fix + (double)s_fbin[b]);
            }
        }
        ++k;
    }

    // ---- drain: stores complete, loads in flight landed, TMEM freed
    if (lane < 2) bulk_wait_all();
    if (tid == 0) {
        if (abort) {
            for (int b = 0; b < 2; ++b)
                if (((inflight >> b) & 1u) && !mbar_wait_bounded(full_bar(b), (ph >> b) & 1u, kStageWaitNs))
                    atomicOr(hdr->status, 2);
        }
    }
    if constexpr (TCR) {
        // after a give-up, products may still be in flight: each issuing thread commits its
        // tensor-core work to the drain barrier, which completes once all of it has landed;
        // it is waited for (bounded) before the TMEM is freed, bit 2 if it never completes
        if (abort) {
            if ((tid & 63) == 0) tc_commit(smem_u32(s_drainbar));
            if (tid == 0 && !mbar_wait_bounded(smem_u32(s_drainbar), 0, kTcWaitNs)) atomicOr(hdr->status, 2);
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tc_dealloc(tc_base, kTcCols);
        }
    }
}

}  // namespace cresso
