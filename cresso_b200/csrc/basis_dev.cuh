// Device helpers for the separable spectral carriers.
//
// Every carrier of the reference pack (cresso_v5.py:295-348) factorises over
// the two axes of a 2-D tensor (a 1-D tensor is a single row):
//   complex modes (mode % 4 in {0, 2, 3}, and the zero mode):
//       raw_cos(i, j) = a1(i) b1(j) - a2(i) b2(j),  raw_sin = a1 b2 + a2 b1
//   product modes (mode % 4 == 1):
//       raw_cos(i, j) = a1(i) b1(j),                raw_sin = a2(i) b2(j)
// and the normalised carrier is (raw - mu) * inv (cresso_v5.py:138-142);
// mu / inv come from the closed-form stats of the tables.
//
// A reconstruction  sum_k alpha_k cos_k + beta_k sin_k  with coefficients
// already multiplied by inv (alpha' = alpha * inv_c, beta' = beta * inv_s)
// becomes, per element,   K + sum_k a1_k(i) U_k(j) + a2_k(i) V_k(j)
// where U, V depend only on the column and K = -sum alpha' mu_c + beta' mu_s.
// A projection  sum_ij x_ij raw_k(i, j)  accumulates z1_k = sum_i x a1_k(i),
// z2_k = sum_i x a2_k(i) down each column and contracts with b1, b2 at the end.
#pragma once

#include "cresso_common.cuh"

namespace cresso {

// Loads (a1_k, a2_k) of row `gr` of a row table for modes 0..RM-1.  The
// table may sit in global or (staged) shared memory: plain generic loads.
template <int RM>
__device__ __forceinline__ void load_row(const float* __restrict__ rowtab, int64_t gr, float (&a1)[RM], float (&a2)[RM]) {
    const float4* p = reinterpret_cast<const float4*>(rowtab + gr * (2 * RM));
#pragma unroll
    for (int q = 0; q < RM / 2; ++q) {
        float4 v = p[q];
        a1[2 * q] = v.x;
        a2[2 * q] = v.y;
        a1[2 * q + 1] = v.z;
        a2[2 * q + 1] = v.w;
    }
}

// Loads (b1_k, b2_k) of global column `gc`.
template <int RM>
__device__ __forceinline__ void load_col(const float* __restrict__ coltab, int64_t gcols, int64_t gc, float (&b1)[RM],
                                         float (&b2)[RM]) {
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        b1[k] = __ldg(coltab + (2 * k) * gcols + gc);
        b2[k] = __ldg(coltab + (2 * k + 1) * gcols + gc);
    }
}

// Column factors of a reconstruction with inv-folded coefficients (alpha', beta').
template <int RM>
__device__ __forceinline__ void make_uv(const float (&b1)[RM], const float (&b2)[RM], const float* __restrict__ alpha,
                                        const float* __restrict__ beta, float (&U)[RM], float (&V)[RM]) {
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        const float al = alpha[k], be = beta[k];
        if (mode_is_product(k)) {
            U[k] = al * b1[k];
            V[k] = be * b2[k];
        } else {
            U[k] = al * b1[k] + be * b2[k];
            V[k] = be * b1[k] - al * b2[k];
        }
    }
}

template <int RM>
__device__ __forceinline__ float recon_dot(float K, const float (&a1)[RM], const float (&a2)[RM], const float (&U)[RM],
                                           const float (&V)[RM]) {
    float s = K;
#pragma unroll
    for (int k = 0; k < RM; ++k) s = fmaf(a1[k], U[k], fmaf(a2[k], V[k], s));
    return s;
}

// Mode 0 of every CRESSO5 carrier pack is the zero-frequency mode, whose
// tables are a = (1, 0), b = (1, 0): its reconstruction term is the constant
// alpha'_0 (folded into K by the finalize kernels) and its projection is the
// plain sum.  The streaming passes therefore loop over modes 1..RM-1 only.
template <int RM>
__device__ __forceinline__ float recon_dot_nz(float K, const float (&a1)[RM], const float (&a2)[RM],
                                              const float (&U)[RM], const float (&V)[RM]) {
    float s = K;
#pragma unroll
    for (int k = 1; k < RM; ++k) s = fmaf(a1[k], U[k], fmaf(a2[k], V[k], s));
    return s;
}

// Adds the column contraction of (z1, z2) into (C, S): C_k += sum x raw_cos_k, S_k += sum x raw_sin_k.
template <int RM>
__device__ __forceinline__ void contract_col(const float (&b1)[RM], const float (&b2)[RM], const float (&z1)[RM],
                                             const float (&z2)[RM], double (&C)[RM], double (&S)[RM]) {
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        const double B1 = b1[k], B2 = b2[k], Z1 = z1[k], Z2 = z2[k];
        if (mode_is_product(k)) {
            C[k] += B1 * Z1;
            S[k] += B2 * Z2;
        } else {
            C[k] += B1 * Z1 - B2 * Z2;
            S[k] += B2 * Z1 + B1 * Z2;
        }
    }
}

// Shrinkage of the redundant carrier sum, 1/sqrt(max(1, 0.7 log2(R+1)))  (cresso_v5.py:368).
__host__ __device__ inline double recon_shrink(int rank) {
    double v = 0.7 * log2((double)rank + 1.0);
    return 1.0 / sqrt(v > 1.0 ? v : 1.0);
}

// Per-mode normalisation record in the shape workspace: carrier = (raw - mu) * inv
// (mu = 0, inv = 1 for the unnormalised zero mode); mhat = mean of the carrier;
// rawmean = mean of the raw separable product.
struct ModeStats {
    double mu_c, inv_c, mu_s, inv_s, mhat_c, mhat_s, rawmean_c, rawmean_s;
};

}  // namespace cresso
