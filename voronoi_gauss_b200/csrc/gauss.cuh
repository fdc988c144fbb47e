// Site Gaussians: conics A = R(q / |q|) diag(1 / (exp(2 clamp(ls, -20, 20)) + floor^2)) R^T and the chain
// rule from dL/dA back to dL/dls and dL/dq (the quantities of vgf.cu:339-421). Shared by the conic kernels
// (conic.cu), the NeRF-sampler field kernels (field.cu) and the inference packing (infer_pack.cu), which
// evaluate each site's conic once per call instead of rebuilding its rotation for every sample.
//
// Storage of a symmetric 3 x 3 conic: (xx, xy, xz, yy, yz, zz); an off-diagonal entry stands for both
// A_ab and A_ba, so dL/d(xy) = dL/dA_01 + dL/dA_10.
//
// Gradient of the rotation: with P = dL/dR, its symmetric parts s_ab = P_ab + P_ba and antisymmetric parts
// a_ab = P_ab - P_ba, differentiating R(w, x, y, z) of a unit quaternion gives
//   dL/dw = 2 (x a_21 + y a_02 + z a_10)
//   dL/dx = 2 (y s_01 + z s_02 + w a_21) - 4 x (P_11 + P_22)
//   dL/dy = 2 (x s_01 + z s_12 + w a_02) - 4 y (P_00 + P_22)
//   dL/dz = 2 (x s_02 + y s_12 + w a_10) - 4 z (P_00 + P_11)
// and the normalisation q / |q| removes the radial part: dL/dq = (g - (g . u) u) / |q|.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vg {

struct ConicLocal {
    float u[4];   // unit quaternion (w, x, y, z)
    float len;    // |q|, at least 1e-12
    float R[9];   // rotation, row-major
    float iv[3];  // 1 / (s_k^2 + floor^2)
    float s2[3];  // s_k^2 = exp(2 clamp(ls_k))
};

// Rotation of a unit quaternion from its pairwise products.
__device__ __forceinline__ void rotation(const float (&u)[4], float (&R)[9]) {
    const float w = u[0], x = u[1], y = u[2], z = u[3];
    const float xx = x * x, yy = y * y, zz = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    R[0] = 1.f - 2.f * (yy + zz), R[1] = 2.f * (xy - wz), R[2] = 2.f * (xz + wy);
    R[3] = 2.f * (xy + wz), R[4] = 1.f - 2.f * (xx + zz), R[5] = 2.f * (yz - wx);
    R[6] = 2.f * (xz - wy), R[7] = 2.f * (yz + wx), R[8] = 1.f - 2.f * (xx + yy);
}

__device__ __forceinline__ void conic_local(const float* __restrict__ ls, const float* __restrict__ quat, int64_t i,
                                            float floor2, ConicLocal& L) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(quat) + i);
    const float raw[4] = {q.x, q.y, q.z, q.w};
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) sq += raw[k] * raw[k];
    L.len = fmaxf(sqrtf(sq), 1e-12f);
#pragma unroll
    for (int k = 0; k < 4; ++k) L.u[k] = raw[k] / L.len;
    rotation(L.u, L.R);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        L.s2[k] = __expf(2.f * fminf(fmaxf(__ldg(ls + 3 * i + k), -20.f), 20.f));
        L.iv[k] = 1.f / (L.s2[k] + floor2);
    }
}

// A in storage order: A_ab = sum_k R_ak iv_k R_bk.
__device__ __forceinline__ void conic_of(const ConicLocal& L, float (&A)[6]) {
    float RS[9];  // R diag(iv)
#pragma unroll
    for (int e = 0; e < 9; ++e) RS[e] = L.R[e] * L.iv[e % 3];
    constexpr int kRow[6] = {0, 0, 0, 1, 1, 2}, kCol[6] = {0, 1, 2, 1, 2, 2};
#pragma unroll
    for (int s = 0; s < 6; ++s) {
        const int a = kRow[s], b = kCol[s];
        A[s] = RS[3 * a] * L.R[3 * b] + RS[3 * a + 1] * L.R[3 * b + 1] + RS[3 * a + 2] * L.R[3 * b + 2];
    }
}

// dL/dls (3) and dL/dq (4) from dL/dA in storage order. The log-scale gradient is taken at the clamped
// value, as the reference's kernel does.
__device__ __forceinline__ void conic_grad(const ConicLocal& L, const float (&g)[6], float (&g_ls)[3], float4& g_quat) {
    // symmetric dL/dA as a full matrix (off-diagonal storage entries split over both halves)
    const float G[9] = {g[0], 0.5f * g[1], 0.5f * g[2], 0.5f * g[1], g[3], 0.5f * g[4], 0.5f * g[2], 0.5f * g[4], g[5]};
    float GR[9];  // G R
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            float acc = 0.f;
#pragma unroll
            for (int m = 0; m < 3; ++m) acc += G[3 * a + m] * L.R[3 * m + k];
            GR[3 * a + k] = acc;
        }
    float P[9];  // dL/dR = 2 G R diag(iv)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        float diag = 0.f;  // (R^T G R)_kk = dL/d iv_k
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            diag += L.R[3 * a + k] * GR[3 * a + k];
            P[3 * a + k] = 2.f * GR[3 * a + k] * L.iv[k];
        }
        g_ls[k] = diag * (-2.f * L.s2[k] * L.iv[k] * L.iv[k]);  // d iv / d ls = -2 s^2 iv^2
    }
    const float w = L.u[0], x = L.u[1], y = L.u[2], z = L.u[3];
    const float s01 = P[1] + P[3], s02 = P[2] + P[6], s12 = P[5] + P[7];
    const float a21 = P[7] - P[5], a02 = P[2] - P[6], a10 = P[3] - P[1];
    float gq[4];
    gq[0] = 2.f * (x * a21 + y * a02 + z * a10);
    gq[1] = 2.f * (y * s01 + z * s02 + w * a21) - 4.f * x * (P[4] + P[8]);
    gq[2] = 2.f * (x * s01 + z * s12 + w * a02) - 4.f * y * (P[0] + P[8]);
    gq[3] = 2.f * (x * s02 + y * s12 + w * a10) - 4.f * z * (P[0] + P[4]);
    const float radial = gq[0] * w + gq[1] * x + gq[2] * y + gq[3] * z;
    g_quat = make_float4((gq[0] - radial * w) / L.len, (gq[1] - radial * x) / L.len, (gq[2] - radial * y) / L.len,
                         (gq[3] - radial * z) / L.len);
}

}  // namespace vg
