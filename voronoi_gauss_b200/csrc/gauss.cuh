// Site Gaussians: conics A = R(q / |q|) diag(1 / (exp(2 clamp(ls, -20, 20)) + floor^2)) R^T and the
// chain rule from dL/dA back to dL/dls and dL/dq (the formulas of vgf.cu:339-421). Shared by the conic
// kernels (conic.cu) and the NeRF-sampler field kernels (field.cu), which evaluate each site's conic
// once per call instead of rebuilding its rotation for every sample that sees it.
//
// Storage of a symmetric 3 x 3 conic: (xx, xy, xz, yy, yz, zz); an off-diagonal entry stands for both
// A_ab and A_ba, so dL/d(xy) = dL/dA_01 + dL/dA_10.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vg {

struct ConicLocal {
    float qn[4], qnorm, R[9], iv[3], s2[3];
};

__device__ __forceinline__ void conic_local(const float* __restrict__ ls, const float* __restrict__ quat, int64_t i,
                                            float floor2, ConicLocal& L) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(quat) + i);
    L.qnorm = fmaxf(sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w), 1e-12f);
    const float w = q.x / L.qnorm, a = q.y / L.qnorm, b = q.z / L.qnorm, c = q.w / L.qnorm;
    L.qn[0] = w, L.qn[1] = a, L.qn[2] = b, L.qn[3] = c;
    L.R[0] = 1.f - 2.f * (b * b + c * c), L.R[1] = 2.f * (a * b - w * c), L.R[2] = 2.f * (a * c + w * b);
    L.R[3] = 2.f * (a * b + w * c), L.R[4] = 1.f - 2.f * (a * a + c * c), L.R[5] = 2.f * (b * c - w * a);
    L.R[6] = 2.f * (a * c - w * b), L.R[7] = 2.f * (b * c + w * a), L.R[8] = 1.f - 2.f * (a * a + b * b);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float s = __expf(2.f * fminf(fmaxf(__ldg(ls + 3 * i + k), -20.f), 20.f));
        L.s2[k] = s;
        L.iv[k] = 1.f / (s + floor2);
    }
}

// A in storage order.
__device__ __forceinline__ void conic_of(const ConicLocal& L, float (&A)[6]) {
    const float* R = L.R;
    int e = 0;
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = a; b < 3; ++b)
            A[e++] = R[3 * a] * R[3 * b] * L.iv[0] + R[3 * a + 1] * R[3 * b + 1] * L.iv[1] +
                     R[3 * a + 2] * R[3 * b + 2] * L.iv[2];
}

// dL/dls (3) and dL/dq (4) from dL/dA in storage order. The log-scale gradient is taken at the clamped
// value, as the reference does.
__device__ __forceinline__ void conic_grad(const ConicLocal& L, const float (&g)[6], float (&g_ls)[3], float4& g_quat) {
    const float* R = L.R;
    const float G[9] = {g[0], 0.5f * g[1], 0.5f * g[2], 0.5f * g[1], g[3], 0.5f * g[4], 0.5f * g[2], 0.5f * g[4], g[5]};
    float GR[9];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int k = 0; k < 3; ++k) GR[3 * a + k] = G[3 * a] * R[k] + G[3 * a + 1] * R[3 + k] + G[3 * a + 2] * R[6 + k];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float g_iv = R[k] * GR[k] + R[3 + k] * GR[3 + k] + R[6 + k] * GR[6 + k];  // (R^T G R)_kk
        g_ls[k] = g_iv * (-2.f * L.s2[k] * L.iv[k] * L.iv[k]);
    }
    float dR[9];  // dL/dR = 2 G R diag(iv)
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int k = 0; k < 3; ++k) dR[3 * a + k] = 2.f * GR[3 * a + k] * L.iv[k];
    const float w = L.qn[0], x = L.qn[1], y = L.qn[2], z = L.qn[3];
    float dq[4];
    dq[0] = 2.f * (-z * dR[1] + y * dR[2] + z * dR[3] - x * dR[5] - y * dR[6] + x * dR[7]);
    dq[1] = 2.f * (y * dR[1] + z * dR[2] + y * dR[3] - 2.f * x * dR[4] - w * dR[5] + z * dR[6] + w * dR[7] -
                   2.f * x * dR[8]);
    dq[2] = 2.f * (-2.f * y * dR[0] + x * dR[1] + w * dR[2] + x * dR[3] + z * dR[5] - w * dR[6] + z * dR[7] -
                   2.f * y * dR[8]);
    dq[3] = 2.f * (-2.f * z * dR[0] - w * dR[1] + x * dR[2] + w * dR[3] - 2.f * z * dR[4] + y * dR[5] + x * dR[6] +
                   y * dR[7]);
    const float proj = dq[0] * w + dq[1] * x + dq[2] * y + dq[3] * z;
    g_quat.x = (dq[0] - proj * w) / L.qnorm, g_quat.y = (dq[1] - proj * x) / L.qnorm;
    g_quat.z = (dq[2] - proj * y) / L.qnorm, g_quat.w = (dq[3] - proj * z) / L.qnorm;
}

}  // namespace vg
