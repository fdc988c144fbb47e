// Conics of the site Gaussians and their gradients, one thread per site (the reference's
// vgf.cu:339-421 formulas): A = R(q / |q|) diag(1 / (exp(2 clamp(ls, -20, 20)) + floor^2)) R^T stored as
// (xx, xy, xz, yy, yz, zz); the backward maps dL/dA to dL/dls and dL/dq (with the projection for the
// normalised quaternion). Elementwise, 52 bytes in / 24 out per site: HBM-bound and small next to
// the traversal.
#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 256;

struct Local {
    float qn[4], qnorm, R[9], iv[3], s2[3];
};

__device__ __forceinline__ void local(const float* __restrict__ ls, const float* __restrict__ quat, int64_t i,
                                      float floor2, Local& L) {
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

__global__ void __launch_bounds__(kBlock)
    conic_forward_kernel(const float* __restrict__ ls, const float* __restrict__ quat, int64_t n, float floor2,
                         float* __restrict__ A) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (i >= n) return;
    Local L;
    local(ls, quat, i, floor2, L);
    const float* R = L.R;
    float out[6];
    int e = 0;
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = a; b < 3; ++b)
            out[e++] = R[3 * a] * R[3 * b] * L.iv[0] + R[3 * a + 1] * R[3 * b + 1] * L.iv[1] +
                       R[3 * a + 2] * R[3 * b + 2] * L.iv[2];
    float2* o = reinterpret_cast<float2*>(A + 6 * i);
    o[0] = make_float2(out[0], out[1]), o[1] = make_float2(out[2], out[3]), o[2] = make_float2(out[4], out[5]);
}

__global__ void __launch_bounds__(kBlock)
    conic_backward_kernel(const float* __restrict__ ls, const float* __restrict__ quat, int64_t n, float floor2,
                          const float* __restrict__ gA, float* __restrict__ g_ls, float* __restrict__ g_quat) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (i >= n) return;
    Local L;
    local(ls, quat, i, floor2, L);
    const float* R = L.R;
    const float2* gp = reinterpret_cast<const float2*>(gA + 6 * i);
    const float2 g01 = __ldg(gp), g23 = __ldg(gp + 1), g45 = __ldg(gp + 2);
    // symmetric dL/dA: an off-diagonal storage entry stands for A_ab and A_ba
    const float G[9] = {g01.x, 0.5f * g01.y, 0.5f * g23.x, 0.5f * g01.y, g23.y,
                        0.5f * g45.x, 0.5f * g23.x, 0.5f * g45.x, g45.y};
    float GR[9];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int k = 0; k < 3; ++k) GR[3 * a + k] = G[3 * a] * R[k] + G[3 * a + 1] * R[3 + k] + G[3 * a + 2] * R[6 + k];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float g_iv = R[k] * GR[k] + R[3 + k] * GR[3 + k] + R[6 + k] * GR[6 + k];  // (R^T G R)_kk
        g_ls[3 * i + k] = g_iv * (-2.f * L.s2[k] * L.iv[k] * L.iv[k]);
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
    float4 gq;
    gq.x = (dq[0] - proj * w) / L.qnorm, gq.y = (dq[1] - proj * x) / L.qnorm;
    gq.z = (dq[2] - proj * y) / L.qnorm, gq.w = (dq[3] - proj * z) / L.qnorm;
    reinterpret_cast<float4*>(g_quat)[i] = gq;
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

cudaError_t conic_forward(const float* log_scale, const float* quat, int64_t n, float floor2, float* A,
                          cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    conic_forward_kernel<<<blocks(n), kBlock, 0, st>>>(log_scale, quat, n, floor2, A);
    return cudaGetLastError();
}

cudaError_t conic_backward(const float* log_scale, const float* quat, int64_t n, float floor2, const float* gA,
                           float* g_ls, float* g_quat, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    conic_backward_kernel<<<blocks(n), kBlock, 0, st>>>(log_scale, quat, n, floor2, gA, g_ls, g_quat);
    return cudaGetLastError();
}

}  // namespace vg
