// Conics of the site Gaussians and their gradients, one thread per site (the quantities of the
// reference's vgf.cu:339-421): A = sum_k c_k a_k a_k^T over the principal axes of q / |q| with weights
// 1 / (exp(2 clamp(ls, -20, 20)) + floor^2), stored as (xx, xy, xz, yy, yz, zz); the backward maps dL/dA
// to dL/dls and dL/dq (gauss.cuh). Elementwise, 28 bytes in / 24 out per site (forward): HBM-bound and
// small next to the traversal.
#include "gauss.cuh"
#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 256;

__global__ void __launch_bounds__(kBlock)
    conic_forward_kernel(const float* __restrict__ ls, const float* __restrict__ quat, int64_t n, float floor2,
                         float* __restrict__ A) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (i >= n) return;
    float out[6];
    gauss_conic(gauss_axes(ls, quat, i, floor2), out);
    float2* o = reinterpret_cast<float2*>(A + 6 * i);
    o[0] = make_float2(out[0], out[1]), o[1] = make_float2(out[2], out[3]), o[2] = make_float2(out[4], out[5]);
}

__global__ void __launch_bounds__(kBlock)
    conic_backward_kernel(const float* __restrict__ ls, const float* __restrict__ quat, int64_t n, float floor2,
                          const float* __restrict__ gA, float* __restrict__ g_ls, float* __restrict__ g_quat) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (i >= n) return;
    const GaussAxes ax = gauss_axes(ls, quat, i, floor2);
    const float2* gp = reinterpret_cast<const float2*>(gA + 6 * i);
    const float2 g01 = __ldg(gp), g23 = __ldg(gp + 1), g45 = __ldg(gp + 2);
    const float g[6] = {g01.x, g01.y, g23.x, g23.y, g45.x, g45.y};
    float gl[3];
    float4 gq;
    gauss_conic_grad(ax, g, gl, gq);
#pragma unroll
    for (int k = 0; k < 3; ++k) g_ls[3 * i + k] = gl[k];
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
