// Site Gaussians in principal-axis form, and the chain rule back to their log-scales and quaternions.
//
// A site's Gaussian is given by a log-scale ls (3) and a quaternion q (4) (vgf.cu:339-421 computes the
// same quantities). With u = q / max(|q|, 1e-12) = (w, v), a_k the k-th principal axis (the k-th column
// of the rotation of u) and the axis weights c_k = 1 / (exp(2 clamp(ls_k, -20, 20)) + floor^2), the conic
// is a sum of three weighted outer products,
//     A = sum_k c_k a_k a_k^T,
// stored as the six entries (xx, xy, xz, yy, yz, zz); an off-diagonal entry stands for both A_ab and
// A_ba, so a gradient of the storage entry xy is dL/dA_01 + dL/dA_10.
//
// Backward. Let G be the symmetric matrix of dL/dA (diagonal entries as given, each off-diagonal one
// half of its storage gradient). Then
//     dL/dc_k   = a_k . (G a_k),          dc_k/dls_k = -2 var_k c_k^2 (var_k = exp(2 clamp(ls_k)), taken at
//                                                      the clamped value, as the reference's kernel does),
//     dL/da_k   = 2 c_k G a_k.
// The axes move with u only by rotation: a left perturbation u -> (1, omega / 2) (x) u turns every axis
// by omega, da_k = omega x a_k, so dL = omega . tau with the torque tau = sum_k a_k x dL/da_k. For a
// tangent change du = (dw, dv) of the unit quaternion, omega = 2 (w dv - dw v + v x dv), hence
//     dL/dw = -2 tau . v,        dL/dv = 2 (w tau + tau x v),
// a vector already orthogonal to u (the normalisation's radial part drops out), and dL/dq is it divided
// by max(|q|, 1e-12).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vg {

struct GaussAxes {
    float4 unit;     // u = (w, x, y, z) = q / len
    float len;       // max(|q|, 1e-12)
    float3 axis[3];  // principal axes a_k (unit vectors)
    float c[3];      // axis weights 1 / (var_k + floor^2)
    float var[3];    // squared scales exp(2 clamp(ls_k, -20, 20))
};

__device__ __forceinline__ float3 f3_cross(const float3 a, const float3 b) {
    return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}

__device__ __forceinline__ float f3_dot(const float3 a, const float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

// Principal axes and weights of site `site` (log-scales (N, 3) and quaternions (N, 4) in the caller's
// order). floor2 = floor^2 is added to every squared scale.
__device__ __forceinline__ GaussAxes gauss_axes(const float* __restrict__ log_scale, const float* __restrict__ quat,
                                                int64_t site, float floor2) {
    GaussAxes g;
    const float4 q = __ldg(reinterpret_cast<const float4*>(quat) + site);
    g.len = fmaxf(sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w), 1e-12f);
    const float w = q.x / g.len, x = q.y / g.len, y = q.z / g.len, z = q.w / g.len;
    g.unit = make_float4(w, x, y, z);
    // columns of the rotation of (w, x, y, z)
    g.axis[0] = make_float3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y));
    g.axis[1] = make_float3(2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x));
    g.axis[2] = make_float3(2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float l = fminf(fmaxf(__ldg(log_scale + 3 * site + k), -20.f), 20.f);
        g.var[k] = __expf(2.f * l);
        g.c[k] = 1.f / (g.var[k] + floor2);
    }
    return g;
}

// A = sum_k c_k a_k a_k^T in storage order (xx, xy, xz, yy, yz, zz).
__device__ __forceinline__ void gauss_conic(const GaussAxes& g, float (&A)[6]) {
#pragma unroll
    for (int e = 0; e < 6; ++e) A[e] = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float3 a = g.axis[k];
        const float3 ca = make_float3(g.c[k] * a.x, g.c[k] * a.y, g.c[k] * a.z);
        A[0] += ca.x * a.x, A[1] += ca.x * a.y, A[2] += ca.x * a.z;
        A[3] += ca.y * a.y, A[4] += ca.y * a.z, A[5] += ca.z * a.z;
    }
}

// dL/dls (3) and dL/dq (4) from dL/dA given in storage order.
__device__ __forceinline__ void gauss_conic_grad(const GaussAxes& g, const float (&gA)[6], float (&g_ls)[3],
                                                 float4& g_quat) {
    const float hxy = 0.5f * gA[1], hxz = 0.5f * gA[2], hyz = 0.5f * gA[4];
    float3 tau = make_float3(0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float3 a = g.axis[k];
        const float3 Ga = make_float3(gA[0] * a.x + hxy * a.y + hxz * a.z, hxy * a.x + gA[3] * a.y + hyz * a.z,
                                      hxz * a.x + hyz * a.y + gA[5] * a.z);
        g_ls[k] = f3_dot(a, Ga) * (-2.f * g.var[k] * g.c[k] * g.c[k]);
        const float3 t = f3_cross(a, Ga);
        const float s = 2.f * g.c[k];
        tau.x += s * t.x, tau.y += s * t.y, tau.z += s * t.z;
    }
    const float3 v = make_float3(g.unit.y, g.unit.z, g.unit.w);
    const float3 txv = f3_cross(tau, v);
    const float w = g.unit.x, inv = 1.f / g.len;
    g_quat = make_float4(-2.f * f3_dot(tau, v) * inv, 2.f * (w * tau.x + txv.x) * inv,
                         2.f * (w * tau.y + txv.y) * inv, 2.f * (w * tau.z + txv.z) * inv);
}

}  // namespace vg
