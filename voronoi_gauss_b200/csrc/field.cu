// NeRF-sampler field kernels: the nearest-site walk of sorted ray samples and the neighbourhood density
// and colour fields at arbitrary sample points, with their gradients (vgf.cu:51-335, bound at
// vgf.cu:438-533). Used by the proposal-sampler renderer (render.py:43-106 of the reference).
//
// One thread per ray (walk) or per sample (fields) over the Morton-packed graph (vg_common.cuh). The
// reference rebuilds each neighbour's rotation from its quaternion for every sample (a square root,
// seven divisions and three exponentials per neighbour); here a prepass evaluates every site's conic
// once per call into a 32-byte record, so a neighbour costs one 16-byte edge load, two 16-byte record
// loads and a 3 x 3 quadratic form:
//
//   gauss (N, 2) float4, internal order: (A xx, xy, xz, yy), (A yz, zz, min(raw, 30), 0)
//            A = scale x conic(log_scale, quat, floor 0); scale = 1 / scale_mult^2 (density proposals)
//   sh    (N, S4) float4, the packed SH rows of the foam field pack (colour only)
//   acc   (N, 2 + S4) float4 gradient accumulators: (g_raw, g_A[0..2]), (g_A[3..5], 0), g_sh rows
//
// The backward passes accumulate dL/dA per site with vector atomics and finish with one thread per site
// that applies the conic chain rule (gauss.cuh) and scatters to the caller's (original-order) tensors:
// g_ls, g_quat, and g_raw (density) or g_sh (colour). Mathematically the same gradients as the
// reference's per-sample scatter_gauss_grad (vgf.cu:126-153); the summation order differs.
//
// With a workspace sized for the sample count (vg_field_workspace_bytes), the backward passes instead
// bucket the samples by cell and reuse the cell-major scatter of the foam backward (foam.cu): a sample's
// density and colour gradients take the same per-neighbour form there (dL/dsigma times the density
// Gaussian; the normalised colour weight a_k with its m_min / 1 / sum a), so one 64-byte item per sample
// in its cell's bucket feeds cm_scatter_bucketed, and one thread per site applies the conic chain rule.
#include <cub/device/device_scan.cuh>

#include <algorithm>

#include "gauss.cuh"
#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 128;
constexpr int kPrepBlock = 256;

__global__ void __launch_bounds__(kPrepBlock)
    gauss_pack_kernel(const int* __restrict__ perm, int n, const float* __restrict__ raw, const float* __restrict__ ls,
                      const float* __restrict__ quat, float scale, const float* __restrict__ sh, int nc, int s4,
                      float4* __restrict__ gauss, float4* __restrict__ shp) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = __ldg(perm + i);
    float A[6];
    gauss_conic(gauss_axes(ls, quat, o, 0.f), A);
    gauss[2 * static_cast<int64_t>(i)] = make_float4(A[0] * scale, A[1] * scale, A[2] * scale, A[3] * scale);
    gauss[2 * static_cast<int64_t>(i) + 1] =
        make_float4(A[4] * scale, A[5] * scale, raw != nullptr ? fminf(__ldg(raw + o), 30.f) : 0.f, 0.f);
    if (shp == nullptr) return;
    const float* s = sh + 48 * o;
    float4* q = shp + static_cast<int64_t>(s4) * i;
    for (int v = 0; v < s4; ++v) {
        float f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) f[u] = 4 * v + u < nc ? __ldg(s + 4 * v + u) : 0.f;
        q[v] = make_float4(f[0], f[1], f[2], f[3]);
    }
}

// Greedy walk of every sample of a ray from the previous sample's site (vgf.cu:51-78): a step moves to
// the first neighbour, in adjacency order, strictly closer to x than the best so far.
__global__ void __launch_bounds__(kBlock)
    walk_kernel(GraphView g, const float* __restrict__ o, const float* __restrict__ d, const float* __restrict__ z,
                const int* __restrict__ start, int64_t B, int S, int* __restrict__ site, int* __restrict__ steps,
                int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= B) return;
    const float o0 = __ldg(o + 3 * r), o1 = __ldg(o + 3 * r + 1), o2 = __ldg(o + 3 * r + 2);
    const float d0 = __ldg(d + 3 * r), d1 = __ldg(d + 3 * r + 1), d2 = __ldg(d + 3 * r + 2);
    const int s0 = __ldg(start + r);
    int* out = site + r * S;
    if (s0 < 0 || s0 >= g.n) {
        for (int s = 0; s < S; ++s) out[s] = -1;
        steps[r] = 0;
        atomicOr(status, kErrBadSite);
        return;
    }
    int cur = __ldg(g.inv + s0), total = 0, err = 0;
    const float* zr = z + r * S;
    for (int s = 0; s < S; ++s) {
        const float t = __ldg(zr + s);
        const float x0 = along(o0, t, d0), x1 = along(o1, t, d1), x2 = along(o2, t, d2);
        int e0 = __ldg(g.off + cur), e1 = __ldg(g.off + cur + 1);
        const float4 P = __ldg(g.edge + e0);
        const float u0 = __fsub_rn(x0, P.x), u1 = __fsub_rn(x1, P.y), u2 = __fsub_rn(x2, P.z);
        float bd = dot3c(u0, u1, u2, u0, u1, u2);
        int it = 0;
        for (; it < kWalkCap; ++it) {
            int best = cur;
            for (int e = e0 + 1; e < e1; ++e) {
                const float4 E = __ldg(g.edge + e);
                const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
                const float dq = dot3c(v0, v1, v2, v0, v1, v2);
                if (dq < bd) bd = dq, best = site_of(E);
            }
            if (best == cur) break;
            cur = best;
            ++total;
            e0 = __ldg(g.off + cur), e1 = __ldg(g.off + cur + 1);
        }
        if (it == kWalkCap) err |= kErrWalkCap;
        out[s] = __ldg(g.perm + cur);
    }
    steps[r] = total;
    if (err) atomicOr(status, err);
}

// Internal id of the sample's site, or -1 (status flagged) when it is not a site of the graph.
__device__ __forceinline__ int sample_cell(const GraphView& g, const int* __restrict__ site, int64_t t, int* status) {
    const int i = __ldg(site + t);
    if (i < 0 || i >= g.n) {
        atomicOr(status, kErrBadSite);
        return -1;
    }
    return __ldg(g.inv + i);
}

__device__ __forceinline__ void load_x(const float* __restrict__ x, int64_t t, float& x0, float& x1, float& x2) {
    x0 = __ldg(x + 3 * t), x1 = __ldg(x + 3 * t + 1), x2 = __ldg(x + 3 * t + 2);
}

// sigma(x) = sum over N(i) of exp(min(raw_k, 30) - v^T A_k v / 2) (vgf.cu:163-177).
__global__ void __launch_bounds__(kBlock)
    density_forward_kernel(GraphView g, const float4* __restrict__ gauss, const float* __restrict__ x,
                           const int* __restrict__ site, int64_t m, float* __restrict__ sigma, int* status) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= m) return;
    const int c = sample_cell(g, site, t, status);
    if (c < 0) {
        sigma[t] = 0.f;
        return;
    }
    float x0, x1, x2;
    load_x(x, t, x0, x1, x2);
    const int e0 = __ldg(g.off + c), e1 = __ldg(g.off + c + 1);
    float s = 0.f;
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int64_t k = site_of(E);
        const float4 G0 = __ldg(gauss + 2 * k), G1 = __ldg(gauss + 2 * k + 1);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        s += __expf(G1.z - 0.5f * maha(G0, G1, v0, v1, v2));
    }
    sigma[t] = s;
}

// dL/d(conic) of one quadratic form v^T A v with dL/dm = gm, in storage order, into two accumulators
// (head goes to the first slot: g_raw for the density, unused for the colour).
__device__ __forceinline__ void add_conic_grad(float4* __restrict__ acc, float head, float gm, float v0, float v1,
                                               float v2) {
    const float g2 = 2.f * gm;
    atomicAdd(acc, make_float4(head, gm * v0 * v0, g2 * v0 * v1, g2 * v0 * v2));
    atomicAdd(acc + 1, make_float4(gm * v1 * v1, g2 * v1 * v2, gm * v2 * v2, 0.f));
}

// vgf.cu:179-198: contributions c = rho_k G_k(x) with c |g_sigma| <= 1e-12 get no gradient.
__global__ void __launch_bounds__(kBlock)
    density_backward_kernel(GraphView g, const float4* __restrict__ gauss, const float* __restrict__ x,
                            const int* __restrict__ site, int64_t m, const float* __restrict__ g_sigma,
                            float4* __restrict__ acc, int* status) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= m) return;
    const float gs = __ldg(g_sigma + t);
    if (gs == 0.f) return;
    const int c = sample_cell(g, site, t, status);
    if (c < 0) return;
    float x0, x1, x2;
    load_x(x, t, x0, x1, x2);
    const int e0 = __ldg(g.off + c), e1 = __ldg(g.off + c + 1);
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int64_t k = site_of(E);
        const float4 G0 = __ldg(gauss + 2 * k), G1 = __ldg(gauss + 2 * k + 1);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        const float w = __expf(G1.z - 0.5f * maha(G0, G1, v0, v1, v2));
        if (w * fabsf(gs) > 1e-12f) add_conic_grad(acc + 2 * k, gs * w, -0.5f * gs * w, v0, v1, v2);
    }
}

// Unit direction of a sample (vgf.cu:228-232).
__device__ __forceinline__ void unit_dir(const float* __restrict__ dirs, int64_t t, float& dx, float& dy, float& dz) {
    dx = __ldg(dirs + 3 * t), dy = __ldg(dirs + 3 * t + 1), dz = __ldg(dirs + 3 * t + 2);
    const float inv = rsqrtf(fmaxf(dx * dx + dy * dy + dz * dz, 1e-20f));
    dx *= inv, dy *= inv, dz *= inv;
}

// C(x, d) = sum_k a_k max(SH_k(d) + 1/2, 0) / sum_k a_k, a_k = exp(-(m_k - m_min) / 2) (vgf.cu:248-282).
__global__ void __launch_bounds__(kBlock)
    color_forward_kernel(GraphView g, const float4* __restrict__ gauss, FieldView F, const float* __restrict__ x,
                         const float* __restrict__ dirs, const int* __restrict__ site, int64_t m,
                         float* __restrict__ rgb, int* status) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= m) return;
    const int c = sample_cell(g, site, t, status);
    if (c < 0) {
        rgb[3 * t] = rgb[3 * t + 1] = rgb[3 * t + 2] = 0.f;
        return;
    }
    float x0, x1, x2, dx, dy, dz;
    load_x(x, t, x0, x1, x2);
    unit_dir(dirs, t, dx, dy, dz);
    float b[16];
    sh_basis(dx, dy, dz, F.sh_deg, b);
    const int e0 = __ldg(g.off + c), e1 = __ldg(g.off + c + 1);
    Blend B;
    B.reset();
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int k = site_of(E);
        const float4 G0 = __ldg(gauss + 2 * static_cast<int64_t>(k));
        const float4 G1 = __ldg(gauss + 2 * static_cast<int64_t>(k) + 1);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        float col[3];
        site_color(F, k, b, col);
        B.add(maha(G0, G1, v0, v1, v2), col[0], col[1], col[2]);
    }
    rgb[3 * t] = B.sum[0] / B.wsum, rgb[3 * t + 1] = B.sum[1] / B.wsum, rgb[3 * t + 2] = B.sum[2] / B.wsum;
}

// vgf.cu:284-335: for each neighbour with normalised weight a_k >= kMinWeight, dL/dsh_k = a_k dL/dC
// masked by the clamp, and dL/dm_k = -a_k / 2 (<dL/dC, c_k> - <dL/dC, C>).
__global__ void __launch_bounds__(kBlock)
    color_backward_kernel(GraphView g, const float4* __restrict__ gauss, FieldView F, const float* __restrict__ x,
                          const float* __restrict__ dirs, const int* __restrict__ site, int64_t m,
                          const float* __restrict__ rgb, const float* __restrict__ g_rgb, float4* __restrict__ acc,
                          int stride, int* status) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= m) return;
    const float gr = __ldg(g_rgb + 3 * t), gg = __ldg(g_rgb + 3 * t + 1), gb = __ldg(g_rgb + 3 * t + 2);
    if (gr == 0.f && gg == 0.f && gb == 0.f) return;
    const int c = sample_cell(g, site, t, status);
    if (c < 0) return;
    float x0, x1, x2;
    load_x(x, t, x0, x1, x2);
    const int e0 = __ldg(g.off + c), e1 = __ldg(g.off + c + 1);
    float mmin = kInf;
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int64_t k = site_of(E);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        mmin = fminf(mmin, maha(__ldg(gauss + 2 * k), __ldg(gauss + 2 * k + 1), v0, v1, v2));
    }
    float A = 0.f;
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int64_t k = site_of(E);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        A += __expf(-0.5f * (maha(__ldg(gauss + 2 * k), __ldg(gauss + 2 * k + 1), v0, v1, v2) - mmin));
    }
    const float inv_a = 1.f / A;
    const float gCC = gr * __ldg(rgb + 3 * t) + gg * __ldg(rgb + 3 * t + 1) + gb * __ldg(rgb + 3 * t + 2);
    float dx, dy, dz;
    unit_dir(dirs, t, dx, dy, dz);
    float b[16];
    sh_basis(dx, dy, dz, F.sh_deg, b);
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int k = site_of(E);
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        const float mk = maha(__ldg(gauss + 2 * static_cast<int64_t>(k)),
                              __ldg(gauss + 2 * static_cast<int64_t>(k) + 1), v0, v1, v2);
        const float a = __expf(-0.5f * (mk - mmin)) * inv_a;
        if (a < kMinWeight) continue;
        float col[3];
        sh_color(F, k, b, col);
        const float dc[3] = {col[0] > 0.f ? a * gr : 0.f, col[1] > 0.f ? a * gg : 0.f, col[2] > 0.f ? a * gb : 0.f};
        float4* G = acc + static_cast<int64_t>(stride) * k;
        if (dc[0] != 0.f || dc[1] != 0.f || dc[2] != 0.f) {
#pragma unroll
            for (int q = 0; q < 12; ++q) {
                if (q >= F.s4) break;
                const int i0 = 4 * q;
                atomicAdd(G + 2 + q, make_float4(b[i0 / 3] * dc[i0 % 3], b[(i0 + 1) / 3] * dc[(i0 + 1) % 3],
                                                 b[(i0 + 2) / 3] * dc[(i0 + 2) % 3], b[(i0 + 3) / 3] * dc[(i0 + 3) % 3]));
            }
        }
        const float ga = gr * fmaxf(col[0], 0.f) + gg * fmaxf(col[1], 0.f) + gb * fmaxf(col[2], 0.f);
        const float gm = -0.5f * a * (ga - gCC);
        if (gm != 0.f) add_conic_grad(G, 0.f, gm, v0, v1, v2);
    }
}

// One thread per site: the conic chain rule on the accumulated dL/dA, then the per-site outputs in the
// caller's order (g_raw for the density, g_sh (N, 16, 3) for the colour; either may be absent).
__global__ void __launch_bounds__(kPrepBlock)
    field_grad_kernel(const int* __restrict__ perm, int n, const float* __restrict__ ls, const float* __restrict__ quat,
                      const float4* __restrict__ acc, int stride, int nc, float* __restrict__ g_raw,
                      float* __restrict__ g_ls, float* __restrict__ g_quat, float* __restrict__ g_sh) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = __ldg(perm + i);
    const float4* G = acc + static_cast<int64_t>(stride) * i;
    const float4 a0 = G[0], a1 = G[1];
    const float gA[6] = {a0.y, a0.z, a0.w, a1.x, a1.y, a1.z};
    float gl[3];
    float4 gq;
    gauss_conic_grad(gauss_axes(ls, quat, o, 0.f), gA, gl, gq);
#pragma unroll
    for (int k = 0; k < 3; ++k) g_ls[3 * o + k] = gl[k];
    reinterpret_cast<float4*>(g_quat)[o] = gq;
    if (g_raw != nullptr) g_raw[o] = a0.x;
    if (g_sh != nullptr) {
        float4* s = reinterpret_cast<float4*>(g_sh + 48 * o);
        const int s4 = stride - 2;
#pragma unroll
        for (int v = 0; v < 12; ++v) {
            float4 q = v < s4 ? G[2 + v] : make_float4(0.f, 0.f, 0.f, 0.f);
            if (4 * v + 0 >= nc) q.x = 0.f;
            if (4 * v + 1 >= nc) q.y = 0.f;
            if (4 * v + 2 >= nc) q.z = 0.f;
            if (4 * v + 3 >= nc) q.w = 0.f;
            s[v] = q;
        }
    }
}

// ------------------------------------------------------------------------ cell-major backward passes

// Site records in the foam field-pack layout (vg_common.cuh) with one of the two conics: the density
// conic and min(raw, 30) (colour = false) or the colour conic and the SH rows (colour = true).
__global__ void __launch_bounds__(kPrepBlock)
    field_rec_kernel(const int* __restrict__ perm, int n, const float* __restrict__ raw, const float* __restrict__ ls,
                     const float* __restrict__ quat, bool colour, const float* __restrict__ sh, int nc, int s4,
                     float4* __restrict__ rec, float4* __restrict__ shp) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = __ldg(perm + i);
    float A[6];
    gauss_conic(gauss_axes(ls, quat, o, 0.f), A);
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 a0 = make_float4(A[0], A[1], A[2], A[3]);
    float4* r = rec + 4 * static_cast<int64_t>(i);
    if (!colour) {
        r[0] = a0, r[1] = make_float4(A[4], A[5], fminf(__ldg(raw + o), 30.f), 0.f), r[2] = z, r[3] = z;
    } else {
        r[0] = z, r[1] = z, r[2] = a0, r[3] = make_float4(A[4], A[5], 0.f, 0.f);
    }
    float4* q = shp + static_cast<int64_t>(s4) * i;
    const float* sr = sh != nullptr ? sh + 48 * o : nullptr;
    for (int v = 0; v < s4; ++v) {
        float f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) f[u] = sr != nullptr && 4 * v + u < nc ? __ldg(sr + 4 * v + u) : 0.f;
        q[v] = make_float4(f[0], f[1], f[2], f[3]);
    }
}

// Samples [t0, t0 + mp) counted per cell (samples whose site is not a site of the graph are skipped by
// this kernel and by field_items_kernel alike).
__global__ void __launch_bounds__(kBlock)
    sample_count_kernel(const GraphView g, const int* __restrict__ site, int64_t t0, int64_t mp,
                        int* __restrict__ count) {
    const int64_t t = t0 + static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= t0 + mp) return;
    const int i = __ldg(site + t);
    if (i < 0 || i >= g.n) return;
    atomicAdd(count + __ldg(g.inv + i), 1);
}

// One 64-byte item per sample at its place in its cell's bucket: (x, dL/dsigma) | (dL/dC, dL/dC . C) |
// (m_min, 1 / sum of colour weights, 0, 0) | (unit direction, 0). For the colour, m_min and the weight sum
// come from the sample's neighbourhood (vgf.cu:297-312); samples without a gradient get a zero item.
__global__ void __launch_bounds__(kBlock)
    field_items_kernel(GraphView g, FieldView F, const float* __restrict__ x, const float* __restrict__ dirs,
                       const int* __restrict__ site, int64_t t0, int64_t mp, const float* __restrict__ g_sigma,
                       const float* __restrict__ rgb, const float* __restrict__ g_rgb, const int* __restrict__ offsets,
                       int* __restrict__ fill, float4* __restrict__ items, int* status) {
    const int64_t t = t0 + static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (t >= t0 + mp) return;
    const int c = sample_cell(g, site, t, status);
    if (c < 0) return;
    float x0, x1, x2;
    load_x(x, t, x0, x1, x2);
    const int64_t pos = __ldg(offsets + c) + atomicAdd(fill + c, 1);
    float4* it = items + 4 * pos;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g_sigma != nullptr) {
        it[0] = make_float4(x0, x1, x2, __ldg(g_sigma + t)), it[1] = z, it[2] = z, it[3] = z;
        return;
    }
    const float gr = __ldg(g_rgb + 3 * t), gg = __ldg(g_rgb + 3 * t + 1), gb = __ldg(g_rgb + 3 * t + 2);
    if (gr == 0.f && gg == 0.f && gb == 0.f) {
        it[0] = make_float4(x0, x1, x2, 0.f), it[1] = z, it[2] = z, it[3] = z;
        return;
    }
    const int e0 = __ldg(g.off + c), e1 = __ldg(g.off + c + 1);
    float mmin = kInf;
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const float4* fr = F.rec + kFieldVec * static_cast<int64_t>(site_of(E));
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        mmin = fminf(mmin, maha(__ldg(fr + 2), __ldg(fr + 3), v0, v1, v2));
    }
    float A = 0.f;
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const float4* fr = F.rec + kFieldVec * static_cast<int64_t>(site_of(E));
        const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
        A += __expf(-0.5f * (maha(__ldg(fr + 2), __ldg(fr + 3), v0, v1, v2) - mmin));
    }
    float dx, dy, dz;
    unit_dir(dirs, t, dx, dy, dz);
    const float gCC = gr * __ldg(rgb + 3 * t) + gg * __ldg(rgb + 3 * t + 1) + gb * __ldg(rgb + 3 * t + 2);
    it[0] = make_float4(x0, x1, x2, 0.f);
    it[1] = make_float4(gr, gg, gb, gCC);
    it[2] = make_float4(mmin, 1.f / A, 0.f, 0.f);
    it[3] = make_float4(dx, dy, dz, 0.f);
}

// One thread per site: the gradient pack (N, 64) of the cell-major scatter -> the caller's outputs via
// the conic chain rule of the density (colour = false: g_raw, g_dA) or colour (g_cA, g_sh) Gaussian.
__global__ void __launch_bounds__(kPrepBlock)
    field_pack_grad_kernel(const int* __restrict__ perm, int n, const float* __restrict__ ls,
                           const float* __restrict__ quat, const float4* __restrict__ grad, bool colour, int nc,
                           float* __restrict__ g_raw, float* __restrict__ g_ls, float* __restrict__ g_quat,
                           float* __restrict__ g_sh) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = __ldg(perm + i);
    const float4* G = grad + (kGradStride / 4) * static_cast<int64_t>(i);
    float gA[6];
    if (!colour) {
        const float4 d0 = G[0], d1 = G[1];
        gA[0] = d0.y, gA[1] = d0.z, gA[2] = d0.w, gA[3] = d1.x, gA[4] = d1.y, gA[5] = d1.z;
        g_raw[o] = d0.x;
    } else {
        const float4 c0 = G[2], c1 = G[3];
        gA[0] = c0.x, gA[1] = c0.y, gA[2] = c0.z, gA[3] = c0.w, gA[4] = c1.x, gA[5] = c1.y;
        float4* sd = reinterpret_cast<float4*>(g_sh + 48 * o);
#pragma unroll
        for (int v = 0; v < 12; ++v) {
            float4 q = G[4 + v];
            if (4 * v + 0 >= nc) q.x = 0.f;
            if (4 * v + 1 >= nc) q.y = 0.f;
            if (4 * v + 2 >= nc) q.z = 0.f;
            if (4 * v + 3 >= nc) q.w = 0.f;
            sd[v] = q;
        }
    }
    float gl[3];
    float4 gq;
    gauss_conic_grad(gauss_axes(ls, quat, o, 0.f), gA, gl, gq);
#pragma unroll
    for (int k = 0; k < 3; ++k) g_ls[3 * o + k] = gl[k];
    reinterpret_cast<float4*>(g_quat)[o] = gq;
}

inline int blocks(int64_t n, int bs) { return static_cast<int>((n + bs - 1) / bs); }

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct FieldLayout {
    size_t gauss, sh, acc, total;
    int s4, stride;
};

FieldLayout field_layout(int64_t n, int sh_deg, int kind) {
    FieldLayout L{};
    const bool color = kind >= 2, backward = kind == 1 || kind == 3;
    L.s4 = color ? sh_vec4(sh_deg) : 0;
    L.stride = 2 + L.s4;
    size_t at = 0;
    L.gauss = at, at += al256(32 * static_cast<size_t>(n));
    L.sh = at, at += al256(16 * static_cast<size_t>(L.s4) * n);
    L.acc = at, at += backward ? al256(16 * static_cast<size_t>(L.stride) * n) : 0;
    L.total = at;
    return L;
}

constexpr int64_t kFieldPass = int64_t(1) << 25;  // samples bucketed at once (2 GB of items)

struct FieldCmLayout {
    size_t rec, sh, grad, items, count, fill, offsets, chunks, counter, temp, temp_bytes, total;
    int s4;
    int64_t pass;
};

// Scratch of the cell-major backward of n sites and m samples (passes of at most kFieldPass samples).
FieldCmLayout field_cm_layout(int64_t n, int sh_deg, bool colour, int64_t m) {
    FieldCmLayout L{};
    L.s4 = colour ? sh_vec4(sh_deg) : 1;
    L.pass = std::max<int64_t>(1, std::min<int64_t>(m, kFieldPass));
    size_t at = 0;
    auto take = [&](size_t b) {
        const size_t h = at;
        at += al256(b);
        return h;
    };
    L.rec = take(16 * kFieldVec * static_cast<size_t>(n));
    L.sh = take(16 * static_cast<size_t>(L.s4) * n);
    L.grad = take(4 * kGradStride * static_cast<size_t>(n));
    L.items = take(64 * static_cast<size_t>(L.pass));
    L.count = take(4 * static_cast<size_t>(n + 1));
    L.fill = take(4 * static_cast<size_t>(n));
    L.offsets = take(4 * static_cast<size_t>(n + 1));
    L.chunks = take(16 * static_cast<size_t>(L.pass / 32 + n + 1));
    L.counter = take(16);
    size_t scan = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan, static_cast<const int*>(nullptr), static_cast<int*>(nullptr),
                                  static_cast<int>(n + 1));
    L.temp_bytes = scan;
    L.temp = take(scan);
    L.total = at;
    return L;
}

// The cell-major backward of the density (g_sigma non-null) or colour field into the caller's outputs.
cudaError_t field_backward_cm(const GraphView& g, const float* raw, const float* ls, const float* quat,
                              const float* sh, int sh_deg, const float* x, const float* dirs, const int* site,
                              int64_t m, const float* g_sigma, const float* rgb, const float* g_rgb, float* g_raw,
                              float* g_ls, float* g_quat, float* g_sh, void* ws, int* status, cudaStream_t st) {
    const bool colour = g_sigma == nullptr;
    const FieldCmLayout L = field_cm_layout(g.n, sh_deg, colour, m);
    char* b = static_cast<char*>(ws);
    float4* rec = reinterpret_cast<float4*>(b + L.rec);
    float4* shp = reinterpret_cast<float4*>(b + L.sh);
    float* grad = reinterpret_cast<float*>(b + L.grad);
    float4* items = reinterpret_cast<float4*>(b + L.items);
    int* count = reinterpret_cast<int*>(b + L.count);
    int* fill = reinterpret_cast<int*>(b + L.fill);
    int* offsets = reinterpret_cast<int*>(b + L.offsets);
    int4* chunks = reinterpret_cast<int4*>(b + L.chunks);
    int* counter = reinterpret_cast<int*>(b + L.counter);
    const int nc = 3 * sh_coeffs(sh_deg);
    field_rec_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(g.perm, g.n, raw, ls, quat, colour,
                                                                     colour ? sh : nullptr, nc, L.s4, rec, shp);
    cudaError_t e = cudaMemsetAsync(grad, 0, 4 * kGradStride * static_cast<size_t>(g.n), st);
    if (e != cudaSuccess) return e;
    const FieldView F{rec, shp, colour ? sh_deg : 0, L.s4};
    for (int64_t t0 = 0; t0 < m; t0 += L.pass) {
        const int64_t mp = std::min<int64_t>(L.pass, m - t0);
        e = cudaMemsetAsync(count, 0, 4 * static_cast<size_t>(g.n + 1), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(fill, 0, 4 * static_cast<size_t>(g.n), st);
        if (e != cudaSuccess) return e;
        sample_count_kernel<<<blocks(mp, kBlock), kBlock, 0, st>>>(g, site, t0, mp, count);
        size_t tb = L.temp_bytes;
        e = cub::DeviceScan::ExclusiveSum(b + L.temp, tb, count, offsets, g.n + 1, st);
        if (e != cudaSuccess) return e;
        field_items_kernel<<<blocks(mp, kBlock), kBlock, 0, st>>>(g, F, x, dirs, site, t0, mp, g_sigma, rgb, g_rgb,
                                                                  offsets, fill, items, status);
        e = cm_scatter_bucketed(g, F, items, offsets, chunks, counter, grad, st);
        if (e != cudaSuccess) return e;
    }
    field_pack_grad_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(
        g.perm, g.n, ls, quat, reinterpret_cast<const float4*>(grad), colour, nc, g_raw, g_ls, g_quat, g_sh);
    return cudaGetLastError();
}

}  // namespace

size_t field_workspace(int64_t n_sites, int sh_deg, int kind) { return field_layout(n_sites, sh_deg, kind).total; }

size_t field_cm_workspace(int64_t n_sites, int sh_deg, int kind, int64_t n_samples) {
    if (kind != 1 && kind != 3) return 0;
    return field_cm_layout(n_sites, sh_deg, kind == 3, n_samples).total;
}

cudaError_t sampler_walk(const GraphView& g, const float* o, const float* d, const float* z, const int* start,
                         int64_t n_rays, int n_samples, int* site, int* steps, int* status, cudaStream_t st) {
    if (n_rays == 0) return cudaSuccess;
    walk_kernel<<<blocks(n_rays, kBlock), kBlock, 0, st>>>(g, o, d, z, start, n_rays, n_samples, site, steps, status);
    return cudaGetLastError();
}

cudaError_t density_field(const GraphView& g, const float* raw, const float* ls, const float* quat, const float* x,
                          const int* site, int64_t m, float inv_mult2, bool backward, const float* g_sigma, float* sigma,
                          float* g_raw, float* g_ls, float* g_quat, void* ws, size_t ws_bytes, int* status,
                          cudaStream_t st) {
    if (backward && m > 0 && ws_bytes >= field_cm_workspace(g.n, 0, 1, m))
        return field_backward_cm(g, raw, ls, quat, nullptr, 0, x, nullptr, site, m, g_sigma, nullptr, nullptr, g_raw,
                                 g_ls, g_quat, nullptr, ws, status, st);
    const FieldLayout L = field_layout(g.n, 0, backward ? 1 : 0);
    char* b = static_cast<char*>(ws);
    float4* gauss = reinterpret_cast<float4*>(b + L.gauss);
    gauss_pack_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(g.perm, g.n, raw, ls, quat,
                                                                      backward ? 1.f : inv_mult2, nullptr, 0, 0, gauss,
                                                                      nullptr);
    if (!backward) {
        if (m > 0) density_forward_kernel<<<blocks(m, kBlock), kBlock, 0, st>>>(g, gauss, x, site, m, sigma, status);
        return cudaGetLastError();
    }
    float4* acc = reinterpret_cast<float4*>(b + L.acc);
    cudaError_t e = cudaMemsetAsync(acc, 0, 16 * static_cast<size_t>(L.stride) * g.n, st);
    if (e != cudaSuccess) return e;
    if (m > 0)
        density_backward_kernel<<<blocks(m, kBlock), kBlock, 0, st>>>(g, gauss, x, site, m, g_sigma, acc, status);
    field_grad_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(g.perm, g.n, ls, quat, acc, L.stride, 0, g_raw,
                                                                      g_ls, g_quat, nullptr);
    return cudaGetLastError();
}

cudaError_t color_field(const GraphView& g, const float* ls, const float* quat, const float* sh, int sh_deg,
                        const float* x, const float* dirs, const int* site, int64_t m, bool backward, const float* rgb_in,
                        const float* g_rgb, float* rgb, float* g_ls, float* g_quat, float* g_sh, void* ws,
                        size_t ws_bytes, int* status, cudaStream_t st) {
    if (backward && m > 0 && ws_bytes >= field_cm_workspace(g.n, sh_deg, 3, m))
        return field_backward_cm(g, nullptr, ls, quat, sh, sh_deg, x, dirs, site, m, nullptr, rgb_in, g_rgb, nullptr,
                                 g_ls, g_quat, g_sh, ws, status, st);
    const FieldLayout L = field_layout(g.n, sh_deg, backward ? 3 : 2);
    char* b = static_cast<char*>(ws);
    float4* gauss = reinterpret_cast<float4*>(b + L.gauss);
    float4* shp = reinterpret_cast<float4*>(b + L.sh);
    const int nc = 3 * sh_coeffs(sh_deg);
    gauss_pack_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(g.perm, g.n, nullptr, ls, quat, 1.f, sh, nc,
                                                                      L.s4, gauss, shp);
    const FieldView F{nullptr, shp, sh_deg, L.s4};
    if (!backward) {
        if (m > 0)
            color_forward_kernel<<<blocks(m, kBlock), kBlock, 0, st>>>(g, gauss, F, x, dirs, site, m, rgb, status);
        return cudaGetLastError();
    }
    float4* acc = reinterpret_cast<float4*>(b + L.acc);
    cudaError_t e = cudaMemsetAsync(acc, 0, 16 * static_cast<size_t>(L.stride) * g.n, st);
    if (e != cudaSuccess) return e;
    if (m > 0)
        color_backward_kernel<<<blocks(m, kBlock), kBlock, 0, st>>>(g, gauss, F, x, dirs, site, m, rgb_in, g_rgb, acc,
                                                                    L.stride, status);
    field_grad_kernel<<<blocks(g.n, kPrepBlock), kPrepBlock, 0, st>>>(g.perm, g.n, ls, quat, acc, L.stride, nc,
                                                                      nullptr, g_ls, g_quat, g_sh);
    return cudaGetLastError();
}

}  // namespace vg
