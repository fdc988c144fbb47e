// Interaction-point rendering (the reference's foam.cu path), one thread per ray.
//
// Samples are x(near), every crossing of a Voronoi face and x(far) (or the last crossing before
// T < t_thresh); consecutive samples bound a segment inside one cell, composited with the trapezoid
// rule (foam.cu:1-16). Rays of a 4x8 pixel tile sit in one warp, so the 32 threads walk through the
// same cells and their 16-byte edge / 64-byte site gathers coalesce into broadcasts. One pass over a
// cell's neighbourhood yields the exit face, the density and the colour blend of the sample.
//
// Training forward records every sample (t, original site, sigma, C rgb, m_min, 1 / sum of colour
// weights) in the reference's (B, K, 8) record format; the backward pass replays the records front to
// back with the reference's suffix formula (foam.cu:16, 428-467) and re-traces rays with more than K
// samples. Gradients go to the (N, 64) gradient pack with 16-byte vector atomics.
#include "render_core.cuh"

namespace vg {
namespace {

constexpr int kBlock = 128;
constexpr int kSlots = 8;

__device__ __forceinline__ void store_sample(float* __restrict__ rec, int64_t r, int K, int s, const Sample& P,
                                             const int* __restrict__ perm) {
    if (s >= K) return;
    float4* q = reinterpret_cast<float4*>(rec + (r * K + s) * kRecord);
    q[0] = make_float4(P.t, __int_as_float(__ldg(perm + P.cell)), P.sigma, P.C0);
    q[1] = make_float4(P.C1, P.C2, P.mmin, P.inv_a);
}

__device__ __forceinline__ void load_sample(const float* __restrict__ rec, int64_t r, int K, int s,
                                            const float (&o)[3], const float (&d)[3], const int* __restrict__ inv,
                                            Sample& P, bool& has_c) {
    const float4* q = reinterpret_cast<const float4*>(rec + (r * K + s) * kRecord);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    P.t = a.x;
    P.x0 = along(o[0], P.t, d[0]), P.x1 = along(o[1], P.t, d[1]), P.x2 = along(o[2], P.t, d[2]);
    P.cell = __ldg(inv + __float_as_int(a.y));
    P.sigma = a.z;
    P.C0 = a.w, P.C1 = b.x, P.C2 = b.y, P.mmin = b.z, P.inv_a = b.w;
    has_c = P.inv_a > 0.f;
}

__device__ __forceinline__ void load_ray(const RayView& R, int64_t r, float (&o)[3], float (&d)[3], float& near,
                                         float& far) {
#pragma unroll
    for (int a = 0; a < 3; ++a) o[a] = __ldg(R.o + 3 * r + a), d[a] = __ldg(R.d + 3 * r + a);
    near = __ldg(R.near + r), far = __ldg(R.far + r);
}

template <bool RECORD>
__global__ void __launch_bounds__(kBlock)
    foam_forward_kernel(GraphView g, FieldView F, RayView R, FoamCfg c, Outputs out, int* status) {
    __shared__ float4 cache_mem[kSlots * kBlock];
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    ColorCache<kSlots> cache{cache_mem + threadIdx.x, kBlock};
    cache.init();
    float o[3], d[3], near, far;
    load_ray(R, r, o, d, near, far);
    float b[16];
    sh_basis(d[0], d[1], d[2], F.sh_deg, b);
    int err = 0, walk_steps = 0, n_samples = 1, n_color = 0;
    const int K = c.record_cap;
    int cur = walk_to(g, __ldg(g.inv + __ldg(R.start + r)), along(o[0], near, d[0]), along(o[1], near, d[1]),
                      along(o[2], near, d[2]), walk_steps, err);
    Sample P;
    float t_exit;
    int next;
    eval_sample(g, F, cur, near, o, d, b, cache, true, P, t_exit, next);
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, dep = 0.f;
    int it = 0;
    for (; it < kMaxCells; ++it) {
        const bool last = next < 0 || t_exit >= far;
        Sample Q;
        float t_exit_q;
        int next_q;
        eval_sample(g, F, last ? P.cell : next, last ? far : fmaxf(t_exit, P.t), o, d, b, cache, !last, Q, t_exit_q,
                    next_q);
        ++n_samples;
        const float delta = Q.t - P.t;
        const float alpha = 1.f - __expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        if (w > c.w_thresh) {
            acc0 += w * 0.5f * (P.C0 + Q.C0);
            acc1 += w * 0.5f * (P.C1 + Q.C1);
            acc2 += w * 0.5f * (P.C2 + Q.C2);
            dep += w * 0.5f * (P.t + Q.t);
            ++n_color;
        }
        T *= 1.f - alpha;
        if (RECORD) store_sample(out.rec, r, K, n_samples - 2, P, g.perm);
        P = Q;
        t_exit = t_exit_q, next = next_q;
        if (last || T < c.t_thresh) break;
    }
    if (it == kMaxCells) err |= kErrCellCap;
    if (RECORD) store_sample(out.rec, r, K, n_samples - 1, P, g.perm);
    out.rgb[3 * r] = acc0, out.rgb[3 * r + 1] = acc1, out.rgb[3 * r + 2] = acc2;
    out.T[r] = T;
    out.depth[r] = dep;
    out.stats[3 * r] = n_samples, out.stats[3 * r + 1] = n_color, out.stats[3 * r + 2] = walk_steps;
    if (err) atomicOr(status, err);
}

__global__ void __launch_bounds__(kBlock)
    foam_backward_kernel(GraphView g, FieldView F, RayView R, FoamCfg c, GradIn gi, float* __restrict__ grad,
                         int* status) {
    __shared__ float4 cache_mem[kSlots * kBlock];
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    ColorCache<kSlots> cache{cache_mem + threadIdx.x, kBlock};
    cache.init();
    float o[3], d[3], near, far;
    load_ray(R, r, o, d, near, far);
    float b[16];
    sh_basis(d[0], d[1], d[2], F.sh_deg, b);
    const float gR0 = __ldg(gi.g_rgb + 3 * r), gR1 = __ldg(gi.g_rgb + 3 * r + 1), gR2 = __ldg(gi.g_rgb + 3 * r + 2);
    const float fg0 = __ldg(gi.rgb + 3 * r), fg1 = __ldg(gi.rgb + 3 * r + 1), fg2 = __ldg(gi.rgb + 3 * r + 2);
    const float gT_final = __ldg(gi.g_T + r) * __ldg(gi.T + r);
    const int K = gi.record_cap;
    const int s_fwd = __ldg(gi.stats + 3 * r);
    const int n_stored = gi.rec != nullptr && K > 0 && s_fwd <= K ? s_fwd : 0;
    int err = 0;
    Sample P;
    bool has_p = true;
    float t_exit = kInf;
    int next = -1;
    if (n_stored > 0) {
        load_sample(gi.rec, r, K, 0, o, d, g.inv, P, has_p);
    } else {
        int walk_steps = 0;
        const int cur = walk_to(g, __ldg(g.inv + __ldg(R.start + r)), along(o[0], near, d[0]),
                                along(o[1], near, d[1]), along(o[2], near, d[2]), walk_steps, err);
        eval_sample(g, F, cur, near, o, d, b, cache, true, P, t_exit, next);
    }
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    float gs_pending = 0.f, gP0 = 0.f, gP1 = 0.f, gP2 = 0.f;  // gradients of P from the segment before it
    for (int it = 0; it < kMaxCells; ++it) {
        Sample Q;
        bool last, has_q = true;
        float t_exit_q = kInf;
        int next_q = -1;
        if (n_stored > 0) {
            if (it + 1 >= n_stored) break;
            load_sample(gi.rec, r, K, it + 1, o, d, g.inv, Q, has_q);
            last = it + 2 >= n_stored;
        } else {
            last = next < 0 || t_exit >= far;
            eval_sample(g, F, last ? P.cell : next, last ? far : fmaxf(t_exit, P.t), o, d, b, cache, !last, Q,
                        t_exit_q, next_q);
        }
        const float delta = Q.t - P.t;
        const float alpha = 1.f - __expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        const float T_next = T * (1.f - alpha);
        const bool active = w > c.w_thresh;
        float c0 = 0.f, c1 = 0.f, c2 = 0.f;
        if (active) {
            c0 = 0.5f * (P.C0 + Q.C0), c1 = 0.5f * (P.C1 + Q.C1), c2 = 0.5f * (P.C2 + Q.C2);
            acc0 += w * c0, acc1 += w * c1, acc2 += w * c2;
        }
        float g_sbar = gR0 * (T_next * c0 - (fg0 - acc0)) + gR1 * (T_next * c1 - (fg1 - acc1)) +
                       gR2 * (T_next * c2 - (fg2 - acc2));
        g_sbar = delta * (g_sbar - gT_final);
        const float h0 = active ? 0.5f * w * gR0 : 0.f, h1 = active ? 0.5f * w * gR1 : 0.f,
                    h2 = active ? 0.5f * w * gR2 : 0.f;
        scatter_sample(g, F, P, gs_pending + 0.5f * g_sbar, gP0 + h0, gP1 + h1, gP2 + h2, has_p, b, cache, grad);
        gs_pending = 0.5f * g_sbar;
        gP0 = h0, gP1 = h1, gP2 = h2;
        T = T_next;
        P = Q;
        has_p = has_q;
        t_exit = t_exit_q, next = next_q;
        if (last || T < c.t_thresh) break;
    }
    scatter_sample(g, F, P, gs_pending, gP0, gP1, gP2, has_p, b, cache, grad);
    if (err) atomicOr(status, err);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

cudaError_t foam_forward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                         const Outputs& out, int* status, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    if (c.record_cap > 0 && out.rec != nullptr)
        foam_forward_kernel<true><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, out, status);
    else
        foam_forward_kernel<false><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, out, status);
    return cudaGetLastError();
}

cudaError_t foam_backward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                          const GradIn& gi, float* grad, int* status, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    foam_backward_kernel<<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, gi, grad, status);
    return cudaGetLastError();
}

}  // namespace vg
