// Fixed-step ray marching (the reference's march.cu path), one thread per ray.
//
// Samples are the midpoints of steps dt inside [near, mid] and n_bg steps uniform in disparity over
// [mid, far] (march.cu:143-153). At every sample the thread walks greedily from the previous site to
// the nearest one, sums the density Gaussians of its neighbourhood and, when the sample's weight
// exceeds w_thresh, blends the colour Gaussians (march.cu:221-262). The backward pass re-marches the
// ray with identical arithmetic (march.cu:264-345); its samples' gradients go to the cell-major scatter
// of foam.cu (items bucketed by cell) when the workspace allows, else per lane with 16-byte atomics.
#include "prof.cuh"
#include "render_core.cuh"

namespace vg {
namespace {

constexpr int kBlock = 128;

__global__ void __launch_bounds__(kBlock)
    march_forward_kernel(GraphView g, FieldView F, RayView R, MarchCfg c, Outputs out, int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    Schedule M;
    schedule_of(R, c, r, M);
    float b[16];
    sh_basis(M.d[0], M.d[1], M.d[2], F.sh_deg, b);
    int err = 0, cur = __ldg(g.inv + __ldg(R.start + r)), n_samples = 0, n_color = 0, walk_steps = 0;
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, dep = 0.f;
    for (int k = 0; k < M.n_total; ++k) {
        float t, delta;
        schedule_step(M, c, k, t, delta);
        Sample S;
        S.t = t;
        S.x0 = along(M.o[0], t, M.d[0]), S.x1 = along(M.o[1], t, M.d[1]), S.x2 = along(M.o[2], t, M.d[2]);
        cur = walk_nearest(g, cur, S.x0, S.x1, S.x2, walk_steps, err);
        S.cell = cur;
        const float alpha = 1.f - __expf(-eval_density(g, F, cur, S.x0, S.x1, S.x2) * delta);
        const float w = T * alpha;
        ++n_samples;
        if (w > c.w_thresh) {
            eval_color(g, F, b, S);
            acc0 += w * S.C0, acc1 += w * S.C1, acc2 += w * S.C2;
            dep += w * t;
            ++n_color;
        }
        T *= 1.f - alpha;
        if (T < c.t_thresh) break;
    }
    out.rgb[3 * r] = acc0, out.rgb[3 * r + 1] = acc1, out.rgb[3 * r + 2] = acc2;
    out.T[r] = T;
    out.depth[r] = dep;
    out.stats[3 * r] = n_samples, out.stats[3 * r + 1] = n_color, out.stats[3 * r + 2] = walk_steps;
    if (err) atomicOr(status, err);
}

__global__ void __launch_bounds__(kBlock)
    march_backward_kernel(GraphView g, FieldView F, RayView R, MarchCfg c, GradIn gi, float* __restrict__ grad,
                          int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    Schedule M;
    schedule_of(R, c, r, M);
    float b[16];
    sh_basis(M.d[0], M.d[1], M.d[2], F.sh_deg, b);
    const float gR0 = __ldg(gi.g_rgb + 3 * r), gR1 = __ldg(gi.g_rgb + 3 * r + 1), gR2 = __ldg(gi.g_rgb + 3 * r + 2);
    const float fg0 = __ldg(gi.rgb + 3 * r), fg1 = __ldg(gi.rgb + 3 * r + 1), fg2 = __ldg(gi.rgb + 3 * r + 2);
    const float tail_grad = __ldg(gi.g_T + r) * __ldg(gi.T + r);
    int err = 0, cur = __ldg(g.inv + __ldg(R.start + r)), walk_steps = 0;
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    for (int k = 0; k < M.n_total; ++k) {
        float t, delta;
        schedule_step(M, c, k, t, delta);
        Sample S;
        S.t = t;
        S.x0 = along(M.o[0], t, M.d[0]), S.x1 = along(M.o[1], t, M.d[1]), S.x2 = along(M.o[2], t, M.d[2]);
        cur = walk_nearest(g, cur, S.x0, S.x1, S.x2, walk_steps, err);
        S.cell = cur;
        const float alpha = 1.f - __expf(-eval_density(g, F, cur, S.x0, S.x1, S.x2) * delta);
        const float w = T * alpha;
        const float T_after = T * (1.f - alpha);
        const bool active = w > c.w_thresh;
        S.C0 = S.C1 = S.C2 = 0.f, S.mmin = 0.f, S.inv_a = 0.f;
        if (active) {
            eval_color(g, F, b, S);
            acc0 += w * S.C0, acc1 += w * S.C1, acc2 += w * S.C2;
        }
        float gsig = gR0 * (T_after * S.C0 - (fg0 - acc0)) + gR1 * (T_after * S.C1 - (fg1 - acc1)) +
                     gR2 * (T_after * S.C2 - (fg2 - acc2));
        gsig = delta * (gsig - tail_grad);
        sample_grads(g, F, S, gsig, active ? w * gR0 : 0.f, active ? w * gR1 : 0.f, active ? w * gR2 : 0.f, active,
                     b, grad);
        T = T_after;
        if (T < c.t_thresh) break;
    }
    if (err) atomicOr(status, err);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

cudaError_t march_forward(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                          const Outputs& out, int* status, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    {
        ProfScope ps(kProfMarchFwd, st);
        march_forward_kernel<<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, out, status);
    }
    return cudaGetLastError();
}

cudaError_t march_backward(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                           const GradIn& gi, float* grad, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    if (cm_ws != nullptr && cm_bytes >= march_backward_workspace(g.n, R.n))
        return march_backward_cm(g, F, R, c, gi, grad, status, cm_ws, st);
    march_backward_kernel<<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, gi, grad, status);
    return cudaGetLastError();
}

}  // namespace vg
