// Inference renderer on the packed inference layout of render.pack_foam (foam_infer.cu:376-435 is the
// interface it replaces). The layout is self-first: cell c owns the edge run [offsets[c], offsets[c+1]),
// whose first record is the site itself, each record a float4 (p_j, half2(r2_j, lam_j)) with the site id
// in a parallel array; per-site rows attr (N, 5 x float4) = density conic + min(raw, 30) | colour conic |
// baked colour; SH in fp32 or fp16.
//
// One thread per ray (rays of a pixel tile share a warp). The samples are those of the training renderer:
// x(near), every exit-face crossing and x(far). Every sample scans its cell's run once for the exit face,
// the density (neighbours farther than sqrt(r2) skipped) and the colour, which, by mode, is
//   exact  the smallest colour Mahalanobis distance m_min only (neighbours whose bound r2 lam is not
//          below the current m_min are skipped); segments with weight > w_thresh then blend their two
//          end samples in a second scan over the neighbours within m_min + color_cut;
//   fused  an online blend in the same scan over the neighbours within m + color_cut of the running
//          minimum;
//   baked  the same blend of the per-view site colours of bake_colors.
// Site colours max(SH_k(d) + 1/2, 0) depend only on the ray direction, so each ray keeps a direct-mapped
// cache of 8 of them in shared memory. Stages 0 and 1 are the reference's ablations: exit faces only, and
// exit faces + density. Per-ray stats (B, 5): samples, coloured segments, walk steps, density terms
// evaluated, SH evaluations; these counts follow the reference's skipping and caching rules, so they
// match its kernel's.
#include "infer_core.cuh"
#include "prof.cuh"

namespace vg {
namespace infer {
namespace {

template <int STAGE, int MODE, bool HALF>
__global__ void __launch_bounds__(kThreads)
    infer_kernel(Layout L, InferCfg cfg, RayView R, Outputs out, int* status) {
    __shared__ float4 cache_mem[kSlots * kThreads];
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (r >= R.n) return;
    if (cfg.only_over != nullptr && __ldg(cfg.only_over + r) <= cfg.over) return;
    SlotCache<HALF> cache{cache_mem + threadIdx.x};
    cache.clear();
    float o[3], d[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) o[a] = __ldg(R.o + 3 * r + a), d[a] = __ldg(R.d + 3 * r + a);
    const float t_near = __ldg(R.near + r), t_far = __ldg(R.far + r);
    const int max_samples = cfg.cap != nullptr ? __ldg(cfg.cap + r) : INT_MAX;
    float b[16];
    sh_basis(d[0], d[1], d[2], STAGE >= 2 && MODE != kBakedColour ? cfg.sh_deg : 0, b);
    int err = 0, walk_steps = 0, n_dens = 0, n_sh = 0, n_samples = 1, n_coloured = 0;

    const int first = nearest_site(L, __ldg(R.start + r), along(o[0], t_near, d[0]), along(o[1], t_near, d[1]),
                                   along(o[2], t_near, d[2]), walk_steps, err);
    CellScan S;
    scan_cell<STAGE, MODE, HALF>(L, cfg, first, t_near, o, d, b, cache, true, S, n_dens, n_sh);
    Sample P;
    take<STAGE, MODE, HALF>(P, S, t_near, first);
    float T = 1.f, fg[3] = {0.f, 0.f, 0.f}, depth = 0.f;
    bool done = false;  // the ray ended (far plane, unbounded cell, sample cap or opacity) within kMaxCells
    for (int cell = 0; cell < kMaxCells && !done; ++cell) {
        const bool last = S.next == INT_MAX || S.t_exit >= t_far || n_samples + 1 >= max_samples;
        const float tQ = last ? t_far : fmaxf(S.t_exit, P.t);
        const int cQ = last ? P.cell : S.next;
        scan_cell<STAGE, MODE, HALF>(L, cfg, cQ, tQ, o, d, b, cache, !last, S, n_dens, n_sh);
        ++n_samples;
        Sample Q;
        take<STAGE, MODE, HALF>(Q, S, tQ, cQ);
        const float alpha = 1.f - __expf(-0.5f * (P.sigma + Q.sigma) * (Q.t - P.t));
        const float w = T * alpha;
        if (STAGE >= 2 && w > cfg.w_thresh) {
            if (MODE == kExact) {
                if (!P.coloured) exact_colour<HALF>(L, cfg, P, o, d, b, cache, n_sh);
                exact_colour<HALF>(L, cfg, Q, o, d, b, cache, n_sh);
            }
#pragma unroll
            for (int a = 0; a < 3; ++a) fg[a] += w * 0.5f * (P.rgb[a] + Q.rgb[a]);
            depth += w * 0.5f * (P.t + Q.t);
            ++n_coloured;
        }
        T *= 1.f - alpha;
        P = Q;
        done = last || T < cfg.t_thresh;
    }
    if (!done) err |= kErrCellCap;
#pragma unroll
    for (int a = 0; a < 3; ++a) out.rgb[3 * r + a] = fg[a];
    out.T[r] = T;
    out.depth[r] = depth;
    int* s = out.stats + 5 * r;
    s[0] = n_samples, s[1] = n_coloured, s[2] = walk_steps, s[3] = n_dens, s[4] = n_sh;
    if (err) atomicOr(status, err);
}

template <int STAGE, int MODE, bool HALF>
void launch(const Layout& L, const InferCfg& cfg, const RayView& R, const Outputs& out, int* status, cudaStream_t st) {
    const int blocks = static_cast<int>((R.n + kThreads - 1) / kThreads);
    ProfScope ps(kProfInfer, st);
    infer_kernel<STAGE, MODE, HALF><<<blocks, kThreads, 0, st>>>(L, cfg, R, out, status);
}

}  // namespace
}  // namespace infer

cudaError_t foam_infer(const InferNet& net, const InferCfg& cfg, const RayView& R, const Outputs& out, int* status,
                       cudaStream_t st) {
    using namespace infer;
    if (R.n == 0) return cudaSuccess;
    const Layout L{net};
    const bool half = net.sh_half != 0;
    if (cfg.stage == 0) {
        launch<0, kExact, false>(L, cfg, R, out, status, st);
    } else if (cfg.stage == 1) {
        launch<1, kExact, false>(L, cfg, R, out, status, st);
    } else if (cfg.color_mode == kBakedColour) {
        launch<2, kBakedColour, false>(L, cfg, R, out, status, st);
    } else if (cfg.color_mode == kExact) {
        if (half)
            launch<2, kExact, true>(L, cfg, R, out, status, st);
        else
            launch<2, kExact, false>(L, cfg, R, out, status, st);
    } else if (half) {
        launch<2, kFusedColour, true>(L, cfg, R, out, status, st);
    } else {
        launch<2, kFusedColour, false>(L, cfg, R, out, status, st);
    }
    return cudaGetLastError();
}

}  // namespace vg
