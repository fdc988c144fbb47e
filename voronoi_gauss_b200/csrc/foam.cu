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
#include <algorithm>
#include <cub/device/device_scan.cuh>

#include "prof.cuh"
#include "render_core.cuh"

// Tuning constants, chosen by measurement on B200 (config-3 scenes at 1080p); the alternatives tried and
// rejected are recorded with their times in the design notes of this repository:
//   kFwdMinBlocks / kBwdMinBlocks / kColorMinBlocks / kScatterMinBlocks  minimum resident blocks of 128
//                  threads per SM of the traversal, the per-ray backward, the colour pass and the scatter
//                  (their register budgets)
//   kChunk         samples of one cell per warp in the cell-major passes (two per lane in the colour
//                  pass), which sets how often a cell's neighbourhood is reloaded
//   kReplicaMaxN   largest neighbourhood size (self included) for which cm_scatter_kernel spreads a
//                  chunk's (neighbour, sample) pairs over all 32 lanes as replicas of each neighbour;
//                  larger cells get one lane per neighbour
//   kScatterUnroll samples of a chunk whose dependent chains one scatter lane interleaves
#ifndef VG_FWD_MINB
#define VG_FWD_MINB 6
#endif
#ifndef VG_BWD_MINB
#define VG_BWD_MINB 1
#endif
#ifndef VG_COLOR_MINB
#define VG_COLOR_MINB 1
#endif
#ifndef VG_SCATTER_MINB
#define VG_SCATTER_MINB 3
#endif
#ifndef VG_SCATTER_UNROLL
#define VG_SCATTER_UNROLL 1
#endif

namespace vg {
namespace {

constexpr int kBlock = 128;
constexpr int kChunk = 64;
constexpr int kReplicaMaxN = 16;
constexpr int kScatterUnroll = VG_SCATTER_UNROLL;

// deferred: the colour fields are filled later; the last field marks the samples that need one (-1)
// orig: the original id of P's site (loaded when P was evaluated, so the store does not wait for it)
__device__ __forceinline__ void put_record(float* __restrict__ rec, int64_t r, int K, int s, const Sample& P,
                                             bool has_c, bool deferred, int orig) {
    if (s >= K) return;
    float4* q = reinterpret_cast<float4*>(rec + (r * K + s) * kRecord);
    q[0] = make_float4(P.t, __int_as_float(orig), P.sigma, deferred ? 0.f : P.C0);
    q[1] = deferred ? make_float4(0.f, 0.f, 0.f, has_c ? -1.f : 0.f)
                    : make_float4(P.C1, P.C2, P.mmin, has_c ? P.inv_a : 0.f);
}

// The two float4 of record s of ray r.
__device__ __forceinline__ void load_record(const float* __restrict__ rec, int64_t r, int K, int s, float4 (&q)[2]) {
    const float4* p = reinterpret_cast<const float4*>(rec + (r * K + s) * kRecord);
    q[0] = __ldg(p), q[1] = __ldg(p + 1);
}

// A sample from its record's two float4.
__device__ __forceinline__ void decode_record(const float4 (&q)[2], const float (&o)[3], const float (&d)[3],
                                              const int* __restrict__ inv, Sample& P, bool& has_c) {
    const float4 a = q[0], b = q[1];
    P.t = a.x;
    P.x0 = along(o[0], P.t, d[0]), P.x1 = along(o[1], P.t, d[1]), P.x2 = along(o[2], P.t, d[2]);
    P.cell = __ldg(inv + __float_as_int(a.y));
    P.sigma = a.z;
    P.C0 = a.w, P.C1 = b.x, P.C2 = b.y, P.mmin = b.z, P.inv_a = b.w;
    has_c = P.inv_a > 0.f;
}

__device__ __forceinline__ void get_record(const float* __restrict__ rec, int64_t r, int K, int s,
                                           const float (&o)[3], const float (&d)[3], const int* __restrict__ inv,
                                           Sample& P, bool& has_c) {
    float4 q[2];
    load_record(rec, r, K, s, q);
    decode_record(q, o, d, inv, P, has_c);
}

__device__ __forceinline__ void load_ray(const RayView& R, int64_t r, float (&o)[3], float (&d)[3], float& near,
                                         float& far) {
#pragma unroll
    for (int a = 0; a < 3; ++a) o[a] = __ldg(R.o + 3 * r + a), d[a] = __ldg(R.d + 3 * r + a);
    near = __ldg(R.near + r), far = __ldg(R.far + r);
}

// What the forward does with colours: evaluate them inline for the segments that need them (every ray,
// or only the rays with more samples than records), or defer them to the cell-major colour pass and
// only mark, in the record's last field, the samples that need one (-1; 0 otherwise).
enum FwdMode { kImmediate = 0, kImmediateOverflow = 1, kDeferred = 2 };

template <bool RECORD, int MODE>
__global__ void __launch_bounds__(kBlock, VG_FWD_MINB)
    foam_forward_kernel(GraphView g, FieldView F, RayView R, FoamCfg c, Outputs out, int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    const int K = c.record_cap;
    if (MODE == kImmediateOverflow && __ldg(out.stats + 3 * r) <= K) return;
    if (MODE == kImmediateOverflow && (c.cm_count != nullptr || c.all_count != nullptr)) {
        // the deferred traversal counted this ray's records; it leaves the cell-major passes
        int* cnt = c.cm_count != nullptr ? c.cm_count + (r / c.cm_rays) * c.cm_stride : nullptr;
        int* all = c.all_count != nullptr ? c.all_count + (r / c.cm_rays) * c.cm_stride : nullptr;
        for (int s = 0; s < K; ++s) {
            const float* q = out.rec + (r * K + s) * kRecord;
            const int cell = __ldg(g.inv + __float_as_int(q[1]));
            if (cnt != nullptr && q[7] < 0.f) atomicAdd(cnt + cell, -1);
            if (all != nullptr) atomicAdd(all + cell, -1);
        }
    }
    constexpr bool kDefer = MODE == kDeferred;
    float o[3], d[3], near, far;
    load_ray(R, r, o, d, near, far);
    float b[16];
    if (!kDefer) sh_basis(d[0], d[1], d[2], F.sh_deg, b);
    int err = 0, walk_steps = 0, n_samples = 1, n_color = 0;
    int cur = walk_nearest(g, __ldg(g.inv + __ldg(R.start + r)), along(o[0], near, d[0]), along(o[1], near, d[1]),
                      along(o[2], near, d[2]), walk_steps, err);
    Sample P;
    float t_exit;
    int next;
    eval_sample<false>(g, F, cur, near, o, d, b, true, P, t_exit, next);
    int p_orig = RECORD ? __ldg(g.perm + P.cell) : 0;
    bool has_p = false;
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, dep = 0.f;
    int it = 0;
    for (; it < kMaxCells; ++it) {
        const bool last = next < 0 || t_exit >= far;
        Sample Q;
        float t_exit_q;
        int next_q;
        eval_sample<false>(g, F, last ? P.cell : next, last ? far : fmaxf(t_exit, P.t), o, d, b, !last, Q, t_exit_q,
                           next_q);
        bool has_q = false;
        const int q_orig = RECORD ? __ldg(g.perm + Q.cell) : 0;
        ++n_samples;
        const float delta = Q.t - P.t;
        const float alpha = 1.f - __expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        if (w > c.w_thresh) {
            if (kDefer) {
                has_p = has_q = true;  // marked: coloured by the cell-major pass
            } else {
                // lazy colours: only the samples bordering a segment with weight > w_thresh need one
                if (!has_p) eval_color(g, F, b, P), has_p = true;
                eval_color(g, F, b, Q), has_q = true;
                acc0 += w * 0.5f * (P.C0 + Q.C0);
                acc1 += w * 0.5f * (P.C1 + Q.C1);
                acc2 += w * 0.5f * (P.C2 + Q.C2);
            }
            dep += w * 0.5f * (P.t + Q.t);
            ++n_color;
        }
        T *= 1.f - alpha;
        if (RECORD) put_record(out.rec, r, K, n_samples - 2, P, has_p, kDefer, p_orig);
        if (kDefer && has_p && n_samples - 2 < K && c.cm_count != nullptr)
            atomicAdd(c.cm_count + (r / c.cm_rays) * c.cm_stride + P.cell, 1);
        if (kDefer && n_samples - 2 < K && c.all_count != nullptr)
            atomicAdd(c.all_count + (r / c.cm_rays) * c.cm_stride + P.cell, 1);
        P = Q;
        p_orig = q_orig;
        has_p = has_q;
        t_exit = t_exit_q, next = next_q;
        if (last || T < c.t_thresh) break;
    }
    if (it == kMaxCells) err |= kErrCellCap;
    if (RECORD) put_record(out.rec, r, K, n_samples - 1, P, has_p, kDefer, p_orig);
    if (kDefer && has_p && n_samples - 1 < K && c.cm_count != nullptr)
        atomicAdd(c.cm_count + (r / c.cm_rays) * c.cm_stride + P.cell, 1);
    if (kDefer && n_samples - 1 < K && c.all_count != nullptr)
        atomicAdd(c.all_count + (r / c.cm_rays) * c.cm_stride + P.cell, 1);
    if (!kDefer) out.rgb[3 * r] = acc0, out.rgb[3 * r + 1] = acc1, out.rgb[3 * r + 2] = acc2;
    out.T[r] = T;
    out.depth[r] = dep;
    out.stats[3 * r] = n_samples, out.stats[3 * r + 1] = n_color, out.stats[3 * r + 2] = walk_steps;
    if (err) atomicOr(status, err);
}

// ------------------------------------------------------------------- cell-major colours (forward)
//
// Deferred colours: the traversal marks the samples that border a segment with weight > w_thresh;
// those samples are bucketed by cell (the counting sort of the backward) and a warp evaluates up to
// 32 samples of one cell at a time, one lane per sample: every lane walks the same neighbour list, so
// the edge, site-record and SH loads are warp-uniform broadcasts. The blend visits the neighbours in
// the cell's order with the same arithmetic as eval_color, so the colours are bit-identical to the
// inline path; cmf_composite_kernel then sums the segments of every ray from its records.

// Samples of a ray chunk counted per cell (the backward's item buckets). One warp per ray, lanes over its
// samples: the records of a ray are read as contiguous 32-byte sectors.
__global__ void __launch_bounds__(kBlock)
    cmf_count_kernel(const float* __restrict__ rec, const int* __restrict__ stats, const int* __restrict__ inv,
                     int64_t r0, int64_t n, int K, int* __restrict__ count) {
    const int64_t rl = (static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (rl >= n) return;
    const int64_t r = r0 + rl;
    const int S = __ldg(stats + 3 * r);
    if (S > K) return;
    for (int s = lane; s < S; s += 32) {
        const float* q = rec + (r * K + s) * kRecord;
        atomicAdd(count + __ldg(inv + __float_as_int(__ldg(q + 1))), 1);
    }
}

// The slots of the samples that need a colour, counting-sorted by cell (one warp per ray).
__global__ void __launch_bounds__(kBlock)
    cmf_bucket_kernel(const float* __restrict__ rec, const int* __restrict__ stats, const int* __restrict__ inv,
                      int64_t r0, int64_t n, int K, const int* __restrict__ offsets, int* __restrict__ fill,
                      int* __restrict__ order) {
    const int64_t rl = (static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (rl >= n) return;
    const int64_t r = r0 + rl;
    const int S = __ldg(stats + 3 * r);
    if (S > K) return;
    for (int s = lane; s < S; s += 32) {
        const float* q = rec + (r * K + s) * kRecord;
        if (__ldg(q + 7) < 0.f) {
            const int cell = __ldg(inv + __float_as_int(__ldg(q + 1)));
            order[__ldg(offsets + cell) + atomicAdd(fill + cell, 1)] = static_cast<int>(rl * K + s);
        }
    }
}

template <int S4>
__global__ void __launch_bounds__(kBlock, VG_COLOR_MINB)
    cmf_color_kernel(GraphView g, FieldView F, RayView R, float* __restrict__ rec, int K,
                     const int* __restrict__ order, const int4* __restrict__ chunks, const int* __restrict__ n_chunks_ptr,
                     int64_t r0) {
    constexpr int kPer = kChunk / 32;  // samples per lane
    constexpr int kNv = 3 + S4;        // float4 per staged neighbour: edge, colour conic (2), SH rows
    __shared__ float4 nbr_smem[(kBlock / 32) * 32 * kNv];
    float4* nbr = nbr_smem + (threadIdx.x >> 5) * 32 * kNv;
    const int lane = threadIdx.x & 31;
    const int n_chunks = *n_chunks_ptr;
    const int warps = gridDim.x * (kBlock / 32);
    for (int ch = blockIdx.x * (kBlock / 32) + (threadIdx.x >> 5); ch < n_chunks; ch += warps) {
        const int4 C = __ldg(chunks + ch);
        int64_t slot[kPer];
        float x[kPer][3], b[kPer][16];
        Blend B[kPer];
#pragma unroll
        for (int p = 0; p < kPer; ++p) {
            const int li = lane + 32 * p;
            slot[p] = -1;
            x[p][0] = x[p][1] = x[p][2] = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) b[p][k] = 0.f;
            B[p].reset();
            if (li < C.z) {
                const int sl = __ldg(order + C.y + li);
                const int64_t r = r0 + sl / K, s = sl % K;
                slot[p] = r * K + s;
                const float t = rec[slot[p] * kRecord];
                float o[3], d[3];
#pragma unroll
                for (int a = 0; a < 3; ++a) o[a] = __ldg(R.o + 3 * r + a), d[a] = __ldg(R.d + 3 * r + a);
                x[p][0] = along(o[0], t, d[0]), x[p][1] = along(o[1], t, d[1]), x[p][2] = along(o[2], t, d[2]);
                sh_basis(d[0], d[1], d[2], F.sh_deg, b[p]);
            }
        }
        const int e0 = __ldg(g.off + C.x), e1 = __ldg(g.off + C.x + 1);
        // the cell's neighbour data, up to 32 neighbours at a time, staged in shared memory by one lane
        // each (all loads in flight together), then read back as warp-wide broadcasts
        for (int eb = e0; eb < e1; eb += 32) {
            const int nb = min(32, e1 - eb);
            __syncwarp();
            if (lane < nb) {
                const float4 E = __ldg(g.edge + eb + lane);
                const int j = site_of(E);
                const float4* fr = F.rec + kFieldVec * static_cast<int64_t>(j);
                const float4* sp = F.sh + static_cast<int64_t>(S4) * j;
                float4* dst = nbr + lane * kNv;
                dst[0] = E, dst[1] = __ldg(fr + 2), dst[2] = __ldg(fr + 3);
#pragma unroll
                for (int q = 0; q < S4; ++q) dst[3 + q] = __ldg(sp + q);
            }
            __syncwarp();
            for (int k = 0; k < nb; ++k) {  // warp-uniform: one cell per chunk
                const float4* src = nbr + k * kNv;
                const float4 E = src[0], r2 = src[1], r3 = src[2];
                float4 coef[S4];
#pragma unroll
                for (int q = 0; q < S4; ++q) coef[q] = src[3 + q];
#pragma unroll
                for (int p = 0; p < kPer; ++p) {
                    const float v0 = x[p][0] - E.x, v1 = x[p][1] - E.y, v2 = x[p][2] - E.z;
                    float c[3] = {0.5f, 0.5f, 0.5f};
#pragma unroll
                    for (int q = 0; q < S4; ++q) {
                        const float f[4] = {coef[q].x, coef[q].y, coef[q].z, coef[q].w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int i = 4 * q + u;
                            if (i < 48) c[i % 3] += b[p][i / 3] * f[u];
                        }
                    }
                    B[p].add(maha(r2, r3, v0, v1, v2), fmaxf(c[0], 0.f), fmaxf(c[1], 0.f), fmaxf(c[2], 0.f));
                }
            }
        }
#pragma unroll
        for (int p = 0; p < kPer; ++p) {
            if (slot[p] < 0) continue;
            const float inv_a = 1.f / B[p].wsum;
            float* q = rec + slot[p] * kRecord;
            q[3] = B[p].sum[0] * inv_a;
            reinterpret_cast<float4*>(q)[1] = make_float4(B[p].sum[1] * inv_a, B[p].sum[2] * inv_a, B[p].m_min, inv_a);
        }
    }
}

// Sums the coloured segments of every fully recorded ray from its records (same arithmetic as the
// traversal, so the weights and the set of coloured segments are the same).
__global__ void __launch_bounds__(kBlock)
    cmf_composite_kernel(const float* __restrict__ rec, const int* __restrict__ stats, int64_t n, int K,
                         float w_thresh, float* __restrict__ rgb) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= n) return;
    const int S = __ldg(stats + 3 * r);
    if (S > K) return;
    const float4* q = reinterpret_cast<const float4*>(rec + r * K * kRecord);
    float4 a0 = __ldg(q), a1 = __ldg(q + 1);
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    for (int s = 1; s < S; ++s) {
        const float4 b0 = __ldg(q + 2 * s), b1 = __ldg(q + 2 * s + 1);
        const float delta = b0.x - a0.x;
        const float alpha = 1.f - __expf(-0.5f * (a0.z + b0.z) * delta);
        const float w = T * alpha;
        if (w > w_thresh) {
            acc0 += w * 0.5f * (a0.w + b0.w);
            acc1 += w * 0.5f * (a1.x + b1.x);
            acc2 += w * 0.5f * (a1.y + b1.y);
        }
        T *= 1.f - alpha;
        a0 = b0, a1 = b1;
    }
    rgb[3 * r] = acc0, rgb[3 * r + 1] = acc1, rgb[3 * r + 2] = acc2;
}

// Per-sample item of the cell-major backward, written by the replay (replay_items_kernel) and consumed by
// cm_scatter_kernel: 64 bytes at the sample's place in its cell's bucket,
//   (x, gs) | (gC, gC . C) | (m_min, 1 / sum of colour weights or 0, 0, 0) | (d, 0)
// where every recorded sample gets an item (zero gradients for the samples that have none).

// What the per-ray backward does: scatter each sample's gradients to the sites of its neighbourhood, for
// every ray or only for the rays that were not recorded in full (the fully recorded ones go through
// replay_items_kernel and the cell-major scatter).
enum BwdMode { kScatterAll = 0, kScatterRetraced = 1 };

struct ItemOut {
    float4* items;         // the bucketed items
    int* count;            // (N + 1) samples per cell
    int64_t r0;            // first ray of the chunk
    int64_t n;             // rays in the chunk
    const int* offsets;    // first bucket position of every cell
    int* fill;             // bucket fill cursors
    int64_t cap;           // item slots of the buffer
    const int* bad;        // set by bucket_check_kernel when the buckets do not fit the buffer
    int* status;
};

template <int MODE>
__global__ void __launch_bounds__(kBlock, VG_BWD_MINB)
    foam_backward_kernel(GraphView g, FieldView F, RayView R, FoamCfg c, GradIn gi, float* __restrict__ grad,
                         int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    {
        const int K_ = gi.record_cap;
        const bool replayable = gi.rec != nullptr && K_ > 0 && __ldg(gi.stats + 3 * r) <= K_;
        if (MODE == kScatterRetraced && replayable) return;
    }
    float o[3], d[3], near, far;
    load_ray(R, r, o, d, near, far);
    float b[16];
    sh_basis(d[0], d[1], d[2], F.sh_deg, b);
    const float gR0 = __ldg(gi.g_rgb + 3 * r), gR1 = __ldg(gi.g_rgb + 3 * r + 1), gR2 = __ldg(gi.g_rgb + 3 * r + 2);
    const float fg0 = __ldg(gi.rgb + 3 * r), fg1 = __ldg(gi.rgb + 3 * r + 1), fg2 = __ldg(gi.rgb + 3 * r + 2);
    const float tail_grad = __ldg(gi.g_T + r) * __ldg(gi.T + r);
    const int K = gi.record_cap;
    const int s_fwd = __ldg(gi.stats + 3 * r);
    const int n_stored = gi.rec != nullptr && K > 0 && s_fwd <= K ? s_fwd : 0;
    int err = 0;
    Sample P;
    bool has_p = true;
    float t_exit = kInf;
    int next = -1;
    if (n_stored > 0) {
        get_record(gi.rec, r, K, 0, o, d, g.inv, P, has_p);
    } else {
        int walk_steps = 0;
        const int cur = walk_nearest(g, __ldg(g.inv + __ldg(R.start + r)), along(o[0], near, d[0]),
                                along(o[1], near, d[1]), along(o[2], near, d[2]), walk_steps, err);
        eval_sample<true>(g, F, cur, near, o, d, b, true, P, t_exit, next);
    }
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    float carry_sigma = 0.f, gP0 = 0.f, gP1 = 0.f, gP2 = 0.f;  // gradients of P from the segment before it
    for (int it = 0; it < kMaxCells; ++it) {
        Sample Q;
        bool last, has_q = true;
        float t_exit_q = kInf;
        int next_q = -1;
        if (n_stored > 0) {
            if (it + 1 >= n_stored) break;
            get_record(gi.rec, r, K, it + 1, o, d, g.inv, Q, has_q);
            last = it + 2 >= n_stored;
        } else {
            last = next < 0 || t_exit >= far;
            eval_sample<true>(g, F, last ? P.cell : next, last ? far : fmaxf(t_exit, P.t), o, d, b, !last, Q, t_exit_q,
                              next_q);
        }
        const float delta = Q.t - P.t;
        const float alpha = 1.f - __expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        const float T_after = T * (1.f - alpha);
        const bool active = w > c.w_thresh;
        float c0 = 0.f, c1 = 0.f, c2 = 0.f;
        if (active) {
            // colours of records written without them (foam.cu:443-445)
            if (!has_p) eval_color(g, F, b, P), has_p = true;
            if (!has_q) eval_color(g, F, b, Q), has_q = true;
            c0 = 0.5f * (P.C0 + Q.C0), c1 = 0.5f * (P.C1 + Q.C1), c2 = 0.5f * (P.C2 + Q.C2);
            acc0 += w * c0, acc1 += w * c1, acc2 += w * c2;
        }
        float g_opacity = gR0 * (T_after * c0 - (fg0 - acc0)) + gR1 * (T_after * c1 - (fg1 - acc1)) +
                       gR2 * (T_after * c2 - (fg2 - acc2));
        g_opacity = delta * (g_opacity - tail_grad);
        const float h0 = active ? 0.5f * w * gR0 : 0.f, h1 = active ? 0.5f * w * gR1 : 0.f,
                    h2 = active ? 0.5f * w * gR2 : 0.f;
        sample_grads(g, F, P, carry_sigma + 0.5f * g_opacity, gP0 + h0, gP1 + h1, gP2 + h2, has_p, b, grad);
        carry_sigma = 0.5f * g_opacity;
        gP0 = h0, gP1 = h1, gP2 = h2;
        T = T_after;
        P = Q;
        has_p = has_q;
        t_exit = t_exit_q, next = next_q;
        if (last || T < c.t_thresh) break;
    }
    sample_grads(g, F, P, carry_sigma, gP0, gP1, gP2, has_p, b, grad);
    if (err) atomicOr(status, err);
}

// The replay of a fully recorded ray into 64-byte items of its samples' cell buckets (foam_backward_kernel's
// arithmetic, items instead of atomics). A record is loaded one segment before it is decoded, and a
// sample's place in its bucket (the fill cursor's ticket) is taken when its record is decoded, one
// segment before its item is written, so both round trips overlap a segment's arithmetic. The loop is
// unrolled in pairs with the two samples (and their record buffers) trading the roles P and Q, so no
// value still in flight is copied between registers.
struct Ticketed {
    Sample S;
    bool has_c;
    int base, tick, limit;  // first position of the sample's cell bucket, its ticket in it, the bucket's end
    float4 raw[2];   // the next record this slot decodes
};

__device__ __forceinline__ void replay_decode(const GradIn& gi, const ItemOut& io, const GraphView& g, int64_t r,
                                              int K, int s, const float (&o)[3], const float (&d)[3], Ticketed& X) {
    get_record(gi.rec, r, K, s, o, d, g.inv, X.S, X.has_c);
    X.base = __ldg(io.offsets + X.S.cell), X.limit = __ldg(io.offsets + X.S.cell + 1);
    X.tick = atomicAdd(io.fill + X.S.cell, 1);
}

// decodes the record already loaded into X.raw
__device__ __forceinline__ void replay_decode_loaded(const ItemOut& io, const GraphView& g, const float (&o)[3],
                                                     const float (&d)[3], Ticketed& X) {
    decode_record(X.raw, o, d, g.inv, X.S, X.has_c);
    X.base = __ldg(io.offsets + X.S.cell), X.limit = __ldg(io.offsets + X.S.cell + 1);
    X.tick = atomicAdd(io.fill + X.S.cell, 1);
}

// Writes X's item at its place; a ticket beyond its cell's bucket (counts that do not belong to these
// records) drops the item and sets kErrBuckets instead of writing outside the bucket.
__device__ __forceinline__ void replay_put(const ItemOut& io, const Ticketed& X, float gs, float gC0, float gC1,
                                           float gC2, bool has_c, const float (&dir)[3]) {
    const int pos = X.base + X.tick;
    if (pos >= X.limit || pos < 0 || pos >= io.cap) {
        atomicOr(io.status, kErrBuckets);
        return;
    }
    const Sample& P = X.S;
    const bool do_c = has_c && (gC0 != 0.f || gC1 != 0.f || gC2 != 0.f);
    const float gCC = do_c ? gC0 * P.C0 + gC1 * P.C1 + gC2 * P.C2 : 0.f;
    float4* it = io.items + 4 * static_cast<int64_t>(pos);
    it[0] = make_float4(P.x0, P.x1, P.x2, gs);
    it[1] = make_float4(do_c ? gC0 : 0.f, do_c ? gC1 : 0.f, do_c ? gC2 : 0.f, gCC);
    it[2] = make_float4(P.mmin, do_c ? P.inv_a : 0.f, 0.f, 0.f);
    it[3] = make_float4(dir[0], dir[1], dir[2], 0.f);
}

__global__ void __launch_bounds__(kBlock, VG_BWD_MINB)
    replay_items_kernel(GraphView g, FieldView F, RayView R, FoamCfg c, GradIn gi, ItemOut io) {
    const int64_t r = io.r0 + static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= io.r0 + io.n) return;
    const int K = gi.record_cap;
    const int n_stored = __ldg(gi.stats + 3 * r);
    if (gi.rec == nullptr || K <= 0 || n_stored > K || n_stored <= 0 || *io.bad) return;
    float o[3], d[3], near, far;
    load_ray(R, r, o, d, near, far);
    float b[16];
    sh_basis(d[0], d[1], d[2], F.sh_deg, b);
    const float gR0 = __ldg(gi.g_rgb + 3 * r), gR1 = __ldg(gi.g_rgb + 3 * r + 1), gR2 = __ldg(gi.g_rgb + 3 * r + 2);
    const float fg0 = __ldg(gi.rgb + 3 * r), fg1 = __ldg(gi.rgb + 3 * r + 1), fg2 = __ldg(gi.rgb + 3 * r + 2);
    const float tail_grad = __ldg(gi.g_T + r) * __ldg(gi.T + r);
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    float carry_sigma = 0.f, gP0 = 0.f, gP1 = 0.f, gP2 = 0.f;  // gradients of P from the segment before it
    // segment k between P (record k) and Q (record k + 1, decoded here); writes P's item; false when the
    // replay ends after it
    auto segment = [&](Ticketed& P, Ticketed& Q, int k) -> bool {
        replay_decode_loaded(io, g, o, d, Q);                                  // record k + 1
        if (k + 2 < n_stored) load_record(gi.rec, r, K, k + 2, P.raw);          // P's slot decodes it next
        const bool last = k + 2 >= n_stored;
        const float delta = Q.S.t - P.S.t;
        const float alpha = 1.f - __expf(-0.5f * (P.S.sigma + Q.S.sigma) * delta);
        const float w = T * alpha;
        const float T_after = T * (1.f - alpha);
        const bool active = w > c.w_thresh;
        float c0 = 0.f, c1 = 0.f, c2 = 0.f;
        if (active) {
            // colours of records written without them (foam.cu:443-445)
            if (!P.has_c) eval_color(g, F, b, P.S), P.has_c = true;
            if (!Q.has_c) eval_color(g, F, b, Q.S), Q.has_c = true;
            c0 = 0.5f * (P.S.C0 + Q.S.C0), c1 = 0.5f * (P.S.C1 + Q.S.C1), c2 = 0.5f * (P.S.C2 + Q.S.C2);
            acc0 += w * c0, acc1 += w * c1, acc2 += w * c2;
        }
        float g_opacity = gR0 * (T_after * c0 - (fg0 - acc0)) + gR1 * (T_after * c1 - (fg1 - acc1)) +
                          gR2 * (T_after * c2 - (fg2 - acc2));
        g_opacity = delta * (g_opacity - tail_grad);
        const float h0 = active ? 0.5f * w * gR0 : 0.f, h1 = active ? 0.5f * w * gR1 : 0.f,
                    h2 = active ? 0.5f * w * gR2 : 0.f;
        replay_put(io, P, carry_sigma + 0.5f * g_opacity, gP0 + h0, gP1 + h1, gP2 + h2, P.has_c, d);
        carry_sigma = 0.5f * g_opacity;
        gP0 = h0, gP1 = h1, gP2 = h2;
        T = T_after;
        return !(last || T < c.t_thresh);
    };
    Ticketed X0, X1;
    replay_decode(gi, io, g, r, K, 0, o, d, X0);
    if (n_stored > 1) load_record(gi.rec, r, K, 1, X1.raw);
    int k = 0;          // segments done; the current P is record k
    bool p_is_1 = false;  // whether the current P is X1
    for (;;) {
        if (k + 1 >= n_stored || k >= kMaxCells) break;
        const bool go = segment(X0, X1, k);
        ++k, p_is_1 = true;
        if (!go || k + 1 >= n_stored || k >= kMaxCells) break;
        const bool go2 = segment(X1, X0, k);
        ++k, p_is_1 = false;
        if (!go2) break;
    }
    if (p_is_1)
        replay_put(io, X1, carry_sigma, gP0, gP1, gP2, X1.has_c, d);
    else
        replay_put(io, X0, carry_sigma, gP0, gP1, gP2, X0.has_c, d);
    // every recorded sample was counted into its bucket: fill the places of any the replay did not reach
    // with zero-gradient items (the replay follows the forward, so normally there are none)
    for (int s2 = k + 1; s2 < n_stored; ++s2) {
        Ticketed Z;
        replay_decode(gi, io, g, r, K, s2, o, d, Z);
        replay_put(io, Z, 0.f, 0.f, 0.f, 0.f, false, d);
    }
}

// ----------------------------------------------------------------------------- cell-major scatter
//
// The gradient of a sample goes to the ~20 sites of its cell's neighbourhood. Thread-per-ray scatter
// issues one set of atomics per (sample, site); but the rays of a view cross each visited cell many
// times (~70 samples per cell at 1080p), so the samples are bucketed by cell (counting sort over the
// cells) and a warp processes up to 32 samples of one cell with ONE LANE PER NEIGHBOUR SITE: the lane
// keeps its site's field record and SH coefficients in registers, loops over the samples (staged in
// shared memory, read as broadcasts), accumulates the site's gradient in registers and issues one set
// of 16-byte atomics per (chunk, site).

// Buckets given by per-cell counts that may come from the caller (vg_foam_backward_counted): their
// offsets must be non-decreasing and end within the item buffer, else the pass is dropped (*bad = 1,
// kErrBuckets) before anything is written or chunked.
__global__ void __launch_bounds__(kBlock)
    bucket_check_kernel(const int* __restrict__ offsets, int n_cells, int64_t cap, int* bad, int* status) {
    const int i = blockIdx.x * kBlock + threadIdx.x;
    if (i > n_cells) return;
    const int a = __ldg(offsets + i);
    const bool ok = i == n_cells ? a >= 0 && a <= cap : a >= 0 && __ldg(offsets + i + 1) >= a;
    if (!ok) *bad = 1, atomicOr(status, kErrBuckets);
}

// Chunks of at most kChunk samples of one cell: (cell, first position in order, count). Nothing when
// bucket_check_kernel rejected the buckets (bad may be null).
__global__ void __launch_bounds__(kBlock)
    cm_chunks_kernel(const int* __restrict__ offsets, int n_cells, int4* __restrict__ chunks, int* n_chunks,
                     const int* bad) {
    if (bad != nullptr && *bad) return;
    const int i = blockIdx.x * kBlock + threadIdx.x;
    const int lane = threadIdx.x & 31;
    int cnt = 0, a = 0;
    if (i < n_cells) a = __ldg(offsets + i), cnt = __ldg(offsets + i + 1) - a;
    const int nch = (cnt + kChunk - 1) / kChunk;
    int incl = nch;  // warp inclusive scan of the chunk counts, one atomic per warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    int base = 0;
    if (lane == 31 && incl > 0) base = atomicAdd(n_chunks, incl);
    base = __shfl_sync(0xffffffffu, base, 31);
    const int first = base + incl - nch;
    for (int c = 0; c < nch; ++c) chunks[first + c] = make_int4(i, a + kChunk * c, min(kChunk, cnt - kChunk * c), 0);
}

// Shared-memory image of one staged sample: x, gs | gC, gC.C | m_min, 1/sum a, -, - | SH basis (16).
constexpr int kItemVec = 7;

// 16-byte asynchronous copy global -> shared (sm_80+ cp.async, L2 only), its group commit and wait.
__device__ __forceinline__ void cp_async16(float4* smem, const float4* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Gradient sums of one neighbour site over a range of a chunk's samples.
template <int S4>
struct PairAcc {
    float ad[8];        // g_raw, g_dA[6], -
    float ac[6];        // g_cA[6]
    float ash[4 * S4];  // g_sh
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int u = 0; u < 8; ++u) ad[u] = 0.f;
#pragma unroll
        for (int u = 0; u < 6; ++u) ac[u] = 0.f;
#pragma unroll
        for (int u = 0; u < 4 * S4; ++u) ash[u] = 0.f;
    }
    // adds the sums held by lane `src` (every lane of the warp takes part; lanes with take == false
    // discard what they receive)
    __device__ __forceinline__ void pull(int src, bool take) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float v = __shfl_sync(0xffffffffu, ad[u], src);
            if (take) ad[u] += v;
        }
#pragma unroll
        for (int u = 0; u < 6; ++u) {
            const float v = __shfl_sync(0xffffffffu, ac[u], src);
            if (take) ac[u] += v;
        }
#pragma unroll
        for (int u = 0; u < 4 * S4; ++u) {
            const float v = __shfl_sync(0xffffffffu, ash[u], src);
            if (take) ash[u] += v;
        }
    }
    __device__ __forceinline__ void flush(float* __restrict__ grad, int j) const {
        float* G = grad + kGradStride * static_cast<int64_t>(j);
        const float4 d0 = make_float4(ad[0], ad[1], ad[2], ad[3]), d1 = make_float4(ad[4], ad[5], ad[6], 0.f);
        const float4 c0 = make_float4(ac[0], ac[1], ac[2], ac[3]), c1 = make_float4(ac[4], ac[5], 0.f, 0.f);
        if (nonzero(d0)) red4(G, d0);
        if (nonzero(d1)) red4(G + 4, d1);
        if (nonzero(c0)) red4(G + 8, c0);
        if (nonzero(c1)) red4(G + 12, c1);
#pragma unroll
        for (int qq = 0; qq < S4; ++qq) {
            const float4 v = make_float4(ash[4 * qq], ash[4 * qq + 1], ash[4 * qq + 2], ash[4 * qq + 3]);
            if (nonzero(v)) red4(G + 16 + 4 * qq, v);
        }
    }
};

// Adds to A the gradients of the neighbour site of edge e from the staged samples [s0, s1) of a chunk
// (the per-sample formulas of foam.cu:303-343 with the sample's items); returns the site.
template <int S4>
__device__ __forceinline__ int scatter_range(const GraphView& g, const FieldView& F, int e, const float4* st, int s0,
                                             int s1, PairAcc<S4>& A) {
    const float4 E = __ldg(g.edge + e);
    const int j = site_of(E);
    if (s0 >= s1) return j;
    const float4* fr = F.rec + kFieldVec * static_cast<int64_t>(j);
    const float4 r0_ = __ldg(fr), r1_ = __ldg(fr + 1), r2_ = __ldg(fr + 2), r3_ = __ldg(fr + 3);
    float4 coef[S4];
#pragma unroll
    for (int q = 0; q < S4; ++q) coef[q] = __ldg(F.sh + static_cast<int64_t>(S4) * j + q);
#pragma unroll kScatterUnroll
    for (int i = s0; i < s1; ++i) {
        const float4* q = st + kItemVec * i;
        const float4 q0 = q[0];
        const float v0 = q0.x - E.x, v1 = q0.y - E.y, v2 = q0.z - E.z;
        const float gs = q0.w;
        if (gs != 0.f) {
            const float gc = gs * __expf(r1_.z - 0.5f * maha(r0_, r1_, v0, v1, v2));
            if (fabsf(gc) > 1e-12f) {
                const float gm = -0.5f * gc;
                A.ad[0] += gc, A.ad[1] += gm * v0 * v0, A.ad[2] += 2.f * gm * v0 * v1, A.ad[3] += 2.f * gm * v0 * v2;
                A.ad[4] += gm * v1 * v1, A.ad[5] += 2.f * gm * v1 * v2, A.ad[6] += gm * v2 * v2;
            }
        }
        const float4 q1 = q[1], q2 = q[2];
        if (q2.y > 0.f) {  // the sample has a colour gradient
            const float a = __expf(-0.5f * (maha(r2_, r3_, v0, v1, v2) - q2.x)) * q2.y;
            if (a >= kMinWeight) {
                float b[16];
                const float4 b0 = q[3], b1 = q[4], b2 = q[5], b3 = q[6];
                b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w, b[4] = b1.x, b[5] = b1.y, b[6] = b1.z;
                b[7] = b1.w, b[8] = b2.x, b[9] = b2.y, b[10] = b2.z, b[11] = b2.w, b[12] = b3.x;
                b[13] = b3.y, b[14] = b3.z, b[15] = b3.w;
                // SH colour of the neighbour in two interleaved partial sums per channel (even / odd
                // basis functions): half the length of each dependent FMA chain
                float c[3] = {0.5f, 0.5f, 0.5f}, h[3] = {0.f, 0.f, 0.f};
#pragma unroll
                for (int qq = 0; qq < S4; ++qq) {
                    const float f[4] = {coef[qq].x, coef[qq].y, coef[qq].z, coef[qq].w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int k = 4 * qq + u;
                        if (k < 48) {
                            if ((k / 3) & 1)
                                h[k % 3] += b[k / 3] * f[u];
                            else
                                c[k % 3] += b[k / 3] * f[u];
                        }
                    }
                }
                c[0] += h[0], c[1] += h[1], c[2] += h[2];
                const float dc[3] = {c[0] > 0.f ? a * q1.x : 0.f, c[1] > 0.f ? a * q1.y : 0.f,
                                     c[2] > 0.f ? a * q1.z : 0.f};
#pragma unroll
                for (int k = 0; k < 4 * S4; ++k)
                    if (k < 48) A.ash[k] += b[k / 3] * dc[k % 3];
                const float ga = q1.x * fmaxf(c[0], 0.f) + q1.y * fmaxf(c[1], 0.f) + q1.z * fmaxf(c[2], 0.f);
                const float gm = -0.5f * a * (ga - q1.w);
                A.ac[0] += gm * v0 * v0, A.ac[1] += 2.f * gm * v0 * v1, A.ac[2] += 2.f * gm * v0 * v2;
                A.ac[3] += gm * v1 * v1, A.ac[4] += 2.f * gm * v1 * v2, A.ac[5] += gm * v2 * v2;
            }
        }
    }
    return j;
}


// The (neighbour, sample) pairs of a chunk of a cell with n <= kReplicaMaxN neighbour sites (self
// included) spread over the 32 lanes: R = 32 / n replicas of every neighbour, replica r taking the r-th
// of R slices of the samples. Replicas of a neighbour combine their sums with warp shuffles, then one
// lane per neighbour adds them to the gradient pack. Same sums as one lane per neighbour, in another
// order.
template <int S4>
__device__ __forceinline__ void replicated_scatter(const GraphView& g, const FieldView& F, const float4* st, int e0,
                                                   int n, int cnt, int lane, float* __restrict__ grad) {
    PairAcc<S4> A;
    A.zero();
    const int R = 32 / n;
    const int j = lane % n, r = lane / n;
    int site = 0;
    if (r < R) site = scatter_range<S4>(g, F, e0 + j, st, (r * cnt) / R, ((r + 1) * cnt) / R, A);
    for (int u = 1; u < R; ++u) A.pull(min(lane + u * n, 31), lane < n);
    if (lane < n) A.flush(grad, site);
}

// Where cm_scatter_kernel finds a chunk's samples: 64-byte items stored contiguously per cell (kBucketed,
// the foam backward), or 64-byte items reached through the cell-sorted index array (kIndexed, the march
// backward).
enum StageMode { kBucketed = 0, kIndexed = 1 };

// With kAsync the bucketed stage returns through its copy-ahead loop, so the generic loop below is
// unreachable in that instantiation (and removed); nvcc's note about it is silenced for this kernel only.
#pragma nv_diag_suppress 128
template <int S4, int STAGE>
__global__ void __launch_bounds__(kBlock, VG_SCATTER_MINB)
    cm_scatter_kernel(GraphView g, FieldView F, const float4* __restrict__ items, const int* __restrict__ order,
                      const int4* __restrict__ chunks, const int* __restrict__ n_chunks_ptr, float* __restrict__ grad) {
    constexpr bool kAsync = STAGE == kBucketed;
    __shared__ float4 smem[(kBlock / 32) * kChunk * kItemVec];
    __shared__ float4 raw_smem[kAsync ? (kBlock / 32) * kChunk * 4 : 1];
    const int lane = threadIdx.x & 31;
    float4* st = smem + (threadIdx.x >> 5) * kChunk * kItemVec;
    const int n_chunks = *n_chunks_ptr;
    const int warps = gridDim.x * (kBlock / 32);
    if (kAsync) {
        // items of chunk i+1 are copied while chunk i is scattered: wait for the copy, expand the items
        // (SH basis of the direction) into the staging area, start the next copy, then scatter
        float4* raw = raw_smem + (threadIdx.x >> 5) * kChunk * 4;
        int ch = blockIdx.x * (kBlock / 32) + (threadIdx.x >> 5);
        int4 C = make_int4(0, 0, 0, 0);
        if (ch < n_chunks) {
            C = __ldg(chunks + ch);
            for (int k = lane; k < 4 * C.z; k += 32) cp_async16(raw + k, items + 4 * static_cast<int64_t>(C.y) + k);
            cp_async_commit();
        }
        for (; ch < n_chunks; ch += warps) {
            cp_async_wait_all();
            __syncwarp();
            for (int li = lane; li < C.z; li += 32) {
                const float4 i3 = raw[4 * li + 3];
                float b[16];
                sh_basis(i3.x, i3.y, i3.z, F.sh_deg, b);
                float4* q = st + kItemVec * li;
                q[0] = raw[4 * li], q[1] = raw[4 * li + 1], q[2] = raw[4 * li + 2];
                q[3] = make_float4(b[0], b[1], b[2], b[3]);
                q[4] = make_float4(b[4], b[5], b[6], b[7]);
                q[5] = make_float4(b[8], b[9], b[10], b[11]);
                q[6] = make_float4(b[12], b[13], b[14], b[15]);
            }
            __syncwarp();
            const int4 Cur = C;
            if (ch + warps < n_chunks) {
                C = __ldg(chunks + ch + warps);
                for (int k = lane; k < 4 * C.z; k += 32)
                    cp_async16(raw + k, items + 4 * static_cast<int64_t>(C.y) + k);
                cp_async_commit();
            }
            const int e0 = __ldg(g.off + Cur.x), e1 = __ldg(g.off + Cur.x + 1);
            if (e1 - e0 <= kReplicaMaxN) {
                replicated_scatter<S4>(g, F, st, e0, e1 - e0, Cur.z, lane, grad);
            } else {
                for (int e = e0 + lane; e < e1; e += 32) {
                    PairAcc<S4> A;
                    A.zero();
                    const int j = scatter_range<S4>(g, F, e, st, 0, Cur.z, A);
                    A.flush(grad, j);
                }
            }
            __syncwarp();
        }
        return;
    }
    for (int ch = blockIdx.x * (kBlock / 32) + (threadIdx.x >> 5); ch < n_chunks; ch += warps) {
        const int4 C = __ldg(chunks + ch);
        const int cell = C.x, cnt = C.z;
        for (int li = lane; li < cnt; li += 32) {  // stage the chunk's 64-byte items
            const int64_t at = STAGE == kIndexed ? __ldg(order + C.y + li) : static_cast<int64_t>(C.y) + li;
            const float4* it = items + 4 * at;
            const float4 i3 = __ldg(it + 3);
            float b[16];
            sh_basis(i3.x, i3.y, i3.z, F.sh_deg, b);
            float4* q = st + kItemVec * li;
            q[0] = __ldg(it), q[1] = __ldg(it + 1), q[2] = __ldg(it + 2);
            q[3] = make_float4(b[0], b[1], b[2], b[3]);
            q[4] = make_float4(b[4], b[5], b[6], b[7]);
            q[5] = make_float4(b[8], b[9], b[10], b[11]);
            q[6] = make_float4(b[12], b[13], b[14], b[15]);
        }
        __syncwarp();
        const int e0 = __ldg(g.off + cell), e1 = __ldg(g.off + cell + 1);
        if (e1 - e0 <= kReplicaMaxN) {
            replicated_scatter<S4>(g, F, st, e0, e1 - e0, cnt, lane, grad);
        } else {
            for (int e = e0 + lane; e < e1; e += 32) {  // one neighbour site per lane
                PairAcc<S4> A;
                A.zero();
                const int j = scatter_range<S4>(g, F, e, st, 0, cnt, A);
                A.flush(grad, j);
            }
        }
        __syncwarp();
    }
}

#pragma nv_diag_default 128

// ------------------------------------------------------------ cell-major backward of the march path
//
// The march backward (march.cu) re-marches every ray; instead of scattering each sample's gradients
// per lane, march_items_kernel writes the first kMarchCap samples of a ray as 64-byte items (the direct
// item layout, with the sample's cell in the third vector) at slot (ray, sample) and counts them per
// cell; march_bucket_kernel sorts the slots by cell and cm_scatter_kernel<kIndexed> scatters them.
// Samples beyond kMarchCap are scattered per lane, as before.

__global__ void __launch_bounds__(kBlock)
    march_items_kernel(GraphView g, FieldView F, RayView R, MarchCfg c, GradIn gi, float* __restrict__ grad,
                       float4* __restrict__ items, int* __restrict__ n_items, int* __restrict__ count, int64_t r0,
                       int64_t nr, int cap, int* status) {
    const int64_t rl = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (rl >= nr) return;
    const int64_t r = r0 + rl;
    Schedule M;
    schedule_of(R, c, r, M);
    float b[16];
    sh_basis(M.d[0], M.d[1], M.d[2], F.sh_deg, b);
    const float gR0 = __ldg(gi.g_rgb + 3 * r), gR1 = __ldg(gi.g_rgb + 3 * r + 1), gR2 = __ldg(gi.g_rgb + 3 * r + 2);
    const float fg0 = __ldg(gi.rgb + 3 * r), fg1 = __ldg(gi.rgb + 3 * r + 1), fg2 = __ldg(gi.rgb + 3 * r + 2);
    const float tail_grad = __ldg(gi.g_T + r) * __ldg(gi.T + r);
    int err = 0, cur = __ldg(g.inv + __ldg(R.start + r)), walk_steps = 0, k = 0;
    float T = 1.f, acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    for (; k < M.n_total; ++k) {
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
        const float gC0 = active ? w * gR0 : 0.f, gC1 = active ? w * gR1 : 0.f, gC2 = active ? w * gR2 : 0.f;
        if (k < cap) {
            const bool do_c = active && (gC0 != 0.f || gC1 != 0.f || gC2 != 0.f);
            float4* it = items + 4 * (rl * cap + k);
            it[0] = make_float4(S.x0, S.x1, S.x2, gsig);
            it[1] = make_float4(do_c ? gC0 : 0.f, do_c ? gC1 : 0.f, do_c ? gC2 : 0.f,
                                do_c ? gC0 * S.C0 + gC1 * S.C1 + gC2 * S.C2 : 0.f);
            it[2] = make_float4(S.mmin, do_c ? S.inv_a : 0.f, __int_as_float(cur), 0.f);
            it[3] = make_float4(M.d[0], M.d[1], M.d[2], 0.f);
            atomicAdd(count + cur, 1);
        } else {
            sample_grads(g, F, S, gsig, gC0, gC1, gC2, active, b, grad);
        }
        T = T_after;
        if (T < c.t_thresh) {
            ++k;
            break;
        }
    }
    n_items[rl] = min(k, cap);
    if (err) atomicOr(status, err);
}

// Counting sort of the march items by cell (one thread per item slot).
__global__ void __launch_bounds__(kBlock)
    march_bucket_kernel(const float4* __restrict__ items, const int* __restrict__ n_items, int64_t nr, int cap,
                        const int* __restrict__ offsets, int* __restrict__ fill, int* __restrict__ order) {
    const int64_t slot = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (slot >= nr * cap) return;
    if (static_cast<int>(slot % cap) >= __ldg(n_items + slot / cap)) return;
    const int cell = __float_as_int(__ldg(items + 4 * slot + 2).z);
    order[__ldg(offsets + cell) + atomicAdd(fill + cell, 1)] = static_cast<int>(slot);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

namespace {

constexpr int64_t kCmItems = int64_t(1) << 26;  // samples bucketed at once (2-4 GB of items)
constexpr int kMarchCap = 256;                    // march samples per ray taken cell-major

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct CmLayout {
    size_t items, n_items, order, count, fill, offsets, chunks, counter, temp, temp_bytes, total;
    int64_t rays_per_pass;
};

// Scratch of the cell-major passes over rays [r0, r0 + rays_per_pass): per-sample items (backward
// only), the cell-sorted order, per-cell counts / fill cursors / offsets, the chunk list, a counter and
// the CUB scan storage.
CmLayout cm_layout(int64_t n_sites, int64_t n_rays, int K, bool with_items, bool with_order = true,
                   int item_bytes = 64) {
    CmLayout L{};
    if (K <= 0 || n_rays <= 0) return L;
    L.rays_per_pass = std::max<int64_t>(1, std::min<int64_t>(n_rays, kCmItems / K));
    const int64_t slots = L.rays_per_pass * K;
    size_t at = 0;
    auto take = [&](size_t b) {
        const size_t h = at;
        at += al256(b);
        return h;
    };
    L.items = take(with_items ? static_cast<size_t>(item_bytes) * slots : 0);
    L.n_items = take(with_items ? 4 * L.rays_per_pass : 0);
    L.order = take(with_order ? 4 * slots : 0);
    const int64_t passes = (n_rays + L.rays_per_pass - 1) / L.rays_per_pass;
    L.count = take(4 * (n_sites + 1) * (with_items ? 1 : passes));
    L.fill = take(4 * n_sites);
    L.offsets = take(4 * (n_sites + 1));
    L.chunks = take(16 * (slots / 32 + n_sites + 1));
    L.counter = take(16);
    size_t scan = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan, static_cast<const int*>(nullptr), static_cast<int*>(nullptr),
                                  static_cast<int>(n_sites + 1));
    L.temp_bytes = scan;
    L.temp = take(scan);
    L.total = at;
    return L;
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace

int64_t foam_count_entries(int64_t n_sites, int64_t n_rays, int record_cap) {
    const CmLayout L = cm_layout(n_sites, n_rays, record_cap, false);
    if (L.rays_per_pass <= 0) return 0;
    return (n_rays + L.rays_per_pass - 1) / L.rays_per_pass * (n_sites + 1);
}

size_t foam_backward_workspace(int64_t n_sites, int64_t n_rays, int record_cap) {
    return cm_layout(n_sites, n_rays, record_cap, true, false).total;
}

cudaError_t cm_scatter_bucketed(const GraphView& g, const FieldView& F, const float4* items, const int* offsets,
                                int4* chunks, int* counter, float* grad, cudaStream_t st) {
    const int n = g.n;
    cudaError_t e = cudaMemsetAsync(counter, 0, 16, st);
    if (e != cudaSuccess) return e;
    cm_chunks_kernel<<<blocks(n), kBlock, 0, st>>>(offsets, n, chunks, counter, nullptr);
    const int grid = sm_count() * 3;
    ProfScope ps(kProfScatter, st);
    switch (F.s4) {
        case 1: cm_scatter_kernel<1, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
        case 3: cm_scatter_kernel<3, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
        case 7: cm_scatter_kernel<7, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
        default: cm_scatter_kernel<12, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
    }
    return cudaGetLastError();
}

size_t march_backward_workspace(int64_t n_sites, int64_t n_rays) {
    return cm_layout(n_sites, n_rays, kMarchCap, true, true, 64).total;
}

cudaError_t march_backward_cm(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                              const GradIn& gi, float* grad, int* status, void* cm_ws, cudaStream_t st) {
    const CmLayout L = cm_layout(g.n, R.n, kMarchCap, true, true, 64);
    char* b = static_cast<char*>(cm_ws);
    float4* items = reinterpret_cast<float4*>(b + L.items);
    int* n_items = reinterpret_cast<int*>(b + L.n_items);
    int* order = reinterpret_cast<int*>(b + L.order);
    int* count = reinterpret_cast<int*>(b + L.count);
    int* fill = reinterpret_cast<int*>(b + L.fill);
    int* offsets = reinterpret_cast<int*>(b + L.offsets);
    int4* chunks = reinterpret_cast<int4*>(b + L.chunks);
    int* counter = reinterpret_cast<int*>(b + L.counter);
    const int n = g.n;
    const int grid = sm_count() * 3;
    for (int64_t r0 = 0; r0 < R.n; r0 += L.rays_per_pass) {
        const int64_t nr = std::min<int64_t>(L.rays_per_pass, R.n - r0);
        cudaError_t e = cudaMemsetAsync(count, 0, 4 * static_cast<size_t>(n + 1), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(fill, 0, 4 * static_cast<size_t>(n), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(counter, 0, 16, st);
        if (e != cudaSuccess) return e;
        {
            ProfScope ps(kProfMarchItems, st);
            march_items_kernel<<<blocks(nr), kBlock, 0, st>>>(g, F, R, c, gi, grad, items, n_items, count, r0, nr,
                                                              kMarchCap, status);
        }
        size_t tb = L.temp_bytes;
        e = cub::DeviceScan::ExclusiveSum(b + L.temp, tb, count, offsets, n + 1, st);
        if (e != cudaSuccess) return e;
        march_bucket_kernel<<<blocks(nr * kMarchCap), kBlock, 0, st>>>(items, n_items, nr, kMarchCap, offsets, fill,
                                                                        order);
        cm_chunks_kernel<<<blocks(n), kBlock, 0, st>>>(offsets, n, chunks, counter, nullptr);
        ProfScope ps(kProfScatter, st);
        switch (F.s4) {
            case 1: cm_scatter_kernel<1, kIndexed><<<grid, kBlock, 0, st>>>(g, F, items, order, chunks, counter, grad); break;
            case 3: cm_scatter_kernel<3, kIndexed><<<grid, kBlock, 0, st>>>(g, F, items, order, chunks, counter, grad); break;
            case 7: cm_scatter_kernel<7, kIndexed><<<grid, kBlock, 0, st>>>(g, F, items, order, chunks, counter, grad); break;
            default: cm_scatter_kernel<12, kIndexed><<<grid, kBlock, 0, st>>>(g, F, items, order, chunks, counter, grad); break;
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Records kept per ray when the caller keeps none (record_cap 0): the no-record forward still defers
// colours, with scratch records for passes of kCmItems / kScratchK rays.
constexpr int kScratchK = 256;

size_t foam_forward_workspace(int64_t n_sites, int64_t n_rays, int record_cap) {
    if (n_rays <= 0) return 0;
    if (record_cap > 0) return cm_layout(n_sites, n_rays, record_cap, false).total;
    const CmLayout L = cm_layout(n_sites, n_rays, kScratchK, false);
    return L.total + al256(static_cast<size_t>(L.rays_per_pass) * kScratchK * kRecord * sizeof(float));
}

namespace {

// Traversal with deferred colours over the rays of R (records out.rec of capacity c.record_cap, all
// rays of R recorded), inline colours for the rays with more samples than records, then the
// cell-major colour passes and the composite.
cudaError_t forward_deferred(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                             const Outputs& out, int* status, const CmLayout& L, char* b, cudaStream_t st) {
    const int K = c.record_cap;
    int* count_all = reinterpret_cast<int*>(b + L.count);
    FoamCfg cc = c;
    {
        // the traversal counts the samples that need a colour per (pass, cell) as it marks them
        const int64_t passes = (R.n + L.rays_per_pass - 1) / L.rays_per_pass;
        cudaError_t e = cudaMemsetAsync(count_all, 0, 4 * static_cast<size_t>(g.n + 1) * passes, st);
        if (e == cudaSuccess && cc.all_count != nullptr)
            e = cudaMemsetAsync(cc.all_count, 0, 4 * static_cast<size_t>(g.n + 1) * passes, st);
        if (e != cudaSuccess) return e;
        cc.cm_count = count_all, cc.cm_rays = L.rays_per_pass, cc.cm_stride = g.n + 1;
    }
    {
        ProfScope ps(kProfTraversal, st);
        foam_forward_kernel<true, kDeferred><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, cc, out, status);
    }
    foam_forward_kernel<true, kImmediateOverflow><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, cc, out, status);
    int* order = reinterpret_cast<int*>(b + L.order);
    int* fill = reinterpret_cast<int*>(b + L.fill);
    int* offsets = reinterpret_cast<int*>(b + L.offsets);
    int4* chunks = reinterpret_cast<int4*>(b + L.chunks);
    int* counter = reinterpret_cast<int*>(b + L.counter);
    const int n = g.n;
    const int grid = sm_count() * 8;
    for (int64_t r0 = 0; r0 < R.n; r0 += L.rays_per_pass) {
        const int64_t nr = std::min<int64_t>(L.rays_per_pass, R.n - r0);
        int* count = count_all + (r0 / L.rays_per_pass) * static_cast<int64_t>(n + 1);
        cudaError_t e = cudaMemsetAsync(fill, 0, 4 * static_cast<size_t>(n), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(counter, 0, 16, st);
        if (e != cudaSuccess) return e;
        size_t tb = L.temp_bytes;
        e = cub::DeviceScan::ExclusiveSum(b + L.temp, tb, count, offsets, n + 1, st);
        if (e != cudaSuccess) return e;
        cmf_bucket_kernel<<<blocks(32 * nr), kBlock, 0, st>>>(out.rec, out.stats, g.inv, r0, nr, K, offsets, fill,
                                                               order);
        cm_chunks_kernel<<<blocks(n), kBlock, 0, st>>>(offsets, n, chunks, counter, nullptr);
        ProfScope ps(kProfColor, st);
        switch (F.s4) {
            case 1: cmf_color_kernel<1><<<grid, kBlock, 0, st>>>(g, F, R, out.rec, K, order, chunks, counter, r0); break;
            case 3: cmf_color_kernel<3><<<grid, kBlock, 0, st>>>(g, F, R, out.rec, K, order, chunks, counter, r0); break;
            case 7: cmf_color_kernel<7><<<grid, kBlock, 0, st>>>(g, F, R, out.rec, K, order, chunks, counter, r0); break;
            default: cmf_color_kernel<12><<<grid, kBlock, 0, st>>>(g, F, R, out.rec, K, order, chunks, counter, r0);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    cmf_composite_kernel<<<blocks(R.n), kBlock, 0, st>>>(out.rec, out.stats, R.n, K, c.w_thresh, out.rgb);
    return cudaGetLastError();
}

}  // namespace

cudaError_t foam_forward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                         const Outputs& out, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    const int K = c.record_cap;
    const bool record = K > 0 && out.rec != nullptr;
    const bool room = cm_ws != nullptr && cm_bytes >= foam_forward_workspace(g.n, R.n, K);
    char* b = static_cast<char*>(cm_ws);
    if (record) {
        if (!room) {
            ProfScope ps(kProfTraversal, st);
            foam_forward_kernel<true, kImmediate><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, out, status);
            return cudaGetLastError();
        }
        return forward_deferred(g, F, R, c, out, status, cm_layout(g.n, R.n, K, false), b, st);
    }
    if (!room) {
        ProfScope ps(kProfTraversal, st);
        foam_forward_kernel<false, kImmediate><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, out, status);
        return cudaGetLastError();
    }
    // no records wanted: scratch records for one pass of rays at a time
    const CmLayout L = cm_layout(g.n, R.n, kScratchK, false);
    float* scratch_rec = reinterpret_cast<float*>(b + L.total);
    FoamCfg cs = c;
    cs.record_cap = kScratchK;
    for (int64_t r0 = 0; r0 < R.n; r0 += L.rays_per_pass) {
        const int64_t nr = std::min<int64_t>(L.rays_per_pass, R.n - r0);
        const RayView Rs{R.o + 3 * r0, R.d + 3 * r0, R.start + r0, R.near + r0, nullptr, R.far + r0, nr};
        const Outputs os{out.rgb + 3 * r0, out.T + r0, out.depth + r0, out.stats + 3 * r0, scratch_rec};
        const cudaError_t e = forward_deferred(g, F, Rs, cs, os, status, L, b, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t foam_backward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                          const GradIn& gi, float* grad, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    const int K = gi.record_cap;
    const CmLayout L = cm_layout(g.n, R.n, K, true, false);
    if (gi.rec == nullptr || K <= 0 || cm_ws == nullptr || cm_bytes < L.total ||
        L.total == 0) {
        foam_backward_kernel<kScatterAll><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, gi, grad, status);
        return cudaGetLastError();
    }
    // rays with more samples than records: re-traced and scattered per ray
    foam_backward_kernel<kScatterRetraced><<<blocks(R.n), kBlock, 0, st>>>(g, F, R, c, gi, grad, status);
    char* b = static_cast<char*>(cm_ws);
    float4* items = reinterpret_cast<float4*>(b + L.items);
    int* count = reinterpret_cast<int*>(b + L.count);
    int* fill = reinterpret_cast<int*>(b + L.fill);
    int* offsets = reinterpret_cast<int*>(b + L.offsets);
    int4* chunks = reinterpret_cast<int4*>(b + L.chunks);
    int* counter = reinterpret_cast<int*>(b + L.counter);
    const int n = g.n;
    const int grid = sm_count() * 3;
    for (int64_t r0 = 0; r0 < R.n; r0 += L.rays_per_pass) {
        const int64_t nr = std::min<int64_t>(L.rays_per_pass, R.n - r0);
        // samples per cell of this pass: kept by the forward (c.all_count), else counted from the records
        int* pass_count = c.all_count != nullptr ? c.all_count + (r0 / L.rays_per_pass) * static_cast<int64_t>(n + 1)
                                                 : count;
        cudaError_t e = cudaMemsetAsync(fill, 0, 4 * static_cast<size_t>(n), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(counter, 0, 16, st);
        if (e == cudaSuccess && c.all_count == nullptr) e = cudaMemsetAsync(count, 0, 4 * static_cast<size_t>(n + 1), st);
        if (e != cudaSuccess) return e;
        int* bad = counter + 1;  // zeroed with the chunk counter
        const ItemOut io{items, pass_count, r0, nr, offsets, fill, L.rays_per_pass * K, bad, status};
        size_t tb = L.temp_bytes;
        if (c.all_count == nullptr)
            cmf_count_kernel<<<blocks(32 * nr), kBlock, 0, st>>>(gi.rec, gi.stats, g.inv, r0, nr, K, count);
        e = cub::DeviceScan::ExclusiveSum(b + L.temp, tb, pass_count, offsets, n + 1, st);
        if (e != cudaSuccess) return e;
        bucket_check_kernel<<<blocks(n + 1), kBlock, 0, st>>>(offsets, n, io.cap, bad, status);
        {
            ProfScope ps(kProfReplay, st);
            replay_items_kernel<<<blocks(nr), kBlock, 0, st>>>(g, F, R, c, gi, io);
        }
        cm_chunks_kernel<<<blocks(n), kBlock, 0, st>>>(offsets, n, chunks, counter, bad);
        ProfScope ps(kProfScatter, st);
        switch (F.s4) {
            case 1: cm_scatter_kernel<1, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
            case 3: cm_scatter_kernel<3, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
            case 7: cm_scatter_kernel<7, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
            default: cm_scatter_kernel<12, kBucketed><<<grid, kBlock, 0, st>>>(g, F, items, nullptr, chunks, counter, grad); break;
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace vg
