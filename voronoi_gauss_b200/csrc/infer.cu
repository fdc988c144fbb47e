// Inference rendering on the reference's packed inference layout (foam_infer.cu:1-25, built by
// render.py:pack_foam): one thread per ray; the self-first neighbourhood of a cell is one run of
// float4 edges (p_j, half2(r2_j, lam_j)), per-site records attr (N, 5 x float4) and SH in fp32 or fp16.
//
// One pass over a cell's edges gives the exit face, the density (skipping neighbours beyond sqrt(r2))
// and either the smallest colour Mahalanobis distance (lazy colours, blended in a second pass for the
// segments with weight > w_thresh), an online colour blend (fused) or a blend of baked per-view site
// colours (baked). Site colours max(SH_k(d) + 1/2, 0) are kept in an 8-slot per-ray direct-mapped cache
// in shared memory. STAGE 0 / 1 are the reference's ablations (exit faces only / + density).
// Per-ray stats (B, 5): samples, coloured segments, walk steps, density terms, SH evaluations.
#include <cuda_fp16.h>

#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 128;
constexpr int kCache = 8;
// unroll factor of the per-cell edge loop (loads of later edges issued before earlier arithmetic)
#ifndef VG_INFER_UNROLL
#define VG_INFER_UNROLL 2
#endif
constexpr int kInferUnroll = VG_INFER_UNROLL;
constexpr int kLazy = 0, kBaked = 1, kFused = 2;

struct Net {
    const float4* __restrict__ points;
    const int* __restrict__ offsets;
    const int* __restrict__ nbr;
    const float4* __restrict__ edge;
    const float4* __restrict__ attr;
    const float4* __restrict__ sh;
    const int* __restrict__ orig;
};

__device__ __forceinline__ bool before(const Net& N, int k, int j) {
    return N.orig != nullptr ? __ldg(N.orig + k) < __ldg(N.orig + j) : k < j;
}

__device__ __forceinline__ float2 cutoffs(const float4& e) {
    const float w = e.w;
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

template <bool HALF>
__device__ __forceinline__ void site_color(const Net& N, int k, const float (&b)[16], float (&c)[3]) {
    c[0] = c[1] = c[2] = 0.5f;
    if (HALF) {
        const float4* s = N.sh + 6 * static_cast<int64_t>(k);
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const float4 f = __ldg(s + q);
            const __half2* h = reinterpret_cast<const __half2*>(&f);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float2 p = __half22float2(h[u]);
                const int i0 = 8 * q + 2 * u, i1 = i0 + 1;
                c[i0 % 3] += b[i0 / 3] * p.x;
                c[i1 % 3] += b[i1 / 3] * p.y;
            }
        }
    } else {
        const float4* s = N.sh + 12 * static_cast<int64_t>(k);
#pragma unroll
        for (int q = 0; q < 12; ++q) {
            const float4 f = __ldg(s + q);
            const float v[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) c[(4 * q + u) % 3] += b[(4 * q + u) / 3] * v[u];
        }
    }
    c[0] = fmaxf(c[0], 0.f), c[1] = fmaxf(c[1], 0.f), c[2] = fmaxf(c[2], 0.f);
}

struct Cache {
    float4* col;  // slot s of this thread at col[s * kBlock]
    template <bool HALF>
    __device__ __forceinline__ void get(const Net& N, int k, const float (&b)[16], float (&c)[3], int& n_sh) {
        float4& e = col[(k & (kCache - 1)) * kBlock];
        const float4 v = e;
        if (__float_as_int(v.w) == k) {
            c[0] = v.x, c[1] = v.y, c[2] = v.z;
            return;
        }
        site_color<HALF>(N, k, b, c);
        e = make_float4(c[0], c[1], c[2], __int_as_float(k));
        ++n_sh;
    }
};

__device__ __forceinline__ int walk(const Net& N, int c, float x0, float x1, float x2, int& steps, int& err) {
    for (int it = 0; it < kWalkCap; ++it) {
        const float4 pc = __ldg(N.points + c);
        const float u0 = __fsub_rn(x0, pc.x), u1 = __fsub_rn(x1, pc.y), u2 = __fsub_rn(x2, pc.z);
        float bd = dot3c(u0, u1, u2, u0, u1, u2);
        int bk = c;
        const int e0 = __ldg(N.offsets + c), e1 = __ldg(N.offsets + c + 1);
        for (int e = e0 + 1; e < e1; ++e) {
            const float4 ed = __ldg(N.edge + e);
            const int k = __ldg(N.nbr + e);
            const float v0 = __fsub_rn(x0, ed.x), v1 = __fsub_rn(x1, ed.y), v2 = __fsub_rn(x2, ed.z);
            const float dk = dot3c(v0, v1, v2, v0, v1, v2);
            if (dk < bd || (dk == bd && before(N, k, bk))) bd = dk, bk = k;
        }
        if (bk == c) return c;
        c = bk;
        ++steps;
    }
    err |= kErrWalkCap;
    return c;
}

struct CellOut {
    float sigma, mmin, t_exit;
    int next;
    Blend B;
};

template <int STAGE, int COLOR, bool HALF>
__device__ __forceinline__ void eval_cell(const Net& N, const InferCfg& M, int c, float t, const float (&o)[3],
                                          const float (&d)[3], const float (&b)[16], Cache& cc, bool want_exit,
                                          CellOut& out, int& n_dens, int& n_sh) {
    constexpr bool BLEND = COLOR != kLazy;
    const float4 pc = __ldg(N.points + c);
    const float x0 = along(o[0], t, d[0]), x1 = along(o[1], t, d[1]), x2 = along(o[2], t, d[2]);
    const int e0 = __ldg(N.offsets + c), e1 = __ldg(N.offsets + c + 1);
    out.sigma = 0.f, out.mmin = kInf, out.t_exit = kInf, out.next = INT_MAX;
    blend_init(out.B);
#pragma unroll kInferUnroll
    for (int e = e0; e < e1; ++e) {
        const float4 ed = __ldg(N.edge + e);
        const int k = __ldg(N.nbr + e);
        if (want_exit && e > e0) {
            const float n0 = __fsub_rn(ed.x, pc.x), n1 = __fsub_rn(ed.y, pc.y), n2 = __fsub_rn(ed.z, pc.z);
            const float dn = dot3c(n0, n1, n2, d[0], d[1], d[2]);
            if (dn > 0.f) {
                const float m0 = __fmaf_rn(0.5f, __fadd_rn(ed.x, pc.x), -o[0]);
                const float m1 = __fmaf_rn(0.5f, __fadd_rn(ed.y, pc.y), -o[1]);
                const float m2 = __fmaf_rn(0.5f, __fadd_rn(ed.z, pc.z), -o[2]);
                const float tt = __fdiv_rn(dot3c(m0, m1, m2, n0, n1, n2), dn);
                if (tt < out.t_exit || (tt == out.t_exit && (out.next == INT_MAX || before(N, k, out.next))))
                    out.t_exit = tt, out.next = k;
            }
        }
        if (STAGE >= 1) {
            const float v0 = __fsub_rn(x0, ed.x), v1 = __fsub_rn(x1, ed.y), v2 = __fsub_rn(x2, ed.z);
            const float r2 = dot3c(v0, v1, v2, v0, v1, v2);
            const float2 cut = cutoffs(ed);
            const float4* a = N.attr + 5 * static_cast<int64_t>(k);
            if (r2 <= cut.x) {
                const float4 q0 = __ldg(a), q1 = __ldg(a + 1);
                out.sigma += __expf(q1.z - 0.5f * maha(q0, q1, v0, v1, v2));
                ++n_dens;
            }
            if (STAGE >= 2) {
                const float lb = r2 * cut.y;
                if (BLEND ? lb <= out.B.m + M.color_cut : lb < out.mmin) {
                    const float4 q2 = __ldg(a + 2), q3 = __ldg(a + 3);
                    const float m = maha(q2, q3, v0, v1, v2);
                    if (BLEND) {
                        if (m <= out.B.m + M.color_cut) {
                            float c3[3];
                            if (COLOR == kBaked) {
                                const float4 q4 = __ldg(a + 4);
                                c3[0] = q4.x, c3[1] = q4.y, c3[2] = q4.z;
                            } else {
                                cc.get<HALF>(N, k, b, c3, n_sh);
                            }
                            blend_add(out.B, m, c3[0], c3[1], c3[2]);
                        }
                    } else {
                        out.mmin = fminf(out.mmin, m);
                    }
                }
            }
        }
    }
}

template <bool HALF>
__device__ __forceinline__ void color_lazy(const Net& N, const InferCfg& M, int c, float t, float mmin,
                                           const float (&o)[3], const float (&d)[3], const float (&b)[16], Cache& cc,
                                           float (&C)[3], int& n_sh) {
    const float x0 = along(o[0], t, d[0]), x1 = along(o[1], t, d[1]), x2 = along(o[2], t, d[2]);
    const int e0 = __ldg(N.offsets + c), e1 = __ldg(N.offsets + c + 1);
    const float cut = mmin + M.color_cut;
    float A = 0.f, r = 0.f, g = 0.f, bl = 0.f;
    for (int e = e0; e < e1; ++e) {
        const float4 ed = __ldg(N.edge + e);
        const float v0 = __fsub_rn(x0, ed.x), v1 = __fsub_rn(x1, ed.y), v2 = __fsub_rn(x2, ed.z);
        if (dot3c(v0, v1, v2, v0, v1, v2) * cutoffs(ed).y > cut) continue;
        const int k = __ldg(N.nbr + e);
        const float4* a = N.attr + 5 * static_cast<int64_t>(k);
        const float4 q2 = __ldg(a + 2), q3 = __ldg(a + 3);
        const float m = maha(q2, q3, v0, v1, v2);
        if (m > cut) continue;
        const float w = __expf(-0.5f * (m - mmin));
        float c3[3];
        cc.get<HALF>(N, k, b, c3, n_sh);
        A += w, r += w * c3[0], g += w * c3[1], bl += w * c3[2];
    }
    const float inv = 1.f / A;
    C[0] = r * inv, C[1] = g * inv, C[2] = bl * inv;
}

template <int STAGE, int COLOR, bool HALF>
__global__ void __launch_bounds__(kBlock)
    infer_kernel(Net N, InferCfg M, RayView R, Outputs out, int* status) {
    constexpr bool BLEND = STAGE >= 2 && COLOR != kLazy;
    __shared__ float4 cache_mem[kCache * kBlock];
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (r >= R.n) return;
    Cache cc{cache_mem + threadIdx.x};
#pragma unroll
    for (int i = 0; i < kCache; ++i) cc.col[i * kBlock] = make_float4(0.f, 0.f, 0.f, __int_as_float(-1));
    const float o[3] = {__ldg(R.o + 3 * r), __ldg(R.o + 3 * r + 1), __ldg(R.o + 3 * r + 2)};
    const float d[3] = {__ldg(R.d + 3 * r), __ldg(R.d + 3 * r + 1), __ldg(R.d + 3 * r + 2)};
    const float t_near = __ldg(R.near + r), t_far = __ldg(R.far + r);
    const int max_samples = M.cap != nullptr ? __ldg(M.cap + r) : INT_MAX;
    float b[16];
    sh_basis(d[0], d[1], d[2], STAGE >= 2 && COLOR != kBaked ? M.sh_deg : 0, b);
    int err = 0, walk_steps = 0, n_dens = 0, n_sh = 0;
    int c = walk(N, __ldg(R.start + r), along(o[0], t_near, d[0]), along(o[1], t_near, d[1]),
                 along(o[2], t_near, d[2]), walk_steps, err);
    CellOut P;
    eval_cell<STAGE, COLOR, HALF>(N, M, c, t_near, o, d, b, cc, true, P, n_dens, n_sh);
    float tP = t_near, sP = P.sigma, mP = P.mmin, CP[3] = {0.f, 0.f, 0.f};
    float t_exit = P.t_exit;
    int next = P.next;
    bool hasP = false;
    int cP = c;
    if (BLEND) {
        const float inv = 1.f / P.B.a;
        CP[0] = P.B.r * inv, CP[1] = P.B.g * inv, CP[2] = P.B.b * inv, hasP = true;
    }
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f}, dep = 0.f;
    int n_samples = 1, n_color = 0, it = 0;
    for (; it < kMaxCells; ++it) {
        const bool last = next == INT_MAX || t_exit >= t_far || n_samples + 1 >= max_samples;
        const float tQ = last ? t_far : fmaxf(t_exit, tP);
        const int cQ = last ? c : next;
        CellOut Q;
        eval_cell<STAGE, COLOR, HALF>(N, M, cQ, tQ, o, d, b, cc, !last, Q, n_dens, n_sh);
        ++n_samples;
        const float delta = tQ - tP;
        const float alpha = 1.f - __expf(-0.5f * (sP + Q.sigma) * delta);
        const float w = T * alpha;
        float CQ[3] = {0.f, 0.f, 0.f};
        bool hasQ = false;
        if (BLEND) {
            const float inv = 1.f / Q.B.a;
            CQ[0] = Q.B.r * inv, CQ[1] = Q.B.g * inv, CQ[2] = Q.B.b * inv, hasQ = true;
        }
        if (STAGE >= 2 && w > M.w_thresh) {
            if (!BLEND) {
                if (!hasP) color_lazy<HALF>(N, M, cP, tP, mP, o, d, b, cc, CP, n_sh);
                color_lazy<HALF>(N, M, cQ, tQ, Q.mmin, o, d, b, cc, CQ, n_sh);
                hasQ = true;
            }
#pragma unroll
            for (int a = 0; a < 3; ++a) acc[a] += w * 0.5f * (CP[a] + CQ[a]);
            dep += w * 0.5f * (tP + tQ);
            ++n_color;
        }
        T *= 1.f - alpha;
        tP = tQ, sP = Q.sigma, mP = Q.mmin, hasP = hasQ, cP = cQ, c = cQ;
        t_exit = Q.t_exit, next = Q.next;
#pragma unroll
        for (int a = 0; a < 3; ++a) CP[a] = CQ[a];
        if (last || T < M.t_thresh) break;
    }
    if (it == kMaxCells) err |= kErrCellCap;
#pragma unroll
    for (int a = 0; a < 3; ++a) out.rgb[3 * r + a] = acc[a];
    out.T[r] = T;
    out.depth[r] = dep;
    int* s = out.stats + 5 * r;
    s[0] = n_samples, s[1] = n_color, s[2] = walk_steps, s[3] = n_dens, s[4] = n_sh;
    if (err) atomicOr(status, err);
}

template <int STAGE, int COLOR, bool HALF>
void launch(const Net& N, const InferCfg& M, const RayView& R, const Outputs& out, int* status, cudaStream_t st) {
    infer_kernel<STAGE, COLOR, HALF>
        <<<static_cast<int>((R.n + kBlock - 1) / kBlock), kBlock, 0, st>>>(N, M, R, out, status);
}

}  // namespace

cudaError_t foam_infer(const InferNet& in, const InferCfg& M, const RayView& R, const Outputs& out, int* status,
                       cudaStream_t st) {
    if (R.n == 0) return cudaSuccess;
    const Net N{in.points, in.offsets, in.nbr, in.edge, in.attr, static_cast<const float4*>(in.sh), in.orig};
    const bool half = in.sh_half != 0;
    if (M.stage == 0)
        launch<0, kLazy, false>(N, M, R, out, status, st);
    else if (M.stage == 1)
        launch<1, kLazy, false>(N, M, R, out, status, st);
    else if (M.color_mode == kBaked)
        launch<2, kBaked, false>(N, M, R, out, status, st);
    else if (M.color_mode == kLazy)
        half ? launch<2, kLazy, true>(N, M, R, out, status, st) : launch<2, kLazy, false>(N, M, R, out, status, st);
    else
        half ? launch<2, kFused, true>(N, M, R, out, status, st) : launch<2, kFused, false>(N, M, R, out, status, st);
    return cudaGetLastError();
}

}  // namespace vg
