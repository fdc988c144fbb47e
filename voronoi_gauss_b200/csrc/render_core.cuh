// Per-sample evaluation and gradient scattering shared by the foam (interaction-point) and march
// (fixed-step) kernels. One thread owns one ray; every routine makes one pass over the contiguous
// self-first neighbourhood of a cell (16-byte edge records) and gathers the 64-byte site records of
// the neighbours it needs.
#pragma once

#include "vg_common.cuh"

namespace vg {

// unroll factor of the neighbour loops of eval_sample / eval_density (loads of later neighbours are
// issued before the arithmetic of earlier ones; measured best on B200)
constexpr int kSampleUnroll = 4;

// One sample of a ray: position, the cell whose neighbourhood evaluates it, density and colour.
struct Sample {
    float t, x0, x1, x2;
    int cell;  // internal id
    float sigma;
    float C0, C1, C2, mmin, inv_a;
};

// Density sum_k exp(min(raw_k, 30) - v^T dA_k v / 2) over {cell} U adj(cell) (foam.cu:211-221), with
// COLOR the colour blend of the neighbourhood (foam.cu:224-249, one online pass) and, when want_exit,
// the exit face of the cell along the ray (foam.cu:185-209; next = -1 when unbounded ahead).
template <bool COLOR>
__device__ __forceinline__ void eval_sample(const GraphView& g, const FieldView& F, int cell, float t,
                                            const float (&o)[3], const float (&d)[3], const float (&b)[16],
                                            bool want_exit, Sample& S, float& t_exit, int& next) {
    S.t = t;
    S.x0 = along(o[0], t, d[0]), S.x1 = along(o[1], t, d[1]), S.x2 = along(o[2], t, d[2]);
    S.cell = cell;
    const int e0 = __ldg(g.off + cell), e1 = __ldg(g.off + cell + 1);
    const float4 Pc = __ldg(g.edge + e0);
    float sigma = 0.f;
    Blend B;
    B.reset();
    t_exit = kInf, next = -1;
#pragma unroll kSampleUnroll
    for (int e = e0; e < e1; ++e) {
        const float4 E = e == e0 ? Pc : __ldg(g.edge + e);
        const int j = site_of(E);
        if (want_exit && e > e0) exit_candidate(E, Pc.x, Pc.y, Pc.z, o, d, t_exit, next, g.perm);
        const float v0 = S.x0 - E.x, v1 = S.x1 - E.y, v2 = S.x2 - E.z;
        const float4* r = F.rec + kFieldVec * static_cast<int64_t>(j);
        const float4 r0 = __ldg(r), r1 = __ldg(r + 1);
        sigma += __expf(r1.z - 0.5f * maha(r0, r1, v0, v1, v2));
        if (COLOR) {
            const float4 r2 = __ldg(r + 2), r3 = __ldg(r + 3);
            float c[3];
            site_color(F, j, b, c);
            B.add(maha(r2, r3, v0, v1, v2), c[0], c[1], c[2]);
        }
    }
    S.sigma = sigma;
    if (COLOR) {
        S.mmin = B.m_min;
        S.inv_a = 1.f / B.wsum;
        S.C0 = B.sum[0] * S.inv_a, S.C1 = B.sum[1] * S.inv_a, S.C2 = B.sum[2] * S.inv_a;
    } else {
        S.mmin = 0.f, S.inv_a = 0.f, S.C0 = S.C1 = S.C2 = 0.f;
    }
}

// Density only (march.cu:182-192).
__device__ __forceinline__ float eval_density(const GraphView& g, const FieldView& F, int cell, float x0, float x1,
                                              float x2) {
    const int e0 = __ldg(g.off + cell), e1 = __ldg(g.off + cell + 1);
    float sigma = 0.f;
#pragma unroll kSampleUnroll
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int j = site_of(E);
        const float v0 = x0 - E.x, v1 = x1 - E.y, v2 = x2 - E.z;
        const float4* r = F.rec + kFieldVec * static_cast<int64_t>(j);
        const float4 r0 = __ldg(r), r1 = __ldg(r + 1);
        sigma += __expf(r1.z - 0.5f * maha(r0, r1, v0, v1, v2));
    }
    return sigma;
}

// Colour only (march.cu:195-219): fills S.C*, S.mmin, S.inv_a for the sample at S.x in S.cell.
__device__ __forceinline__ void eval_color(const GraphView& g, const FieldView& F, const float (&b)[16], Sample& S) {
    const int e0 = __ldg(g.off + S.cell), e1 = __ldg(g.off + S.cell + 1);
    Blend B;
    B.reset();
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int j = site_of(E);
        const float v0 = S.x0 - E.x, v1 = S.x1 - E.y, v2 = S.x2 - E.z;
        const float4* r = F.rec + kFieldVec * static_cast<int64_t>(j);
        const float4 r2 = __ldg(r + 2), r3 = __ldg(r + 3);
        float c[3];
        site_color(F, j, b, c);
        B.add(maha(r2, r3, v0, v1, v2), c[0], c[1], c[2]);
    }
    S.mmin = B.m_min;
    S.inv_a = 1.f / B.wsum;
    S.C0 = B.sum[0] * S.inv_a, S.C1 = B.sum[1] * S.inv_a, S.C2 = B.sum[2] * S.inv_a;
}

__device__ __forceinline__ void red4(float* p, float a, float b, float c, float d) {
    atomicAdd(reinterpret_cast<float4*>(p), make_float4(a, b, c, d));
}

__device__ __forceinline__ void red4(float* p, const float4& v) { atomicAdd(reinterpret_cast<float4*>(p), v); }

// Gradients of one sample into the gradient pack: gs = dL/dsigma, gC = dL/dC, has_c whether the
// sample's colour exists (foam.cu:303-343). Four floats per atomic (16-byte vector reductions).
__device__ __forceinline__ void sample_grads(const GraphView& g, const FieldView& F, const Sample& P, float gs,
                                             float gC0, float gC1, float gC2, bool has_c, const float (&b)[16],
                                             float* __restrict__ grad) {
    const bool do_c = has_c && (gC0 != 0.f || gC1 != 0.f || gC2 != 0.f);
    if (gs == 0.f && !do_c) return;
    const float gCC = gC0 * P.C0 + gC1 * P.C1 + gC2 * P.C2;
    const int e0 = __ldg(g.off + P.cell), e1 = __ldg(g.off + P.cell + 1);
    for (int e = e0; e < e1; ++e) {
        const float4 E = __ldg(g.edge + e);
        const int j = site_of(E);
        const float v0 = P.x0 - E.x, v1 = P.x1 - E.y, v2 = P.x2 - E.z;
        const float4* r = F.rec + kFieldVec * static_cast<int64_t>(j);
        float* G = grad + kGradStride * static_cast<int64_t>(j);
        if (gs != 0.f) {
            const float4 r0 = __ldg(r), r1 = __ldg(r + 1);
            const float gc = gs * __expf(r1.z - 0.5f * maha(r0, r1, v0, v1, v2));
            if (fabsf(gc) > 1e-12f) {
                const float gm = -0.5f * gc;
                red4(G, gc, gm * v0 * v0, 2.f * gm * v0 * v1, 2.f * gm * v0 * v2);
                red4(G + 4, gm * v1 * v1, 2.f * gm * v1 * v2, gm * v2 * v2, 0.f);
            }
        }
        if (do_c) {
            const float4 r2 = __ldg(r + 2), r3 = __ldg(r + 3);
            const float a = __expf(-0.5f * (maha(r2, r3, v0, v1, v2) - P.mmin)) * P.inv_a;
            if (a < kMinWeight) continue;
            float c[3];
            site_color(F, j, b, c);  // max(SH + 1/2, 0): positive exactly where the unclamped value is
            const float dc[3] = {c[0] > 0.f ? a * gC0 : 0.f, c[1] > 0.f ? a * gC1 : 0.f, c[2] > 0.f ? a * gC2 : 0.f};
            if (dc[0] != 0.f || dc[1] != 0.f || dc[2] != 0.f) {
#pragma unroll
                for (int q = 0; q < 12; ++q) {
                    if (q >= F.s4) break;
                    float f[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = 4 * q + u;
                        f[u] = i < 48 ? b[i / 3] * dc[i % 3] : 0.f;
                    }
                    red4(G + 16 + 4 * q, f[0], f[1], f[2], f[3]);
                }
            }
            const float ga = gC0 * c[0] + gC1 * c[1] + gC2 * c[2];
            const float gm = -0.5f * a * (ga - gCC);
            if (gm != 0.f) {
                red4(G + 8, gm * v0 * v0, 2.f * gm * v0 * v1, 2.f * gm * v0 * v2, gm * v1 * v1);
                red4(G + 12, 2.f * gm * v1 * v2, gm * v2 * v2, 0.f, 0.f);
            }
        }
    }
}

__device__ __forceinline__ bool nonzero(const float4& v) { return v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f; }

// ---------------------------------------------------------------------------------- fixed steps

// A ray of the fixed-step march: n_in midpoint steps of dt in [near, mid], then n_bg steps uniform in
// disparity over [mid, far] (march.cu:134-153).
struct Schedule {
    float o[3], d[3];
    float near, mid, far;
    int n_in, n_total;
};

__device__ __forceinline__ void schedule_of(const RayView& R, const MarchCfg& c, int64_t r, Schedule& M) {
#pragma unroll
    for (int a = 0; a < 3; ++a) M.o[a] = __ldg(R.o + 3 * r + a), M.d[a] = __ldg(R.d + 3 * r + a);
    M.near = __ldg(R.near + r), M.mid = __ldg(R.mid + r), M.far = __ldg(R.far + r);
    M.n_in = M.mid > M.near ? static_cast<int>(ceilf(__fdiv_rn(__fsub_rn(M.mid, M.near), c.dt))) : 0;
    M.n_total = M.n_in + c.n_bg;
}

__device__ __forceinline__ void schedule_step(const Schedule& M, const MarchCfg& c, int k, float& t, float& delta) {
    if (k < M.n_in) {
        const float t0 = __fmaf_rn(static_cast<float>(k), c.dt, M.near), t1 = fminf(__fadd_rn(t0, c.dt), M.mid);
        t = __fmul_rn(0.5f, __fadd_rn(t0, t1)), delta = __fsub_rn(t1, t0);
    } else {
        const float i0 = __fdiv_rn(1.f, M.mid), i1 = __fdiv_rn(1.f, M.far), di = __fsub_rn(i1, i0);
        const float nb = static_cast<float>(c.n_bg);
        const float u0 = __fdiv_rn(static_cast<float>(k - M.n_in), nb);
        const float u1 = __fdiv_rn(static_cast<float>(k - M.n_in + 1), nb);
        t = __fdiv_rn(1.f, __fmaf_rn(__fmul_rn(0.5f, __fadd_rn(u0, u1)), di, i0));
        delta = __fsub_rn(__fdiv_rn(1.f, __fmaf_rn(u1, di, i0)), __fdiv_rn(1.f, __fmaf_rn(u0, di, i0)));
    }
}

}  // namespace vg
