// Device side of the inference renderer on the packed inference layout of render.pack_foam, shared by
// the per-ray kernel (infer.cu) and the deferred-colour pipeline (infer_cm.cu): the layout accessor, the
// per-cell scan (exit face, density and, by mode, colour), site colours and the greedy walk. Every value
// that decides a sample or a colour is computed here once, so both pipelines produce the same samples,
// weights and colours bit for bit.
#pragma once

#include <cuda_fp16.h>

#include "vg_common.cuh"

namespace vg {
namespace infer {

constexpr int kThreads = 128;
constexpr int kSlots = 8;  // colour cache entries per ray (a power of two)
// unroll factor of the per-cell edge scan (loads of later edges issued before earlier arithmetic)
#ifndef VG_INFER_UNROLL
#define VG_INFER_UNROLL 2
#endif
constexpr int kScanUnroll = VG_INFER_UNROLL;
constexpr int kAttrRows = 5;                               // float4 rows per site in attr
enum ColourMode { kExact = 0, kBakedColour = 1, kFusedColour = 2 };  // the API's color_mode values

// The inference layout as one thread reads it.
struct Layout {
    InferNet net;
    __device__ __forceinline__ int first(int c) const { return __ldg(net.offsets + c); }
    __device__ __forceinline__ int end(int c) const { return __ldg(net.offsets + c + 1); }
    __device__ __forceinline__ float4 record(int e) const { return __ldg(net.edge + e); }
    __device__ __forceinline__ int site(int e) const { return __ldg(net.nbr + e); }
    __device__ __forceinline__ float4 centre(int c) const { return __ldg(net.points + c); }
    __device__ __forceinline__ const float4* rows(int k) const { return net.attr + kAttrRows * static_cast<int64_t>(k); }
    // tie-break order of sites: their ids before any renumbering
    __device__ __forceinline__ int rank(int k) const { return net.orig != nullptr ? __ldg(net.orig + k) : k; }
};

// (r2, lam) of an edge record: beyond squared distance r2 the site's density is negligible, lam bounds the
// eigenvalues of its colour conic from below (so m >= r2 lam).
__device__ __forceinline__ float2 record_bounds(const float4& rec) {
    const float packed = rec.w;
    return __half22float2(*reinterpret_cast<const __half2*>(&packed));
}

__device__ __forceinline__ float dist2(float x0, float x1, float x2, const float4& p) {
    const float v0 = __fsub_rn(x0, p.x), v1 = __fsub_rn(x1, p.y), v2 = __fsub_rn(x2, p.z);
    return dot3c(v0, v1, v2, v0, v1, v2);
}

// float4 rows of one site's SH coefficients in the layout: 6 rows of fp16 or 12 rows of fp32.
template <bool HALF>
constexpr int coef_rows() { return HALF ? 6 : 12; }

// The 48 SH coefficients in (basis function, channel) order from a site's coefficient rows (global or
// shared memory).
template <bool HALF>
__device__ __forceinline__ void unpack_coefficients(const float4 (&rows)[coef_rows<HALF>()], float (&f)[48]) {
    if (HALF) {
#pragma unroll
        for (int q = 0; q < coef_rows<HALF>(); ++q) {
            const float4 v = rows[q];
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float2 pair = __half22float2(h[u]);
                f[8 * q + 2 * u] = pair.x, f[8 * q + 2 * u + 1] = pair.y;
            }
        }
    } else {
#pragma unroll
        for (int q = 0; q < coef_rows<HALF>(); ++q) {
            const float4 v = rows[q];
            f[4 * q] = v.x, f[4 * q + 1] = v.y, f[4 * q + 2] = v.z, f[4 * q + 3] = v.w;
        }
    }
}

// The coefficient rows of site k from the layout's SH array.
template <bool HALF>
__device__ __forceinline__ void load_coefficient_rows(const void* sh, int k, float4 (&rows)[coef_rows<HALF>()]) {
    const float4* row = static_cast<const float4*>(sh) + coef_rows<HALF>() * static_cast<int64_t>(k);
#pragma unroll
    for (int q = 0; q < coef_rows<HALF>(); ++q) rows[q] = __ldg(row + q);
}

// max(SH(d) + 1/2, 0) from the coefficients f and the basis b of the ray direction; each channel sums the
// basis functions in order. Every colour of the inference renderers goes through this one sum.
__device__ __forceinline__ void colour_sum(const float (&f)[48], const float (&b)[16], float (&rgb)[3]) {
    rgb[0] = rgb[1] = rgb[2] = 0.5f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) rgb[ch] += b[j] * f[3 * j + ch];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) rgb[ch] = fmaxf(rgb[ch], 0.f);
}

// max(SH_k(d) + 1/2, 0) of site k.
template <bool HALF>
__device__ __forceinline__ void clamped_colour(const void* sh, int k, const float (&b)[16], float (&rgb)[3]) {
    float4 rows[coef_rows<HALF>()];
    load_coefficient_rows<HALF>(sh, k, rows);
    float f[48];
    unpack_coefficients<HALF>(rows, f);
    colour_sum(f, b, rgb);
}

// Direct-mapped per-ray cache of clamped site colours in shared memory: entry k mod kSlots holds
// (rgb, k); a miss evaluates the SH, replaces the entry and counts one SH evaluation.
template <bool HALF>
struct SlotCache {
    float4* entry0;  // this thread's first entry; entries kThreads apart
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int s = 0; s < kSlots; ++s) entry0[s * kThreads] = make_float4(0.f, 0.f, 0.f, __int_as_float(-1));
    }
    __device__ __forceinline__ void colour(const Layout& L, int k, const float (&b)[16], float (&rgb)[3],
                                           int& n_sh) {
        float4& slot = entry0[(k & (kSlots - 1)) * kThreads];
        const float4 held = slot;
        if (__float_as_int(held.w) == k) {
            rgb[0] = held.x, rgb[1] = held.y, rgb[2] = held.z;
            return;
        }
        clamped_colour<HALF>(L.net.sh, k, b, rgb);
        slot = make_float4(rgb[0], rgb[1], rgb[2], __int_as_float(k));
        ++n_sh;
    }
};

// Greedy walk on the layout to the site nearest to x (steps to the neighbour with the smallest squared
// distance; equal distances go to the smaller rank).
__device__ __forceinline__ int nearest_site(const Layout& L, int c, float x0, float x1, float x2, int& steps,
                                            int& err) {
    for (int it = 0; it < kWalkCap; ++it) {
        float best = dist2(x0, x1, x2, L.centre(c));
        int arg = c;
        const int e1 = L.end(c);
        for (int e = L.first(c) + 1; e < e1; ++e) {
            const int k = L.site(e);
            const float dk = dist2(x0, x1, x2, L.record(e));
            if (dk < best || (dk == best && L.rank(k) < L.rank(arg))) best = dk, arg = k;
        }
        if (arg == c) return c;
        c = arg;
        ++steps;
    }
    err |= kErrWalkCap;
    return c;
}

// What one scan of a cell yields for the sample at o + t d.
struct CellScan {
    float sigma;   // density
    float m_min;   // smallest colour Mahalanobis distance among the neighbours not skipped (exact mode)
    Blend mix;     // blended colour (fused / baked modes)
    float t_exit;  // exit-face distance along the ray, kInf when none was asked for or none lies ahead
    int next;      // the cell behind the exit face, INT_MAX when none
};

// Crossing of the face between cell site pc and neighbour record p along the ray, when the ray moves
// towards the neighbour (d . (p - pc) > 0): the t where o + t d reaches the bisector plane.
__device__ __forceinline__ bool face_crossing(const float4& p, const float4& pc, const float (&o)[3],
                                              const float (&d)[3], float& t) {
    const float n0 = __fsub_rn(p.x, pc.x), n1 = __fsub_rn(p.y, pc.y), n2 = __fsub_rn(p.z, pc.z);
    const float towards = dot3c(n0, n1, n2, d[0], d[1], d[2]);
    if (!(towards > 0.f)) return false;
    const float h0 = __fmaf_rn(0.5f, __fadd_rn(p.x, pc.x), -o[0]);
    const float h1 = __fmaf_rn(0.5f, __fadd_rn(p.y, pc.y), -o[1]);
    const float h2 = __fmaf_rn(0.5f, __fadd_rn(p.z, pc.z), -o[2]);
    t = __fdiv_rn(dot3c(h0, h1, h2, n0, n1, n2), towards);
    return true;
}

template <int STAGE, int MODE, bool HALF>
__device__ __forceinline__ void scan_cell(const Layout& L, const InferCfg& cfg, int c, float t, const float (&o)[3],
                                          const float (&d)[3], const float (&b)[16], SlotCache<HALF>& cache,
                                          bool find_exit, CellScan& S, int& n_dens, int& n_sh) {
    constexpr bool kMix = MODE != kExact;
    const float4 pc = L.centre(c);
    const float x0 = along(o[0], t, d[0]), x1 = along(o[1], t, d[1]), x2 = along(o[2], t, d[2]);
    S.sigma = 0.f, S.m_min = kInf, S.t_exit = kInf, S.next = INT_MAX;
    S.mix.reset();
    const int e0 = L.first(c), e1 = L.end(c);
#pragma unroll kScanUnroll
    for (int e = e0; e < e1; ++e) {
        const float4 rec = L.record(e);
        const int k = L.site(e);
        float tc;
        if (find_exit && e != e0 && face_crossing(rec, pc, o, d, tc) &&
            (tc < S.t_exit || (tc == S.t_exit && (S.next == INT_MAX || L.rank(k) < L.rank(S.next)))))
            S.t_exit = tc, S.next = k;
        if (STAGE < 1) continue;
        const float v0 = __fsub_rn(x0, rec.x), v1 = __fsub_rn(x1, rec.y), v2 = __fsub_rn(x2, rec.z);
        const float r2 = dot3c(v0, v1, v2, v0, v1, v2);
        const float2 bound = record_bounds(rec);
        const float4* row = L.rows(k);
        if (r2 <= bound.x) {
            const float4 conic_a = __ldg(row), conic_b = __ldg(row + 1);  // conic_b.z = min(raw, 30)
            S.sigma += __expf(conic_b.z - 0.5f * maha(conic_a, conic_b, v0, v1, v2));
            ++n_dens;
        }
        if (STAGE < 2) continue;
        const float floor_m = r2 * bound.y;  // no colour distance of this neighbour is below it
        if (kMix ? !(floor_m <= S.mix.m_min + cfg.color_cut) : !(floor_m < S.m_min)) continue;
        const float m = maha(__ldg(row + 2), __ldg(row + 3), v0, v1, v2);
        if (!kMix) {
            S.m_min = fminf(S.m_min, m);
            continue;
        }
        if (!(m <= S.mix.m_min + cfg.color_cut)) continue;
        float rgb[3];
        if (MODE == kBakedColour) {
            const float4 baked = __ldg(row + 4);
            rgb[0] = baked.x, rgb[1] = baked.y, rgb[2] = baked.z;
        } else {
            cache.colour(L, k, b, rgb, n_sh);
        }
        S.mix.add(m, rgb[0], rgb[1], rgb[2]);
    }
}

// One sample along the ray and its colour once known.
struct Sample {
    float t, sigma, m_min;
    float rgb[3];
    bool coloured;
    int cell;
};

// Exact-mode colour of sample s: the blend of the neighbours of its cell within m_min + color_cut.
template <bool HALF>
__device__ __forceinline__ void exact_colour(const Layout& L, const InferCfg& cfg, Sample& s, const float (&o)[3],
                                             const float (&d)[3], const float (&b)[16], SlotCache<HALF>& cache,
                                             int& n_sh) {
    const float x0 = along(o[0], s.t, d[0]), x1 = along(o[1], s.t, d[1]), x2 = along(o[2], s.t, d[2]);
    const float limit = s.m_min + cfg.color_cut;
    float wsum = 0.f, sum[3] = {0.f, 0.f, 0.f};
    const int e1 = L.end(s.cell);
    for (int e = L.first(s.cell); e < e1; ++e) {
        const float4 rec = L.record(e);
        const float v0 = __fsub_rn(x0, rec.x), v1 = __fsub_rn(x1, rec.y), v2 = __fsub_rn(x2, rec.z);
        if (dot3c(v0, v1, v2, v0, v1, v2) * record_bounds(rec).y > limit) continue;
        const int k = L.site(e);
        const float4* row = L.rows(k);
        const float m = maha(__ldg(row + 2), __ldg(row + 3), v0, v1, v2);
        if (m > limit) continue;
        const float a = __expf(-0.5f * (m - s.m_min));
        float rgb[3];
        cache.colour(L, k, b, rgb, n_sh);
        wsum += a, sum[0] += a * rgb[0], sum[1] += a * rgb[1], sum[2] += a * rgb[2];
    }
    const float inv = 1.f / wsum;
    s.rgb[0] = sum[0] * inv, s.rgb[1] = sum[1] * inv, s.rgb[2] = sum[2] * inv;
    s.coloured = true;
}

template <int STAGE, int MODE, bool HALF>
__device__ __forceinline__ void take(Sample& s, const CellScan& S, float t, int cell) {
    s.t = t, s.sigma = S.sigma, s.m_min = S.m_min, s.cell = cell;
    s.coloured = STAGE >= 2 && MODE != kExact;
    if (s.coloured)
        S.mix.mean(s.rgb);
    else
        s.rgb[0] = s.rgb[1] = s.rgb[2] = 0.f;
}

}  // namespace infer
}  // namespace vg
