// Shared device code of the B200 Voronoi-Gaussian renderer (sm_100a).
//
// Data layout in HBM (built by pack.cu, read by foam.cu / march.cu):
//
//   graph pack (once per scene graph; sites renumbered along a 30-bit Morton curve)
//     perm  (N)      internal id -> original id (ties are broken on original ids, as the reference)
//     inv   (N)      original id -> internal id
//     off   (N + 1)  self-first CSR offsets, internal order
//     edge  (N + M)  float4 (p_j.x, p_j.y, p_j.z, bits(internal j)); the first edge of a cell is the
//                    cell's own site, so one pass over 16-byte records gives the site, its Delaunay
//                    neighbours and their positions (exit faces, walks and neighbourhood sums)
//   field pack (per call, internal order)
//     rec   (N, 4) float4: (dA xx, xy, xz, yy), (dA yz, zz, min(raw, 30), 0),
//                          (cA xx, xy, xz, yy), (cA yz, zz, 0, 0)          64 B per site
//     sh    (N, S4) float4: the 3 (sh_deg + 1)^2 used SH coefficients, channel-interleaved as in the
//                           reference (coefficient j, channel c at 3 j + c), zero-padded to float4
//   gradient pack (backward, internal order; summed with vector atomics and, across GPUs, NCCL)
//     grad  (N, 64) float: g_raw, g_dA[6], 0 | g_cA[6], 0, 0 | g_sh[48]   256 B per site
//
// Arithmetic that decides which cells a ray visits (walk distances, exit-face parameters, sample
// positions) uses explicit round-to-nearest intrinsics in the order nvcc contracts the reference's
// source (a0 b0 + a1 b1 + a2 b2 -> fma(a2, b2, fma(a0, b0, a1 b1)), o + t d -> fma(t, d, o)), so the
// cell sequences do not depend on this compiler's contraction choices.
#pragma once

#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

namespace vg {

constexpr float kInf = 3.402823466e38f;  // largest finite float: "no exit face yet" (foam.cu:27)
constexpr int kWalkCap = 4096;           // greedy walk steps per query (foam.cu:29)
constexpr int kMaxCells = 8192;          // cells per ray (foam.cu:30)
constexpr float kMinWeight = 1e-7f;      // normalised colour weights below get no gradient (foam.cu:31)
constexpr int kRecord = 8;               // floats per recorded sample (foam.cu:274)
constexpr int kGradStride = 64;          // floats per site in the gradient pack
constexpr int kFieldVec = 4;             // float4 per site in the field pack

// error bits written to the status word of a launch
constexpr int kErrWalkCap = 1;   // a greedy walk hit kWalkCap
constexpr int kErrCellCap = 2;   // a ray hit kMaxCells
constexpr int kErrBadSite = 4;   // a start or sample site outside [0, N): that ray or sample is skipped
constexpr int kErrBuckets = 8;   // per-cell sample counts that do not fit the records: the cell-major items
                                 // that fall outside their cell's bucket (or all of a pass's, when the
                                 // counts' buckets overflow the item buffer) are dropped

inline __host__ __device__ int sh_coeffs(int deg) { return (deg + 1) * (deg + 1); }
inline __host__ __device__ int sh_vec4(int deg) { return (3 * sh_coeffs(deg) + 3) / 4; }

struct GraphView {
    const int* perm;
    const int* inv;
    const int* off;
    const float4* edge;
    int n;
};

struct FieldView {
    const float4* rec;  // (N, 4)
    const float4* sh;   // (N, S4)
    int sh_deg;
    int s4;
};

// ------------------------------------------------------------------------------------- arithmetic

__device__ __forceinline__ float dot3c(float a0, float a1, float a2, float b0, float b1, float b2) {
    return __fmaf_rn(a2, b2, __fmaf_rn(a0, b0, __fmul_rn(a1, b1)));
}

__device__ __forceinline__ float along(float o, float t, float d) { return __fmaf_rn(t, d, o); }

// v^T A v of a conic stored (xx, xy, xz, yy) | (yz, zz, ., .) (foam.cu:101-105).
__device__ __forceinline__ float maha(const float4& a, const float4& b, float v0, float v1, float v2) {
    return a.x * v0 * v0 + a.w * v1 * v1 + b.y * v2 * v2 + 2.f * (a.y * v0 * v1 + a.z * v0 * v2 + b.x * v1 * v2);
}

// Real SH basis up to degree 3 (foam.cu:118-141): the normalisation constants of each band, with the
// reference's signs, times the Cartesian polynomials of the standard real basis; functions above `deg`
// are zero.
namespace shc {
constexpr float k0 = 0.28209479177387814f;                                                   // l = 0
constexpr float k1 = 0.4886025119029199f;                                                    // l = 1
constexpr float k2xy = 1.0925484305920792f, k2z = 0.31539156525252005f, k2d = 0.5462742152960396f;  // l = 2
constexpr float k3a = 0.5900435899266435f, k3b = 2.890611442640554f, k3c = 0.4570457994644658f,
                k3z = 0.3731763325901154f, k3d = 1.445305721320277f;                          // l = 3
}  // namespace shc

__device__ __forceinline__ void sh_basis(float x, float y, float z, int deg, float (&b)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = 0.f;
    b[0] = shc::k0;
    if (deg >= 1) b[1] = -shc::k1 * y, b[2] = shc::k1 * z, b[3] = -shc::k1 * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    b[4] = shc::k2xy * x * y, b[5] = -shc::k2xy * y * z, b[6] = shc::k2z * (2.f * zz - xx - yy);
    b[7] = -shc::k2xy * x * z, b[8] = shc::k2d * (xx - yy);
    if (deg < 3) return;
    const float around = 4.f * zz - xx - yy;  // shared by the two m = +-1 functions of band 3
    b[9] = -shc::k3a * y * (3.f * xx - yy), b[10] = shc::k3b * x * y * z, b[11] = -shc::k3c * y * around;
    b[12] = shc::k3z * z * (2.f * zz - 3.f * xx - 3.f * yy), b[13] = -shc::k3c * x * around;
    b[14] = shc::k3d * z * (xx - yy), b[15] = -shc::k3a * x * (xx - 3.f * yy);
}

// SH_k(d) + 1/2 per channel (unclamped) from the packed coefficients of site k.
__device__ __forceinline__ void sh_color(const FieldView& F, int k, const float (&b)[16], float (&c)[3]) {
    c[0] = c[1] = c[2] = 0.5f;
    const float4* s = F.sh + static_cast<int64_t>(F.s4) * k;
#pragma unroll
    for (int q = 0; q < 12; ++q) {
        if (q >= F.s4) break;
        const float4 v = __ldg(s + q);
        const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = 4 * q + u;
            if (i < 48) c[i % 3] += b[i / 3] * f[u];
        }
    }
}

__device__ __forceinline__ int site_of(const float4& e) { return __float_as_int(e.w); }

// (t, k) precedes (bt, bk) with ties broken by the smaller original index.
__device__ __forceinline__ bool better(float t, int k, float bt, int bk, const int* __restrict__ perm) {
    if (t < bt) return true;
    if (t == bt) return bk < 0 || __ldg(perm + k) < __ldg(perm + bk);
    return false;
}

// Greedy walk on the packed graph to the nearest site of x, ties to the smaller original index
// (foam.cu:163-181): each step moves to the neighbour minimising (|x - p|^2, original id).
__device__ __forceinline__ int walk_nearest(const GraphView& g, int cur, float x0, float x1, float x2, int& steps,
                                       int& err) {
    for (int it = 0; it < kWalkCap; ++it) {
        const int e0 = __ldg(g.off + cur), e1 = __ldg(g.off + cur + 1);
        float bd = kInf;
        int bk = -1;
        for (int e = e0; e < e1; ++e) {
            const float4 E = __ldg(g.edge + e);
            const float v0 = __fsub_rn(x0, E.x), v1 = __fsub_rn(x1, E.y), v2 = __fsub_rn(x2, E.z);
            const float dk = dot3c(v0, v1, v2, v0, v1, v2);
            const int k = site_of(E);
            if (better(dk, k, bd, bk, g.perm)) bd = dk, bk = k;
        }
        if (bk == cur || bk < 0) return cur;
        cur = bk;
        ++steps;
    }
    err |= kErrWalkCap;
    return cur;
}

// Exit-face candidate of cell c (site pc) through the face shared with neighbour E (foam.cu:191-205).
__device__ __forceinline__ void exit_candidate(const float4& E, float pc0, float pc1, float pc2, const float (&o)[3],
                                               const float (&d)[3], float& bt, int& bk, const int* __restrict__ perm) {
    const float n0 = __fsub_rn(E.x, pc0), n1 = __fsub_rn(E.y, pc1), n2 = __fsub_rn(E.z, pc2);
    const float dn = dot3c(n0, n1, n2, d[0], d[1], d[2]);
    if (dn > 0.f) {
        const float m0 = __fmaf_rn(0.5f, __fadd_rn(E.x, pc0), -o[0]);
        const float m1 = __fmaf_rn(0.5f, __fadd_rn(E.y, pc1), -o[1]);
        const float m2 = __fmaf_rn(0.5f, __fadd_rn(E.z, pc2), -o[2]);
        const float t = __fdiv_rn(dot3c(m0, m1, m2, n0, n1, n2), dn);
        const int k = site_of(E);
        if (better(t, k, bt, bk, perm)) bt = t, bk = k;
    }
}

// Online normalised blend sum_k a_k c_k / sum_k a_k with a_k = exp(-(m_k - m_min) / 2): the sums are
// kept relative to the smallest m seen so far and rescaled when a smaller one arrives, so one pass gives
// the quantity of the reference's two passes (foam.cu:224-249).
struct Blend {
    float m_min, wsum, sum[3];
    __device__ __forceinline__ void reset() { m_min = kInf, wsum = sum[0] = sum[1] = sum[2] = 0.f; }
    __device__ __forceinline__ void add(float m, float r, float g, float b) {
        if (m < m_min) {
            const float shrink = __expf(-0.5f * (m_min - m));
            wsum *= shrink, sum[0] *= shrink, sum[1] *= shrink, sum[2] *= shrink;
            m_min = m;
        }
        const float a = __expf(-0.5f * (m - m_min));
        wsum += a, sum[0] += a * r, sum[1] += a * g, sum[2] += a * b;
    }
    // the blended colour sum / wsum
    __device__ __forceinline__ void mean(float (&c)[3]) const {
        const float inv = 1.f / wsum;
        c[0] = sum[0] * inv, c[1] = sum[1] * inv, c[2] = sum[2] * inv;
    }
};

// Clamped site colour max(SH_k(d) + 1/2, 0) of site k for the ray direction of basis b.
__device__ __forceinline__ void site_color(const FieldView& F, int k, const float (&b)[16], float (&c)[3]) {
    sh_color(F, k, b, c);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) c[ch] = fmaxf(c[ch], 0.f);
}

// ------------------------------------------------------------------------------ host-side launchers

struct RayView {
    const float* o;
    const float* d;
    const int* start;  // original site ids
    const float* near;
    const float* mid;  // march only
    const float* far;
    int64_t n;
};

struct FoamCfg {
    float t_thresh, w_thresh;
    int record_cap;
    // set by foam_forward for the deferred traversal: per-pass counts of the samples that need a
    // colour, cm_count[(ray / cm_rays) * cm_stride + cell] (null: not counted)
    int* cm_count = nullptr;
    int64_t cm_rays = 1;
    int cm_stride = 0;
    // per-pass counts of every recorded sample of the fully recorded rays, all_count[pass * (N + 1) + cell]
    // (the backward's item buckets): filled by the deferred forward, read by the backward instead of
    // counting the records again (null: not kept)
    int* all_count = nullptr;
};

struct MarchCfg {
    float dt;
    int n_bg;
    float t_thresh, w_thresh;
};

struct Outputs {
    float* rgb;
    float* T;
    float* depth;
    int* stats;
    float* rec;
};

struct GradIn {
    const float* rgb;
    const float* T;
    const float* g_rgb;
    const float* g_T;
    const float* rec;
    const int* stats;
    int record_cap;
};

// capi.cu: records the message returned by vg_last_error on this thread and returns code
int set_error(int code, const char* msg);

// pack.cu
size_t graph_pack_bytes(int64_t n, int64_t m);
cudaError_t graph_pack(const float* points, const int* offsets, const int* adj, int64_t n, int64_t m, void* pack,
                       size_t bytes, cudaStream_t st);
GraphView graph_view(const void* pack, int64_t n, int64_t m);
size_t field_bytes(int64_t n, int sh_deg);
cudaError_t field_pack(const GraphView& g, const float* raw, const float* dA, const float* cA, const float* sh,
                       int sh_deg, void* field, cudaStream_t st);
FieldView field_view(const void* field, int64_t n, int sh_deg);
cudaError_t grad_unpack(const GraphView& g, const float* grad, int sh_deg, float* g_raw, float* g_dA, float* g_cA,
                        float* g_sh, cudaStream_t st);

// foam.cu. The forward takes optional scratch (cm_ws, foam_forward_workspace bytes) for the cell-major
// colour pass of the rays whose samples all fit in the records; without it colours are evaluated inline.
size_t foam_forward_workspace(int64_t n_sites, int64_t n_rays, int record_cap);
cudaError_t foam_forward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                         const Outputs& out, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st);
// Scratch of the cell-major backward (rays fully recorded in records of capacity record_cap).
size_t foam_backward_workspace(int64_t n_sites, int64_t n_rays, int record_cap);
// int32 entries of FoamCfg::all_count for a call of n_rays rays with records of capacity record_cap
int64_t foam_count_entries(int64_t n_sites, int64_t n_rays, int record_cap);
cudaError_t foam_backward(const GraphView& g, const FieldView& F, const RayView& R, const FoamCfg& c,
                          const GradIn& gi, float* grad, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st);

// march.cu
cudaError_t march_forward(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                          const Outputs& out, int* status, cudaStream_t st);
// The backward takes optional scratch (march_backward_workspace bytes) for the cell-major scatter.
cudaError_t march_backward(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                           const GradIn& gi, float* grad, int* status, void* cm_ws, size_t cm_bytes, cudaStream_t st);
// foam.cu: the cell-major gradient scatter of 64-byte items stored contiguously per cell (offsets (N + 1)
// of the cells' item runs; item layout: (x, dL/dsigma) | (dL/dC, dL/dC . C) | (m_min, 1 / sum of colour
// weights or 0, -, -) | (unit direction, -)) into the gradient pack grad (N, 64); chunks holds
// (items / 32 + N + 1) int4, counter 16 bytes.
cudaError_t cm_scatter_bucketed(const GraphView& g, const FieldView& F, const float4* items, const int* offsets,
                                int4* chunks, int* counter, float* grad, cudaStream_t st);
// foam.cu: the cell-major part of the march backward
size_t march_backward_workspace(int64_t n_sites, int64_t n_rays);
cudaError_t march_backward_cm(const GraphView& g, const FieldView& F, const RayView& R, const MarchCfg& c,
                              const GradIn& gi, float* grad, int* status, void* cm_ws, cudaStream_t st);

// conic.cu
// floor2 = floor^2 rounded to float once (the reference passes static_cast<float>(floor * floor))
cudaError_t conic_forward(const float* log_scale, const float* quat, int64_t n, float floor2, float* A,
                          cudaStream_t st);
cudaError_t conic_backward(const float* log_scale, const float* quat, int64_t n, float floor2, const float* gA,
                           float* g_ls, float* g_quat, cudaStream_t st);

// field.cu: the NeRF-sampler field kernels. kind: 0 density forward, 1 density backward, 2 colour
// forward, 3 colour backward. inv_mult2 = 1 / scale_mult^2 (forward only; the backward uses 1).
size_t field_workspace(int64_t n_sites, int sh_deg, int kind);
// scratch of the cell-major backward (kind 1 or 3) of n_samples samples; a backward given at least this
// much takes that path
size_t field_cm_workspace(int64_t n_sites, int sh_deg, int kind, int64_t n_samples);
cudaError_t sampler_walk(const GraphView& g, const float* o, const float* d, const float* z, const int* start,
                         int64_t n_rays, int n_samples, int* site, int* steps, int* status, cudaStream_t st);
cudaError_t density_field(const GraphView& g, const float* raw, const float* ls, const float* quat, const float* x,
                          const int* site, int64_t m, float inv_mult2, bool backward, const float* g_sigma, float* sigma,
                          float* g_raw, float* g_ls, float* g_quat, void* ws, size_t ws_bytes, int* status,
                          cudaStream_t st);
cudaError_t color_field(const GraphView& g, const float* ls, const float* quat, const float* sh, int sh_deg,
                        const float* x, const float* dirs, const int* site, int64_t m, bool backward, const float* rgb_in,
                        const float* g_rgb, float* rgb, float* g_ls, float* g_quat, float* g_sh, void* ws,
                        size_t ws_bytes, int* status, cudaStream_t st);

// infer_pack.cu: the inference layout of render.pack_foam / bake_colors. g (the graph pack) renumbers
// the sites in Morton order when non-null; floor2 = fp32(scale_floor^2), log_eps = fp32(log eps_density).
size_t infer_pack_workspace(int64_t n_sites);
cudaError_t infer_pack(const GraphView* g, int64_t n, const float* points, const int* offsets, const int* adj,
                       const float* raw, const float* d_ls, const float* d_quat, const float* c_ls,
                       const float* c_quat, const float* sh, float floor2, float log_eps, int with_eps, int sh_half,
                       float* points4, int* offsets_out, int* nbr, float* edge, float* attr, void* sh_out,
                       float* sh32, int* orig, void* ws, cudaStream_t st);
cudaError_t bake_colors(const float* points4, const float* sh32, int sh_deg, int64_t n, float cx, float cy, float cz,
                        float* attr, cudaStream_t st);

// rays.cu: camera rays in pixel-tile order (th = 0: row-major) and nearest sites by greedy walks.
// K_inv, c2w: host 3 x 3 row-major; centre: host 3.
cudaError_t camera_rays(const float* K_inv, const float* c2w, const float* centre, int W, int H, int th, int tw,
                        float* o, float* d, cudaStream_t st);
cudaError_t nearest_sites(const GraphView& g, const float* queries, int64_t n_queries, int* out, int* status,
                          cudaStream_t st);

// infer.cu
struct InferNet {
    const float4* points;
    const int* offsets;
    const int* nbr;
    const float4* edge;
    const float4* attr;
    const void* sh;
    const int* orig;
    int sh_half;
};
struct InferCfg {
    float t_thresh, w_thresh, color_cut;
    int sh_deg, color_mode, stage;
    const int* cap;
    // when set, the per-ray kernel renders only the rays r with only_over[r] > over (the rays that the
    // deferred pipeline could not hold)
    const int* only_over = nullptr;
    int over = 0;
};
cudaError_t foam_infer(const InferNet& N, const InferCfg& c, const RayView& R, const Outputs& out, int* status,
                       cudaStream_t st);
// Stage-2 rendering with deferred, cell-major colours (infer_cm.cu) from the layout and its trace records
// (infer_trace_records: 12 floats per edge); workspace of foam_infer_workspace(N, B) bytes. Outputs rgb /
// T / depth and stats columns 0-3 as foam_infer; column 4 counts the SH evaluations of the cell-major pass.
size_t foam_infer_workspace(int64_t n_sites, int64_t n_rays);
cudaError_t infer_trace_records(const InferNet& N, int64_t n_edges, float* recs, cudaStream_t st);
cudaError_t foam_infer_deferred(const InferNet& N, const float* trace_recs, int64_t n_sites, const InferCfg& c,
                                const RayView& R, const Outputs& out, int* status, void* ws, size_t ws_bytes,
                                cudaStream_t st);

}  // namespace vg
