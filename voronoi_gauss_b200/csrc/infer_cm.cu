// Inference rendering with deferred, cell-major colours on the packed inference layout (the stage-2
// work of foam_infer.cu:286-361, behind the interface of foam_infer.cu:376-435).
//
// Measured on the reference's own kernel (config 2, fast configuration), finding the samples (exit faces)
// and their densities is about 30 % of a frame and the colours the other 70 %: every sample blends the
// SH colours of its neighbourhood in the per-ray scan, gathering 96-192 bytes of coefficients per
// neighbour from a thread whose 31 warp-mates want other sites. Here the frame runs in four passes:
//
//   trace      one thread per ray (rays of a 4x8 pixel tile per warp): the samples, their densities and
//              the compositing weights exactly as the per-ray kernel, no colour. The samples that border
//              a segment with weight > w_thresh are kept per ray (position, the weight of the segment that
//              ends at the sample when that segment is coloured) and counted per cell.
//   bucket     the kept samples counting-sorted by cell (scan of the counts, one warp per ray to place).
//   colour     one warp per chunk of up to 64 samples of one cell: the cell's neighbour data (edge record,
//              colour conic, SH rows) is staged in shared memory once and read as broadcasts; each lane
//              blends two samples with the arithmetic of the per-ray scan (same neighbour order, same
//              skips, same colour sum), so the colours are bit-identical to it.
//   composite  one thread per ray: the coloured segments summed in ray order with the per-ray kernel's
//              expression, so the image is bit-identical too.
//
// A ray with more than kKept kept samples is rendered whole by the per-ray kernel afterwards (its kept
// samples are coloured and discarded). Per-ray stats: columns 0-3 (samples, coloured segments, walk
// steps, density terms) as the per-ray kernel; column 4 counts the SH colours the cell-major pass
// evaluated for the ray's samples (no per-ray colour cache here).
#include <cub/device/device_scan.cuh>

#include <algorithm>

#include "infer_core.cuh"
#include "prof.cuh"

namespace vg {
namespace infer {
namespace {

constexpr int kKept = 96;                          // kept samples per ray
constexpr int64_t kPassSlots = int64_t(1) << 26;   // kept-sample slots per pass of rays
constexpr int kChunkSamples = 64;                  // samples of one cell per warp in the colour pass
#ifndef VG_TRACE_MINB
#define VG_TRACE_MINB 8
#endif
constexpr int kTraceMinBlocks = VG_TRACE_MINB;     // resident blocks of the trace per SM (its register budget)

// The trace's per-edge records, built from the layout (once per layout: the caller keeps them): edge e of
// cell c's run as three
// float4 = (p_j, half2(r2_j, lam_j)) | density conic (xx, xy, xz, yy) of site j | (yz, zz, min(raw_j, 30),
// bits(j)), i.e. the edge record followed by the rows attr[j, 0:8] with the site id in the unused slot.
// A cell's neighbourhood is then one contiguous run of 48-byte records, and the density terms need no
// gather through the site ids.
__global__ void __launch_bounds__(kThreads)
    trace_records_kernel(Layout L, int64_t n_edges, float4* __restrict__ recs) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (e >= n_edges) return;
    const int k = L.site(static_cast<int>(e));
    const float4* row = L.rows(k);
    const float4 b = __ldg(row + 1);
    recs[3 * e] = L.record(static_cast<int>(e));
    recs[3 * e + 1] = __ldg(row);
    recs[3 * e + 2] = make_float4(b.x, b.y, b.z, __int_as_float(k));
}

// The exit face and density of the sample at o + t d in cell c from the trace records: the arithmetic,
// neighbour order and skips of scan_cell<1> (infer_core.cuh), so both give the same samples and weights.
__device__ __forceinline__ void trace_scan(const Layout& L, const float4* __restrict__ recs, int c, float t,
                                           const float (&o)[3], const float (&d)[3], bool find_exit, CellScan& S,
                                           int& n_dens) {
    const int e0 = L.first(c), e1 = L.end(c);
    const float4 pc = __ldg(recs + 3 * static_cast<int64_t>(e0));  // the self-first run starts with the site
    const float x0 = along(o[0], t, d[0]), x1 = along(o[1], t, d[1]), x2 = along(o[2], t, d[2]);
    S.sigma = 0.f, S.t_exit = kInf, S.next = INT_MAX;
#pragma unroll kScanUnroll
    for (int e = e0; e < e1; ++e) {
        const float4* q = recs + 3 * static_cast<int64_t>(e);
        const float4 rec = __ldg(q), ca = __ldg(q + 1), cb = __ldg(q + 2);
        const int k = __float_as_int(cb.w);
        float tc;
        if (find_exit && e != e0 && face_crossing(rec, pc, o, d, tc) &&
            (tc < S.t_exit || (tc == S.t_exit && (S.next == INT_MAX || L.rank(k) < L.rank(S.next)))))
            S.t_exit = tc, S.next = k;
        const float v0 = __fsub_rn(x0, rec.x), v1 = __fsub_rn(x1, rec.y), v2 = __fsub_rn(x2, rec.z);
        const float r2 = dot3c(v0, v1, v2, v0, v1, v2);
        if (r2 <= record_bounds(rec).x) {
            S.sigma += __expf(cb.z - 0.5f * maha(ca, cb, v0, v1, v2));
            ++n_dens;
        }
    }
}

struct Kept {
    float4* slot;   // (rays of the pass, kKept): x, weight of the coloured segment ending here (0: none);
                    // the colour pass replaces x by the sample's colour
    int* cell;      // (rays of the pass, kKept) cell of the sample
    int* n_kept;    // (rays of the pass) samples kept (more than kKept: rendered per ray)
    int* count;     // (N + 1) kept samples per cell
    int* fill;      // (N) bucket cursors
    int* offsets;   // (N + 1) first bucket position per cell
    int* order;     // slots sorted by cell
    int4* chunks;   // (cell, first position in order, count)
    int* counter;   // number of chunks
};

__global__ void __launch_bounds__(kThreads, kTraceMinBlocks)
    trace_kernel(Layout L, const float4* __restrict__ recs, InferCfg cfg, RayView R, Outputs out, Kept K, int64_t nr,
                 int* status) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (r >= nr) return;
    float o[3], d[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) o[a] = __ldg(R.o + 3 * r + a), d[a] = __ldg(R.d + 3 * r + a);
    const float t_near = __ldg(R.near + r), t_far = __ldg(R.far + r);
    const int max_samples = cfg.cap != nullptr ? __ldg(cfg.cap + r) : INT_MAX;
    int err = 0, walk_steps = 0, n_dens = 0, n_samples = 1, n_coloured = 0, kept = 0;
    float4* slot = K.slot + r * kKept;
    int* slot_cell = K.cell + r * kKept;
    auto keep = [&](float t, int cell, float w_before) {
        if (kept < kKept) {
            slot[kept] = make_float4(along(o[0], t, d[0]), along(o[1], t, d[1]), along(o[2], t, d[2]), w_before);
            slot_cell[kept] = cell;
            atomicAdd(K.count + cell, 1);
        }
        ++kept;
    };

    const int first = nearest_site(L, __ldg(R.start + r), along(o[0], t_near, d[0]), along(o[1], t_near, d[1]),
                                   along(o[2], t_near, d[2]), walk_steps, err);
    CellScan S;
    trace_scan(L, recs, first, t_near, o, d, true, S, n_dens);
    float tP = t_near, sigmaP = S.sigma;
    int cP = first;
    bool keptP = false;
    float T = 1.f, depth = 0.f;
    bool done = false;
    for (int cell = 0; cell < kMaxCells && !done; ++cell) {
        const bool last = S.next == INT_MAX || S.t_exit >= t_far || n_samples + 1 >= max_samples;
        const float tQ = last ? t_far : fmaxf(S.t_exit, tP);
        const int cQ = last ? cP : S.next;
        trace_scan(L, recs, cQ, tQ, o, d, !last, S, n_dens);
        ++n_samples;
        const float alpha = 1.f - __expf(-0.5f * (sigmaP + S.sigma) * (tQ - tP));
        const float w = T * alpha;
        bool keptQ = false;
        if (w > cfg.w_thresh) {
            if (!keptP) keep(tP, cP, 0.f);
            keep(tQ, cQ, w);
            keptQ = true;
            depth += w * 0.5f * (tP + tQ);
            ++n_coloured;
        }
        T *= 1.f - alpha;
        tP = tQ, sigmaP = S.sigma, cP = cQ, keptP = keptQ;
        done = last || T < cfg.t_thresh;
    }
    if (!done) err |= kErrCellCap;
    out.T[r] = T;
    out.depth[r] = depth;
    int* s = out.stats + 5 * r;
    s[0] = n_samples, s[1] = n_coloured, s[2] = walk_steps, s[3] = n_dens, s[4] = 0;
    K.n_kept[r] = kept;
    if (err) atomicOr(status, err);
}

// The kept slots of the pass's rays counting-sorted by cell; one warp per ray.
__global__ void __launch_bounds__(kThreads) bucket_kernel(Kept K, int64_t nr) {
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= nr) return;
    const int n = min(__ldg(K.n_kept + r), kKept);
    for (int k = lane; k < n; k += 32) {
        const int64_t sl = r * kKept + k;
        const int c = __ldg(K.cell + sl);
        K.order[__ldg(K.offsets + c) + atomicAdd(K.fill + c, 1)] = static_cast<int>(sl);
    }
}

// Chunks of at most kChunkSamples samples of one cell: (cell, first position in order, count).
__global__ void __launch_bounds__(kThreads) chunks_kernel(const int* __restrict__ offsets, int n_cells,
                                                          int4* __restrict__ chunks, int* n_chunks) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    const int lane = threadIdx.x & 31;
    int cnt = 0, a = 0;
    if (i < n_cells) a = __ldg(offsets + i), cnt = __ldg(offsets + i + 1) - a;
    const int nch = (cnt + kChunkSamples - 1) / kChunkSamples;
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
    for (int c = 0; c < nch; ++c)
        chunks[first + c] = make_int4(i, a + kChunkSamples * c, min(kChunkSamples, cnt - kChunkSamples * c), 0);
}

// What the colour pass stages per neighbour: its edge record, colour conic (two rows) and either its SH
// coefficients (as 12 fp32 rows, fp16 ones converted once while staging) or its baked colour.
template <int MODE>
constexpr int staged_rows() { return 3 + (MODE == kBakedColour ? 1 : 12); }

template <int MODE, bool HALF>
__global__ void __launch_bounds__(kThreads)
    colour_kernel(Layout L, InferCfg cfg, RayView R, Kept K, const int* __restrict__ n_chunks_ptr,
                  int* __restrict__ stats) {
    constexpr int kPer = kChunkSamples / 32;  // samples per lane
    constexpr int kNv = staged_rows<MODE>();
    constexpr int kCoef = coef_rows<HALF>();
    __shared__ float4 smem[(kThreads / 32) * 32 * kNv];
    float4* nbr = smem + (threadIdx.x >> 5) * 32 * kNv;
    const int lane = threadIdx.x & 31;
    const int n_chunks = *n_chunks_ptr;
    const int warps = gridDim.x * (kThreads / 32);
    for (int ch = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); ch < n_chunks; ch += warps) {
        const int4 C = __ldg(K.chunks + ch);
        int64_t sl[kPer];
        float x[kPer][3], b[kPer][16], w_before[kPer], m_min[kPer];
        Blend mix[kPer];
        int n_sh[kPer];
#pragma unroll
        for (int p = 0; p < kPer; ++p) {
            const int li = lane + 32 * p;
            sl[p] = -1;
            x[p][0] = x[p][1] = x[p][2] = 0.f;
            w_before[p] = 0.f, m_min[p] = kInf, n_sh[p] = 0;
            mix[p].reset();
#pragma unroll
            for (int j = 0; j < 16; ++j) b[p][j] = 0.f;
            if (li < C.z) {
                sl[p] = __ldg(K.order + C.y + li);
                const float4 X = K.slot[sl[p]];
                x[p][0] = X.x, x[p][1] = X.y, x[p][2] = X.z, w_before[p] = X.w;
                const int64_t r = sl[p] / kKept;
                if (MODE != kBakedColour)
                    sh_basis(__ldg(R.d + 3 * r), __ldg(R.d + 3 * r + 1), __ldg(R.d + 3 * r + 2), cfg.sh_deg, b[p]);
            }
        }
        const int e0 = L.first(C.x), e1 = L.end(C.x);
        // exact colours take two scans of the neighbours (the smallest distance, then the blend); the fused
        // and baked blends one
        constexpr int kScans = MODE == kExact ? 2 : 1;
#pragma unroll 1
        for (int scan = 0; scan < kScans; ++scan) {
            for (int eb = e0; eb < e1; eb += 32) {
                const int nb = min(32, e1 - eb);
                if (scan == 0 || e1 - e0 > 32) {  // a cell of <= 32 neighbours stays staged for the second scan
                    __syncwarp();
                    if (lane < nb) {
                        const float4 E = L.record(eb + lane);
                        const float4* row = L.rows(L.site(eb + lane));
                        float4* dst = nbr + lane * kNv;
                        dst[0] = E, dst[1] = __ldg(row + 2), dst[2] = __ldg(row + 3);
                        if (MODE == kBakedColour) {
                            dst[3] = __ldg(row + 4);
                        } else {
                            float4 rows[kCoef];
                            load_coefficient_rows<HALF>(L.net.sh, L.site(eb + lane), rows);
                            float f[48];
                            unpack_coefficients<HALF>(rows, f);
#pragma unroll
                            for (int q = 0; q < 12; ++q)
                                dst[3 + q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                        }
                    }
                    __syncwarp();
                }
                for (int k = 0; k < nb; ++k) {  // warp-uniform: one cell per chunk
                    const float4* src = nbr + k * kNv;
                    const float4 E = src[0], ca = src[1], cb = src[2];
                    const float lam = record_bounds(E).y;
                    bool want[kPer];
                    float m[kPer], v[kPer][3];
                    bool any = false;
#pragma unroll
                    for (int p = 0; p < kPer; ++p) {
                        want[p] = false;
                        if (sl[p] < 0) continue;
                        v[p][0] = __fsub_rn(x[p][0], E.x), v[p][1] = __fsub_rn(x[p][1], E.y);
                        v[p][2] = __fsub_rn(x[p][2], E.z);
                        const float floor_m = dot3c(v[p][0], v[p][1], v[p][2], v[p][0], v[p][1], v[p][2]) * lam;
                        if (MODE == kExact && scan == 0) {
                            // the smallest colour distance (skip: bound not below the current minimum)
                            if (!(floor_m < m_min[p])) continue;
                            m_min[p] = fminf(m_min[p], maha(ca, cb, v[p][0], v[p][1], v[p][2]));
                        } else if (MODE == kExact) {
                            const float limit = m_min[p] + cfg.color_cut;
                            if (floor_m > limit) continue;
                            m[p] = maha(ca, cb, v[p][0], v[p][1], v[p][2]);
                            want[p] = !(m[p] > limit);
                        } else {
                            if (!(floor_m <= mix[p].m_min + cfg.color_cut)) continue;
                            m[p] = maha(ca, cb, v[p][0], v[p][1], v[p][2]);
                            want[p] = m[p] <= mix[p].m_min + cfg.color_cut;
                        }
                        any |= want[p];
                    }
                    if (!any) continue;
                    float rgb[3];
                    float f[48];
                    if (MODE == kBakedColour) {
                        const float4 baked = src[3];
                        rgb[0] = baked.x, rgb[1] = baked.y, rgb[2] = baked.z;
                    } else {
#pragma unroll
                        for (int q = 0; q < 12; ++q) {
                            const float4 c4 = src[3 + q];
                            f[4 * q] = c4.x, f[4 * q + 1] = c4.y, f[4 * q + 2] = c4.z, f[4 * q + 3] = c4.w;
                        }
                    }
#pragma unroll
                    for (int p = 0; p < kPer; ++p) {
                        if (!want[p]) continue;
                        if (MODE != kBakedColour) colour_sum(f, b[p], rgb), ++n_sh[p];
                        if (MODE == kExact) {
                            const float a = __expf(-0.5f * (m[p] - m_min[p]));
                            mix[p].wsum += a, mix[p].sum[0] += a * rgb[0], mix[p].sum[1] += a * rgb[1];
                            mix[p].sum[2] += a * rgb[2];
                        } else {
                            mix[p].add(m[p], rgb[0], rgb[1], rgb[2]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int p = 0; p < kPer; ++p) {
            if (sl[p] < 0) continue;
            float c[3];
            mix[p].mean(c);
            K.slot[sl[p]] = make_float4(c[0], c[1], c[2], w_before[p]);
            if (n_sh[p]) atomicAdd(stats + 5 * (sl[p] / kKept) + 4, n_sh[p]);
        }
    }
}

// The coloured segments of every ray held by the pass, in ray order (the per-ray kernel's expression).
__global__ void __launch_bounds__(kThreads) composite_kernel(Kept K, int64_t nr, float* __restrict__ rgb) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (r >= nr) return;
    const int n = __ldg(K.n_kept + r);
    if (n > kKept) return;  // rendered per ray
    const float4* slot = K.slot + r * kKept;
    float fg[3] = {0.f, 0.f, 0.f}, prev[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < n; ++k) {
        const float4 v = slot[k];
        const float cur[3] = {v.x, v.y, v.z};
        const float w = v.w;
        if (w > 0.f) {
#pragma unroll
            for (int a = 0; a < 3; ++a) fg[a] += w * 0.5f * (prev[a] + cur[a]);
        }
        prev[0] = cur[0], prev[1] = cur[1], prev[2] = cur[2];
    }
    rgb[3 * r] = fg[0], rgb[3 * r + 1] = fg[1], rgb[3 * r + 2] = fg[2];
}

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct KeptLayout {
    size_t slot, cell, n_kept, count, fill, offsets, order, chunks, counter, temp, temp_bytes, total;
    int64_t rays_per_pass;
};

KeptLayout kept_layout(int64_t n_sites, int64_t n_rays) {
    KeptLayout L{};
    if (n_rays <= 0) return L;
    L.rays_per_pass = std::max<int64_t>(1, std::min<int64_t>(n_rays, kPassSlots / kKept));
    const int64_t slots = L.rays_per_pass * kKept;
    size_t at = 0;
    auto take = [&](size_t bytes) {
        const size_t h = at;
        at += al256(bytes);
        return h;
    };
    L.slot = take(16 * static_cast<size_t>(slots));
    L.cell = take(4 * static_cast<size_t>(slots));
    L.n_kept = take(4 * static_cast<size_t>(L.rays_per_pass));
    L.count = take(4 * static_cast<size_t>(n_sites + 1));
    L.fill = take(4 * static_cast<size_t>(n_sites));
    L.offsets = take(4 * static_cast<size_t>(n_sites + 1));
    L.order = take(4 * static_cast<size_t>(slots));
    L.chunks = take(16 * static_cast<size_t>(slots / kChunkSamples + n_sites + 1));
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
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int MODE, bool HALF>
void launch_colour(const Layout& L, const InferCfg& cfg, const RayView& R, const Kept& K, int* stats, cudaStream_t st) {
    ProfScope ps(kProfInferColour, st);
    colour_kernel<MODE, HALF><<<sm_count() * 8, kThreads, 0, st>>>(L, cfg, R, K, K.counter, stats);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kThreads - 1) / kThreads); }

}  // namespace
}  // namespace infer

size_t foam_infer_workspace(int64_t n_sites, int64_t n_rays) { return infer::kept_layout(n_sites, n_rays).total; }

cudaError_t infer_trace_records(const InferNet& net, int64_t n_edges, float* recs, cudaStream_t st) {
    using namespace infer;
    if (n_edges == 0) return cudaSuccess;
    trace_records_kernel<<<blocks(n_edges), kThreads, 0, st>>>(Layout{net}, n_edges, reinterpret_cast<float4*>(recs));
    return cudaGetLastError();
}

cudaError_t foam_infer_deferred(const InferNet& net, const float* trace_recs, int64_t n_sites, const InferCfg& cfg,
                                const RayView& R, const Outputs& out, int* status, void* ws, size_t ws_bytes,
                                cudaStream_t st) {
    using namespace infer;
    if (R.n == 0) return cudaSuccess;
    const KeptLayout KL = kept_layout(n_sites, R.n);
    if (cfg.stage < 2 || trace_recs == nullptr || ws == nullptr || ws_bytes < KL.total)
        return foam_infer(net, cfg, R, out, status, st);
    const Layout L{net};
    char* base = static_cast<char*>(ws);
    Kept K{reinterpret_cast<float4*>(base + KL.slot), reinterpret_cast<int*>(base + KL.cell),
           reinterpret_cast<int*>(base + KL.n_kept), reinterpret_cast<int*>(base + KL.count),
           reinterpret_cast<int*>(base + KL.fill), reinterpret_cast<int*>(base + KL.offsets),
           reinterpret_cast<int*>(base + KL.order), reinterpret_cast<int4*>(base + KL.chunks),
           reinterpret_cast<int*>(base + KL.counter)};
    const int n = static_cast<int>(n_sites);
    const bool half = net.sh_half != 0;
    const float4* recs = reinterpret_cast<const float4*>(trace_recs);
    for (int64_t r0 = 0; r0 < R.n; r0 += KL.rays_per_pass) {
        const int64_t nr = std::min<int64_t>(KL.rays_per_pass, R.n - r0);
        const RayView Rp{R.o + 3 * r0, R.d + 3 * r0, R.start + r0, R.near + r0, nullptr, R.far + r0, nr};
        const Outputs op{out.rgb + 3 * r0, out.T + r0, out.depth + r0, out.stats + 5 * r0, nullptr};
        InferCfg cp = cfg;
        if (cfg.cap != nullptr) cp.cap = cfg.cap + r0;
        cudaError_t e = cudaMemsetAsync(K.count, 0, 4 * static_cast<size_t>(n + 1), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(K.fill, 0, 4 * static_cast<size_t>(n), st);
        if (e == cudaSuccess) e = cudaMemsetAsync(K.counter, 0, 16, st);
        if (e != cudaSuccess) return e;
        {
            ProfScope ps(kProfInfer, st);
            trace_kernel<<<blocks(nr), kThreads, 0, st>>>(L, recs, cp, Rp, op, K, nr, status);
        }
        size_t tb = KL.temp_bytes;
        e = cub::DeviceScan::ExclusiveSum(base + KL.temp, tb, K.count, K.offsets, n + 1, st);
        if (e != cudaSuccess) return e;
        bucket_kernel<<<blocks(32 * nr), kThreads, 0, st>>>(K, nr);
        chunks_kernel<<<blocks(n), kThreads, 0, st>>>(K.offsets, n, K.chunks, K.counter);
        if (cfg.color_mode == kBakedColour)
            launch_colour<kBakedColour, false>(L, cp, Rp, K, op.stats, st);
        else if (cfg.color_mode == kExact)
            half ? launch_colour<kExact, true>(L, cp, Rp, K, op.stats, st)
                 : launch_colour<kExact, false>(L, cp, Rp, K, op.stats, st);
        else
            half ? launch_colour<kFusedColour, true>(L, cp, Rp, K, op.stats, st)
                 : launch_colour<kFusedColour, false>(L, cp, Rp, K, op.stats, st);
        composite_kernel<<<blocks(nr), kThreads, 0, st>>>(K, nr, op.rgb);
        // the rays that kept more samples than there are slots: the whole ray per thread
        cp.only_over = K.n_kept, cp.over = kKept;
        e = foam_infer(net, cp, Rp, op, status, st);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

}  // namespace vg
