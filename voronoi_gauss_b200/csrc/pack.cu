// Layout transforms around the traversal kernels (see vg_common.cuh for the formats).
//
//   graph_pack  points (N, 3), CSR offsets (N + 1), adj (M) in original order
//               -> Morton-ordered self-first neighbourhoods of float4 (p_j, internal j)
//               Morton codes: 10 bits per axis of the points' bounding box, the quantisation of
//               render.py:168-176 (morton_order), sorted stably so equal codes keep index order.
//   field_pack  raw (N), dA (N, 6), cA (N, 6), sh (N, 16, 3) -> 64-byte site records + packed SH
//   grad_unpack gradient pack (N, 64) -> g_raw (N), g_dA (N, 6), g_cA (N, 6), g_sh (N, 16, 3)
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 256;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct PackLayout {
    size_t perm, inv, off, edge, bbox, keys_in, keys_out, vals_in, sizes, temp, temp_bytes, total;
};

// Byte offsets of the sections of a graph pack; the CUB scratch comes last, so the views (with_temp =
// false) do not need the CUB size queries.
PackLayout layout(int64_t n, int64_t m, bool with_temp) {
    PackLayout L{};
    size_t at = 0;
    auto take = [&](size_t bytes) {
        const size_t here = at;
        at += align256(bytes);
        return here;
    };
    L.perm = take(4 * n);
    L.inv = take(4 * n);
    L.off = take(4 * (n + 1));
    L.edge = take(16 * (n + m));
    L.bbox = take(32);
    L.keys_in = take(4 * n);
    L.keys_out = take(4 * n);
    L.vals_in = take(4 * n);
    L.sizes = take(4 * (n + 1));
    if (!with_temp) {
        L.total = at;
        return L;
    }
    size_t sort_bytes = 0, scan_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, static_cast<const unsigned*>(nullptr),
                                    static_cast<unsigned*>(nullptr), static_cast<const int*>(nullptr),
                                    static_cast<int*>(nullptr), static_cast<int>(n), 0, 30);
    cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<const int*>(nullptr), static_cast<int*>(nullptr),
                                  static_cast<int>(n + 1));
    L.temp_bytes = sort_bytes > scan_bytes ? sort_bytes : scan_bytes;
    L.temp = take(L.temp_bytes);
    L.total = at;
    return L;
}

__device__ __forceinline__ int ordered(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float unordered(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff); }

__global__ void bbox_init(int* bb) {
    if (threadIdx.x < 3) bb[threadIdx.x] = INT_MAX, bb[3 + threadIdx.x] = INT_MIN;
}

__global__ void __launch_bounds__(kBlock) bbox_kernel(const float* __restrict__ p, int n, int* bb) {
    int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {INT_MIN, INT_MIN, INT_MIN};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const int v = ordered(p[3 * static_cast<int64_t>(i) + a]);
            lo[a] = min(lo[a], v), hi[a] = max(hi[a], v);
        }
    }
#pragma unroll
    for (int a = 0; a < 3; ++a) {
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            lo[a] = min(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], s));
            hi[a] = max(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], s));
        }
    }
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int a = 0; a < 3; ++a) atomicMin(bb + a, lo[a]), atomicMax(bb + 3 + a, hi[a]);
    }
}

__global__ void __launch_bounds__(kBlock)
    morton_kernel(const float* __restrict__ p, int n, const int* __restrict__ bb, unsigned* __restrict__ keys,
                  int* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    unsigned code = 0;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        const float lo = unordered(bb[a]), hi = unordered(bb[3 + a]);
        const float ext = fmaxf(__fsub_rn(hi, lo), 1e-12f);
        const float f = __fmul_rn(__fdiv_rn(__fsub_rn(p[3 * static_cast<int64_t>(i) + a], lo), ext), 1023.f);
        const int q = min(max(static_cast<int>(f), 0), 1023);
#pragma unroll
        for (int b = 0; b < 10; ++b) code |= static_cast<unsigned>((q >> b) & 1) << (3 * b + a);
    }
    keys[i] = code;
    vals[i] = i;
}

__global__ void __launch_bounds__(kBlock)
    inverse_kernel(const int* __restrict__ perm, const int* __restrict__ offsets, int n, int* __restrict__ inv,
                   int* __restrict__ sizes) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > n) return;
    if (i == n) {
        sizes[n] = 0;
        return;
    }
    const int o = perm[i];
    inv[o] = i;
    sizes[i] = offsets[o + 1] - offsets[o] + 1;
}

__global__ void __launch_bounds__(kBlock)
    edge_kernel(const float* __restrict__ p, const int* __restrict__ offsets, const int* __restrict__ adj,
                const int* __restrict__ perm, const int* __restrict__ inv, const int* __restrict__ off, int n,
                float4* __restrict__ edge) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int o = perm[i];
    const int64_t base = off[i];
    const int64_t o3 = 3 * static_cast<int64_t>(o);
    edge[base] = make_float4(p[o3], p[o3 + 1], p[o3 + 2], __int_as_float(i));
    const int a0 = offsets[o], a1 = offsets[o + 1];
    for (int e = a0; e < a1; ++e) {
        const int j = adj[e];
        const int64_t j3 = 3 * static_cast<int64_t>(j);
        edge[base + 1 + (e - a0)] = make_float4(p[j3], p[j3 + 1], p[j3 + 2], __int_as_float(inv[j]));
    }
}

// Zeroes the components of a float4 row v of SH coefficients at or beyond nc.
__device__ __forceinline__ float4 sh_row_masked(float4 x, int v, int nc) {
    if (4 * v + 0 >= nc) x.x = 0.f;
    if (4 * v + 1 >= nc) x.y = 0.f;
    if (4 * v + 2 >= nc) x.z = 0.f;
    if (4 * v + 3 >= nc) x.w = 0.f;
    return x;
}

// Site records and SH rows in internal (Morton) order. The conic part is one thread per site; the SH rows
// (s4 float4 per site, 48 floats per site in the parameter) are copied by the whole warp over its 32 sites
// row after row, so every load and store instruction moves contiguous 16-byte pieces.
__global__ void __launch_bounds__(kBlock)
    field_kernel(const int* __restrict__ perm, int n, const float* __restrict__ raw, const float* __restrict__ dA,
                 const float* __restrict__ cA, const float* __restrict__ sh, int nc, int s4, float4* __restrict__ rec,
                 float4* __restrict__ shp) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31, i0 = i - lane;
    if (i0 >= n) return;  // whole warp
    const int64_t o = i < n ? perm[i] : 0;
    if (i < n) {
        const float2* a = reinterpret_cast<const float2*>(dA + 6 * o);
        const float2* c = reinterpret_cast<const float2*>(cA + 6 * o);
        const float2 a0 = a[0], a1 = a[1], a2 = a[2], c0 = c[0], c1 = c[1], c2 = c[2];
        float4* r = rec + 4 * static_cast<int64_t>(i);
        r[0] = make_float4(a0.x, a0.y, a1.x, a1.y);
        r[1] = make_float4(a2.x, a2.y, fminf(raw[o], 30.f), 0.f);
        r[2] = make_float4(c0.x, c0.y, c1.x, c1.y);
        r[3] = make_float4(c2.x, c2.y, 0.f, 0.f);
    }
    const float4* sh4 = reinterpret_cast<const float4*>(sh);
    const int sites = min(32, n - i0), total = sites * s4;
    for (int f = lane; f < 32 * s4; f += 32) {  // warp-uniform trip count
        const int site = f / s4, v = f - site * s4;
        const int64_t os = __shfl_sync(0xffffffffu, o, site & 31);
        if (f < total) shp[static_cast<int64_t>(s4) * i0 + f] = sh_row_masked(__ldg(sh4 + 12 * os + v), v, nc);
    }
}

__global__ void __launch_bounds__(kBlock)
    unpack_kernel(const int* __restrict__ perm, int n, const float4* __restrict__ grad, int nc,
                  float* __restrict__ g_raw, float* __restrict__ g_dA, float* __restrict__ g_cA,
                  float* __restrict__ g_sh) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31, i0 = i - lane;
    if (i0 >= n) return;  // whole warp
    const int64_t o = i < n ? perm[i] : 0;
    if (i < n) {
        const float4* G = grad + (kGradStride / 4) * static_cast<int64_t>(i);
        const float4 d0 = G[0], d1 = G[1], c0 = G[2], c1 = G[3];
        g_raw[o] = d0.x;
        float2* a = reinterpret_cast<float2*>(g_dA + 6 * o);
        a[0] = make_float2(d0.y, d0.z), a[1] = make_float2(d0.w, d1.x), a[2] = make_float2(d1.y, d1.z);
        float2* c = reinterpret_cast<float2*>(g_cA + 6 * o);
        c[0] = make_float2(c0.x, c0.y), c[1] = make_float2(c0.z, c0.w), c[2] = make_float2(c1.x, c1.y);
    }
    // the 12 SH-gradient rows of the warp's 32 sites, row after row by the whole warp (contiguous 16-byte
    // pieces per instruction on both sides)
    float4* s4 = reinterpret_cast<float4*>(g_sh);
    const int sites = min(32, n - i0), total = sites * 12;
    for (int f = lane; f < 32 * 12; f += 32) {  // warp-uniform trip count
        const int site = f / 12, v = f - site * 12;
        const int64_t os = __shfl_sync(0xffffffffu, o, site & 31);
        if (f < total)
            s4[12 * os + v] = sh_row_masked(grad[(kGradStride / 4) * static_cast<int64_t>(i0 + site) + 4 + v], v, nc);
    }
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

size_t graph_pack_bytes(int64_t n, int64_t m) { return layout(n, m, true).total; }

GraphView graph_view(const void* pack, int64_t n, int64_t m) {
    const PackLayout L = layout(n, m, false);
    const char* b = static_cast<const char*>(pack);
    return {reinterpret_cast<const int*>(b + L.perm), reinterpret_cast<const int*>(b + L.inv),
            reinterpret_cast<const int*>(b + L.off), reinterpret_cast<const float4*>(b + L.edge), static_cast<int>(n)};
}

cudaError_t graph_pack(const float* points, const int* offsets, const int* adj, int64_t n, int64_t m, void* pack,
                       size_t bytes, cudaStream_t st) {
    const PackLayout L = layout(n, m, true);
    if (bytes < L.total) return cudaErrorInvalidValue;
    char* b = static_cast<char*>(pack);
    int* perm = reinterpret_cast<int*>(b + L.perm);
    int* inv = reinterpret_cast<int*>(b + L.inv);
    int* off = reinterpret_cast<int*>(b + L.off);
    float4* edge = reinterpret_cast<float4*>(b + L.edge);
    int* bb = reinterpret_cast<int*>(b + L.bbox);
    unsigned* kin = reinterpret_cast<unsigned*>(b + L.keys_in);
    unsigned* kout = reinterpret_cast<unsigned*>(b + L.keys_out);
    int* vin = reinterpret_cast<int*>(b + L.vals_in);
    int* sizes = reinterpret_cast<int*>(b + L.sizes);
    void* temp = b + L.temp;
    const int N = static_cast<int>(n);
    bbox_init<<<1, 32, 0, st>>>(bb);
    bbox_kernel<<<min(blocks(n), 1184), kBlock, 0, st>>>(points, N, bb);
    morton_kernel<<<blocks(n), kBlock, 0, st>>>(points, N, bb, kin, vin);
    size_t tb = L.temp_bytes;
    cudaError_t err = cub::DeviceRadixSort::SortPairs(temp, tb, kin, kout, vin, perm, N, 0, 30, st);
    if (err != cudaSuccess) return err;
    inverse_kernel<<<blocks(n + 1), kBlock, 0, st>>>(perm, offsets, N, inv, sizes);
    tb = L.temp_bytes;
    err = cub::DeviceScan::ExclusiveSum(temp, tb, sizes, off, N + 1, st);
    if (err != cudaSuccess) return err;
    edge_kernel<<<blocks(n), kBlock, 0, st>>>(points, offsets, adj, perm, inv, off, N, edge);
    return cudaGetLastError();
}

size_t field_bytes(int64_t n, int sh_deg) {
    return align256(16 * kFieldVec * static_cast<size_t>(n)) + align256(16 * sh_vec4(sh_deg) * static_cast<size_t>(n));
}

FieldView field_view(const void* field, int64_t n, int sh_deg) {
    const char* b = static_cast<const char*>(field);
    return {reinterpret_cast<const float4*>(b), reinterpret_cast<const float4*>(b + align256(16 * kFieldVec * n)),
            sh_deg, sh_vec4(sh_deg)};
}

cudaError_t field_pack(const GraphView& g, const float* raw, const float* dA, const float* cA, const float* sh,
                       int sh_deg, void* field, cudaStream_t st) {
    char* b = static_cast<char*>(field);
    float4* rec = reinterpret_cast<float4*>(b);
    float4* shp = reinterpret_cast<float4*>(b + align256(16 * kFieldVec * static_cast<size_t>(g.n)));
    field_kernel<<<blocks(g.n), kBlock, 0, st>>>(g.perm, g.n, raw, dA, cA, sh, 3 * sh_coeffs(sh_deg), sh_vec4(sh_deg),
                                                 rec, shp);
    return cudaGetLastError();
}

cudaError_t grad_unpack(const GraphView& g, const float* grad, int sh_deg, float* g_raw, float* g_dA, float* g_cA,
                        float* g_sh, cudaStream_t st) {
    unpack_kernel<<<blocks(g.n), kBlock, 0, st>>>(g.perm, g.n, reinterpret_cast<const float4*>(grad),
                                                  3 * sh_coeffs(sh_deg), g_raw, g_dA, g_cA, g_sh);
    return cudaGetLastError();
}

}  // namespace vg
