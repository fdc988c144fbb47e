// The inference layout of render.pack_foam (render.py:179-225) and bake_colors (render.py:228-235),
// built on the device instead of by a chain of torch gathers:
//
//   points (N, 4)      (p, 0)
//   offsets (N + 1)    self-first CSR: cell i owns edges [offsets[i], offsets[i + 1]), its own site first
//   nbr (N + M)        site of every edge
//   edge (N + M, 4)    (p_j, bits of half2(r2_j, lam_j)): r2 the squared distance beyond which
//                      rho_j G_j < eps_density (inf when eps_density = 0), lam the smallest eigenvalue of
//                      the colour conic; both rounded to the safe side by 2^-9 before the fp16 rounding
//   attr (N, 20)       (dA[6], min(raw, 30), 0, cA[6], 0, 0, baked rgb[3], 0)
//   sh (N, 16, 3)      fp32 or fp16;  orig (N) = perm when renumbered
//
// Two passes of one thread per site: site records (and each site's half2 cut, by original id), then the
// cells' edge runs. With reorder the sites take the Morton order of the graph pack (the same 10-bit
// quantisation and stable sort as render.morton_order), whose self-first CSR offsets are the renumbered
// offsets of the layout. Every value is computed with the operations, in the order and rounding, of the
// torch code it replaces (correctly rounded expf / division, fp32(floor^2), fp32(log eps)), so the
// layout is bit-identical to pack_foam run on the GPU.
#include <cuda_fp16.h>

#include "gauss.cuh"
#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float max_var(const float* __restrict__ ls, int64_t o, float floor2) {
    float m = -kInf;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float c = fminf(fmaxf(__ldg(ls + 3 * o + k), -20.f), 20.f);
        m = fmaxf(m, __fadd_rn(expf(__fmul_rn(2.f, c)), floor2));
    }
    return m;
}

__global__ void __launch_bounds__(kBlock)
    site_kernel(const int* __restrict__ perm, int n, const float* __restrict__ points, const float* __restrict__ raw,
                const float* __restrict__ d_ls, const float* __restrict__ d_quat, const float* __restrict__ c_ls,
                const float* __restrict__ c_quat, const float* __restrict__ sh, float floor2, float log_eps,
                int with_eps, int sh_half, float4* __restrict__ points4, float* __restrict__ attr,
                void* __restrict__ sh_out, float* __restrict__ sh32, int* __restrict__ orig, float* __restrict__ cut) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = perm != nullptr ? __ldg(perm + i) : i;
    const float rc = fminf(__ldg(raw + o), 30.f);
    float r2 = __int_as_float(0x7f800000);  // +inf
    if (with_eps) {
        const float over = fmaxf(__fsub_rn(rc, log_eps), 0.f);
        r2 = __fmul_rn(__fmul_rn(__fmul_rn(2.f, max_var(d_ls, o, floor2)), over), 1.001953125f);
    }
    float lam = __fdiv_rn(1.f, max_var(c_ls, o, floor2));
    lam = fminf(__fmul_rn(lam, 0.998046875f), 65000.f);
    const __half2 h = __floats2half2_rn(r2, lam);
    cut[o] = *reinterpret_cast<const float*>(&h);
    points4[i] = make_float4(__ldg(points + 3 * o), __ldg(points + 3 * o + 1), __ldg(points + 3 * o + 2), 0.f);
    float A[6], C[6];
    gauss_conic(gauss_axes(d_ls, d_quat, o, floor2), A);
    gauss_conic(gauss_axes(c_ls, c_quat, o, floor2), C);
    float* a = attr + 20 * static_cast<int64_t>(i);
#pragma unroll
    for (int k = 0; k < 6; ++k) a[k] = A[k], a[8 + k] = C[k];
    a[6] = rc, a[7] = 0.f;
#pragma unroll
    for (int k = 14; k < 20; ++k) a[k] = 0.f;
    const float* s = sh + 48 * o;
    for (int k = 0; k < 48; ++k) {
        const float v = __ldg(s + k);
        if (sh_half)
            static_cast<__half*>(sh_out)[48 * static_cast<int64_t>(i) + k] = __float2half_rn(v);
        else
            static_cast<float*>(sh_out)[48 * static_cast<int64_t>(i) + k] = v;
        if (sh32 != nullptr) sh32[48 * static_cast<int64_t>(i) + k] = v;
    }
    if (orig != nullptr) orig[i] = static_cast<int>(o);
}

__global__ void __launch_bounds__(kBlock)
    edge_kernel(const int* __restrict__ perm, const int* __restrict__ inv, const int* __restrict__ new_off, int n,
                const float* __restrict__ points, const int* __restrict__ offsets, const int* __restrict__ adj,
                const float* __restrict__ cut, int* __restrict__ offsets_out, int* __restrict__ nbr,
                float4* __restrict__ edge) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > n) return;
    if (i == n) {
        offsets_out[n] = perm != nullptr ? __ldg(new_off + n) : __ldg(offsets + n) + n;
        return;
    }
    const int o = perm != nullptr ? __ldg(perm + i) : i;
    const int base = perm != nullptr ? __ldg(new_off + i) : __ldg(offsets + i) + i;
    offsets_out[i] = base;
    const int a0 = __ldg(offsets + o), a1 = __ldg(offsets + o + 1);
    for (int j = 0; j <= a1 - a0; ++j) {
        const int64_t src = j == 0 ? o : __ldg(adj + a0 + j - 1);
        nbr[base + j] = perm != nullptr ? __ldg(inv + src) : static_cast<int>(src);
        edge[base + j] = make_float4(__ldg(points + 3 * src), __ldg(points + 3 * src + 1), __ldg(points + 3 * src + 2),
                                     __ldg(cut + src));
    }
}

// max(SH_k(d_k) + 1/2, 0) for the unit direction d_k from the camera centre to site k, into attr[16:19]
// (render.py:228-235).
__global__ void __launch_bounds__(kBlock)
    bake_kernel(const float4* __restrict__ points4, const float* __restrict__ sh32, int sh_deg, int n, float cx,
                float cy, float cz, float* __restrict__ attr) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float4 p = __ldg(points4 + i);
    float dx = p.x - cx, dy = p.y - cy, dz = p.z - cz;
    const float inv = 1.f / fmaxf(sqrtf(dx * dx + dy * dy + dz * dz), 1e-12f);
    dx *= inv, dy *= inv, dz *= inv;
    float b[16];
    sh_basis(dx, dy, dz, sh_deg, b);
    const float* s = sh32 + 48 * static_cast<int64_t>(i);
    float c[3] = {0.f, 0.f, 0.f};
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) c[ch] += b[j] * __ldg(s + 3 * j + ch);
    float* a = attr + 20 * static_cast<int64_t>(i);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) a[16 + ch] = fmaxf(c[ch] + 0.5f, 0.f);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

size_t infer_pack_workspace(int64_t n_sites) { return ((4 * static_cast<size_t>(n_sites)) + 255) & ~size_t(255); }

cudaError_t infer_pack(const GraphView* g, int64_t n, const float* points, const int* offsets, const int* adj,
                       const float* raw, const float* d_ls, const float* d_quat, const float* c_ls,
                       const float* c_quat, const float* sh, float floor2, float log_eps, int with_eps, int sh_half,
                       float* points4, int* offsets_out, int* nbr, float* edge, float* attr, void* sh_out,
                       float* sh32, int* orig, void* ws, cudaStream_t st) {
    const int* perm = g != nullptr ? g->perm : nullptr;
    float* cut = static_cast<float*>(ws);
    site_kernel<<<blocks(n), kBlock, 0, st>>>(perm, static_cast<int>(n), points, raw, d_ls, d_quat, c_ls, c_quat, sh,
                                               floor2, log_eps, with_eps, sh_half, reinterpret_cast<float4*>(points4),
                                               attr, sh_out, sh32, g != nullptr ? orig : nullptr, cut);
    edge_kernel<<<blocks(n + 1), kBlock, 0, st>>>(perm, g != nullptr ? g->inv : nullptr, g != nullptr ? g->off : nullptr,
                                                   static_cast<int>(n), points, offsets, adj, cut, offsets_out, nbr,
                                                   reinterpret_cast<float4*>(edge));
    return cudaGetLastError();
}

cudaError_t bake_colors(const float* points4, const float* sh32, int sh_deg, int64_t n, float cx, float cy, float cz,
                        float* attr, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    bake_kernel<<<blocks(n), kBlock, 0, st>>>(reinterpret_cast<const float4*>(points4), sh32, sh_deg,
                                               static_cast<int>(n), cx, cy, cz, attr);
    return cudaGetLastError();
}

}  // namespace vg
