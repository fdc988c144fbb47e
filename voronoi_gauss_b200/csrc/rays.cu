// Scene preparation on the device, the two host steps either side of the renderers in render_image
// (render.py:260-266):
//
//   camera_rays    pinhole rays of a W x H image (colmap.py:129-134): d = c2w K^-1 (px + 0.5, py + 0.5, 1),
//                  normalised, origin the camera centre; written in th x tw pixel-tile order (the
//                  bench_infer.py:37-41 ordering: tiles row-major, pixels row-major inside a tile, partial
//                  tiles at the right and bottom edges kept), so that a warp's 32 rays share cells.
//   nearest_sites  the site nearest to each query point (sites.py:38-39, a k-d tree on the host in the
//                  reference): a greedy walk on the Delaunay graph from the first site of the Morton
//                  order, exact because a site that is not the nearest always has a strictly closer
//                  Delaunay neighbour; distance ties go to the smaller original index.
#include "vg_common.cuh"

namespace vg {
namespace {

constexpr int kBlock = 256;

// Position of pixel (x, y) in the tile order.
__device__ __forceinline__ int64_t tile_rank(int x, int y, int W, int H, int th, int tw) {
    const int ty = y / th, tx = x / tw;
    const int h = min(th, H - ty * th), w = min(tw, W - tx * tw);
    return static_cast<int64_t>(ty) * th * W + static_cast<int64_t>(tx) * tw * h + (y % th) * w + (x % tw);
}

__global__ void __launch_bounds__(kBlock)
    camera_rays_kernel(float k00, float k01, float k02, float k11, float k12, float r00, float r01, float r02,
                       float r10, float r11, float r12, float r20, float r21, float r22, float cx, float cy, float cz,
                       int W, int H, int th, int tw, float* __restrict__ o, float* __restrict__ d) {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (p >= static_cast<int64_t>(W) * H) return;
    const int x = static_cast<int>(p % W), y = static_cast<int>(p / W);
    const float u = x + 0.5f, v = y + 0.5f;
    // K^-1 of a pinhole camera is upper triangular: (k00 u + k01 v + k02, k11 v + k12, 1)
    const float a = k00 * u + k01 * v + k02, b = k11 * v + k12;
    float dx = r00 * a + r01 * b + r02, dy = r10 * a + r11 * b + r12, dz = r20 * a + r21 * b + r22;
    const float inv = 1.f / sqrtf(dx * dx + dy * dy + dz * dz);
    dx *= inv, dy *= inv, dz *= inv;
    const int64_t r = th > 0 ? tile_rank(x, y, W, H, th, tw) : p;
    o[3 * r] = cx, o[3 * r + 1] = cy, o[3 * r + 2] = cz;
    d[3 * r] = dx, d[3 * r + 1] = dy, d[3 * r + 2] = dz;
}

__global__ void __launch_bounds__(kBlock)
    nearest_kernel(GraphView g, const float* __restrict__ q, int64_t nq, int* __restrict__ out, int* status) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (i >= nq) return;
    int steps = 0, err = 0;
    const int c = walk_nearest(g, 0, __ldg(q + 3 * i), __ldg(q + 3 * i + 1), __ldg(q + 3 * i + 2), steps, err);
    out[i] = __ldg(g.perm + c);
    if (err) atomicOr(status, err);
}

inline int blocks(int64_t n) { return static_cast<int>((n + kBlock - 1) / kBlock); }

}  // namespace

cudaError_t camera_rays(const float* K_inv, const float* c2w, const float* centre, int W, int H, int th, int tw,
                        float* o, float* d, cudaStream_t st) {
    const int64_t n = static_cast<int64_t>(W) * H;
    if (n == 0) return cudaSuccess;
    camera_rays_kernel<<<blocks(n), kBlock, 0, st>>>(K_inv[0], K_inv[1], K_inv[2], K_inv[4], K_inv[5], c2w[0], c2w[1],
                                                      c2w[2], c2w[3], c2w[4], c2w[5], c2w[6], c2w[7], c2w[8],
                                                      centre[0], centre[1], centre[2], W, H, th, tw, o, d);
    return cudaGetLastError();
}

cudaError_t nearest_sites(const GraphView& g, const float* queries, int64_t n_queries, int* out, int* status,
                          cudaStream_t st) {
    if (n_queries == 0) return cudaSuccess;
    nearest_kernel<<<blocks(n_queries), kBlock, 0, st>>>(g, queries, n_queries, out, status);
    return cudaGetLastError();
}

}  // namespace vg
