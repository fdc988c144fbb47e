/*
 * TEST INFRASTRUCTURE ONLY — not part of the product.
 *
 * CPU restatement (fp32, one thread per block of rays) of the reference's hot path, used as the
 * checker by tests/, by __graft_entry__.smoke() and as bench.py's CPU baseline. The product
 * (voronoi_gauss_b200, libvgb200.so) never links, loads or calls this library.
 *
 * Every function follows the reference kernel it names, operation by operation:
 *   vgo_foam_forward / vgo_foam_backward   csrc/foam.cu:163-469 (walk, exit faces, density, colour,
 *                                          trapezoid compositing, records, forward-order replay)
 *   vgo_march_forward / vgo_march_backward csrc/march.cu:134-345
 *   vgo_conic_forward / vgo_conic_backward csrc/vgf.cu:339-421
 *   vgo_foam_infer                         csrc/foam_infer.cu:50-361 (self-first packed layout)
 *   vgo_walk, vgo_density_*, vgo_color_*   csrc/vgf.cu:51-335 (NeRF-sampler field kernels)
 * All arrays are host memory in the reference layouts (float32 / int32, row-major).
 * Gradient outputs are accumulated (+=): the caller zero-fills them.
 */
#ifndef VG_ORACLE_H
#define VG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int vgo_foam_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                     const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                     const float* o, const float* d, const int32_t* start, const float* near,
                     const float* far, int64_t n_rays, float t_thresh, float w_thresh, int record_cap,
                     float* rgb, float* T, float* depth, int32_t* stats, float* rec, int n_threads);

int vgo_foam_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                      const float* o, const float* d, const int32_t* start, const float* near,
                      const float* far, int64_t n_rays, float t_thresh, float w_thresh, const float* rgb,
                      const float* T, const float* g_rgb, const float* g_T, const float* rec, int record_cap,
                      const int32_t* stats, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                      int n_threads);

int vgo_march_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                      const float* o, const float* d, const int32_t* start, const float* near,
                      const float* mid, const float* far, int64_t n_rays, float dt, int n_bg,
                      float t_thresh, float w_thresh, float* rgb, float* T, float* depth, int32_t* stats,
                      int n_threads);

int vgo_march_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                       const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                       const float* o, const float* d, const int32_t* start, const float* near,
                       const float* mid, const float* far, int64_t n_rays, float dt, int n_bg,
                       float t_thresh, float w_thresh, const float* rgb, const float* T,
                       const float* g_rgb, const float* g_T, float* g_raw, float* g_dA, float* g_cA,
                       float* g_sh, int n_threads);

void vgo_conic_forward(const float* log_scale, const float* quat, int64_t n, float floor, float* A);
void vgo_conic_backward(const float* log_scale, const float* quat, int64_t n, float floor, const float* gA,
                        float* g_ls, float* g_quat);

/* NeRF-sampler field kernels (vgf.cu:51-335), single-threaded; gradients accumulated (+=).
 * vgo_walk: site (B, S), steps (B). vgo_density_*: sigma (M) / g_raw (N), g_ls (N, 3), g_quat (N, 4).
 * vgo_color_*: rgb (M, 3) / g_ls, g_quat, g_sh (N, 16, 3). */
int vgo_walk(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites, const float* o,
             const float* d, const float* z, const int32_t* start, int64_t n_rays, int n_samples, int32_t* site,
             int32_t* steps);
int vgo_density_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                        const float* raw, const float* ls, const float* quat, const float* x, const int32_t* site,
                        int64_t m, double scale_mult, float* sigma);
int vgo_density_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                         const float* raw, const float* ls, const float* quat, const float* x, const int32_t* site,
                         int64_t m, const float* grad_sigma, float* g_raw, float* g_ls, float* g_quat);
int vgo_color_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* ls, const float* quat, const float* sh, int sh_deg, const float* x,
                      const float* dirs, const int32_t* site, int64_t m, float* rgb);
int vgo_color_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                       const float* ls, const float* quat, const float* sh, int sh_deg, const float* x,
                       const float* dirs, const int32_t* site, int64_t m, const float* rgb, const float* grad_rgb,
                       float* g_ls, float* g_quat, float* g_sh);

/* sh: float32 (N, 16, 3) when sh_half == 0, else IEEE binary16 bits (N, 16, 3); sh may be NULL for
 * baked colours. orig and cap may be NULL (n_orig / n_cap == 0). */
int vgo_foam_infer(const float* points4, const int32_t* offsets, const int32_t* nbr, const float* edge,
                   const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites,
                   const float* o, const float* d, const int32_t* start, const float* near, const float* far,
                   int64_t n_rays, float t_thresh, float w_thresh, float color_cut, int color_mode, int stage,
                   const int32_t* cap, const int32_t* orig, float* rgb, float* T, float* depth,
                   int32_t* stats, int n_threads);

#ifdef __cplusplus
}
#endif

#endif
