/*
 * libvgb200 — B200 (sm_100a) renderer of Voronoi-Gaussian radiance fields, C ABI.
 *
 * Drop-in boundary for the CUDA extensions of daovietanh190499/voronoi-gauss. Each entry point below
 * replaces one pybind11 function of the reference (file:line of the reference given beside it): same
 * argument meaning, layouts and output semantics, with torch tensors replaced by raw device pointers
 * and element counts, outputs allocated by the caller, and an integer status instead of a Python
 * exception.
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise; all arrays are C-contiguous, float32 or
 *     int32 exactly as in the reference (foam.cu:34-37 CHECK_INPUT, foam.cu:481-494).
 *   - `stream` is a cudaStream_t (0 = legacy default stream); work is enqueued asynchronously on the
 *     device that is current on the calling thread, nothing synchronises the host.
 *   - `workspace` is caller-allocated device scratch of at least the size returned by the matching
 *     *_workspace_bytes function (256-byte aligned). The library allocates no device memory.
 *   - Return value: VG_OK (0) or an error code; vg_last_error() gives a message (thread-local).
 *     Loop caps (4096 walk steps, 8192 cells per ray, foam.cu:29-30) truncate as in the reference;
 *     vg_status() reports, after the stream has been synchronised, whether a launch hit one.
 *
 * Scene graph. The reference passes (points, offsets, adj) to every call and keeps them fixed
 * (ext.Graph, ext.py:46-58). Here they are packed once by vg_graph_pack into a caller buffer (Morton-
 * ordered self-first neighbourhoods of 16-byte records); every render call takes that pack instead.
 */
#ifndef VGB200_H
#define VGB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    VG_OK = 0,
    VG_ERR_INVALID_ARG = 1,  /* shape / dtype / size / null pointer: the reference's TORCH_CHECK */
    VG_ERR_WORKSPACE = 2,    /* workspace or pack buffer smaller than required */
    VG_ERR_CUDA = 3          /* a CUDA launch or runtime call failed */
};

/* Library version (major * 10000 + minor * 100 + patch). */
int vg_version(void);

/* Message of the last error on this thread ("" if none). */
const char* vg_last_error(void);

/* Bits of the status word accumulated by the render launches since the last vg_status_reset():
 * 1 = a greedy walk hit its 4096-step cap, 2 = a ray hit the 8192-cell cap, 4 = a start or sample site
 * outside [0, N) was skipped, 8 = the per-cell counts given to vg_foam_backward_counted do not belong to
 * its records (samples that found no place in their cell's bucket, or a whole pass whose buckets do not
 * fit the item buffer, were left out of the gradients). Synchronises the device. */
int vg_status(int* bits);
int vg_status_reset(void);

/* ---------------------------------------------------------------------------------- scene graph */

/* Bytes of the packed graph of n_sites sites with n_adj adjacency entries. */
size_t vg_graph_pack_bytes(int64_t n_sites, int64_t n_adj);

/* Packs (points (N, 3) float32, offsets (N + 1) int32, adj (M) int32) — the CSR Delaunay adjacency
 * of ext.Graph (ext.py:46-52) — into `pack`. Replaces the per-call (points, offsets, adj) triple of
 * every function below. */
int vg_graph_pack(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                  int64_t n_adj, void* pack, size_t pack_bytes, void* stream);

/* ------------------------------------------------------------------------- interaction points */

/* Workspace of vg_foam_forward / vg_march_forward (backward = 0), of vg_foam_backward /
 * vg_march_backward (backward = 1), of vg_foam_backward_packed (backward = 2), or of vg_march_backward
 * with its cell-major gradient scatter (backward = 3: more memory, faster), for n_sites sites at SH
 * degree sh_deg, n_rays rays and records of capacity record_cap (0 for march). */
size_t vg_foam_workspace_bytes(int64_t n_sites, int sh_deg, int64_t n_rays, int record_cap, int backward);

/* foam_forward (foam.cu:505-526): rendering at the ray / Voronoi-face interaction points.
 * raw (N), dA (N, 6), cA (N, 6), sh (N, 16, 3); o, d (B, 3); start (B) site near each origin;
 * near, far (B). Outputs rgb (B, 3) foreground colour, T (B) final transmittance, depth (B),
 * stats (B, 3) int32 = (samples, coloured segments, walk steps); with record_cap K > 0 also
 * rec (B, K, 8) = the first K samples of every ray (t, site bits, sigma, C rgb, m_min, 1 / sum of
 * colour weights) for vg_foam_backward; rec may be NULL when K == 0. */
int vg_foam_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                    const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                    const int32_t* start, const float* near, const float* far, int64_t n_rays, float t_thresh,
                    float w_thresh, int record_cap, float* rgb, float* T, float* depth, int32_t* stats,
                    float* rec, void* workspace, size_t workspace_bytes, void* stream);

/* foam_backward (foam.cu:528-558): gradients g_raw (N), g_dA (N, 6), g_cA (N, 6), g_sh (N, 16, 3)
 * (overwritten) of sum(g_rgb * rgb) + sum(g_T * T). Replays the records of rays with
 * stats[r, 0] <= record_cap and re-traces the others (record_cap = 0: re-trace every ray). */
int vg_foam_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                     const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                     const int32_t* start, const float* near, const float* far, int64_t n_rays,
                     float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                     const float* g_T, const float* rec, int record_cap, const int32_t* stats, float* g_raw,
                     float* g_dA, float* g_cA, float* g_sh, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Training variants of vg_foam_forward / vg_foam_backward with no reference counterpart: the forward
 * also writes, into `counts` (vg_foam_counts_bytes, int32, caller-owned until the backward), how many of
 * its recorded samples fall into each cell per pass of the cell-major backward, which the backward then
 * reads instead of counting the records again. Same arguments and results otherwise; the forward needs
 * the full vg_foam_workspace_bytes(..., backward = 0) workspace and record_cap > 0, and the backward
 * must get the records, stats and counts of that forward with the same rays and record_cap. */
size_t vg_foam_counts_bytes(int64_t n_sites, int64_t n_rays, int record_cap);
int vg_foam_forward_counted(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                            const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                            const int32_t* start, const float* near, const float* far, int64_t n_rays,
                            float t_thresh, float w_thresh, int record_cap, float* rgb, float* T, float* depth,
                            int32_t* stats, float* rec, int32_t* counts, void* workspace, size_t workspace_bytes,
                            void* stream);
int vg_foam_backward_counted(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                             const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                             const int32_t* start, const float* near, const float* far, int64_t n_rays,
                             float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                             const float* g_T, const float* rec, int record_cap, const int32_t* stats,
                             const int32_t* counts, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                             void* workspace, size_t workspace_bytes, void* stream);

/* The two halves of vg_foam_backward, for data-parallel training: the gradients of this device's
 * rays are summed into grad_pack (N, 64) float32 (zero-filled first when zero_first != 0; layout
 * g_raw, g_dA[6], 0, g_cA[6], 0, 0, g_sh[48] in packed site order), which can be all-reduced across
 * devices before vg_grad_unpack writes the reference's four gradient arrays. No reference
 * counterpart: the reference is single-GPU. */
int vg_foam_backward_packed(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                            const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                            const int32_t* start, const float* near, const float* far, int64_t n_rays,
                            float t_thresh, float w_thresh, const float* rgb, const float* T,
                            const float* g_rgb, const float* g_T, const float* rec, int record_cap,
                            const int32_t* stats, float* grad_pack, int zero_first, void* workspace,
                            size_t workspace_bytes, void* stream);
int vg_grad_unpack(const void* pack, int64_t n_sites, int64_t n_adj, const float* grad_pack, int sh_deg,
                   float* g_raw, float* g_dA, float* g_cA, float* g_sh, void* stream);

/* vg_foam_forward for callers that cannot allocate device memory while rendering (a plugin inside a
 * host that owns a fixed memory pool, a real-time viewer that reserves all buffers at start-up, a
 * process whose device memory belongs to another framework's allocator). No counterpart in the
 * reference. Same arguments and outputs as vg_foam_forward without the workspace: the per-site
 * scratch lives in a static device array (32 MiB, allocated when the library loads on a device and
 * held by every device that loads it until exit), so n_sites is limited to 131072 (VG_ERR_WORKSPACE
 * beyond). The first call on a device looks up that array's address (make it before any stream
 * capture). Calls share the array: calls that overlap on the GPU race and must be ordered by the
 * caller (e.g. one stream). Allocates and frees nothing. What the field records leave of the array
 * serves as the cell-major colour pass's workspace when that fits (small ray batches of small scenes);
 * otherwise colours are evaluated inline along each ray (same image, slower). */
int vg_foam_forward_noalloc(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                            const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                            const int32_t* start, const float* near, const float* far, int64_t n_rays,
                            float t_thresh, float w_thresh, int record_cap, float* rgb, float* T, float* depth,
                            int32_t* stats, float* rec, void* stream);

/* ------------------------------------------------------------------------------- fixed steps */

/* march_forward (march.cu:383-403): midpoints of steps dt in [near, mid], n_bg disparity steps in
 * [mid, far]; outputs as vg_foam_forward without records. */
int vg_march_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                     const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                     const int32_t* start, const float* near, const float* mid, const float* far, int64_t n_rays,
                     float dt, int n_bg, float t_thresh, float w_thresh, float* rgb, float* T, float* depth,
                     int32_t* stats, void* workspace, size_t workspace_bytes, void* stream);

/* march_backward (march.cu:405-429): re-marches every ray; gradients overwritten. Given the larger
 * workspace of vg_foam_workspace_bytes(..., backward = 3), the samples' gradients are bucketed by cell
 * and scattered cell-major; with the backward = 1 size, per sample. */
int vg_march_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                      const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                      const int32_t* start, const float* near, const float* mid, const float* far, int64_t n_rays,
                      float dt, int n_bg, float t_thresh, float w_thresh, const float* rgb, const float* T,
                      const float* g_rgb, const float* g_T, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------- conics */

/* conic_forward (vgf.cu:535-546): A (N, 6) = R(q) diag(1 / (exp(2 clamp(ls)) + floor^2)) R^T. */
int vg_conic_forward(const float* log_scale, const float* quat, int64_t n, double floor, float* A, void* stream);

/* conic_backward (vgf.cu:548-561): g_ls (N, 3), g_quat (N, 4) from gA (N, 6). */
int vg_conic_backward(const float* log_scale, const float* quat, int64_t n, double floor, const float* gA,
                      float* g_ls, float* g_quat, void* stream);

/* ------------------------------------------------------------------ NeRF-sampler field kernels */

/* walk (vgf.cu:438-456): nearest site of every sample o + z d of the (B, S) sorted sample depths z,
 * each found by a greedy walk from the previous sample's site (the first from start[r]); a step moves
 * to the first neighbour, in adjacency order, strictly closer than the current best. Outputs
 * site (B, S) int32 original site ids and steps (B) int32 walk steps per ray. A start outside [0, N)
 * gives site -1 for that ray and sets status bit 4. */
int vg_walk(const void* pack, int64_t n_sites, int64_t n_adj, const float* o, const float* d, const float* z,
            const int32_t* start, int64_t n_rays, int64_t n_samples, int32_t* site, int32_t* steps,
            void* stream);

/* Workspace of the field functions for n_sites sites and n_samples samples: kind 0
 * vg_density_forward, 1 vg_density_backward, 2 vg_color_forward, 3 vg_color_backward (sh_deg used by 2
 * and 3). A backward given this much buckets its samples by cell and scatters the gradients
 * cell-major; given only the size for n_samples = 0, it scatters them per sample. */
size_t vg_field_workspace_bytes(int64_t n_sites, int sh_deg, int kind, int64_t n_samples);

/* density_forward (vgf.cu:458-475): sigma (M) = sum over the neighbourhood {i} U adj(i) of the
 * sample's site i of exp(min(raw_k, 30) - v^T A_k v / 2), A_k the conic of (log_scale, quat) widened
 * by scale_mult (A / scale_mult^2). raw (N), log_scale (N, 3), quat (N, 4), x (M, 3), site (M).
 * A site outside [0, N) gives sigma 0 and sets status bit 4. */
int vg_density_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* log_scale,
                       const float* quat, const float* x, const int32_t* site, int64_t n_samples,
                       double scale_mult, float* sigma, void* workspace, size_t workspace_bytes, void* stream);

/* density_backward (vgf.cu:477-492): g_raw (N), g_ls (N, 3), g_quat (N, 4) (overwritten) of
 * sum(grad_sigma * sigma) at scale_mult 1. */
int vg_density_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* log_scale,
                        const float* quat, const float* x, const int32_t* site, int64_t n_samples,
                        const float* grad_sigma, float* g_raw, float* g_ls, float* g_quat, void* workspace,
                        size_t workspace_bytes, void* stream);

/* color_forward (vgf.cu:494-513): rgb (M, 3) = sum_k a_k max(SH_k(d) + 1/2, 0) / sum_k a_k over the
 * neighbourhood of the sample's site, a_k = exp(-(m_k - min m) / 2), m_k = v^T A_k v with the colour
 * conics of (log_scale, quat); dirs (M, 3) need not be unit; sh (N, 16, 3), sh_deg 0..3. */
int vg_color_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* log_scale, const float* quat,
                     const float* sh, int sh_deg, const float* x, const float* dirs, const int32_t* site,
                     int64_t n_samples, float* rgb, void* workspace, size_t workspace_bytes, void* stream);

/* color_backward (vgf.cu:515-533): g_ls (N, 3), g_quat (N, 4), g_sh (N, 16, 3) (overwritten) of
 * sum(grad_rgb * rgb), rgb the forward's output. */
int vg_color_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* log_scale, const float* quat,
                      const float* sh, int sh_deg, const float* x, const float* dirs, const int32_t* site,
                      int64_t n_samples, const float* rgb, const float* grad_rgb, float* g_ls, float* g_quat,
                      float* g_sh, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------- inference */

/* Workspace of vg_infer_pack. */
size_t vg_infer_pack_workspace_bytes(int64_t n_sites);

/* render.pack_foam (render.py:179-225) on the device: the inference layout of vg_foam_infer from the
 * scene (points (N, 3), offsets (N + 1), adj (M)) and the model parameters (raw (N), d/c log-scales
 * (N, 3), d/c quaternions (N, 4), sh (N, 16, 3) fp32). Outputs points4 (N, 4), offsets_out (N + 1),
 * nbr (N + M), edge (N + M, 4), attr (N, 20) (baked colours zero), sh_out (N, 16, 3) in fp16 when
 * sh_half else fp32, sh32 (N, 16, 3) fp32 in the output order (may be NULL) and, with reorder, orig (N)
 * = the Morton permutation of the graph pack `pack` (which must then be non-null). Bit-identical to
 * pack_foam on the GPU. */
int vg_infer_pack(const void* pack, int64_t n_sites, int64_t n_adj, const float* points, const int32_t* offsets,
                  const int32_t* adj, const float* raw, const float* d_log_scale, const float* d_quat,
                  const float* c_log_scale, const float* c_quat, const float* sh, double scale_floor,
                  double eps_density, int sh_half, int reorder, float* points4, int32_t* offsets_out, int32_t* nbr,
                  float* edge, float* attr, void* sh_out, float* sh32, int32_t* orig, void* workspace,
                  size_t workspace_bytes, void* stream);

/* render.bake_colors (render.py:228-235): attr[:, 16:19] = max(SH_k(d_k) + 1/2, 0) for the unit
 * direction d_k from the camera centre (cx, cy, cz) to site k; points4 and sh32 as written by
 * vg_infer_pack. */
int vg_bake_colors(const float* points4, const float* sh32, int sh_deg, int64_t n_sites, float cx, float cy, float cz,
                   float* attr, void* stream);

/* ------------------------------------------------------------------------------ scene preparation */

/* Pinhole rays of a width x height image (colmap.py:129-134): d = c2w K^-1 (px + 0.5, py + 0.5, 1)
 * normalised, o = centre. K_inv, c2w: HOST 3 x 3 row-major arrays (K_inv of a pinhole camera: row 1
 * column 0 zero, last row (0, 0, 1)); centre: HOST 3 floats. Outputs o, d (W H, 3) on the device, in
 * tile_h x tile_w pixel tiles (tiles row-major, pixels row-major inside a tile; the ray order of
 * bench_infer.py:37-41), or row-major pixels when tile_h == 0. */
int vg_camera_rays(const float* K_inv, const float* c2w, const float* centre, int width, int height, int tile_h,
                   int tile_w, float* o, float* d, void* stream);

/* sites.nearest_sites (sites.py:38-39): the site nearest to each of the n_queries points queries
 * (n_queries, 3), as original ids in site (n_queries) int32, by greedy walks on the packed graph (distance
 * ties to the smaller id). Used for the `start` site of every ray (render.py:263). */
int vg_nearest_sites(const void* pack, int64_t n_sites, int64_t n_adj, const float* queries, int64_t n_queries,
                     int32_t* site, void* stream);

/* foam_infer (foam_infer.cu:376-435) on the packed inference layout of render.pack_foam: points (N, 4),
 * offsets (N + 1) into self-first neighbourhoods, nbr (E), edge (E, 4) = (p, half2(r2, lam)),
 * attr (N, 20), sh (N, 16, 3) float32 (sh_half = 0) or float16 (sh_half = 1, may be NULL for baked
 * colours), orig (N) or NULL, cap (B) or NULL. color_mode 0 lazy / 1 baked / 2 fused; stage 0..2.
 * Outputs rgb (B, 3), T (B), depth (B), stats (B, 5). */
int vg_foam_infer(const float* points, const int32_t* offsets, const int32_t* nbr, const float* edge,
                  const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites, int64_t n_edges,
                  const float* o, const float* d, const int32_t* start, const float* near, const float* far,
                  int64_t n_rays, float t_thresh, float w_thresh, float color_cut, int color_mode, int stage,
                  const int32_t* cap, const int32_t* orig, float* rgb, float* T, float* depth, int32_t* stats,
                  void* stream);

/* Workspace of vg_foam_infer_deferred for n_sites sites and n_rays rays. */
size_t vg_foam_infer_workspace_bytes(int64_t n_sites, int64_t n_rays);

/* Trace records of an inference layout for vg_foam_infer_deferred: records (n_edges, 12) float32, built
 * once per layout and kept by the caller (they change only when nbr, edge or attr change): edge e as
 * (edge[e] | attr[nbr[e], 0:4] | attr[nbr[e], 4:7], bits(nbr[e])), so the traversal reads each cell's
 * neighbourhood with its density conics as one contiguous run. No reference counterpart (an auxiliary
 * layout of foam_infer.cu's inputs). */
int vg_infer_trace_records(const int32_t* nbr, const float* edge, const float* attr, int64_t n_sites, int64_t n_edges,
                           float* records, void* stream);

/* foam_infer (foam_infer.cu:376-435) with deferred, cell-major colours: the same arguments as
 * vg_foam_infer plus the layout's trace records (vg_infer_trace_records) and a caller-allocated workspace. At stage 2 the samples, densities and weights are
 * traced per ray without colours; the samples that border a coloured segment are then sorted by cell and
 * coloured one cell at a time, and composited per ray in order. rgb, T, depth and stats columns 0-3
 * (samples, coloured segments, walk steps, density terms) are those of vg_foam_infer, bit for bit;
 * column 4 counts the SH colours evaluated by the cell-major pass for the ray's samples (vg_foam_infer
 * counts the misses of its per-ray colour cache, as the reference kernel does). Stages 0 and 1 need no
 * workspace and run as vg_foam_infer. */
int vg_foam_infer_deferred(const float* points, const int32_t* offsets, const int32_t* nbr, const float* edge,
                           const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites,
                           int64_t n_edges, const float* o, const float* d, const int32_t* start, const float* near,
                           const float* far, int64_t n_rays, float t_thresh, float w_thresh, float color_cut,
                           int color_mode, int stage, const int32_t* cap, const int32_t* orig,
                           const float* trace_records, float* rgb, float* T, float* depth, int32_t* stats,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------ kernel timing */

/* Measurement aid with no counterpart in the reference (whose benchmarks time whole extension calls).
 * While enabled, every launch of the kernel classes below is bracketed by a pair of CUDA events
 * recorded on that launch's own stream, so a benchmark can read one kernel's device time inside a
 * larger timed region. vg_prof_enable(1) forgets earlier records and starts recording, (0) stops.
 * vg_prof_read waits for the recorded events of one class and returns their summed time in ms and
 * the number of launches. Events are created on the current device; use one device per process while
 * recording. Disabled (the default), the launches carry no events. */
enum {
    VG_PROF_TRAVERSAL = 0,   /* interaction-point traversal of vg_foam_forward */
    VG_PROF_COLOR = 1,       /* cell-major colour pass of vg_foam_forward */
    VG_PROF_REPLAY = 2,      /* record replay of vg_foam_backward (writes the scatter's items) */
    VG_PROF_SCATTER = 3,     /* cell-major gradient scatter (foam, march and field backwards) */
    VG_PROF_INFER = 4,       /* per-ray traversal of vg_foam_infer / vg_foam_infer_deferred */
    VG_PROF_MARCH_FWD = 5,   /* vg_march_forward */
    VG_PROF_MARCH_ITEMS = 6, /* re-march of vg_march_backward writing the scatter's items */
    VG_PROF_INFER_COLOR = 7  /* cell-major colour pass of vg_foam_infer_deferred */
};
int vg_prof_enable(int on);
int vg_prof_read(int kernel, double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif
