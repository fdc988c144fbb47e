// extern "C" entry points of libvgb200 (declared in include/vgb200.h): argument checks with the
// reference's error semantics, workspace carving and dispatch to the kernels.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "vgb200.h"  // include/ (on the -I path)
#include "vg_common.cuh"

namespace {

thread_local std::string g_error;

// status word of the render launches, one per device (module memory; addressed per device below)
__device__ int g_status_word;
constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
std::mutex g_status_mu;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(VG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int* status_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (g_status_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
        g_status_ptr[dev] = static_cast<int*>(p);
    }
    return g_status_ptr[dev];
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

#define REQUIRE(cond, ...)                                   \
    do {                                                     \
        if (!(cond)) return fail(VG_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

int check_scene(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA, const float* cA,
                const float* sh, int sh_deg) {
    REQUIRE(pack != nullptr, "graph pack is null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE(raw && dA && cA && sh, "raw, dA, cA and sh must be non-null");
    REQUIRE(sh_deg >= 0 && sh_deg <= 3, "sh_deg must be in 0..3");
    return VG_OK;
}

int check_rays(int64_t n_rays, const float* o, const float* d, const int32_t* start, const float* near,
               const float* far) {
    REQUIRE(n_rays >= 0, "n_rays must be >= 0");
    REQUIRE(n_rays == 0 || (o && d && start && near && far), "ray arrays must be non-null");
    return VG_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Vector loads / stores of the kernels: conics and their gradients as float2, SH rows as float4,
// records as float4.
int check_alignment(const float* dA, const float* cA, const float* sh, const float* rec) {
    REQUIRE(aligned(dA, 8) && aligned(cA, 8), "conics must be 8-byte aligned");
    REQUIRE(aligned(sh, 16), "sh must be 16-byte aligned");
    REQUIRE(rec == nullptr || aligned(rec, 16), "rec must be 16-byte aligned");
    return VG_OK;
}

size_t field_ws(int64_t n, int deg) { return align256(vg::field_bytes(n, deg)); }
size_t grad_ws(int64_t n) { return align256(static_cast<size_t>(n) * vg::kGradStride * sizeof(float)); }

int check_field(const void* pack, int64_t n_sites, int64_t n_adj, const float* ls, const float* quat, const float* x,
                const int32_t* site, int64_t m, void* workspace, size_t workspace_bytes, int sh_deg, int kind) {
    REQUIRE(pack != nullptr, "graph pack is null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE(ls && quat, "log_scale and quat must be non-null");
    REQUIRE(aligned(quat, 16), "quat must be 16-byte aligned");
    REQUIRE(m >= 0, "n_samples must be >= 0");
    REQUIRE(m == 0 || (x && site), "x and site must be non-null");
    REQUIRE(sh_deg >= 0 && sh_deg <= 3, "sh_deg must be in 0..3");
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const size_t need = vg::field_workspace(n_sites, sh_deg, kind);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    return VG_OK;
}

}  // namespace

namespace vg {
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace vg

extern "C" {

int vg_version(void) { return 100; }

const char* vg_last_error(void) { return g_error.c_str(); }

int vg_status(int* bits) {
    REQUIRE(bits != nullptr, "bits is null");
    int* p = status_ptr();
    if (p == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "vg_status");
    e = cudaMemcpy(bits, p, sizeof(int), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_status");
}

int vg_status_reset(void) {
    int* p = status_ptr();
    if (p == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const cudaError_t e = cudaMemset(p, 0, sizeof(int));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_status_reset");
}

size_t vg_graph_pack_bytes(int64_t n_sites, int64_t n_adj) {
    if (n_sites <= 0 || n_adj < 0) return 0;
    return vg::graph_pack_bytes(n_sites, n_adj);
}

int vg_graph_pack(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites, int64_t n_adj,
                  void* pack, size_t pack_bytes, void* stream) {
    REQUIRE(points && offsets && pack, "points, offsets and pack must be non-null");
    REQUIRE(n_adj == 0 || adj != nullptr, "adj is null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE((reinterpret_cast<uintptr_t>(pack) & 255) == 0, "pack must be 256-byte aligned");
    const size_t need = vg::graph_pack_bytes(n_sites, n_adj);
    if (pack_bytes < need) return fail(VG_ERR_WORKSPACE, "graph pack needs %zu bytes, got %zu", need, pack_bytes);
    const cudaError_t e = vg::graph_pack(points, offsets, adj, n_sites, n_adj, pack, pack_bytes,
                                         static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_graph_pack");
}

size_t vg_foam_workspace_bytes(int64_t n_sites, int sh_deg, int64_t n_rays, int record_cap, int backward) {
    if (n_sites <= 0 || sh_deg < 0 || sh_deg > 3 || n_rays < 0 || record_cap < 0) return 0;
    if (backward == 0) return field_ws(n_sites, sh_deg) + align256(vg::foam_forward_workspace(n_sites, n_rays, record_cap));
    if (backward == 3) return field_ws(n_sites, sh_deg) + grad_ws(n_sites) + align256(vg::march_backward_workspace(n_sites, n_rays));
    const size_t cm = align256(vg::foam_backward_workspace(n_sites, n_rays, record_cap));
    return field_ws(n_sites, sh_deg) + (backward == 1 ? grad_ws(n_sites) : 0) + cm;
}

static int foam_forward_impl(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                             const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                             const int32_t* start, const float* near, const float* far, int64_t n_rays,
                             float t_thresh, float w_thresh, int record_cap, float* rgb, float* T, float* depth,
                             int32_t* stats, float* rec, int32_t* counts, void* workspace, size_t workspace_bytes,
                             void* stream) {
    int rc = check_scene(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg);
    if (rc) return rc;
    if ((rc = check_rays(n_rays, o, d, start, near, far))) return rc;
    REQUIRE(record_cap >= 0, "record_cap must be >= 0");
    REQUIRE(n_rays == 0 || (rgb && T && depth && stats), "outputs must be non-null");
    REQUIRE(record_cap == 0 || n_rays == 0 || rec != nullptr, "rec is null with record_cap > 0");
    if ((rc = check_alignment(dA, cA, sh, record_cap > 0 ? rec : nullptr))) return rc;
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    // with counts, the cell-major forward must run (it keeps them): the full workspace is required
    const size_t need = counts != nullptr ? vg_foam_workspace_bytes(n_sites, sh_deg, n_rays, record_cap, 0)
                                          : field_ws(n_sites, sh_deg);
    if (workspace_bytes < need || workspace == nullptr)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    REQUIRE(counts == nullptr || record_cap > 0, "sample counts need records (record_cap > 0)");
    if (n_rays == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    cudaError_t e = vg::field_pack(g, raw, dA, cA, sh, sh_deg, workspace, st);
    if (e != cudaSuccess) return cuda_fail(e, "field pack");
    const vg::FieldView F = vg::field_view(workspace, n_sites, sh_deg);
    const vg::RayView R{o, d, start, near, nullptr, far, n_rays};
    vg::FoamCfg c{t_thresh, w_thresh, record_cap};
    c.all_count = counts;
    const vg::Outputs out{rgb, T, depth, stats, record_cap > 0 ? rec : nullptr};
    // scratch beyond the field records enables the cell-major colour pass (inline colours otherwise)
    const size_t fw = field_ws(n_sites, sh_deg);
    e = vg::foam_forward(g, F, R, c, out, status, static_cast<char*>(workspace) + fw, workspace_bytes - fw, st);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_foam_forward");
}

int vg_foam_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                    const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                    const int32_t* start, const float* near, const float* far, int64_t n_rays, float t_thresh,
                    float w_thresh, int record_cap, float* rgb, float* T, float* depth, int32_t* stats, float* rec,
                    void* workspace, size_t workspace_bytes, void* stream) {
    return foam_forward_impl(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays, t_thresh,
                             w_thresh, record_cap, rgb, T, depth, stats, rec, nullptr, workspace, workspace_bytes,
                             stream);
}

size_t vg_foam_counts_bytes(int64_t n_sites, int64_t n_rays, int record_cap) {
    if (n_sites <= 0 || n_rays <= 0 || record_cap <= 0) return 0;
    return 4 * static_cast<size_t>(vg::foam_count_entries(n_sites, n_rays, record_cap));
}

int vg_foam_forward_counted(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                            const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                            const int32_t* start, const float* near, const float* far, int64_t n_rays,
                            float t_thresh, float w_thresh, int record_cap, float* rgb, float* T, float* depth,
                            int32_t* stats, float* rec, int32_t* counts, void* workspace, size_t workspace_bytes,
                            void* stream) {
    REQUIRE(n_rays == 0 || counts != nullptr, "counts is null");
    REQUIRE(aligned(counts, 4), "counts must be 4-byte aligned");
    return foam_forward_impl(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays, t_thresh,
                             w_thresh, record_cap, rgb, T, depth, stats, rec, n_rays ? counts : nullptr, workspace,
                             workspace_bytes, stream);
}

static int foam_backward_impl(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                              const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                              const int32_t* start, const float* near, const float* far, int64_t n_rays,
                              float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                              const float* g_T, const float* rec, int record_cap, const int32_t* stats, float* grad,
                              bool zero_first, void* workspace, size_t workspace_bytes, size_t need, size_t cm_off,
                              cudaStream_t st, const int32_t* counts = nullptr) {
    int rc = check_scene(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg);
    if (rc) return rc;
    if ((rc = check_rays(n_rays, o, d, start, near, far))) return rc;
    REQUIRE(record_cap >= 0, "record_cap must be >= 0");
    REQUIRE(n_rays == 0 || (rgb && T && g_rgb && g_T && stats), "rgb, T, g_rgb, g_T and stats must be non-null");
    if ((rc = check_alignment(dA, cA, sh, record_cap > 0 ? rec : nullptr))) return rc;
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    if (workspace_bytes < need || workspace == nullptr)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    cudaError_t e = cudaSuccess;
    if (zero_first) {
        e = cudaMemsetAsync(grad, 0, static_cast<size_t>(n_sites) * vg::kGradStride * sizeof(float), st);
        if (e != cudaSuccess) return cuda_fail(e, "zero gradients");
    }
    if (n_rays == 0) return VG_OK;
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    e = vg::field_pack(g, raw, dA, cA, sh, sh_deg, workspace, st);
    if (e != cudaSuccess) return cuda_fail(e, "field pack");
    const vg::FieldView F = vg::field_view(workspace, n_sites, sh_deg);
    const vg::RayView R{o, d, start, near, nullptr, far, n_rays};
    vg::FoamCfg c{t_thresh, w_thresh, record_cap};
    c.all_count = record_cap > 0 ? const_cast<int32_t*>(counts) : nullptr;  // read only in the backward
    const vg::GradIn gi{rgb, T, g_rgb, g_T, record_cap > 0 ? rec : nullptr, stats, record_cap};
    void* cm = static_cast<char*>(workspace) + cm_off;
    e = vg::foam_backward(g, F, R, c, gi, grad, status, cm, workspace_bytes - cm_off, st);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_foam_backward");
}

static int foam_backward_unpacked(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                                  const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                                  const int32_t* start, const float* near, const float* far, int64_t n_rays,
                                  float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                                  const float* g_T, const float* rec, int record_cap, const int32_t* stats,
                                  const int32_t* counts, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    REQUIRE(g_raw && g_dA && g_cA && g_sh, "gradient outputs must be non-null");
    REQUIRE(aligned(g_dA, 8) && aligned(g_cA, 8) && aligned(g_sh, 16), "gradient outputs misaligned");
    if (sh_deg < 0 || sh_deg > 3) return fail(VG_ERR_INVALID_ARG, "sh_deg must be in 0..3");
    const size_t need = vg_foam_workspace_bytes(n_sites, sh_deg, n_rays, record_cap, 1);
    float* grad = reinterpret_cast<float*>(static_cast<char*>(workspace) + field_ws(n_sites, sh_deg));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = foam_backward_impl(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays,
                                t_thresh, w_thresh, rgb, T, g_rgb, g_T, rec, record_cap, stats, grad, true, workspace,
                                workspace_bytes, need, field_ws(n_sites, sh_deg) + grad_ws(n_sites), st, counts);
    if (rc) return rc;
    const cudaError_t e =
        vg::grad_unpack(vg::graph_view(pack, n_sites, n_adj), grad, sh_deg, g_raw, g_dA, g_cA, g_sh, st);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "gradient unpack");
}

int vg_foam_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                     const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                     const int32_t* start, const float* near, const float* far, int64_t n_rays, float t_thresh,
                     float w_thresh, const float* rgb, const float* T, const float* g_rgb, const float* g_T,
                     const float* rec, int record_cap, const int32_t* stats, float* g_raw, float* g_dA, float* g_cA,
                     float* g_sh, void* workspace, size_t workspace_bytes, void* stream) {
    return foam_backward_unpacked(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays,
                                  t_thresh, w_thresh, rgb, T, g_rgb, g_T, rec, record_cap, stats, nullptr, g_raw, g_dA,
                                  g_cA, g_sh, workspace, workspace_bytes, stream);
}

int vg_foam_backward_counted(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                             const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                             const int32_t* start, const float* near, const float* far, int64_t n_rays,
                             float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                             const float* g_T, const float* rec, int record_cap, const int32_t* stats,
                             const int32_t* counts, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                             void* workspace, size_t workspace_bytes, void* stream) {
    REQUIRE(n_rays == 0 || record_cap == 0 || counts != nullptr, "counts is null");
    return foam_backward_unpacked(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays,
                                  t_thresh, w_thresh, rgb, T, g_rgb, g_T, rec, record_cap, stats, counts, g_raw, g_dA,
                                  g_cA, g_sh, workspace, workspace_bytes, stream);
}

int vg_foam_backward_packed(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                            const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                            const int32_t* start, const float* near, const float* far, int64_t n_rays, float t_thresh,
                            float w_thresh, const float* rgb, const float* T, const float* g_rgb, const float* g_T,
                            const float* rec, int record_cap, const int32_t* stats, float* grad_pack, int zero_first,
                            void* workspace, size_t workspace_bytes, void* stream) {
    REQUIRE(grad_pack != nullptr, "grad_pack is null");
    REQUIRE((reinterpret_cast<uintptr_t>(grad_pack) & 15) == 0, "grad_pack must be 16-byte aligned");
    if (sh_deg < 0 || sh_deg > 3) return fail(VG_ERR_INVALID_ARG, "sh_deg must be in 0..3");
    return foam_backward_impl(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays, t_thresh,
                              w_thresh, rgb, T, g_rgb, g_T, rec, record_cap, stats, grad_pack, zero_first != 0,
                              workspace, workspace_bytes, vg_foam_workspace_bytes(n_sites, sh_deg, n_rays, record_cap, 2),
                              field_ws(n_sites, sh_deg), static_cast<cudaStream_t>(stream));
}

int vg_grad_unpack(const void* pack, int64_t n_sites, int64_t n_adj, const float* grad_pack, int sh_deg,
                   float* g_raw, float* g_dA, float* g_cA, float* g_sh, void* stream) {
    REQUIRE(pack && grad_pack && g_raw && g_dA && g_cA && g_sh, "arguments must be non-null");
    REQUIRE(aligned(grad_pack, 16) && aligned(g_dA, 8) && aligned(g_cA, 8) && aligned(g_sh, 16),
            "gradient arrays misaligned");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(sh_deg >= 0 && sh_deg <= 3, "sh_deg must be in 0..3");
    const cudaError_t e = vg::grad_unpack(vg::graph_view(pack, n_sites, n_adj), grad_pack, sh_deg, g_raw, g_dA, g_cA,
                                          g_sh, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_grad_unpack");
}

int vg_march_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                     const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                     const int32_t* start, const float* near, const float* mid, const float* far, int64_t n_rays,
                     float dt, int n_bg, float t_thresh, float w_thresh, float* rgb, float* T, float* depth,
                     int32_t* stats, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_scene(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg);
    if (rc) return rc;
    if ((rc = check_rays(n_rays, o, d, start, near, far))) return rc;
    REQUIRE(n_rays == 0 || mid != nullptr, "mid is null");
    REQUIRE(n_rays == 0 || (rgb && T && depth && stats), "outputs must be non-null");
    REQUIRE(n_bg >= 0, "n_bg must be >= 0");
    if ((rc = check_alignment(dA, cA, sh, nullptr))) return rc;
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const size_t need = field_ws(n_sites, sh_deg);
    if (workspace_bytes < need || workspace == nullptr)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    if (n_rays == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    cudaError_t e = vg::field_pack(g, raw, dA, cA, sh, sh_deg, workspace, st);
    if (e != cudaSuccess) return cuda_fail(e, "field pack");
    const vg::FieldView F = vg::field_view(workspace, n_sites, sh_deg);
    const vg::RayView R{o, d, start, near, mid, far, n_rays};
    const vg::MarchCfg c{dt, n_bg, t_thresh, w_thresh};
    const vg::Outputs out{rgb, T, depth, stats, nullptr};
    e = vg::march_forward(g, F, R, c, out, status, st);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_march_forward");
}

int vg_march_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* dA,
                      const float* cA, const float* sh, int sh_deg, const float* o, const float* d,
                      const int32_t* start, const float* near, const float* mid, const float* far, int64_t n_rays,
                      float dt, int n_bg, float t_thresh, float w_thresh, const float* rgb, const float* T,
                      const float* g_rgb, const float* g_T, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                      void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_scene(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg);
    if (rc) return rc;
    if ((rc = check_rays(n_rays, o, d, start, near, far))) return rc;
    REQUIRE(n_rays == 0 || mid != nullptr, "mid is null");
    REQUIRE(n_rays == 0 || (rgb && T && g_rgb && g_T), "rgb, T, g_rgb and g_T must be non-null");
    REQUIRE(g_raw && g_dA && g_cA && g_sh, "gradient outputs must be non-null");
    REQUIRE(n_bg >= 0, "n_bg must be >= 0");
    if ((rc = check_alignment(dA, cA, sh, nullptr))) return rc;
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    REQUIRE(aligned(g_dA, 8) && aligned(g_cA, 8) && aligned(g_sh, 16), "gradient outputs misaligned");
    const size_t need = vg_foam_workspace_bytes(n_sites, sh_deg, n_rays, 0, 1);
    if (workspace_bytes < need || workspace == nullptr)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    float* grad = reinterpret_cast<float*>(static_cast<char*>(workspace) + field_ws(n_sites, sh_deg));
    char* cm_ws = static_cast<char*>(workspace) + need;  // cell-major scratch when the caller gave more
    const size_t cm_bytes = workspace_bytes - need;
    cudaError_t e = cudaMemsetAsync(grad, 0, static_cast<size_t>(n_sites) * vg::kGradStride * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "zero gradients");
    if (n_rays > 0) {
        e = vg::field_pack(g, raw, dA, cA, sh, sh_deg, workspace, st);
        if (e != cudaSuccess) return cuda_fail(e, "field pack");
        const vg::FieldView F = vg::field_view(workspace, n_sites, sh_deg);
        const vg::RayView R{o, d, start, near, mid, far, n_rays};
        const vg::MarchCfg c{dt, n_bg, t_thresh, w_thresh};
        const vg::GradIn gi{rgb, T, g_rgb, g_T, nullptr, nullptr, 0};
        e = vg::march_backward(g, F, R, c, gi, grad, status, cm_bytes > 0 ? cm_ws : nullptr, cm_bytes, st);
        if (e != cudaSuccess) return cuda_fail(e, "vg_march_backward");
    }
    e = vg::grad_unpack(g, grad, sh_deg, g_raw, g_dA, g_cA, g_sh, st);
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "gradient unpack");
}

int vg_conic_forward(const float* log_scale, const float* quat, int64_t n, double floor, float* A, void* stream) {
    REQUIRE(n >= 0, "n must be >= 0");
    REQUIRE(n == 0 || (log_scale && quat && A), "arguments must be non-null");
    REQUIRE(aligned(quat, 16) && aligned(A, 8), "quat must be 16-byte and A 8-byte aligned");
    const cudaError_t e = vg::conic_forward(log_scale, quat, n, static_cast<float>(floor * floor), A,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_conic_forward");
}

int vg_conic_backward(const float* log_scale, const float* quat, int64_t n, double floor, const float* gA,
                      float* g_ls, float* g_quat, void* stream) {
    REQUIRE(n >= 0, "n must be >= 0");
    REQUIRE(n == 0 || (log_scale && quat && gA && g_ls && g_quat), "arguments must be non-null");
    REQUIRE(aligned(quat, 16) && aligned(gA, 8) && aligned(g_quat, 16), "conic arrays misaligned");
    const cudaError_t e = vg::conic_backward(log_scale, quat, n, static_cast<float>(floor * floor), gA, g_ls, g_quat,
                                             static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_conic_backward");
}

int vg_walk(const void* pack, int64_t n_sites, int64_t n_adj, const float* o, const float* d, const float* z,
            const int32_t* start, int64_t n_rays, int64_t n_samples, int32_t* site, int32_t* steps, void* stream) {
    REQUIRE(pack != nullptr, "graph pack is null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE(n_rays >= 0 && n_samples >= 0 && n_samples < INT32_MAX, "bad sample counts");
    REQUIRE(n_rays == 0 || (o && d && start && steps), "ray arrays must be non-null");
    REQUIRE(n_rays * n_samples == 0 || (z && site), "z and site must be non-null");
    if (n_rays == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    const cudaError_t e = vg::sampler_walk(g, o, d, z, start, n_rays, static_cast<int>(n_samples), site, steps, status,
                                           static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_walk");
}

size_t vg_field_workspace_bytes(int64_t n_sites, int sh_deg, int kind, int64_t n_samples) {
    if (n_sites <= 0 || kind < 0 || kind > 3 || sh_deg < 0 || sh_deg > 3 || n_samples < 0) return 0;
    return std::max(vg::field_workspace(n_sites, sh_deg, kind),
                    n_samples > 0 ? vg::field_cm_workspace(n_sites, sh_deg, kind, n_samples) : size_t(0));
}

int vg_density_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* log_scale,
                       const float* quat, const float* x, const int32_t* site, int64_t n_samples, double scale_mult,
                       float* sigma, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_field(pack, n_sites, n_adj, log_scale, quat, x, site, n_samples, workspace, workspace_bytes, 0, 0);
    if (rc) return rc;
    REQUIRE(raw != nullptr, "raw must be non-null");
    REQUIRE(n_samples == 0 || sigma != nullptr, "sigma must be non-null");
    REQUIRE(scale_mult != 0.0, "scale_mult must be nonzero");
    if (n_samples == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    const cudaError_t e = vg::density_field(g, raw, log_scale, quat, x, site, n_samples,
                                            static_cast<float>(1.0 / (scale_mult * scale_mult)), false, nullptr, sigma,
                                            nullptr, nullptr, nullptr, workspace, workspace_bytes, status,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_density_forward");
}

int vg_density_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw, const float* log_scale,
                        const float* quat, const float* x, const int32_t* site, int64_t n_samples,
                        const float* grad_sigma, float* g_raw, float* g_ls, float* g_quat, void* workspace,
                        size_t workspace_bytes, void* stream) {
    int rc = check_field(pack, n_sites, n_adj, log_scale, quat, x, site, n_samples, workspace, workspace_bytes, 0, 1);
    if (rc) return rc;
    REQUIRE(raw != nullptr, "raw must be non-null");
    REQUIRE(n_samples == 0 || grad_sigma != nullptr, "grad_sigma must be non-null");
    REQUIRE(g_raw && g_ls && g_quat, "gradient outputs must be non-null");
    REQUIRE(aligned(g_quat, 16), "g_quat must be 16-byte aligned");
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    const cudaError_t e = vg::density_field(g, raw, log_scale, quat, x, site, n_samples, 1.f, true, grad_sigma, nullptr,
                                            g_raw, g_ls, g_quat, workspace, workspace_bytes, status,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_density_backward");
}

int vg_color_forward(const void* pack, int64_t n_sites, int64_t n_adj, const float* log_scale, const float* quat,
                     const float* sh, int sh_deg, const float* x, const float* dirs, const int32_t* site,
                     int64_t n_samples, float* rgb, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_field(pack, n_sites, n_adj, log_scale, quat, x, site, n_samples, workspace, workspace_bytes,
                         sh_deg, 2);
    if (rc) return rc;
    REQUIRE(sh != nullptr, "sh must be non-null");
    REQUIRE(n_samples == 0 || (dirs && rgb), "dirs and rgb must be non-null");
    if (n_samples == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    const cudaError_t e = vg::color_field(g, log_scale, quat, sh, sh_deg, x, dirs, site, n_samples, false, nullptr, nullptr,
                                          rgb, nullptr, nullptr, nullptr, workspace, workspace_bytes, status,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_color_forward");
}

int vg_color_backward(const void* pack, int64_t n_sites, int64_t n_adj, const float* log_scale, const float* quat,
                      const float* sh, int sh_deg, const float* x, const float* dirs, const int32_t* site,
                      int64_t n_samples, const float* rgb, const float* grad_rgb, float* g_ls, float* g_quat,
                      float* g_sh, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_field(pack, n_sites, n_adj, log_scale, quat, x, site, n_samples, workspace, workspace_bytes,
                         sh_deg, 3);
    if (rc) return rc;
    REQUIRE(sh != nullptr, "sh must be non-null");
    REQUIRE(n_samples == 0 || (dirs && rgb && grad_rgb), "dirs, rgb and grad_rgb must be non-null");
    REQUIRE(g_ls && g_quat && g_sh, "gradient outputs must be non-null");
    REQUIRE(aligned(g_quat, 16) && aligned(g_sh, 16), "g_quat and g_sh must be 16-byte aligned");
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::GraphView g = vg::graph_view(pack, n_sites, n_adj);
    const cudaError_t e = vg::color_field(g, log_scale, quat, sh, sh_deg, x, dirs, site, n_samples, true, rgb, grad_rgb,
                                          nullptr, g_ls, g_quat, g_sh, workspace, workspace_bytes, status,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_color_backward");
}

size_t vg_infer_pack_workspace_bytes(int64_t n_sites) {
    return n_sites > 0 ? vg::infer_pack_workspace(n_sites) : 0;
}

int vg_infer_pack(const void* pack, int64_t n_sites, int64_t n_adj, const float* points, const int32_t* offsets,
                  const int32_t* adj, const float* raw, const float* d_log_scale, const float* d_quat,
                  const float* c_log_scale, const float* c_quat, const float* sh, double scale_floor,
                  double eps_density, int sh_half, int reorder, float* points4, int32_t* offsets_out, int32_t* nbr,
                  float* edge, float* attr, void* sh_out, float* sh32, int32_t* orig, void* workspace,
                  size_t workspace_bytes, void* stream) {
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE(points && offsets && (adj || n_adj == 0), "points, offsets and adj must be non-null");
    REQUIRE(raw && d_log_scale && d_quat && c_log_scale && c_quat && sh, "parameters must be non-null");
    REQUIRE(aligned(d_quat, 16) && aligned(c_quat, 16), "quaternions must be 16-byte aligned");
    REQUIRE(points4 && offsets_out && nbr && edge && attr && sh_out, "outputs must be non-null");
    REQUIRE(aligned(points4, 16) && aligned(edge, 16), "points4 and edge must be 16-byte aligned");
    REQUIRE(!reorder || (pack && orig), "reorder needs the graph pack and orig");
    REQUIRE(eps_density >= 0.0, "eps_density must be >= 0");
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const size_t need = vg::infer_pack_workspace(n_sites);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    vg::GraphView g{};
    if (reorder) g = vg::graph_view(pack, n_sites, n_adj);
    const float log_eps = eps_density > 0.0 ? static_cast<float>(std::log(eps_density)) : 0.f;
    const cudaError_t e =
        vg::infer_pack(reorder ? &g : nullptr, n_sites, points, offsets, adj, raw, d_log_scale, d_quat, c_log_scale,
                       c_quat, sh, static_cast<float>(scale_floor * scale_floor), log_eps, eps_density > 0.0, sh_half,
                       points4, offsets_out, nbr, edge, attr, sh_out, sh32, orig, workspace,
                       static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_infer_pack");
}

int vg_bake_colors(const float* points4, const float* sh32, int sh_deg, int64_t n_sites, float cx, float cy, float cz,
                   float* attr, void* stream) {
    REQUIRE(n_sites >= 0 && n_sites < INT32_MAX, "n_sites must be in [0, 2^31)");
    REQUIRE(n_sites == 0 || (points4 && sh32 && attr), "arrays must be non-null");
    REQUIRE(aligned(points4, 16), "points4 must be 16-byte aligned");
    REQUIRE(sh_deg >= 0 && sh_deg <= 3, "sh_deg must be in 0..3");
    const cudaError_t e = vg::bake_colors(points4, sh32, sh_deg, n_sites, cx, cy, cz, attr,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_bake_colors");
}

int vg_camera_rays(const float* K_inv, const float* c2w, const float* centre, int width, int height, int tile_h,
                   int tile_w, float* o, float* d, void* stream) {
    REQUIRE(K_inv && c2w && centre, "K_inv, c2w and centre must be non-null host arrays");
    REQUIRE(width >= 0 && height >= 0, "image size must be >= 0");
    REQUIRE(tile_h >= 0 && (tile_h == 0 || tile_w > 0), "tile sizes must be positive (tile_h 0: row-major)");
    REQUIRE(K_inv[3] == 0.f && K_inv[6] == 0.f && K_inv[7] == 0.f && K_inv[8] == 1.f,
            "K_inv must be the inverse of a pinhole intrinsic matrix (row 1 column 0 zero, last row 0 0 1)");
    REQUIRE(static_cast<int64_t>(width) * height == 0 || (o && d), "o and d must be non-null");
    const cudaError_t e = vg::camera_rays(K_inv, c2w, centre, width, height, tile_h, tile_w, o, d,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_camera_rays");
}

int vg_nearest_sites(const void* pack, int64_t n_sites, int64_t n_adj, const float* queries, int64_t n_queries,
                     int32_t* site, void* stream) {
    REQUIRE(pack != nullptr, "graph pack is null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX, "n_sites must be in [1, 2^31)");
    REQUIRE(n_adj >= 0 && n_sites + n_adj < INT32_MAX, "adjacency too large for int32 offsets");
    REQUIRE(n_queries >= 0, "n_queries must be >= 0");
    REQUIRE(n_queries == 0 || (queries && site), "queries and site must be non-null");
    if (n_queries == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const cudaError_t e = vg::nearest_sites(vg::graph_view(pack, n_sites, n_adj), queries, n_queries, site, status,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_nearest_sites");
}

namespace {

int infer_args(const float* points, const int32_t* offsets, const int32_t* nbr, const float* edge, const float* attr,
               const void* sh, int sh_deg, int64_t n_sites, int64_t n_edges, const float* o, const float* d,
               const int32_t* start, const float* near, const float* far, int64_t n_rays, int color_mode, int stage,
               float* rgb, float* T, float* depth, int32_t* stats) {
    REQUIRE(points && offsets && nbr && edge && attr, "pack arrays must be non-null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX && n_edges >= n_sites && n_edges < INT32_MAX, "bad pack sizes");
    REQUIRE(color_mode >= 0 && color_mode <= 2, "color_mode must be 0 (lazy), 1 (baked) or 2 (fused)");
    REQUIRE(stage >= 0 && stage <= 2, "stage must be 0, 1 or 2");
    REQUIRE(sh_deg >= 0 && sh_deg <= 3, "sh_deg must be in 0..3");
    REQUIRE(color_mode == 1 || stage < 2 || sh != nullptr, "sh must be (N, 16, 3)");
    REQUIRE(aligned(points, 16) && aligned(edge, 16) && aligned(attr, 16) && aligned(sh, 16),
            "points, edge, attr and sh must be 16-byte aligned");
    int rc = check_rays(n_rays, o, d, start, near, far);
    if (rc) return rc;
    REQUIRE(n_rays == 0 || (rgb && T && depth && stats), "outputs must be non-null");
    return VG_OK;
}

}  // namespace

int vg_foam_infer(const float* points, const int32_t* offsets, const int32_t* nbr, const float* edge,
                  const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites, int64_t n_edges,
                  const float* o, const float* d, const int32_t* start, const float* near, const float* far,
                  int64_t n_rays, float t_thresh, float w_thresh, float color_cut, int color_mode, int stage,
                  const int32_t* cap, const int32_t* orig, float* rgb, float* T, float* depth, int32_t* stats,
                  void* stream) {
    int rc = infer_args(points, offsets, nbr, edge, attr, sh, sh_deg, n_sites, n_edges, o, d, start, near, far, n_rays,
                        color_mode, stage, rgb, T, depth, stats);
    if (rc) return rc;
    if (n_rays == 0) return VG_OK;
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::InferNet N{reinterpret_cast<const float4*>(points), offsets, nbr, reinterpret_cast<const float4*>(edge),
                         reinterpret_cast<const float4*>(attr), sh, orig, sh_half};
    const vg::InferCfg c{t_thresh, w_thresh, color_cut, sh_deg, color_mode, stage, cap};
    const vg::RayView R{o, d, start, near, nullptr, far, n_rays};
    const vg::Outputs out{rgb, T, depth, stats, nullptr};
    const cudaError_t e = vg::foam_infer(N, c, R, out, status, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_foam_infer");
}

size_t vg_foam_infer_workspace_bytes(int64_t n_sites, int64_t n_rays) {
    if (n_sites <= 0 || n_sites >= INT32_MAX || n_rays < 0) return 0;
    return vg::foam_infer_workspace(n_sites, n_rays);
}

int vg_infer_trace_records(const int32_t* nbr, const float* edge, const float* attr, int64_t n_sites, int64_t n_edges,
                           float* records, void* stream) {
    REQUIRE(nbr && edge && attr && records, "nbr, edge, attr and records must be non-null");
    REQUIRE(n_sites > 0 && n_sites < INT32_MAX && n_edges >= n_sites && n_edges < INT32_MAX, "bad pack sizes");
    REQUIRE(aligned(edge, 16) && aligned(attr, 16) && aligned(records, 16), "edge, attr and records must be 16-byte aligned");
    const vg::InferNet N{nullptr, nullptr, nbr, reinterpret_cast<const float4*>(edge),
                         reinterpret_cast<const float4*>(attr), nullptr, nullptr, 0};
    const cudaError_t e = vg::infer_trace_records(N, n_edges, records, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_infer_trace_records");
}

int vg_foam_infer_deferred(const float* points, const int32_t* offsets, const int32_t* nbr, const float* edge,
                           const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites,
                           int64_t n_edges, const float* o, const float* d, const int32_t* start, const float* near,
                           const float* far, int64_t n_rays, float t_thresh, float w_thresh, float color_cut,
                           int color_mode, int stage, const int32_t* cap, const int32_t* orig,
                           const float* trace_records, float* rgb, float* T, float* depth, int32_t* stats,
                           void* workspace, size_t workspace_bytes, void* stream) {
    int rc = infer_args(points, offsets, nbr, edge, attr, sh, sh_deg, n_sites, n_edges, o, d, start, near, far, n_rays,
                        color_mode, stage, rgb, T, depth, stats);
    if (rc) return rc;
    if (n_rays == 0) return VG_OK;
    REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    REQUIRE(stage < 2 || (trace_records != nullptr && aligned(trace_records, 16)),
            "trace_records (from vg_infer_trace_records) must be non-null and 16-byte aligned");
    const size_t need = stage == 2 ? vg::foam_infer_workspace(n_sites, n_rays) : 0;
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(VG_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    int* status = status_ptr();
    if (status == nullptr) return fail(VG_ERR_CUDA, "status word unavailable");
    const vg::InferNet N{reinterpret_cast<const float4*>(points), offsets, nbr, reinterpret_cast<const float4*>(edge),
                         reinterpret_cast<const float4*>(attr), sh, orig, sh_half};
    const vg::InferCfg c{t_thresh, w_thresh, color_cut, sh_deg, color_mode, stage, cap};
    const vg::RayView R{o, d, start, near, nullptr, far, n_rays};
    const vg::Outputs out{rgb, T, depth, stats, nullptr};
    const cudaError_t e = vg::foam_infer_deferred(N, trace_records, n_sites, c, R, out, status, workspace,
                                                  workspace_bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VG_OK : cuda_fail(e, "vg_foam_infer_deferred");
}

}  // extern "C"
