// vg_foam_forward_noalloc: the interaction-point forward render for callers that must not allocate
// device memory at render time.
//
// Who needs it: hosts that own all device memory up front and forbid allocations once rendering has
// started — a renderer embedded as a plugin in an application with its own fixed memory pool, a
// real-time viewer that reserves every buffer at start-up so frame times stay predictable, or a
// process whose device memory is already fully handed out to another framework's caching
// allocator. Such callers can still pass the scene, rays and output buffers they own, but cannot
// provide the extra scratch (the packed per-site field records) that vg_foam_forward takes as a
// workspace.
//
// Here that scratch is a file-scope device array of fixed size, allocated by the CUDA runtime when
// the library's module is loaded on a device and held by every device that loads the library until
// the process exits. It fits the field records of at most kMaxSites sites at any SH degree (32 MiB).
// In host code the array's name only stands for the symbol, not a device address: its address on
// the current device is looked up with cudaGetSymbolAddress, once per device, on the first call made
// with that device current; make that first call before any stream capture. No call allocates or
// frees device memory.
//
// The field records take the front of the array; the space behind them serves as the workspace of the
// cell-major colour pass when that pass's workspace fits there (small ray batches of small scenes),
// and otherwise the forward evaluates colours inline along each ray (same image, slower).
//
// All calls share the one array and leave their own records in it. Nothing needs clearing: a call
// writes the records of all its sites before its render kernel reads them. Calls whose work overlaps
// on the GPU (different streams, or several host threads on one device) race on the array, so the
// caller must order them, e.g. by issuing them on one stream.
#include <mutex>

#include "vg_common.cuh"
#include "vgb200.h"

namespace {

constexpr int64_t kMaxSites = int64_t(1) << 17;                    // 131072 sites
constexpr size_t kScratchBytes = size_t(kMaxSites) * (64 + 192);   // 64-byte record + 48 SH floats

static __device__ __align__(256) unsigned char g_field_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

}  // namespace

extern "C" int vg_foam_forward_noalloc(const void* pack, int64_t n_sites, int64_t n_adj, const float* raw,
                                       const float* dA, const float* cA, const float* sh, int sh_deg,
                                       const float* o, const float* d, const int32_t* start, const float* near,
                                       const float* far, int64_t n_rays, float t_thresh, float w_thresh,
                                       int record_cap, float* rgb, float* T, float* depth, int32_t* stats,
                                       float* rec, void* stream) {
    if (n_sites > kMaxSites)
        return vg::set_error(VG_ERR_WORKSPACE, "vg_foam_forward_noalloc: n_sites exceeds the 131072-site limit of its "
                                               "static scratch; use vg_foam_forward with a workspace");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return vg::set_error(VG_ERR_CUDA, "vg_foam_forward_noalloc: no usable current device");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (g_scratch_ptr[dev] == nullptr) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_field_scratch);
            if (e != cudaSuccess || p == nullptr)
                return vg::set_error(VG_ERR_CUDA, "vg_foam_forward_noalloc: cannot address the static scratch");
            g_scratch_ptr[dev] = p;
        }
        scratch = g_scratch_ptr[dev];
    }
    return vg_foam_forward(pack, n_sites, n_adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, n_rays, t_thresh,
                           w_thresh, record_cap, rgb, T, depth, stats, rec, scratch, kScratchBytes, stream);
}
