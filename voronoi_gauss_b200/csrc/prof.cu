// Kernel timing registry behind vg_prof_enable / vg_prof_read (see prof.cuh).
#include <atomic>
#include <mutex>
#include <vector>

#include "prof.cuh"
#include "vg_common.cuh"
#include "vgb200.h"

namespace vg {
namespace {

constexpr int kMaxSlots = 1 << 16;  // event pairs kept per enable period

struct Slot {
    cudaEvent_t begin = nullptr, end = nullptr;
    int kernel = -1;
    bool ended = false;
};

std::atomic<bool> g_on{false};
std::mutex g_mu;
std::vector<Slot> g_slots;  // events are created once and reused across enable periods
int g_used = 0;

}  // namespace

int prof_begin(int kernel, cudaStream_t st) {
    if (!g_on.load(std::memory_order_relaxed)) return -1;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_on.load(std::memory_order_relaxed) || g_used >= kMaxSlots) return -1;
    if (g_used == static_cast<int>(g_slots.size())) {
        Slot s;
        if (cudaEventCreate(&s.begin) != cudaSuccess) return -1;
        if (cudaEventCreate(&s.end) != cudaSuccess) {
            cudaEventDestroy(s.begin);
            return -1;
        }
        g_slots.push_back(s);
    }
    Slot& s = g_slots[g_used];
    if (cudaEventRecord(s.begin, st) != cudaSuccess) return -1;
    s.kernel = kernel;
    s.ended = false;
    return g_used++;
}

void prof_end(int slot, cudaStream_t st) {
    if (slot < 0) return;
    std::lock_guard<std::mutex> lock(g_mu);
    if (slot >= g_used) return;
    g_slots[slot].ended = cudaEventRecord(g_slots[slot].end, st) == cudaSuccess;
}

}  // namespace vg

extern "C" {

int vg_prof_enable(int on) {
    std::lock_guard<std::mutex> lock(vg::g_mu);
    if (on) vg::g_used = 0;
    vg::g_on.store(on != 0);
    return VG_OK;
}

int vg_prof_read(int kernel, double* total_ms, int64_t* launches) {
    if (kernel < 0 || kernel >= vg::kProfKernels || total_ms == nullptr || launches == nullptr)
        return vg::set_error(VG_ERR_INVALID_ARG, "vg_prof_read: bad kernel id or null output");
    std::lock_guard<std::mutex> lock(vg::g_mu);
    double sum = 0.0;
    int64_t n = 0;
    for (int i = 0; i < vg::g_used; ++i) {
        const vg::Slot& s = vg::g_slots[i];
        if (s.kernel != kernel || !s.ended) continue;
        cudaError_t e = cudaEventSynchronize(s.end);
        float ms = 0.f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, s.begin, s.end);
        if (e != cudaSuccess) return vg::set_error(VG_ERR_CUDA, cudaGetErrorString(e));
        sum += ms;
        ++n;
    }
    *total_ms = sum;
    *launches = n;
    return VG_OK;
}

}  // extern "C"
