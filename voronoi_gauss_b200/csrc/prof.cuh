// Kernel timing for measurement (vg_prof_enable / vg_prof_read of the C ABI): while enabled, each
// instrumented launch is bracketed by a pair of CUDA events recorded on its own launch stream, so the
// host can read that kernel's device time inside a larger timed region. Disabled (the default), a scope
// costs one relaxed atomic load.
#pragma once

#include <cuda_runtime.h>

namespace vg {

// Kernel classes timed (the VG_PROF_* values of include/vgb200.h).
enum ProfKernel {
    kProfTraversal = 0,   // foam_forward_kernel: traversal of the interaction-point forward
    kProfColor = 1,       // cmf_color_kernel: cell-major colours
    kProfReplay = 2,      // foam_backward_kernel<items>: record replay writing the scatter's items
    kProfScatter = 3,     // cm_scatter_kernel: cell-major gradient scatter
    kProfInfer = 4,       // infer_kernel / trace_kernel: inference traversal (per ray)
    kProfMarchFwd = 5,    // march_forward_kernel
    kProfMarchItems = 6,  // march_items_kernel: march backward re-march writing items
    kProfInferColour = 7, // colour_kernel of the deferred inference pipeline
    kProfKernels = 8
};

int prof_begin(int kernel, cudaStream_t st);  // slot of the event pair, or -1 when not recording
void prof_end(int slot, cudaStream_t st);

struct ProfScope {
    int slot;
    cudaStream_t st;
    ProfScope(int kernel, cudaStream_t s) : slot(prof_begin(kernel, s)), st(s) {}
    ~ProfScope() { prof_end(slot, st); }
    ProfScope(const ProfScope&) = delete;
    ProfScope& operator=(const ProfScope&) = delete;
};

}  // namespace vg
