// noalloc.cu -- allocation-free variant of the fused field backward.
//
// nerf_b200_field_backward needs a scratch buffer for the per-CTA MLP
// weight-gradient partials, which its caller allocates.  Some callers cannot
// allocate device memory: a host application that owns the whole device
// memory budget and hands plugins only the buffers of a call (an engine or
// renderer plugin with a fixed pool), or a process where a cudaMalloc would
// synchronise the device and stall other work at the wrong moment.  This
// entry point keeps that scratch in a file-scope __device__ array instead,
// so a call allocates nothing; the caller still passes every input and
// output.
//
// The array holds kNoAllocPartialRows rows of 10240 floats (13.1 MB).  It is
// part of the module image, so every GPU that loads the library holds it
// until the process exits.  Its device address is looked up once per device
// with cudaGetSymbolAddress (in host code the symbol name is only a
// host-side stand-in, not a device address), on the first call made with
// that device current; make that first call before any stream capture.  The
// cached address belongs to the device's primary context: after a
// cudaDeviceReset the module is loaded again and the entry point must not be
// called any more in that process.  All
// calls share the array: each launch overwrites every row it uses before
// reading it, so no clearing is needed between calls, but calls whose
// kernels overlap on the GPU (different streams, or different host threads
// on the same device) race on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/nerf_b200.h"
#include "kernels.h"

namespace nb {
namespace {

constexpr uint32_t kNoAllocPartialRows = 320;  // >= 2 CTAs x 148 SMs on B200
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartialRows * kMlpParams];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_ptr[kMaxDevices] = {};

cudaError_t scratch_of_current_device(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess) return e;
        g_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace nb

extern "C" {

NERF_API uint32_t nerf_b200_field_backward_noalloc_max_rows(void) { return nb::kNoAllocPartialRows; }

NERF_API NerfStatus nerf_b200_field_backward_noalloc(const NerfB200GridLayout* layout, const void* params, const float* pos,
                                                     const float* dirs, uint32_t n, const void* feat, const float* dout,
                                                     void* grid_grad, float* mlp_grad, void* stream) {
    if (!layout || layout->n_levels != 16u || !params || !mlp_grad || !grid_grad) return NERF_STATUS_INVALID_USAGE;
    if (n && (!pos || !dirs || !feat || !dout)) return NERF_STATUS_INVALID_USAGE;
    if (n > 0x7FFFFFFFu) return NERF_STATUS_INVALID_USAGE;  // rows are indexed with 32-bit tile counters
    // The tables are read and reduced in 16-byte blocks.
    if ((reinterpret_cast<uintptr_t>(params) & 15u) || (reinterpret_cast<uintptr_t>(grid_grad) & 15u)) return NERF_STATUS_INVALID_USAGE;
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    // Same CTA count as nerf_b200_field_backward, so both give the same sums.
    const uint32_t blocks = nb::field_backward_blocks();
    if (blocks == 0u || blocks > nb::kNoAllocPartialRows) return NERF_STATUS_INVALID_USAGE;  // scratch too small for this GPU
    float* partials = nullptr;
    if (nb::scratch_of_current_device(&partials) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    nb::FieldArgs a{};
    a.lt = nb::make_level_table(*reinterpret_cast<const nb::GridLayout*>(layout));
    a.params16 = params;
    a.mlp_offset = 2u * layout->offset[layout->n_levels];
    a.n_direct = n;
    a.pos_unit = pos;
    a.dirs = dirs;
    a.feat = const_cast<void*>(feat);
    a.dout = reinterpret_cast<const float4*>(dout);
    a.grid_grad = grid_grad;
    a.partials = partials;
    if (nb::launch_field_backward(a, nb::kFieldDirect, blocks, s) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    nb::OptimArgs o{};
    o.partials = partials;
    o.n_partials = blocks;
    o.mlp_grad = mlp_grad;
    return nb::launch_wgrad_reduce(o, s) == cudaSuccess ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR;
}

}  // extern "C"
