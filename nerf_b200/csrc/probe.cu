// probe.cu -- L2 microbenchmarks for the roofline of the hash-grid kernels.
//
// Built into its own library, libnerf_b200_l2probe.so, which only the
// benchmark loads; the product library libnerf_b200.so does not contain it.
//
// The field kernels are bound by L2 (hash-table gathers in the forward,
// f16x2 reductions in the backward), for which no driver-measured peak
// exists.  These two probes measure it on the running GPU:
//   read  every thread streams 16-byte loads over an L2-resident buffer;
//   red   every thread issues red.global.add.noftz.f16x2 (or the 8-byte .v2
//         or 16-byte .v4 form) at hashed addresses of a buffer the size of a
//         hash table.
#include "common.cuh"

#include "probe.h"

namespace nb {
namespace {

__global__ void __launch_bounds__(256) k_probe_read(const uint4* __restrict__ buf, uint64_t n16, uint32_t passes,
                                                    uint32_t* sink) {
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint32_t acc = 0u;
    for (uint32_t p = 0; p < passes; ++p)
        for (uint64_t i = tid; i < n16; i += stride) {
            const uint4 v = __ldcg(buf + i);
            acc ^= v.x ^ v.y ^ v.z ^ v.w;
        }
    if (acc == 0x9E3779B9u) sink[tid & 1023u] = acc;  // keeps the loads live
}

__global__ void __launch_bounds__(256) k_probe_red(uint32_t* buf, uint32_t mask, uint32_t reps, uint32_t vec) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t v = pack_h2(1.0f / 1024.0f, -1.0f / 1024.0f);
    for (uint32_t i = 0; i < reps; ++i) {
        const uint32_t e = hash_u32(tid * 0x9E3779B9u + i) & mask;
        if (vec == 2u) {
            asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};\n" ::"l"(buf + (e & ~3u)), "r"(v), "r"(v),
                         "r"(v), "r"(v)
                         : "memory");
        } else if (vec == 1u) {
            asm volatile("red.global.add.noftz.v2.f16x2 [%0], {%1, %2};\n" ::"l"(buf + (e & ~1u)), "r"(v), "r"(v) : "memory");
        } else {
            red_add_f16x2(buf + e, v);
        }
    }
}

// Gathers at hashed addresses: the access pattern of the hash-table lookups
// (one sector per lane per load).  vec 0: 4-byte loads, 1: 8-byte loads of
// an aligned word pair.
__global__ void __launch_bounds__(256) k_probe_gather(const uint32_t* __restrict__ buf, uint32_t mask, uint32_t reps,
                                                      uint32_t vec, uint32_t* sink) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t acc = 0u;
#pragma unroll 8
    for (uint32_t i = 0; i < reps; ++i) {
        const uint32_t e = hash_u32(tid * 0x9E3779B9u + i) & mask;
        if (vec == 1u) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(buf + (e & ~1u)));
            acc ^= v.x ^ v.y;
        } else {
            acc ^= __ldg(buf + e);
        }
    }
    if (acc == 0x9E3779B9u) sink[tid & 1023u] = acc;  // keeps the loads live
}

uint32_t probe_blocks() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return static_cast<uint32_t>(sms) * 8u;
}

}  // namespace
}  // namespace nb

extern "C" {

NERF_API NerfStatus nerf_b200_probe_l2_read(const void* buf, uint64_t bytes, uint32_t passes, uint32_t* sink, void* stream) {
    if (!buf || !sink || bytes < 16u || (reinterpret_cast<uintptr_t>(buf) & 15u)) return NERF_STATUS_INVALID_USAGE;
    nb::k_probe_read<<<nb::probe_blocks(), 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(buf),
                                                                                         bytes / 16u, passes, sink);
    return cudaGetLastError() == cudaSuccess ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR;
}

NERF_API NerfStatus nerf_b200_probe_l2_red(void* buf, uint32_t words, uint32_t reps, uint32_t vec, uint64_t* ops,
                                           void* stream) {
    if (!buf || words < 4u || (words & (words - 1u)) || (reinterpret_cast<uintptr_t>(buf) & 15u) || vec > 2u)
        return NERF_STATUS_INVALID_USAGE;
    const uint32_t blocks = nb::probe_blocks();
    nb::k_probe_red<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t*>(buf), words - 1u, reps,
                                                                           vec);
    if (ops) *ops = static_cast<uint64_t>(blocks) * 256u * reps;
    return cudaGetLastError() == cudaSuccess ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR;
}

NERF_API NerfStatus nerf_b200_probe_l2_gather(const void* buf, uint32_t words, uint32_t reps, uint32_t vec, uint32_t* sink,
                                              uint64_t* ops, void* stream) {
    if (!buf || !sink || words < 4u || (words & (words - 1u)) || (reinterpret_cast<uintptr_t>(buf) & 15u) || vec > 1u)
        return NERF_STATUS_INVALID_USAGE;
    const uint32_t blocks = nb::probe_blocks();
    nb::k_probe_gather<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint32_t*>(buf), words - 1u,
                                                                              reps, vec, sink);
    if (ops) *ops = static_cast<uint64_t>(blocks) * 256u * reps;
    return cudaGetLastError() == cudaSuccess ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR;
}

}  // extern "C"
