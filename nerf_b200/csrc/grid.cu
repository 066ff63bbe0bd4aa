// grid.cu -- standalone hash-grid encoder kernels (forward gather, backward
// scatter) over unit-cube points.  One thread per (point, level): the 16
// threads of a point write its 64-byte feature row contiguously.
#include "grid.cuh"
#include "kernels.h"

namespace nb {

LevelTable make_level_table(const GridLayout& g) {
    LevelTable t{};
    for (uint32_t l = 0; l < g.n_levels; ++l) {
        t.scale[l] = g.scale[l];
        t.res[l] = g.resolution[l];
        t.dense[l] = g.dense[l];
        t.offset[l] = g.offset[l];
    }
    t.n_levels = g.n_levels;
    t.hash_mask = (1u << g.log2_hashmap_size) - 1u;
    return t;
}

namespace {

__device__ __forceinline__ void load_levels(const LevelTable& lt, LevelParams* lv) {
    if (threadIdx.x < lt.n_levels) {
        const uint32_t l = threadIdx.x;
        lv[l] = LevelParams{lt.scale[l], lt.res[l], lt.dense[l], lt.offset[l]};
    }
    __syncthreads();
}

__global__ void __launch_bounds__(256) k_grid_forward(const LevelTable lt, const float* __restrict__ pos, uint32_t n,
                                                      const uint32_t* __restrict__ params, uint32_t* __restrict__ feat) {
    __shared__ LevelParams lv[kMaxLevels];
    load_levels(lt, lv);
    const uint64_t task = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t L = lt.n_levels;
    if (task >= static_cast<uint64_t>(n) * L) return;
    const uint32_t pt = static_cast<uint32_t>(task / L), l = static_cast<uint32_t>(task % L);
    const float p[3] = {pos[3ull * pt + 0], pos[3ull * pt + 1], pos[3ull * pt + 2]};
    feat[task] = level_forward(params, p, lv[l], lt.hash_mask);
}

__global__ void __launch_bounds__(256) k_grid_backward(const LevelTable lt, const float* __restrict__ pos, uint32_t n,
                                                       const uint32_t* __restrict__ dfeat, uint32_t* grad) {
    __shared__ LevelParams lv[kMaxLevels];
    load_levels(lt, lv);
    const uint64_t task = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t L = lt.n_levels;
    if (task >= static_cast<uint64_t>(n) * L) return;
    const uint32_t pt = static_cast<uint32_t>(task / L), l = static_cast<uint32_t>(task % L);
    const float p[3] = {pos[3ull * pt + 0], pos[3ull * pt + 1], pos[3ull * pt + 2]};
    const float2 d = unpack_h2(dfeat[task]);
    level_backward(grad, p, lv[l], lt.hash_mask, d.x, d.y);
}

}  // namespace

cudaError_t launch_grid_forward(const LevelTable& lt, const float* pos, uint32_t n, const void* params, void* feat,
                                cudaStream_t s) {
    if (n == 0u) return cudaSuccess;
    const uint64_t tasks = static_cast<uint64_t>(n) * lt.n_levels;
    const uint32_t blocks = static_cast<uint32_t>((tasks + 255u) / 256u);
    k_grid_forward<<<blocks, 256, 0, s>>>(lt, pos, n, static_cast<const uint32_t*>(params), static_cast<uint32_t*>(feat));
    return cudaGetLastError();
}

cudaError_t launch_grid_backward(const LevelTable& lt, const float* pos, uint32_t n, const void* dfeat, void* grad,
                                 cudaStream_t s) {
    if (n == 0u) return cudaSuccess;
    const uint64_t tasks = static_cast<uint64_t>(n) * lt.n_levels;
    const uint32_t blocks = static_cast<uint32_t>((tasks + 255u) / 256u);
    k_grid_backward<<<blocks, 256, 0, s>>>(lt, pos, n, static_cast<const uint32_t*>(dfeat), static_cast<uint32_t*>(grad));
    return cudaGetLastError();
}

}  // namespace nb
