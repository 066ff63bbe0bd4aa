// occupancy.cu -- occupancy-grid maintenance (reference backend-cuda.cu:1555-1634).
//
// The reference runs four full-grid kernels per refresh (decay, clear,
// max-update, rebuild with atomicOr).  Here one thread owns one 32-cell
// bitfield word: it decays its cells, folds in the densities of the cells
// that fall in this step's query window (computed by the field kernel in
// occupancy mode), stores the cells back and writes the word, so the grid is
// read and written once and the bitfield needs no atomics.
//   warm-up init (step 0): density = 1, every bit set
//   refresh: density = max(density * decay, sigma) for window cells,
//            density * decay elsewhere; bit = density > threshold
// The window is cells (start + k) mod C, k < update_count, with
// start = frame * update_count mod C.
#include "common.cuh"
#include "kernels.h"

namespace nb {
namespace {

__global__ void __launch_bounds__(256) k_occupancy_update(const OccupancyArgs a) {
    const uint32_t w = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t words = (a.cell_count + 31u) / 32u;
    if (w >= words) return;
    uint32_t mode, frame;
    if (a.direct) {
        mode = a.mode;
        frame = a.frame;
    } else {
        frame = a.state->frame_index;
        mode = occupancy_mode(frame, a.warmup_steps, a.update_interval);
    }
    const uint32_t C = a.cell_count;
    const bool whole = 32u * (w + 1u) <= C;  // the last word of a grid that is not a multiple of 32 goes cell by cell
    float4* d4 = reinterpret_cast<float4*>(a.density + 32ull * w);
    if (mode == kOccWarmupInit) {
        if (whole) {
#pragma unroll
            for (int q = 0; q < 8; ++q) d4[q] = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        } else {
            for (uint32_t c = 32u * w; c < C; ++c) a.density[c] = 1.0f;
        }
        a.bitfield[w] = 0xFFFFFFFFu;
        return;
    }
    if (mode != kOccRefresh) return;
    const uint32_t start = static_cast<uint32_t>(static_cast<unsigned long long>(frame) * a.update_count % C);
    uint32_t word = 0u;
    if (whole) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 v = d4[q];
            float* e = reinterpret_cast<float*>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t c = 32u * w + 4u * q + j;
                float d = __fmul_rn(e[j], a.decay);
                const uint32_t k = c >= start ? c - start : c + (C - start);
                if (k < a.update_count) d = fmaxf(d, a.occ_sigma[k]);
                e[j] = d;
                if (d > a.threshold) word |= 1u << (4u * q + j);
            }
            d4[q] = v;
        }
    } else {
        for (uint32_t c = 32u * w; c < C; ++c) {
            float d = __fmul_rn(a.density[c], a.decay);
            const uint32_t k = c >= start ? c - start : c + (C - start);
            if (k < a.update_count) d = fmaxf(d, a.occ_sigma[k]);
            a.density[c] = d;
            if (d > a.threshold) word |= 1u << (c - 32u * w);
        }
    }
    a.bitfield[w] = word;
}

}  // namespace

cudaError_t launch_occupancy_update(const OccupancyArgs& a, cudaStream_t s) {
    const uint32_t words = (a.cell_count + 31u) / 32u;
    if (words == 0u) return cudaSuccess;
    k_occupancy_update<<<(words + 255u) / 256u, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
