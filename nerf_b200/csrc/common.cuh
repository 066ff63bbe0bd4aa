// common.cuh -- device helpers shared by the sm_100a kernels of libnerf_b200.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "types.h"

#define NB_DEV __device__ __forceinline__

namespace nb {

// ---------------------------------------------------------------------------
// Integer hashing (same function as reference backend-cuda.cu:321-328 and
// :1439-1446) and the uniform draw built on it (:329-332).
// ---------------------------------------------------------------------------
NB_DEV uint32_t hash_u32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}
NB_DEV float rand01(uint32_t seed) {
    return __fdiv_rn(static_cast<float>(hash_u32(seed) & 0x00FFFFFFu), 16777216.0f);
}
NB_DEV uint32_t train_camera(uint32_t frame, uint32_t n_images) {
    return hash_u32(frame * 747796405u + 2891336453u) % n_images;
}
NB_DEV uint32_t occupancy_mode(uint32_t frame, uint32_t warmup, uint32_t interval) {
    if (frame < warmup) return frame == 0u ? kOccWarmupInit : kOccNone;
    return (interval != 0u && frame % interval == 0u) ? kOccRefresh : kOccNone;
}

// ---------------------------------------------------------------------------
// fp16 packing
// ---------------------------------------------------------------------------
NB_DEV uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
NB_DEV float2 unpack_h2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}
NB_DEV float h2f_bits(uint16_t b) {
    __half h = *reinterpret_cast<__half*>(&b);
    return __half2float(h);
}
// Keeps lanes of a packed f16x2 where the mask pair is > 0, zero elsewhere.
NB_DEV uint32_t relu_mask_h2(uint32_t v, uint32_t mask_src) {
    const __half2 m = *reinterpret_cast<__half2*>(&mask_src);
    return v & __hgt2_mask(m, __float2half2_rn(0.0f));  // 0xFFFF per lane where m > 0
}
// ReLU of two fp32 values packed to f16x2.
NB_DEV uint32_t relu_pack_h2(float lo, float hi) { return pack_h2(fmaxf(lo, 0.0f), fmaxf(hi, 0.0f)); }

// ---------------------------------------------------------------------------
// Tensor-core fragments (mma.sync m16n8k16, fp16 in, fp32 accumulate) and
// shared-memory matrix loads.
// A (16x16, row-major): a0 rows 0-7/k 0-7, a1 rows 8-15/k 0-7, a2 rows 0-7/k 8-15, a3 rows 8-15/k 8-15.
// B (16x8, col): b0 k 0-7, b1 k 8-15.  C (16x8): c0,c1 row g cols 2t,2t+1; c2,c3 row g+8.
// with g = lane/4, t = lane%4.
// ---------------------------------------------------------------------------
NB_DEV void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
NB_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
NB_DEV void ldsm_x4(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
NB_DEV void ldsm_x4_t(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

// A fragment of a row-major [row][k] fp16 matrix in shared memory (row stride in halves).
NB_DEV void load_a_rowmajor(uint32_t a[4], const __half* base, uint32_t stride, uint32_t row0, uint32_t k0, uint32_t lane) {
    const uint32_t mi = lane >> 3;
    const uint32_t r = row0 + (lane & 7u) + (mi & 1u) * 8u;
    const uint32_t k = k0 + (mi >> 1) * 8u;
    ldsm_x4(a, base + r * stride + k);
}
// A fragment of A = S^T where S is stored [k][m] (m contiguous): A[m][k] = S[k][m].
NB_DEV void load_a_transposed(uint32_t a[4], const __half* base, uint32_t stride, uint32_t m0, uint32_t k0, uint32_t lane) {
    const uint32_t mi = lane >> 3;
    const uint32_t k = k0 + (lane & 7u) + (mi >> 1) * 8u;
    const uint32_t m = m0 + (mi & 1u) * 8u;
    ldsm_x4_t(a, base + k * stride + m);
}
// B fragments of two n-tiles (n0, n0+8) for B[k][n] = W[n][k], W stored [n][k] (k contiguous).
// b[0],b[1] -> tile n0; b[2],b[3] -> tile n0+8.
NB_DEV void load_b_nk(uint32_t b[4], const __half* base, uint32_t stride, uint32_t n0, uint32_t k0, uint32_t lane) {
    const uint32_t mi = lane >> 3;
    const uint32_t n = n0 + (lane & 7u) + (mi >> 1) * 8u;
    const uint32_t k = k0 + (mi & 1u) * 8u;
    ldsm_x4(b, base + n * stride + k);
}
// B fragments of two n-tiles for B stored [k][n] (n contiguous).
NB_DEV void load_b_kn(uint32_t b[4], const __half* base, uint32_t stride, uint32_t n0, uint32_t k0, uint32_t lane) {
    const uint32_t mi = lane >> 3;
    const uint32_t k = k0 + (lane & 7u) + (mi & 1u) * 8u;
    const uint32_t n = n0 + (mi >> 1) * 8u;
    ldsm_x4_t(b, base + k * stride + n);
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (cp.async); a copy with valid == false
// reads nothing and zero-fills its destination.
// ---------------------------------------------------------------------------
NB_DEV void cp_async16(void* smem, const void* gmem, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
NB_DEV void cp_async4(void* smem, const void* gmem, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 4 : 0)
                 : "memory");
}
NB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
NB_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// Global atomics
// ---------------------------------------------------------------------------
// Adds a packed f16x2 to global memory at L2 without returning the old value.
NB_DEV void red_add_f16x2(void* gptr, uint32_t v) {
    asm volatile("red.global.add.noftz.f16x2 [%0], %1;\n" ::"l"(gptr), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
NB_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
NB_DEV uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace nb
