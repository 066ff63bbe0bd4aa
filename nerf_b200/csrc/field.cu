// field.cu -- fused radiance-field kernels.
//
// The field maps a sample (unit-cube position, view direction) to raw density
// and raw colour:
//   features  = hash grid (16 levels x 2 fp16)                    32
//   density   = W1d relu(W0d features)                 32 -> 64 -> 16
//   colour    = W2c relu(W1c relu(W0c [density16, SH16(dir)]))   32 -> 64 -> 64 -> 16 (3 used)
// raw sigma is density[0]; sigma = exp(raw) (trunc_exp), rgb = sigmoid(raw rgb).
//
// Both kernels are persistent: each CTA of 4 warps loads the MLP weights
// once into padded shared memory and then walks 64-row tiles (16 rows per
// warp).  Matrix products use mma.sync m16n8k16 (fp16 operands, fp32
// accumulation) with activations chained through registers: the C fragment
// of one layer is the A fragment of the next.
//
// The backward kernel recomputes the forward from the stored hash features,
// back-propagates through both MLPs and accumulates the weight gradients of
// all five matrices over its tiles in registers (each warp owns a fixed
// quarter of the 10240 weights); the per-CTA sums go to a partials buffer,
// reduced by the statistics kernel (one GPU) or launch_wgrad_reduce.  The
// feature gradient goes to the hash table with fp16x2 reductions: from a
// separate kernel over the training rows (k_grid_scatter), in the kernel
// itself for the kernel-level entry points.
#include "grid.cuh"
#include "kernels.h"
#include "ray.cuh"

namespace nb {
namespace {

constexpr uint32_t kRows = 64;      // rows per tile
constexpr uint32_t kThreads = 128;  // 4 warps x 16 rows
constexpr uint32_t kL = 16;         // hash levels feeding the 32-wide MLP input
// Training rows written by the forward for the backward: 32 hash features
// (fp16), 16 SH coefficients (fp16) and the unit position (3 fp32 + pad):
// 112 bytes = 28 words.  The kernel-level entry points use plain 32-feature
// rows (16 words).
constexpr uint32_t kTrainRowU32 = 28, kFeatRowU32 = 16;

// Padded shared-memory copies of the five weight matrices (halves).
constexpr uint32_t kS32 = 40, kS64 = 72, kS16 = 24;
constexpr uint32_t kWD0 = 0;                  // 64 x 32
constexpr uint32_t kWD1 = kWD0 + 64 * kS32;   // 16 x 64
constexpr uint32_t kWC0 = kWD1 + 16 * kS64;   // 64 x 32
constexpr uint32_t kWC1 = kWC0 + 64 * kS32;   // 64 x 64
constexpr uint32_t kWC2 = kWC1 + 64 * kS64;   // 16 x 64
constexpr uint32_t kWTotal = kWC2 + 16 * kS64;


__device__ __forceinline__ void copy_matrix(__half* dst, uint32_t stride, const __half* src, uint32_t rows, uint32_t cols) {
    const uint32_t q = cols / 8u;
    for (uint32_t c = threadIdx.x; c < rows * q; c += blockDim.x) {
        const uint32_t r = c / q, k = (c % q) * 8u;
        *reinterpret_cast<uint4*>(dst + r * stride + k) = *reinterpret_cast<const uint4*>(src + r * cols + k);
    }
}

__device__ __forceinline__ void load_weights(__half* w, const __half* mlp, bool density_only) {
    copy_matrix(w + kWD0, kS32, mlp + kMlpD0, 64, 32);
    copy_matrix(w + kWD1, kS64, mlp + kMlpD1, 16, 64);
    if (density_only) return;
    copy_matrix(w + kWC0, kS32, mlp + kMlpC0, 64, 32);
    copy_matrix(w + kWC1, kS64, mlp + kMlpC1, 64, 64);
    copy_matrix(w + kWC2, kS64, mlp + kMlpC2, 16, 64);
}

// Real SH bands 0..3 of a unit direction; evaluation order and rounding
// identical to the CPU oracle's sh4().
__device__ __forceinline__ void sh4(float x, float y, float z, float o[16]) {
    const float xy = __fmul_rn(x, y), xz = __fmul_rn(x, z), yz = __fmul_rn(y, z);
    const float x2 = __fmul_rn(x, x), y2 = __fmul_rn(y, y), z2 = __fmul_rn(z, z);
    o[0] = 0.28209479177387814f;
    o[1] = __fmul_rn(-0.48860251190291987f, y);
    o[2] = __fmul_rn(0.48860251190291987f, z);
    o[3] = __fmul_rn(-0.48860251190291987f, x);
    o[4] = __fmul_rn(1.0925484305920792f, xy);
    o[5] = __fmul_rn(-1.0925484305920792f, yz);
    o[6] = __fsub_rn(__fmul_rn(0.94617469575755997f, z2), 0.31539156525251999f);
    o[7] = __fmul_rn(-1.0925484305920792f, xz);
    o[8] = __fsub_rn(__fmul_rn(0.54627421529603959f, x2), __fmul_rn(0.54627421529603959f, y2));
    o[9] = __fmul_rn(__fmul_rn(0.59004358992664352f, y), __fadd_rn(__fmul_rn(-3.0f, x2), y2));
    o[10] = __fmul_rn(__fmul_rn(2.8906114426405538f, xy), z);
    o[11] = __fmul_rn(__fmul_rn(0.45704579946446572f, y), __fsub_rn(1.0f, __fmul_rn(5.0f, z2)));
    o[12] = __fmul_rn(__fmul_rn(0.3731763325901154f, z), __fsub_rn(__fmul_rn(5.0f, z2), 3.0f));
    o[13] = __fmul_rn(__fmul_rn(0.45704579946446572f, x), __fsub_rn(1.0f, __fmul_rn(5.0f, z2)));
    o[14] = __fmul_rn(__fmul_rn(1.4453057213202769f, z), __fsub_rn(x2, y2));
    o[15] = __fmul_rn(__fmul_rn(0.59004358992664352f, x), __fadd_rn(-x2, __fmul_rn(3.0f, y2)));
}

// out[NT] (n-tiles of 8) = A[KC k-chunks of 16] x W^T with W stored [n][k].
template <int NT, int KC>
__device__ __forceinline__ void gemm_nk(float acc[NT][4], const uint32_t a[KC][4], const __half* W, uint32_t stride,
                                        uint32_t lane) {
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            load_b_nk(b, W, stride, np * 16u, kc * 16u, lane);
            mma16816(acc[2 * np], a[kc], b[0], b[1]);
            mma16816(acc[2 * np + 1], a[kc], b[2], b[3]);
        }
    }
}
// out[NT] = A[KC] x W with W stored [k][n] (the transpose product of the backward pass).
template <int NT, int KC>
__device__ __forceinline__ void gemm_kn(float acc[NT][4], const uint32_t a[KC][4], const __half* W, uint32_t stride,
                                        uint32_t lane) {
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            load_b_kn(b, W, stride, np * 16u, kc * 16u, lane);
            mma16816(acc[2 * np], a[kc], b[0], b[1]);
            mma16816(acc[2 * np + 1], a[kc], b[2], b[3]);
        }
    }
}

// C fragments (NT n-tiles) -> A fragments (NT/2 k-chunks) of the next layer.
template <int NT>
__device__ __forceinline__ void relu_to_a(const float acc[NT][4], uint32_t a[NT / 2][4]) {
#pragma unroll
    for (int kc = 0; kc < NT / 2; ++kc) {
        a[kc][0] = relu_pack_h2(acc[2 * kc][0], acc[2 * kc][1]);
        a[kc][1] = relu_pack_h2(acc[2 * kc][2], acc[2 * kc][3]);
        a[kc][2] = relu_pack_h2(acc[2 * kc + 1][0], acc[2 * kc + 1][1]);
        a[kc][3] = relu_pack_h2(acc[2 * kc + 1][2], acc[2 * kc + 1][3]);
    }
}
template <int NT>
__device__ __forceinline__ void mask_to_a(const float acc[NT][4], const uint32_t h[NT / 2][4], uint32_t a[NT / 2][4]) {
#pragma unroll
    for (int kc = 0; kc < NT / 2; ++kc) {
        a[kc][0] = relu_mask_h2(pack_h2(acc[2 * kc][0], acc[2 * kc][1]), h[kc][0]);
        a[kc][1] = relu_mask_h2(pack_h2(acc[2 * kc][2], acc[2 * kc][3]), h[kc][1]);
        a[kc][2] = relu_mask_h2(pack_h2(acc[2 * kc + 1][0], acc[2 * kc + 1][1]), h[kc][2]);
        a[kc][3] = relu_mask_h2(pack_h2(acc[2 * kc + 1][2], acc[2 * kc + 1][3]), h[kc][3]);
    }
}
// A fragment (k-chunk kc) of a warp's 16 rows -> row-major shared memory.
__device__ __forceinline__ void store_a(__half* base, uint32_t stride, uint32_t row0, uint32_t kc, const uint32_t a[4],
                                        uint32_t lane) {
    const uint32_t g = lane >> 2, t = lane & 3u;
    *reinterpret_cast<uint32_t*>(base + (row0 + g) * stride + kc * 16u + 2u * t) = a[0];
    *reinterpret_cast<uint32_t*>(base + (row0 + g + 8u) * stride + kc * 16u + 2u * t) = a[1];
    *reinterpret_cast<uint32_t*>(base + (row0 + g) * stride + kc * 16u + 8u + 2u * t) = a[2];
    *reinterpret_cast<uint32_t*>(base + (row0 + g + 8u) * stride + kc * 16u + 8u + 2u * t) = a[3];
}

// Shared memory of the forward kernel and the renderer (the renderer appends
// its slots after kFwdBase): weights | feat[64][40] | xc[64][40] | pos[64]
// (unit position) | levels.  The training forward appends two stages of the
// next tile's raw inputs (pos+dt, ray id), filled with cp.async.
struct Smem {
    __half* w;
    __half* feat;
    __half* xc;
    float4* pos;
    LevelParams* lv;
};
constexpr size_t kFwdBase = (kWTotal + 2 * kRows * kS32) * 2 + kRows * 16 + kMaxLevels * 16;
constexpr size_t kFwdStage = kRows * 16 + kRows * 4;
constexpr size_t kFwdSmem = kFwdBase + 2 * kFwdStage;

__device__ __forceinline__ Smem carve(unsigned char* raw) {
    Smem s{};
    s.w = reinterpret_cast<__half*>(raw);
    s.feat = s.w + kWTotal;
    s.xc = s.feat + kRows * kS32;
    s.pos = reinterpret_cast<float4*>(s.xc + kRows * kS32);
    s.lv = reinterpret_cast<LevelParams*>(s.pos + kRows);
    return s;
}
struct FwdStage {
    float4* pos;     // raw pos_dt of the tile
    uint32_t* sray;  // ray id of each row
};
__device__ __forceinline__ FwdStage fwd_stage(unsigned char* raw, uint32_t k) {
    FwdStage st;
    st.pos = reinterpret_cast<float4*>(raw + kFwdBase + k * kFwdStage);
    st.sray = reinterpret_cast<uint32_t*>(st.pos + kRows);
    return st;
}

// Shared memory of the backward kernel: weights | levels | activation
// staging for the weight gradients (hd, dhd, h1, dh1, h2, dh2 [64][72];
// dyd, dyc [64][24]) | two input stages (features [64][40], colour input
// [64][40] whose columns 16..31 hold the SH coefficients, unit position,
// upstream gradient), filled with cp.async one tile ahead.
struct BwdSmem {
    __half* w;
    LevelParams* lv;
    __half *hd, *dhd, *h1, *dh1, *h2, *dh2, *dyd, *dyc;
    __half2* runs;
};
struct BwdStage {
    __half* feat;
    __half* xc;
    float4* pos;
    float4* dout;
};
// The hash-table scatter takes dX through a per-warp [16 rows][kL + 1]
// f16x2 buffer (one row per lane of each half warp, see scatter_runs).
constexpr uint32_t kRunStride = kL + 1;
constexpr size_t kBwdFixed =
    kWTotal * 2 + kMaxLevels * 16 + (6 * kRows * kS64 + 2 * kRows * kS16) * 2 + (kThreads / 32) * 16 * kRunStride * 4;
constexpr size_t kBwdStage = 2 * kRows * kS32 * 2 + 2 * kRows * 16;
constexpr size_t kBwdSmem = kBwdFixed + 2 * kBwdStage;

__device__ __forceinline__ BwdSmem carve_bwd(unsigned char* raw) {
    BwdSmem s{};
    s.w = reinterpret_cast<__half*>(raw);
    s.lv = reinterpret_cast<LevelParams*>(s.w + kWTotal);
    __half* b = reinterpret_cast<__half*>(s.lv + kMaxLevels);
    s.hd = b;
    s.dhd = s.hd + kRows * kS64;
    s.h1 = s.dhd + kRows * kS64;
    s.dh1 = s.h1 + kRows * kS64;
    s.h2 = s.dh1 + kRows * kS64;
    s.dh2 = s.h2 + kRows * kS64;
    s.dyd = s.dh2 + kRows * kS64;
    s.dyc = s.dyd + kRows * kS16;
    s.runs = reinterpret_cast<__half2*>(s.dyc + kRows * kS16);
    return s;
}
__device__ __forceinline__ BwdStage bwd_stage(unsigned char* raw, uint32_t k) {
    BwdStage st;
    st.feat = reinterpret_cast<__half*>(raw + kBwdFixed + k * kBwdStage);
    st.xc = st.feat + kRows * kS32;
    st.pos = reinterpret_cast<float4*>(st.xc + kRows * kS32);
    st.dout = st.pos + kRows;
    return st;
}

__device__ __forceinline__ uint32_t row_count(const FieldArgs& a, int mode) {
    if (mode == kFieldTrain) return a.state->n_samples;
    if (mode == kFieldOccupancy) {
        const uint32_t m = occupancy_mode(a.state->frame_index, a.warmup_steps, a.update_interval);
        return m == kOccRefresh ? a.update_count : 0u;
    }
    return a.n_direct;
}

__device__ __forceinline__ void world_to_unit(const FieldArgs& a, const float pw[3], float u[3]) {
#pragma unroll
    for (int k = 0; k < 3; ++k) u[k] = clamp01(__fdiv_rn(__fsub_rn(pw[k], a.aabb_min[k]), a.aabb_size[k]));
}

__device__ __forceinline__ void write_sh(__half* xc_row, const float d[3], bool valid) {
    float sh[16];
    if (valid) {
        sh4(d[0], d[1], d[2], sh);
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) sh[k] = 0.0f;
    }
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = pack_h2(sh[2 * k], sh[2 * k + 1]);
    uint4* dst = reinterpret_cast<uint4*>(xc_row + 16u);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// Training forward: copies of the next tile's pos+dt and ray ids.
__device__ __forceinline__ void fwd_prefetch(const FieldArgs& a, const FwdStage& st, uint32_t row0, uint32_t n) {
    const uint32_t tid = threadIdx.x;
    if (tid < kRows) {
        const uint32_t r = row0 + tid;
        cp_async16(st.pos + tid, a.pos_dt + (r < n ? r : 0u), r < n);
    } else {
        const uint32_t i = tid - kRows;
        const uint32_t r = row0 + i;
        cp_async4(st.sray + i, a.sample_ray + (r < n ? r : 0u), r < n);
    }
}

// Per-row inputs of a tile: unit position -> s.pos, SH(dir) -> s.xc[:,16:32].
__device__ __forceinline__ void load_rows(const FieldArgs& a, int mode, const Smem& s, const FwdStage* st, uint32_t row0,
                                          uint32_t n) {
    const uint32_t tid = threadIdx.x;
    if (tid >= kRows) return;
    const uint32_t r = row0 + tid;
    float u[3] = {0.0f, 0.0f, 0.0f}, d[3] = {0.0f, 0.0f, 0.0f};
    const bool valid = r < n;
    if (valid) {
        if (mode == kFieldTrain) {
            const float4 p = st->pos[tid];
            const float pw[3] = {p.x, p.y, p.z};
            world_to_unit(a, pw, u);
            const RayRecord& ray = a.rays[st->sray[tid]];
            d[0] = ray.dir[0];
            d[1] = ray.dir[1];
            d[2] = ray.dir[2];
        } else if (mode == kFieldOccupancy) {
            // Cell (cascade after cascade, x fastest) of the round-robin window;
            // its centre in its cascade's box.
            const uint32_t R = a.grid_res, RRR = R * R * R;
            const uint32_t start =
                static_cast<uint32_t>(static_cast<unsigned long long>(a.state->frame_index) * a.update_count % a.cell_count);
            const uint32_t q = static_cast<uint32_t>((static_cast<unsigned long long>(start) + r) % a.cell_count);
            const uint32_t mip = q / RRR, cell = q - mip * RRR;
            const uint32_t z = cell / (R * R), rem = cell - z * R * R, y = rem / R, x = rem - y * R;
            const uint32_t ci[3] = {x, y, z};
            const float s = pow2f(mip);
            float c[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const float lo = mip == 0u ? a.casc.bmn[k] : __fsub_rn(a.casc.c[k], __fmul_rn(a.casc.h[k], s));
                const float step = __fdiv_rn(__fmul_rn(a.casc.bsize[k], s), static_cast<float>(R));
                c[k] = __fmaf_rn(__fadd_rn(static_cast<float>(ci[k]), 0.5f), step, lo);
            }
            world_to_unit(a, c, u);
        } else {
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                if (mode == kFieldDirect) u[k] = a.pos_unit[3ull * r + k];
                d[k] = a.dirs[3ull * r + k];
            }
        }
    }
    s.pos[tid] = make_float4(u[0], u[1], u[2], 0.0f);
    write_sh(s.xc + tid * kS32, d, valid && mode != kFieldOccupancy);
}

// Hash encode of a 64-row tile into feat[64][40] (level l in columns 2l,
// 2l+1).  Warp w takes levels w, w+4, w+8, w+12 and lane j rows j and j+32,
// so one gather instruction reads one level for 32 consecutive rows: on all
// but the finest levels consecutive samples of a ray (or neighbouring pixels
// of a render tile) share cells, and their loads fall into few sectors.  Two
// levels are looked up per round, so each lane has the loads of four
// (row, level) lookups -- 16 to 32 loads -- in flight before it waits.
// ok(row, pos) says whether a row is live; a dead row loads nothing and
// stores zeros.
template <class Gather = LevelGather, class Ok>
__device__ __forceinline__ void encode_rows(const uint32_t* __restrict__ P, const LevelParams* lv, uint32_t hash_mask,
                                            const float4* pos, __half* feat, Ok ok) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t ra = lane, rb = lane + 32u;
    const float4 pa4 = pos[ra], pb4 = pos[rb];
    const bool oka = ok(ra, pa4), okb = ok(rb, pb4);
    const float pa[3] = {oka ? pa4.x : 0.0f, oka ? pa4.y : 0.0f, oka ? pa4.z : 0.0f};
    const float pb[3] = {okb ? pb4.x : 0.0f, okb ? pb4.y : 0.0f, okb ? pb4.z : 0.0f};
#pragma unroll 1
    for (uint32_t i = 0; i < kL / 8u; ++i) {
        const uint32_t l0 = warp + 8u * i, l1 = l0 + 4u;
        const LevelParams lp0 = lv[l0], lp1 = lv[l1];
        Gather g[4];
        gather_level(P, pa, lp0, hash_mask, oka, g[0]);
        gather_level(P, pb, lp0, hash_mask, okb, g[1]);
        gather_level(P, pa, lp1, hash_mask, oka, g[2]);
        gather_level(P, pb, lp1, hash_mask, okb, g[3]);
        const uint32_t v0 = finish_level(g[0]), v1 = finish_level(g[1]), v2 = finish_level(g[2]), v3 = finish_level(g[3]);
        *reinterpret_cast<uint32_t*>(feat + ra * kS32 + 2u * l0) = oka ? v0 : 0u;
        *reinterpret_cast<uint32_t*>(feat + rb * kS32 + 2u * l0) = okb ? v1 : 0u;
        *reinterpret_cast<uint32_t*>(feat + ra * kS32 + 2u * l1) = oka ? v2 : 0u;
        *reinterpret_cast<uint32_t*>(feat + rb * kS32 + 2u * l1) = okb ? v3 : 0u;
    }
}

// Rows of a tile to global memory in 16-byte pieces, one row after another:
// training rows are features | SH | unit position (112 bytes), kernel-level
// rows features only (64 bytes).
__device__ __forceinline__ void store_rows(const FieldArgs& a, const Smem& s, int mode, uint32_t row0, uint32_t n) {
    const uint32_t q_per_row = mode == kFieldTrain ? kTrainRowU32 / 4u : kFeatRowU32 / 4u;
    uint4* dst = static_cast<uint4*>(a.feat);
    for (uint32_t c = threadIdx.x; c < kRows * q_per_row; c += kThreads) {
        const uint32_t r = c / q_per_row, q = c - r * q_per_row;
        if (row0 + r >= n) continue;
        const uint4 v = q < 4u ? *reinterpret_cast<const uint4*>(s.feat + r * kS32 + 8u * q)
                               : (q < 6u ? *reinterpret_cast<const uint4*>(s.xc + r * kS32 + 16u + 8u * (q - 4u))
                                         : *reinterpret_cast<const uint4*>(s.pos + r));
        dst[static_cast<unsigned long long>(row0 + r) * q_per_row + q] = v;
    }
}


__device__ __forceinline__ void load_levels(const LevelTable& lt, LevelParams* lv) {
    if (threadIdx.x < lt.n_levels) {
        const uint32_t l = threadIdx.x;
        lv[l] = LevelParams{lt.scale[l], lt.res[l], lt.dense[l], lt.offset[l]};
    }
}

// Forward chain of one warp's 16 rows.
struct Chain {
    uint32_t xd[2][4];
    uint32_t hd[4][4];
    float yd[2][4];
    uint32_t xc[2][4];
    uint32_t h1[4][4];
    uint32_t h2[4][4];
    float yc[2][4];
};
__device__ __forceinline__ void forward_density(const __half* w, const __half* feat, uint32_t wrow, uint32_t lane, Chain& c) {
    load_a_rowmajor(c.xd[0], feat, kS32, wrow, 0, lane);
    load_a_rowmajor(c.xd[1], feat, kS32, wrow, 16, lane);
    float acc[8][4];
    gemm_nk<8, 2>(acc, c.xd, w + kWD0, kS32, lane);
    relu_to_a<8>(acc, c.hd);
    gemm_nk<2, 4>(c.yd, c.hd, w + kWD1, kS64, lane);
}
__device__ __forceinline__ void forward_colour(const __half* w, const __half* xc, uint32_t wrow, uint32_t lane, Chain& c) {
    c.xc[0][0] = pack_h2(c.yd[0][0], c.yd[0][1]);
    c.xc[0][1] = pack_h2(c.yd[0][2], c.yd[0][3]);
    c.xc[0][2] = pack_h2(c.yd[1][0], c.yd[1][1]);
    c.xc[0][3] = pack_h2(c.yd[1][2], c.yd[1][3]);
    load_a_rowmajor(c.xc[1], xc, kS32, wrow, 16, lane);
    float acc[8][4];
    gemm_nk<8, 2>(acc, c.xc, w + kWC0, kS32, lane);
    relu_to_a<8>(acc, c.h1);
    gemm_nk<8, 4>(acc, c.h1, w + kWC1, kS64, lane);
    relu_to_a<8>(acc, c.h2);
    gemm_nk<2, 4>(c.yc, c.h2, w + kWC2, kS64, lane);
}

__global__ void __launch_bounds__(kThreads) k_field_forward(const FieldArgs a, const int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const Smem s = carve(smem_raw);
    const uint32_t n = row_count(a, mode);
    if (n == 0u) return;
    const __half* mlp = static_cast<const __half*>(a.params16) + a.mlp_offset;
    load_weights(s.w, mlp, mode == kFieldOccupancy);
    load_levels(a.lt, s.lv);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t n_tiles = (n + kRows - 1u) / kRows;
    const bool staged = mode == kFieldTrain;
    if (staged && blockIdx.x < n_tiles) fwd_prefetch(a, fwd_stage(smem_raw, 0), blockIdx.x * kRows, n);
    cp_async_commit();
    uint32_t it = 0;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t row0 = tile * kRows;
        const FwdStage cur = fwd_stage(smem_raw, it & 1u);
        if (staged && tile + gridDim.x < n_tiles) fwd_prefetch(a, fwd_stage(smem_raw, (it + 1u) & 1u), (tile + gridDim.x) * kRows, n);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();  // this tile's stage is visible; the previous tile is done with shared memory
        load_rows(a, mode, s, &cur, row0, n);
        __syncthreads();
        if (mode == kFieldMlp) {  // given features: 64-byte rows into feat[64][40]
            const uint4* src = static_cast<const uint4*>(a.feat);
            for (uint32_t c = threadIdx.x; c < kRows * 4u; c += kThreads) {
                const uint32_t r = c >> 2, q = c & 3u;
                const uint4 v = row0 + r < n ? src[static_cast<unsigned long long>(row0 + r) * 4u + q] : make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(s.feat + r * kS32 + q * 8u) = v;
            }
        } else {
            encode_rows(static_cast<const uint32_t*>(a.params16), s.lv, a.lt.hash_mask, s.pos, s.feat,
                        [&](uint32_t r, const float4&) { return row0 + r < n; });
        }
        __syncthreads();
        if ((mode == kFieldTrain || mode == kFieldDirect) && a.feat != nullptr) store_rows(a, s, mode, row0, n);
        const uint32_t wrow = warp * 16u;
        Chain c;
        forward_density(s.w, s.feat, wrow, lane, c);
        const uint32_t rA = row0 + wrow + g, rB = rA + 8u;
        if (mode == kFieldOccupancy) {
            if (t == 0u) {
                if (rA < n) a.occ_sigma[rA] = expf(c.yd[0][0]);
                if (rB < n) a.occ_sigma[rB] = expf(c.yd[0][2]);
            }
            continue;
        }
        forward_colour(s.w, s.xc, wrow, lane, c);
        const float bA = __shfl_down_sync(0xffffffffu, c.yc[0][0], 1);
        const float bB = __shfl_down_sync(0xffffffffu, c.yc[0][2], 1);
        if (t == 0u) {
            if (rA < n) a.raw[rA] = make_float4(c.yd[0][0], c.yc[0][0], c.yc[0][1], bA);
            if (rB < n) a.raw[rB] = make_float4(c.yd[0][2], c.yc[0][2], c.yc[0][3], bB);
        }
    }
    cp_async_wait<0>();
}

// Training forward without the MLPs (the tensor-core MLP kernel of mlp_tc.cu
// evaluates them from the rows written here): hash encode and SH of 64-row
// tiles, written as the 112-byte training rows.  No weights in shared memory,
// so more CTAs are resident to hide the gathers' latency.
constexpr size_t kEncBase = (2 * kRows * kS32) * 2 + kRows * 16 + kMaxLevels * 16;
constexpr size_t kEncSmem = kEncBase + 2 * kFwdStage;

__global__ void __launch_bounds__(kThreads) k_field_encode(const FieldArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem s{};
    s.w = nullptr;
    s.feat = reinterpret_cast<__half*>(smem_raw);
    s.xc = s.feat + kRows * kS32;
    s.pos = reinterpret_cast<float4*>(s.xc + kRows * kS32);
    s.lv = reinterpret_cast<LevelParams*>(s.pos + kRows);
    auto stage = [&](uint32_t k) {
        FwdStage st;
        st.pos = reinterpret_cast<float4*>(smem_raw + kEncBase + k * kFwdStage);
        st.sray = reinterpret_cast<uint32_t*>(st.pos + kRows);
        return st;
    };
    const uint32_t n = a.state->n_samples;
    if (n == 0u) return;
    load_levels(a.lt, s.lv);
    const uint32_t n_tiles = (n + kRows - 1u) / kRows;
    if (blockIdx.x < n_tiles) fwd_prefetch(a, stage(0), blockIdx.x * kRows, n);
    cp_async_commit();
    uint32_t it = 0;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t row0 = tile * kRows;
        const FwdStage cur = stage(it & 1u);
        if (tile + gridDim.x < n_tiles) fwd_prefetch(a, stage((it + 1u) & 1u), (tile + gridDim.x) * kRows, n);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();  // this tile's stage is visible; the previous tile's rows are stored
        load_rows(a, kFieldTrain, s, &cur, row0, n);
        __syncthreads();
        encode_rows(static_cast<const uint32_t*>(a.params16), s.lv, a.lt.hash_mask, s.pos, s.feat,
                    [&](uint32_t r, const float4&) { return row0 + r < n; });
        __syncthreads();
        store_rows(a, s, kFieldTrain, row0, n);
    }
    cp_async_wait<0>();
}

// ---- weight-gradient ownership: warp w accumulates 20 m16n8 tiles ----
// acc[NT] += (A_s^T)[m0:m0+16, rows] x B_s[rows, n0:n0+8NT] over the tile's 64 rows.
template <int NT>
__device__ __forceinline__ void wgrad_rows(float (*acc)[4], const __half* A_s, uint32_t sa, uint32_t m0, const __half* B_s,
                                           uint32_t sb, uint32_t n0, uint32_t lane) {
#pragma unroll
    for (uint32_t kc = 0; kc < kRows / 16u; ++kc) {
        uint32_t af[4];
        load_a_transposed(af, A_s, sa, m0, kc * 16u, lane);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            load_b_kn(b, B_s, sb, n0 + np * 16u, kc * 16u, lane);
            mma16816(acc[2 * np], af, b[0], b[1]);
            mma16816(acc[2 * np + 1], af, b[2], b[3]);
        }
    }
}
template <int NT>
__device__ __forceinline__ void store_wtiles(const float (*acc)[4], float* out, uint32_t mat, uint32_t in_dim, uint32_t m0,
                                             uint32_t n0, uint32_t lane) {
    const uint32_t g = lane >> 2, t = lane & 3u;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const uint32_t n = n0 + 8u * j + 2u * t;
        out[mat + (m0 + g) * in_dim + n] = acc[j][0];
        out[mat + (m0 + g) * in_dim + n + 1u] = acc[j][1];
        out[mat + (m0 + g + 8u) * in_dim + n] = acc[j][2];
        out[mat + (m0 + g + 8u) * in_dim + n + 1u] = acc[j][3];
    }
}

// Backward: copies of the next tile's inputs.  Training: the 112-byte rows of
// the forward (features -> feat, SH -> xc[:,16:32], unit position -> pos) and
// the upstream gradient.  Direct (kernel-level entry): 64-byte feature rows,
// unit positions and the upstream gradient (SH is computed in the tile).
__device__ __forceinline__ void bwd_prefetch(const FieldArgs& a, int mode, const BwdStage& st, uint32_t row0, uint32_t n) {
    const uint32_t tid = threadIdx.x;
    const uint4* gr = static_cast<const uint4*>(a.feat);
    if (mode == kFieldTrain) {
        for (uint32_t c = tid; c < kRows * 7u; c += kThreads) {
            const uint32_t r = c / 7u, q = c % 7u;
            const bool ok = row0 + r < n;
            void* dst = q < 4u ? static_cast<void*>(st.feat + r * kS32 + q * 8u)
                               : (q < 6u ? static_cast<void*>(st.xc + r * kS32 + 16u + (q - 4u) * 8u) : static_cast<void*>(st.pos + r));
            cp_async16(dst, gr + (ok ? static_cast<unsigned long long>(row0 + r) * 7u + q : 0ull), ok);
        }
    } else {
        for (uint32_t c = tid; c < kRows * 4u; c += kThreads) {
            const uint32_t r = c >> 2, q = c & 3u;
            const bool ok = row0 + r < n;
            cp_async16(st.feat + r * kS32 + q * 8u, gr + (ok ? static_cast<unsigned long long>(row0 + r) * 4u + q : 0ull), ok);
        }
        if (mode == kFieldDirect && tid >= kRows) {
            const uint32_t i = tid - kRows, r = row0 + i;
            const bool ok = r < n;
            float* pp = reinterpret_cast<float*>(st.pos + i);
#pragma unroll
            for (int k = 0; k < 3; ++k) cp_async4(pp + k, a.pos_unit + (ok ? 3ull * r + k : 0ull), ok);
        }
    }
    if (tid < kRows) {
        const uint32_t r = row0 + tid;
        const bool ok = r < n;
        cp_async16(st.dout + tid, a.dout + (ok ? r : 0u), ok);
    }
}

// Scatter of one level for the 16 rows of a half warp (row r in lane r of
// the half).  Consecutive rows are consecutive samples, mostly of one ray,
// and on all but the finest levels runs of them share a cell.  A segmented suffix sum
// of the per-corner contributions (w_c * dX rounded to f16x2, summed in f16x2
// like the L2 reductions they replace) leaves each run's total in its first
// row, which alone issues the corner reductions: fewer reductions, and far
// less contention on the hot entries of coarse levels.  Rows of levels whose
// cell coordinates do not pack into 30 bits (more than 1024 vertices per
// axis) never merge.
template <uint32_t W>
__device__ __forceinline__ void scatter_runs_w(uint32_t* G, const LevelParams lp, uint32_t hash_mask, const float p[3], bool ok,
                                               float d0, float d1, uint32_t r, uint32_t lane) {
    static_assert(W == 16u || W == 32u, "run width");
    constexpr uint32_t kFull = W == 32u ? 0xFFFFFFFFu : 0xFFFFu;
    uint32_t i[3];
    float f[3], w[8];
    level_cell(p, lp, i, f);
    const uint32_t key = (ok && lp.res <= 1024u) ? (i[0] | (i[1] << 10) | (i[2] << 20)) : (0x80000000u | lane);
    const uint32_t next = __shfl_down_sync(0xffffffffu, key, 1, W);
    const uint32_t ends = (__ballot_sync(0xffffffffu, r == W - 1u || next != key) >> (lane & ~(W - 1u))) & kFull;
    const uint32_t end = static_cast<uint32_t>(__ffs(ends & (kFull << r))) - 1u;  // last row of this run
    const bool head = r == 0u || ((ends >> (r - 1u)) & 1u);
    corner_weights(f, w);
    __half2 v[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) v[c] = __floats2half2_rn(w[c] * d0, w[c] * d1);
#pragma unroll
    for (uint32_t o = 1; o < W; o <<= 1) {
        const bool take = r + o <= end;
        if (!__any_sync(0xffffffffu, take)) break;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const __half2 x = __shfl_down_sync(0xffffffffu, v[c], o, W);
            if (take) v[c] = __hadd2(v[c], x);
        }
    }
    if (!(ok && head)) return;
    uint32_t e[8];
    corner_entries(i, lp, hash_mask, e);
#pragma unroll
    for (uint32_t c = 0; c < 8u; c += 2u)
        red_pair(G, e[c], e[c + 1], *reinterpret_cast<const uint32_t*>(&v[c]), *reinterpret_cast<const uint32_t*>(&v[c + 1]));
}
__device__ __forceinline__ void scatter_runs(uint32_t* G, const LevelParams lp, uint32_t hash_mask, const float p[3], bool ok,
                                             float d0, float d1, uint32_t r, uint32_t lane) {
    scatter_runs_w<16u>(G, lp, hash_mask, p, ok, d0, d1, r, lane);
}

// Hash-table scatter of the training backward: warp per 32 consecutive
// rows (lane = row), all 16 levels, runs of rows in one cell merged over the
// whole warp.  Inputs: the feature gradients (fp16 x 32 per row) and the unit
// positions of the training rows.
constexpr uint32_t kScatterThreads = 256;
__global__ void __launch_bounds__(kScatterThreads) k_grid_scatter(const FieldArgs a) {
    __shared__ LevelParams lv[kMaxLevels];
    __shared__ uint32_t dsm[kScatterThreads / 32u][32][kL + 1];  // each lane's row of feature gradients
    load_levels(a.lt, lv);
    __syncthreads();
    const uint32_t n = a.state->n_samples;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t warps = gridDim.x * (kScatterThreads / 32u);
    uint32_t* G = static_cast<uint32_t*>(a.grid_grad);
    const uint4* rows = static_cast<const uint4*>(a.feat);
    const uint4* dfe = static_cast<const uint4*>(a.dfeat);
    for (uint32_t wb = blockIdx.x * (kScatterThreads / 32u) + (threadIdx.x >> 5); wb * 32u < n; wb += warps) {
        const uint32_t r = wb * 32u + lane;
        const bool ok = r < n;
        const uint32_t rr = ok ? r : n - 1u;
        const uint4 pq = rows[static_cast<unsigned long long>(rr) * (kTrainRowU32 / 4u) + 6u];
        const float p[3] = {__uint_as_float(pq.x), __uint_as_float(pq.y), __uint_as_float(pq.z)};
        uint32_t* mine = dsm[threadIdx.x >> 5][lane];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 q = dfe[static_cast<unsigned long long>(rr) * 4u + k];
            mine[4 * k] = q.x;
            mine[4 * k + 1] = q.y;
            mine[4 * k + 2] = q.z;
            mine[4 * k + 3] = q.w;
        }
#pragma unroll 1
        for (uint32_t l = 0; l < kL; ++l) {
            const float2 d = unpack_h2(mine[l]);
            scatter_runs_w<32u>(G, lv[l], a.lt.hash_mask, p, ok, d.x, d.y, lane, lane);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 2) k_field_backward(const FieldArgs a, const int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const BwdSmem s = carve_bwd(smem_raw);
    const uint32_t n = row_count(a, mode);
    const __half* mlp = static_cast<const __half*>(a.params16) + a.mlp_offset;
    load_weights(s.w, mlp, false);
    load_levels(a.lt, s.lv);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint32_t* ggrad = static_cast<uint32_t*>(a.grid_grad);
    float acc[20][4];
#pragma unroll
    for (int i = 0; i < 20; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

    const uint32_t n_tiles = (n + kRows - 1u) / kRows;
    if (blockIdx.x < n_tiles) bwd_prefetch(a, mode, bwd_stage(smem_raw, 0), blockIdx.x * kRows, n);
    cp_async_commit();
    uint32_t it = 0;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t row0 = tile * kRows;
        const BwdStage cur = bwd_stage(smem_raw, it & 1u);
        if (tile + gridDim.x < n_tiles) bwd_prefetch(a, mode, bwd_stage(smem_raw, (it + 1u) & 1u), (tile + gridDim.x) * kRows, n);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();  // this tile's stage is visible; the previous tile's weight gradients are done
        const uint32_t wrow = warp * 16u;
        // Direct rows: each warp computes the SH of its own 16 rows.
        if (mode != kFieldTrain) {
            if (lane < 16u) {
                const uint32_t rr = wrow + lane;
                const bool ok = row0 + rr < n;
                float d[3] = {0.0f, 0.0f, 0.0f};
                if (ok)
                    for (int k = 0; k < 3; ++k) d[k] = a.dirs[3ull * (row0 + rr) + k];
                write_sh(cur.xc + rr * kS32, d, ok);
            }
            __syncwarp();
        }
        Chain c;
        forward_density(s.w, cur.feat, wrow, lane, c);
        forward_colour(s.w, cur.xc, wrow, lane, c);
#pragma unroll
        for (uint32_t kc = 0; kc < 4; ++kc) {
            store_a(s.hd, kS64, wrow, kc, c.hd[kc], lane);
            store_a(s.h1, kS64, wrow, kc, c.h1[kc], lane);
            store_a(s.h2, kS64, wrow, kc, c.h2[kc], lane);
        }
        store_a(cur.xc, kS32, wrow, 0, c.xc[0], lane);

        const float4 dA = cur.dout[wrow + g];  // zero-filled past the last row
        const float4 dB = cur.dout[wrow + g + 8u];
        uint32_t dyc[1][4];
        dyc[0][0] = t == 0u ? pack_h2(dA.y, dA.z) : (t == 1u ? pack_h2(dA.w, 0.0f) : 0u);
        dyc[0][1] = t == 0u ? pack_h2(dB.y, dB.z) : (t == 1u ? pack_h2(dB.w, 0.0f) : 0u);
        dyc[0][2] = 0u;
        dyc[0][3] = 0u;
        store_a(s.dyc, kS16, wrow, 0, dyc[0], lane);

        float acc64[8][4];
        uint32_t dh2[4][4], dh1[4][4];
        gemm_kn<8, 1>(acc64, dyc, s.w + kWC2, kS64, lane);
        mask_to_a<8>(acc64, c.h2, dh2);
        gemm_kn<8, 4>(acc64, dh2, s.w + kWC1, kS64, lane);
        mask_to_a<8>(acc64, c.h1, dh1);
        float dxc[2][4];
        gemm_kn<2, 4>(dxc, dh1, s.w + kWC0, kS32, lane);
        uint32_t dyd[1][4];
        dyd[0][0] = pack_h2(dxc[0][0] + (t == 0u ? dA.x : 0.0f), dxc[0][1]);
        dyd[0][1] = pack_h2(dxc[0][2] + (t == 0u ? dB.x : 0.0f), dxc[0][3]);
        dyd[0][2] = pack_h2(dxc[1][0], dxc[1][1]);
        dyd[0][3] = pack_h2(dxc[1][2], dxc[1][3]);
        uint32_t dhd[4][4];
        gemm_kn<8, 1>(acc64, dyd, s.w + kWD1, kS64, lane);
        mask_to_a<8>(acc64, c.hd, dhd);
        float dxd[4][4];
        gemm_kn<4, 4>(dxd, dhd, s.w + kWD0, kS32, lane);
#pragma unroll
        for (uint32_t kc = 0; kc < 4; ++kc) {
            store_a(s.dh2, kS64, wrow, kc, dh2[kc], lane);
            store_a(s.dh1, kS64, wrow, kc, dh1[kc], lane);
            store_a(s.dhd, kS64, wrow, kc, dhd[kc], lane);
        }
        store_a(s.dyd, kS16, wrow, 0, dyd[0], lane);

        // Hash-table gradient: dX (rounded to f16x2, the precision of the
        // table's gradient) is transposed through shared memory to one row per
        // lane.  Training: the rows go to dfeat for the scatter kernel.
        // Direct: each half warp scatters its 16 rows, half h taking levels
        // h, h+2, ..., with runs of rows in one cell merged (scatter_runs).
        __half2* runs = s.runs + warp * 16u * kRunStride;
#pragma unroll
        for (uint32_t nt = 0; nt < 4u; ++nt) {
            runs[g * kRunStride + 4u * nt + t] = __floats2half2_rn(dxd[nt][0], dxd[nt][1]);
            runs[(g + 8u) * kRunStride + 4u * nt + t] = __floats2half2_rn(dxd[nt][2], dxd[nt][3]);
        }
        __syncwarp();
        if (mode == kFieldTrain || mode == kFieldMlp) {
            uint32_t* df = static_cast<uint32_t*>(a.dfeat);
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) {
                const uint32_t idx = lane + 32u * k, rr = idx >> 4, wd = idx & 15u;
                if (row0 + wrow + rr < n)
                    df[static_cast<unsigned long long>(row0 + wrow + rr) * 16u + wd] =
                        *reinterpret_cast<const uint32_t*>(&runs[rr * kRunStride + wd]);
            }
        } else {
            const uint32_t r = lane & 15u, h = lane >> 4;
            const float4 p4 = cur.pos[wrow + r];
            const float p[3] = {p4.x, p4.y, p4.z};
            const bool ok = row0 + wrow + r < n;
#pragma unroll 1
            for (uint32_t k = 0; k < kL / 2u; ++k) {
                const uint32_t l = 2u * k + h;
                const float2 d = __half22float2(runs[r * kRunStride + l]);
                scatter_runs(ggrad, s.lv[l], a.lt.hash_mask, p, ok, d.x, d.y, r, lane);
            }
        }
        __syncthreads();

        // Weight gradients of the tile, summed into this warp's owned tiles.
        if (warp == 0u) {
#pragma unroll
            for (uint32_t mt = 0; mt < 4; ++mt) wgrad_rows<4>(acc + 4 * mt, s.dhd, kS64, 16u * mt, cur.feat, kS32, 0u, lane);
            wgrad_rows<4>(acc + 16, s.dyd, kS16, 0u, s.hd, kS64, 0u, lane);
        } else if (warp == 1u) {
            wgrad_rows<4>(acc, s.dyd, kS16, 0u, s.hd, kS64, 32u, lane);
#pragma unroll
            for (uint32_t mt = 0; mt < 4; ++mt) wgrad_rows<4>(acc + 4 + 4 * mt, s.dh1, kS64, 16u * mt, cur.xc, kS32, 0u, lane);
        } else if (warp == 2u) {
#pragma unroll
            for (uint32_t mt = 0; mt < 2; ++mt) wgrad_rows<8>(acc + 8 * mt, s.dh2, kS64, 16u * mt, s.h1, kS64, 0u, lane);
            wgrad_rows<4>(acc + 16, s.dyc, kS16, 0u, s.h2, kS64, 0u, lane);
        } else {
#pragma unroll
            for (uint32_t mt = 0; mt < 2; ++mt) wgrad_rows<8>(acc + 8 * mt, s.dh2, kS64, 32u + 16u * mt, s.h1, kS64, 0u, lane);
            wgrad_rows<4>(acc + 16, s.dyc, kS16, 0u, s.h2, kS64, 32u, lane);
        }
        __syncthreads();
    }
    cp_async_wait<0>();

    float* out = a.partials + static_cast<unsigned long long>(blockIdx.x) * kMlpParams;
    if (warp == 0u) {
#pragma unroll
        for (uint32_t mt = 0; mt < 4; ++mt) store_wtiles<4>(acc + 4 * mt, out, kMlpD0, 32u, 16u * mt, 0u, lane);
        store_wtiles<4>(acc + 16, out, kMlpD1, 64u, 0u, 0u, lane);
    } else if (warp == 1u) {
        store_wtiles<4>(acc, out, kMlpD1, 64u, 0u, 32u, lane);
#pragma unroll
        for (uint32_t mt = 0; mt < 4; ++mt) store_wtiles<4>(acc + 4 + 4 * mt, out, kMlpC0, 32u, 16u * mt, 0u, lane);
    } else if (warp == 2u) {
#pragma unroll
        for (uint32_t mt = 0; mt < 2; ++mt) store_wtiles<8>(acc + 8 * mt, out, kMlpC1, 64u, 16u * mt, 0u, lane);
        store_wtiles<4>(acc + 16, out, kMlpC2, 64u, 0u, 0u, lane);
    } else {
#pragma unroll
        for (uint32_t mt = 0; mt < 2; ++mt) store_wtiles<8>(acc + 8 * mt, out, kMlpC1, 64u, 32u + 16u * mt, 0u, lane);
        store_wtiles<4>(acc + 16, out, kMlpC2, 64u, 0u, 32u, lane);
    }
}

// ---------------------------------------------------------------------------
// Renderer.  Persistent CTAs of 4 warps own 64 ray slots.  Every round each
// live slot marches its ray to the next occupied sample (cone-angle steps,
// dt_min = chord / max_steps), the 64 samples go through the fused field as
// one tile, and each slot composites its sample front to back; a slot whose
// transmittance falls below the stop threshold, or whose march leaves the
// box, writes its pixel (white background, round-to-nearest RGBA8) and takes
// the next pixel from a device work counter.  Pixels are enumerated tile by
// tile over the tiles this rank owns (tile t belongs to rank t mod world).
// ---------------------------------------------------------------------------
struct alignas(16) RenderSlot {
    float o[3], d[3];
    float t, tf, dt_min;
    float T, acc0, acc1, acc2;
    uint32_t i, pixel, n, live;  // live: 0 empty, 1 marching, 2 no work left
};
constexpr size_t kRenderSmem = kFwdBase + kRows * sizeof(RenderSlot) + kRows * 16 + kRows * 4;

__device__ __forceinline__ uint32_t pack_rgba(float r, float g, float b) {
    const uint32_t ur = __float2uint_rn(fminf(1.0f, fmaxf(0.0f, r)) * 255.0f);
    const uint32_t ug = __float2uint_rn(fminf(1.0f, fmaxf(0.0f, g)) * 255.0f);
    const uint32_t ub = __float2uint_rn(fminf(1.0f, fmaxf(0.0f, b)) * 255.0f);
    return (255u << 24) | (ub << 16) | (ug << 8) | ur;
}

__global__ void __launch_bounds__(kThreads) k_render(const RenderArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const Smem s = carve(smem_raw);
    RenderSlot* slots = reinterpret_cast<RenderSlot*>(smem_raw + kFwdBase);
    float4* raw_s = reinterpret_cast<float4*>(slots + kRows);
    float* dt_s = reinterpret_cast<float*>(raw_s + kRows);
    const __half* mlp = static_cast<const __half*>(a.params16) + a.mlp_offset;
    load_weights(s.w, mlp, false);
    if (threadIdx.x < a.lt.n_levels) {
        const uint32_t l = threadIdx.x;
        s.lv[l] = LevelParams{a.lt.scale[l], a.lt.res[l], a.lt.dense[l], a.lt.offset[l]};
    }
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t g = lane >> 2, t4 = lane & 3u;
    const AabbConsts box = make_box(a.aabb_min, a.aabb_max, a.aabb_size, a.casc);
    const float cone = cone_angle(a.fx, a.fy);
    // Work enumeration over this rank's tiles.
    const uint32_t tile = a.tile;
    uint32_t tiles_x = 1u, total_q;
    if (tile == 0u) {
        total_q = a.width * a.height;
    } else {
        tiles_x = (a.width + tile - 1u) / tile;
        const uint32_t tiles_y = (a.height + tile - 1u) / tile;
        const uint32_t n_tiles = tiles_x * tiles_y;
        const uint32_t mine = a.tile_rank < n_tiles ? (n_tiles - a.tile_rank + a.tile_world - 1u) / a.tile_world : 0u;
        total_q = mine * tile * tile;
    }
    if (tid < kRows) slots[tid].live = 0u;
    unsigned long long my_samples = 0ull;
    __syncthreads();
    for (;;) {
        bool has_row = false;
        if (tid < kRows) {
            RenderSlot& S = slots[tid];
            for (;;) {
                if (S.live == 2u) break;
                if (S.live == 0u) {
                    const uint32_t q = atomicAdd(a.work_counter, 1u);
                    if (q >= total_q) {
                        S.live = 2u;
                        break;
                    }
                    uint32_t x, y;
                    if (tile == 0u) {
                        x = q % a.width;
                        y = q / a.width;
                    } else {
                        const uint32_t k = q / (tile * tile), p = q % (tile * tile);
                        const uint32_t tt = a.tile_rank + k * a.tile_world;
                        x = (tt % tiles_x) * tile + p % tile;
                        y = (tt / tiles_x) * tile + p / tile;
                        if (x >= a.width || y >= a.height) continue;
                    }
                    const uint32_t pixel = y * a.width + x;
                    Ray ray;
                    const bool hit = camera_ray(a.c2w, a.fx, a.fy, a.cx, a.cy, static_cast<float>(a.height),
                                                __fadd_rn(static_cast<float>(x), 0.5f), __fadd_rn(static_cast<float>(y), 0.5f), ray) &&
                                     clip_aabb(box, ray);
                    if (!hit) {
                        a.rgba[pixel] = pack_rgba(1.0f, 1.0f, 1.0f);
                        if (a.spp) a.spp[pixel] = 0u;
                        continue;
                    }
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        S.o[k] = ray.o[k];
                        S.d[k] = ray.d[k];
                    }
                    S.t = ray.tn;
                    S.tf = ray.tf;
                    S.dt_min = __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(a.max_steps));
                    S.T = 1.0f;
                    S.acc0 = S.acc1 = S.acc2 = 0.0f;
                    S.i = 0u;
                    S.n = 0u;
                    S.pixel = pixel;
                    S.live = 1u;
                }
                // March to the next occupied sample.
                Ray ray;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    ray.o[k] = S.o[k];
                    ray.d[k] = S.d[k];
                }
                float t = S.t, dt = 0.0f, p[3];
                uint32_t i = S.i;
                bool found = false;
                while (t < S.tf && i < a.max_steps) {
                    dt = march_dt(t, S.tf, S.dt_min, cone);
                    ray_point(ray, march_mid(t, dt), p);
                    t = __fadd_rn(t, dt);
                    ++i;
                    if (occupied(a.bitfield, a.grid_res, box, p)) {
                        found = true;
                        break;
                    }
                }
                S.t = t;
                S.i = i;
                if (found) {
                    float u[3];
#pragma unroll
                    for (int k = 0; k < 3; ++k) u[k] = clamp01(__fdiv_rn(__fsub_rn(p[k], box.mn[k]), box.size[k]));
                    s.pos[tid] = make_float4(u[0], u[1], u[2], 1.0f);
                    dt_s[tid] = fmaxf(0.0f, dt);
                    float sh[16];
                    sh4(ray.d[0], ray.d[1], ray.d[2], sh);
                    uint32_t* dst = reinterpret_cast<uint32_t*>(s.xc + tid * kS32 + 16u);
#pragma unroll
                    for (int k = 0; k < 8; ++k) dst[k] = pack_h2(sh[2 * k], sh[2 * k + 1]);
                    has_row = true;
                    break;
                }
                a.rgba[S.pixel] = pack_rgba(S.acc0 + S.T, S.acc1 + S.T, S.acc2 + S.T);
                if (a.spp) a.spp[S.pixel] = S.n;
                S.live = 0u;
            }
            if (!has_row) s.pos[tid] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (!__syncthreads_or(has_row)) break;
        // Encode the tile's live rows (16-byte corner-pair loads: fewer sectors per pixel).
        encode_rows<LevelGatherWide>(static_cast<const uint32_t*>(a.params16), s.lv, a.lt.hash_mask, s.pos, s.feat,
                    [](uint32_t, const float4& p) { return p.w > 0.0f; });
        __syncthreads();
        {
            const uint32_t wrow = warp * 16u;
            Chain c;
            forward_density(s.w, s.feat, wrow, lane, c);
            forward_colour(s.w, s.xc, wrow, lane, c);
            const float bA = __shfl_down_sync(0xffffffffu, c.yc[0][0], 1);
            const float bB = __shfl_down_sync(0xffffffffu, c.yc[0][2], 1);
            if (t4 == 0u) {
                raw_s[wrow + g] = make_float4(c.yd[0][0], c.yc[0][0], c.yc[0][1], bA);
                raw_s[wrow + g + 8u] = make_float4(c.yd[0][2], c.yc[0][2], c.yc[0][3], bB);
            }
        }
        __syncthreads();
        if (tid < kRows && s.pos[tid].w > 0.0f) {
            RenderSlot& S = slots[tid];
            const float4 r = raw_s[tid];
            const float al = __fsub_rn(1.0f, expf(-__fmul_rn(expf(r.x), dt_s[tid])));
            const float w = __fmul_rn(S.T, al);
            S.acc0 = __fadd_rn(S.acc0, __fmul_rn(w, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-r.y)))));
            S.acc1 = __fadd_rn(S.acc1, __fmul_rn(w, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-r.z)))));
            S.acc2 = __fadd_rn(S.acc2, __fmul_rn(w, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-r.w)))));
            S.T = __fmul_rn(S.T, __fsub_rn(1.0f, al));
            ++S.n;
            ++my_samples;
            if (a.stop_transmittance > 0.0f && S.T < a.stop_transmittance) {
                a.rgba[S.pixel] = pack_rgba(S.acc0 + S.T, S.acc1 + S.T, S.acc2 + S.T);
                if (a.spp) a.spp[S.pixel] = S.n;
                S.live = 0u;
            }
        }
        __syncthreads();
    }
    if (a.total_samples && tid < kRows && my_samples) atomicAdd(a.total_samples, my_samples);
}

uint32_t g_render_blocks = 0;

uint32_t g_fwd_blocks = 0, g_bwd_blocks = 0, g_enc_blocks = 0;

}  // namespace

cudaError_t field_init_attributes() {
    cudaError_t e = cudaFuncSetAttribute(k_field_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFwdSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_field_backward, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBwdSmem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, f = 0, b = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&f, k_field_forward, kThreads, kFwdSmem)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_field_backward, kThreads, kBwdSmem)) != cudaSuccess) return e;
    g_fwd_blocks = static_cast<uint32_t>(sms * (f > 0 ? f : 1));
    e = cudaFuncSetAttribute(k_render, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kRenderSmem));
    if (e != cudaSuccess) return e;
    int r = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, k_render, kThreads, kRenderSmem)) != cudaSuccess) return e;
    g_render_blocks = static_cast<uint32_t>(sms * (r > 0 ? r : 1));
    e = cudaFuncSetAttribute(k_field_encode, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kEncSmem));
    if (e != cudaSuccess) return e;
    int en = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&en, k_field_encode, kThreads, kEncSmem)) != cudaSuccess) return e;
    g_enc_blocks = static_cast<uint32_t>(sms * (en > 0 ? en : 1));
    g_bwd_blocks = static_cast<uint32_t>(sms * (b > 0 ? b : 1));
    return cudaSuccess;
}
uint32_t field_forward_blocks() { return g_fwd_blocks; }
uint32_t field_backward_blocks() { return g_bwd_blocks; }

cudaError_t launch_field_forward(const FieldArgs& a, int mode, uint32_t blocks, cudaStream_t s) {
    if (blocks == 0u) return cudaErrorInvalidValue;
    k_field_forward<<<blocks, kThreads, kFwdSmem, s>>>(a, mode);
    return cudaGetLastError();
}
cudaError_t launch_field_encode(const FieldArgs& a, cudaStream_t s) {
    if (g_enc_blocks == 0u || a.feat == nullptr) return cudaErrorInvalidValue;
    k_field_encode<<<g_enc_blocks, kThreads, kEncSmem, s>>>(a);
    return cudaGetLastError();
}
cudaError_t launch_render(const RenderArgs& a, cudaStream_t s) {
    if (g_render_blocks == 0u) return cudaErrorInitializationError;
    k_render<<<g_render_blocks, kThreads, kRenderSmem, s>>>(a);
    return cudaGetLastError();
}
cudaError_t render_init_attributes() { return field_init_attributes(); }

cudaError_t launch_field_backward(const FieldArgs& a, int mode, uint32_t blocks, cudaStream_t s) {
    if (blocks == 0u) return cudaErrorInvalidValue;
    if ((mode == kFieldTrain || mode == kFieldMlp) && a.dfeat == nullptr) return cudaErrorInvalidValue;
    k_field_backward<<<blocks, kThreads, kBwdSmem, s>>>(a, mode);
    return cudaGetLastError();
}

cudaError_t launch_grid_scatter(const FieldArgs& a, cudaStream_t s) {
    if (a.dfeat == nullptr || a.grid_grad == nullptr) return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    k_grid_scatter<<<static_cast<uint32_t>(sms) * 8u, kScatterThreads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
