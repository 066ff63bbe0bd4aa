// mlp_tc.cu -- the field MLPs on the 5th-generation tensor cores (tcgen05).
//
// Same network as field.cu (density 32 -> 64 -> 16, colour [density16, SH16]
// -> 64 -> 64 -> 16, ReLU, fp16 operands rounded at the same points, fp32
// accumulation), evaluated on 128-row tiles with tcgen05.mma: one thread
// issues each layer's MMAs (M = 128 rows, N = 64 or 16 outputs, K = 16 per
// instruction) from shared-memory operands into a tensor-memory accumulator;
// an mbarrier signals completion; every thread then loads its own row from
// tensor memory (row r = lane r), applies the activation, rounds to fp16 and
// writes the row back to shared memory as the next layer's A operand.
// Operands use the K-major interleaved layout of umma.cuh; the weights are
// staged once per CTA.  Persistent CTAs of 4 warps, one tile at a time; the
// CTAs resident on an SM overlap each other's layer round trips.
//
// Every wait on the mbarrier is bounded (one second); a CTA whose MMAs do not
// complete sets the error word, frees its tensor memory and returns.
#include "kernels.h"
#include "umma.cuh"

namespace nb {
namespace {

constexpr uint32_t kTcRows = 128;
constexpr uint32_t kTcThreads = 128;
constexpr uint32_t kTcCols = 64;  // tensor-memory columns per CTA (largest layer output)
// Shared memory (bytes): weights in K-major interleaved layout, the 128 x 32
// layer input (features, then the colour input) and the 128 x 64 hidden layer.
constexpr uint32_t kOffWd0 = 0;              // 64 x 32
constexpr uint32_t kOffWd1 = kOffWd0 + 4096;  // 16 x 64
constexpr uint32_t kOffWc0 = kOffWd1 + 2048;  // 64 x 32
constexpr uint32_t kOffWc1 = kOffWc0 + 4096;  // 64 x 64
constexpr uint32_t kOffWc2 = kOffWc1 + 8192;  // 16 x 64
constexpr uint32_t kOffX = kOffWc2 + 2048;    // 128 x 32
constexpr uint32_t kOffH = kOffX + 8192;      // 128 x 64
constexpr uint32_t kOffBar = kOffH + 16384;   // mbarrier, tensor-memory base
constexpr uint32_t kTcSmem = kOffBar + 16;
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// Row-major [n][k] fp16 weights -> K-major interleaved.
__device__ __forceinline__ void stage_weights(unsigned char* smem, uint32_t off, const __half* w, uint32_t N, uint32_t K) {
    const uint32_t chunks = N * K / 8u;
    for (uint32_t c = threadIdx.x; c < chunks; c += blockDim.x) {
        const uint32_t n = c / (K / 8u), j = c % (K / 8u);
        *reinterpret_cast<uint4*>(smem + off + umma::interleaved_offset(n, 8u * j, K)) =
            *reinterpret_cast<const uint4*>(w + n * K + 8u * j);
    }
}

// Real SH bands 0..3 (the same evaluation as field.cu's sh4).
__device__ __forceinline__ void sh4_tc(float x, float y, float z, float o[16]) {
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

// Eight fp16 values (packed pairs) -> one 16-byte chunk of row r, columns 8j..8j+7.
__device__ __forceinline__ void put_chunk(unsigned char* smem, uint32_t off, uint32_t r, uint32_t j, uint32_t K,
                                          const uint32_t w[4]) {
    *reinterpret_cast<uint4*>(smem + off + umma::interleaved_offset(r, 8u * j, K)) = make_uint4(w[0], w[1], w[2], w[3]);
}

enum : int { kTcRowsMlp = 0, kTcRowsTrain = 1 };

// One row's inputs, loaded a tile ahead of their use: 32 fp16 features, and
// either the 16 fp16 SH coefficients of a training row or the view direction
// of a feature row; the backward also takes the loss-scaled d raw.
struct RowIn {
    uint4 f[4];
    uint4 sh[2];
    float d[3];
    float4 dout;
};
template <int kRowsMode, bool kBwd>
__device__ __forceinline__ void load_row(RowIn& in, const uint4* __restrict__ rows, const float* __restrict__ dirs,
                                         const float4* __restrict__ dout, uint32_t g, bool live) {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    const unsigned long long q = kRowsMode == kTcRowsTrain ? 7ull : 4ull;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) in.f[k] = live ? rows[q * g + k] : z;
    if (kRowsMode == kTcRowsTrain) {
        in.sh[0] = live ? rows[7ull * g + 4] : z;
        in.sh[1] = live ? rows[7ull * g + 5] : z;
    } else {
#pragma unroll
        for (uint32_t k = 0; k < 3u; ++k) in.d[k] = live ? dirs[3ull * g + k] : 0.0f;
    }
    if (kBwd) in.dout = live ? dout[g] : make_float4(0.f, 0.f, 0.f, 0.f);
}
// Features -> row r of the 128 x 32 matrix at x_off; the 16 SH coefficients
// (packed fp16 pairs) -> shp.
template <int kRowsMode>
__device__ __forceinline__ void put_row(unsigned char* smem, uint32_t x_off, uint32_t r, const RowIn& in, bool live,
                                        uint32_t shp[8]) {
#pragma unroll
    for (uint32_t q = 0; q < 4u; ++q) {
        const uint32_t w[4] = {in.f[q].x, in.f[q].y, in.f[q].z, in.f[q].w};
        put_chunk(smem, x_off, r, q, 32u, w);
    }
    if (kRowsMode == kTcRowsTrain) {
        shp[0] = in.sh[0].x; shp[1] = in.sh[0].y; shp[2] = in.sh[0].z; shp[3] = in.sh[0].w;
        shp[4] = in.sh[1].x; shp[5] = in.sh[1].y; shp[6] = in.sh[1].z; shp[7] = in.sh[1].w;
    } else {
        float sh[16];
        if (live) {
            sh4_tc(in.d[0], in.d[1], in.d[2], sh);
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) sh[k] = 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) shp[k] = pack_h2(sh[2 * k], sh[2 * k + 1]);
    }
}

// 64 accumulator columns of this thread's row -> ReLU -> fp16 -> row r of the
// 128 x 64 activation at byte offset dst.
__device__ __forceinline__ void relu_row_to_act(unsigned char* smem, uint32_t taddr, uint32_t dst, uint32_t r) {
#pragma unroll
    for (uint32_t half = 0; half < 2u; ++half) {
        float v[32];
        umma::tmem_ld32(taddr + 32u * half, v);
#pragma unroll
        for (uint32_t j = 0; j < 4u; ++j) {
            uint32_t w[4];
#pragma unroll
            for (uint32_t q = 0; q < 4u; ++q) w[q] = relu_pack_h2(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
            put_chunk(smem, dst, r, 4u * half + j, 64u, w);
        }
    }
}

// One layer: D[128 x N] = A[128 x K] * W[N x K]^T, issued by thread 0.
__device__ __forceinline__ void issue_layer(uint32_t smem_base, uint32_t a_off, uint32_t w_off, uint32_t K, uint32_t N,
                                            uint32_t tmem, uint64_t* bar) {
    umma::fence_after_sync();
    const uint32_t idesc = umma::idesc_f16(kTcRows, N, 0u, 0u);
    for (uint32_t s = 0; s < K / 16u; ++s)
        umma::mma_f16(tmem, umma::desc_k_major(smem_base + a_off, K, s), umma::desc_k_major(smem_base + w_off, K, s), idesc,
                      s > 0u ? 1u : 0u);
    umma::commit(bar);
}

// Waits until the layer's MMAs are complete.  The result is uniform over the
// warp (tensor-memory loads are warp-collective: either the whole warp loads
// or none of it); false when any lane's wait gave up.
__device__ __forceinline__ bool layer_done(uint64_t* bar, uint32_t& phase) {
    const bool ok = umma::mbar_wait(bar, phase, kWaitLimitNs);
    phase ^= 1u;
    umma::fence_after_sync();
    return __all_sync(0xffffffffu, ok);
}
// Shared-memory rows written by all threads become the next MMA's operand;
// tensor-memory reads of all threads are done before the next MMA writes.
// Returns true when any thread of the block saw a failed wait.
__device__ __forceinline__ bool layer_handoff(bool failed) {
    umma::fence_before_sync();
    umma::fence_async_smem();
    return __syncthreads_or(failed ? 1 : 0) != 0;
}

// Rows: 64-byte feature rows with directions (kTcRowsMlp) or the 112-byte
// training rows (kTcRowsTrain: features | SH | position); n from n_ptr when
// non-null.
template <int kRowsMode>
__global__ void __launch_bounds__(kTcThreads) k_mlp_forward_tc(const __half* __restrict__ mlp, const uint4* __restrict__ feat,
                                                                const float* __restrict__ dirs, const uint32_t* __restrict__ n_ptr,
                                                                uint32_t n_direct, float4* __restrict__ raw, uint32_t* error) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffBar + 8);
    const uint32_t tid = threadIdx.x, warp = tid >> 5;
    const uint32_t sbase = smem_u32(smem);
    stage_weights(smem, kOffWd0, mlp + kMlpD0, 64, 32);
    stage_weights(smem, kOffWd1, mlp + kMlpD1, 16, 64);
    stage_weights(smem, kOffWc0, mlp + kMlpC0, 64, 32);
    stage_weights(smem, kOffWc1, mlp + kMlpC1, 64, 64);
    stage_weights(smem, kOffWc2, mlp + kMlpC2, 16, 64);
    if (warp == 0) {
        umma::tmem_alloc(tslot, kTcCols);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(bar, 1);
        umma::fence_mbar_init();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;
    const uint32_t my_lanes = tmem + ((32u * warp) << 16);  // this warp's 32 lanes = rows 32w..32w+31
    const uint32_t n = n_ptr ? *n_ptr : n_direct;
    uint32_t phase = 0;
    bool failed = false;
    const uint32_t n_tiles = (n + kTcRows - 1u) / kTcRows;
    RowIn in;
    load_row<kRowsMode, false>(in, feat, dirs, nullptr, blockIdx.x * kTcRows + tid, blockIdx.x * kTcRows + tid < n);
    for (uint32_t tile = blockIdx.x; tile < n_tiles && !failed; tile += gridDim.x) {
        const uint32_t r = tid, g = tile * kTcRows + tid;
        const bool live = g < n;
        // Features -> X; SH kept for the colour input; the next tile's rows are loaded meanwhile.
        uint32_t shp[8];
        put_row<kRowsMode>(smem, kOffX, r, in, live, shp);
        {
            const uint32_t gn = (tile + gridDim.x) * kTcRows + tid;
            load_row<kRowsMode, false>(in, feat, dirs, nullptr, gn, tile + gridDim.x < n_tiles && gn < n);
        }
        if ((failed = layer_handoff(false))) break;
        // density layer 0
        if (tid == 0) issue_layer(sbase, kOffX, kOffWd0, 32, 64, tmem, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes, kOffH, r);
        if ((failed = layer_handoff(failed))) break;
        // density layer 1 -> raw sigma, colour input [density16 | SH16]
        if (tid == 0) issue_layer(sbase, kOffH, kOffWd1, 64, 16, tmem, bar);
        failed = !layer_done(bar, phase);
        float sigma = 0.0f;
        if (!failed) {
            float yd[16];
            umma::tmem_ld16(my_lanes, yd);
            sigma = yd[0];
            uint32_t w[4];
#pragma unroll
            for (uint32_t j = 0; j < 2u; ++j) {
#pragma unroll
                for (uint32_t q = 0; q < 4u; ++q) w[q] = pack_h2(yd[8 * j + 2 * q], yd[8 * j + 2 * q + 1]);
                put_chunk(smem, kOffX, r, j, 32u, w);
            }
            put_chunk(smem, kOffX, r, 2u, 32u, shp);
            put_chunk(smem, kOffX, r, 3u, 32u, shp + 4);
        }
        if ((failed = layer_handoff(failed))) break;
        // colour layers
        if (tid == 0) issue_layer(sbase, kOffX, kOffWc0, 32, 64, tmem, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes, kOffH, r);
        if ((failed = layer_handoff(failed))) break;
        if (tid == 0) issue_layer(sbase, kOffH, kOffWc1, 64, 64, tmem, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes, kOffH, r);
        if ((failed = layer_handoff(failed))) break;
        if (tid == 0) issue_layer(sbase, kOffH, kOffWc2, 64, 16, tmem, bar);
        failed = !layer_done(bar, phase);
        if (!failed) {
            float yc[16];
            umma::tmem_ld16(my_lanes, yc);
            if (live) raw[g] = make_float4(sigma, yc[0], yc[1], yc[2]);
        }
        if ((failed = layer_handoff(failed))) break;
    }
    if (failed && tid == 0) atomicOr(error, 1u);
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, kTcCols);
}

// ---------------------------------------------------------------------------
// Backward.  Per 128-row tile: the forward is recomputed (activations kept in
// shared memory), then each backward layer issues its input-gradient MMA
// (M = 128 rows) together with the weight-gradient MMA that consumes the same
// upstream gradient (M = 64 weight rows, K = the tile's 128 rows, both
// operands read MN-major from the same shared-memory buffers).  The five
// weight gradients accumulate in tensor memory over all tiles of the CTA and
// are written once, as this CTA's row of the partials buffer.
// ---------------------------------------------------------------------------
constexpr uint32_t kBX0 = kOffX;              // 128 x 32 features
constexpr uint32_t kBXc = kBX0 + 8192;        // 128 x 32 colour input
constexpr uint32_t kBHd = kBXc + 8192;        // 128 x 64
constexpr uint32_t kBH1 = kBHd + 16384;       // 128 x 64
constexpr uint32_t kBH2 = kBH1 + 16384;       // 128 x 64
constexpr uint32_t kBD = kBH2 + 16384;        // 128 x 64: dH2 (masked), then dH1, then dHd
constexpr uint32_t kBYc = kBD + 16384;        // 128 x 16: d raw colour (rgb, zero padded)
constexpr uint32_t kBYd = kBYc + 4096;        // 128 x 16: d density output
constexpr uint32_t kBBar = kBYd + 4096;
constexpr uint32_t kBwdTcSmem = kBBar + 16;
// Tensor-memory columns: layer outputs, then the weight-gradient accumulators
// (M = 64: rows in lanes 0-15 of each 32-lane quarter).
constexpr uint32_t kTOut = 0, kTWd0 = 64, kTWd1t = 96, kTWc0 = 112, kTWc1 = 144, kTWc2t = 208;
constexpr uint32_t kBwdTcCols = 256;

// Masked (ReLU of the stored fp16 activation > 0) upstream gradient of 64
// columns: accumulator row -> fp16 -> row r of kBD.
__device__ __forceinline__ void masked_row_to_d(unsigned char* smem, uint32_t taddr, uint32_t act_off, uint32_t r) {
#pragma unroll
    for (uint32_t half = 0; half < 2u; ++half) {
        float v[32];
        umma::tmem_ld32(taddr + 32u * half, v);
#pragma unroll
        for (uint32_t j = 0; j < 4u; ++j) {
            const uint4 h = *reinterpret_cast<const uint4*>(smem + act_off + umma::interleaved_offset(r, 8u * (4u * half + j), 64u));
            const uint32_t hm[4] = {h.x, h.y, h.z, h.w};
            uint32_t w[4];
#pragma unroll
            for (uint32_t q = 0; q < 4u; ++q) w[q] = relu_mask_h2(pack_h2(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]), hm[q]);
            put_chunk(smem, kBD, r, 4u * half + j, 64u, w);
        }
    }
}

// Input-gradient MMAs: D[128 x N] = A[128 x K] (K-major) * W^T where the
// weight matrix W is stored [K][N] (read MN-major).
__device__ __forceinline__ void issue_dgrad(uint32_t sbase, uint32_t a_off, uint32_t w_off, uint32_t K, uint32_t N, uint32_t tmem) {
    const uint32_t idesc = umma::idesc_f16(kTcRows, N, 0u, 1u);
    for (uint32_t s = 0; s < K / 16u; ++s)
        umma::mma_f16(tmem, umma::desc_k_major(sbase + a_off, K, s), umma::desc_mn_major(sbase + w_off, N, s), idesc,
                      s > 0u ? 1u : 0u);
}
// Weight-gradient MMAs over the tile's 128 rows: D[64 x N] (+)= G^T * X with
// G stored [128][64] and X stored [128][N] (both read MN-major).
__device__ __forceinline__ void issue_wgrad(uint32_t sbase, uint32_t g_off, uint32_t x_off, uint32_t N, uint32_t tmem,
                                            bool first) {
    const uint32_t idesc = umma::idesc_f16(64u, N, 1u, 1u);
    for (uint32_t s = 0; s < kTcRows / 16u; ++s)
        umma::mma_f16(tmem, umma::desc_mn_major(sbase + g_off, 64u, s), umma::desc_mn_major(sbase + x_off, N, s), idesc,
                      (first && s == 0u) ? 0u : 1u);
}

// One M = 64 accumulator (N columns) of this thread's rows -> partials:
// transposed (weight stored [N][64], the accumulator holds its transpose) or not
// (weight stored [64][N]).
template <uint32_t N>
__device__ __forceinline__ void store_wgrad(uint32_t taddr, float* out, uint32_t mat, uint32_t row, bool transposed, bool store) {
    float v[N];
    if constexpr (N == 16) {
        umma::tmem_ld16(taddr, v);
    } else {
#pragma unroll
        for (uint32_t c = 0; c < N / 32u; ++c) umma::tmem_ld32(taddr + 32u * c, v + 32u * c);
    }
    if (!store) return;
#pragma unroll
    for (uint32_t c = 0; c < N; ++c) {
        if (transposed) out[mat + c * 64u + row] = v[c];
        else out[mat + row * N + c] = v[c];
    }
}

template <int kRowsMode>
__global__ void __launch_bounds__(kTcThreads) k_mlp_backward_tc(const __half* __restrict__ mlp, const uint4* __restrict__ rows,
                                                                 const float* __restrict__ dirs, const float4* __restrict__ dout,
                                                                 const uint32_t* __restrict__ n_ptr, uint32_t n_direct,
                                                                 uint4* __restrict__ dfeat, float* __restrict__ partials,
                                                                 uint32_t* error) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kBBar);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kBBar + 8);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t n = n_ptr ? *n_ptr : n_direct;
    stage_weights(smem, kOffWd0, mlp + kMlpD0, 64, 32);
    stage_weights(smem, kOffWd1, mlp + kMlpD1, 16, 64);
    stage_weights(smem, kOffWc0, mlp + kMlpC0, 64, 32);
    stage_weights(smem, kOffWc1, mlp + kMlpC1, 64, 64);
    stage_weights(smem, kOffWc2, mlp + kMlpC2, 16, 64);
    if (warp == 0) {
        umma::tmem_alloc(tslot, kBwdTcCols);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(bar, 1);
        umma::fence_mbar_init();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;
    const uint32_t my_lanes = tmem + ((32u * warp) << 16);
    uint32_t phase = 0;
    bool failed = false, first = true;
    const uint32_t n_tiles = (n + kTcRows - 1u) / kTcRows;
    RowIn in;
    load_row<kRowsMode, true>(in, rows, dirs, dout, blockIdx.x * kTcRows + tid, blockIdx.x * kTcRows + tid < n);
    for (uint32_t tile = blockIdx.x; tile < n_tiles && !failed; tile += gridDim.x) {
        const uint32_t r = tid, g = tile * kTcRows + tid;
        const bool live = g < n;
        // ---- inputs: features -> X0, SH -> Xc[:, 16:32], d raw colour -> Yc; next tile's rows loaded meanwhile ----
        uint32_t shp[8];
        put_row<kRowsMode>(smem, kBX0, r, in, live, shp);
        put_chunk(smem, kBXc, r, 2u, 32u, shp);
        put_chunk(smem, kBXc, r, 3u, 32u, shp + 4);
        const float4 d4 = in.dout;
        {
            const uint32_t w0[4] = {pack_h2(d4.y, d4.z), pack_h2(d4.w, 0.0f), 0u, 0u};
            const uint32_t w1[4] = {0u, 0u, 0u, 0u};
            put_chunk(smem, kBYc, r, 0u, 16u, w0);
            put_chunk(smem, kBYc, r, 1u, 16u, w1);
        }
        {
            const uint32_t gn = (tile + gridDim.x) * kTcRows + tid;
            load_row<kRowsMode, true>(in, rows, dirs, dout, gn, tile + gridDim.x < n_tiles && gn < n);
        }
        if ((failed = layer_handoff(false))) break;
        // ---- forward recompute ----
        if (tid == 0) issue_layer(sbase, kBX0, kOffWd0, 32, 64, tmem + kTOut, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes + kTOut, kBHd, r);
        if ((failed = layer_handoff(failed))) break;
        if (tid == 0) issue_layer(sbase, kBHd, kOffWd1, 64, 16, tmem + kTOut, bar);
        failed = !layer_done(bar, phase);
        if (!failed) {
            float yd[16];
            umma::tmem_ld16(my_lanes + kTOut, yd);
            uint32_t w[4];
#pragma unroll
            for (uint32_t j = 0; j < 2u; ++j) {
#pragma unroll
                for (uint32_t q = 0; q < 4u; ++q) w[q] = pack_h2(yd[8 * j + 2 * q], yd[8 * j + 2 * q + 1]);
                put_chunk(smem, kBXc, r, j, 32u, w);
            }
        }
        if ((failed = layer_handoff(failed))) break;
        if (tid == 0) issue_layer(sbase, kBXc, kOffWc0, 32, 64, tmem + kTOut, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes + kTOut, kBH1, r);
        if ((failed = layer_handoff(failed))) break;
        if (tid == 0) issue_layer(sbase, kBH1, kOffWc1, 64, 64, tmem + kTOut, bar);
        failed = !layer_done(bar, phase);
        if (!failed) relu_row_to_act(smem, my_lanes + kTOut, kBH2, r);
        if ((failed = layer_handoff(failed))) break;
        // ---- backward: colour layer 2 (dH2 = dYc W2; dW2^T += H2^T dYc) ----
        if (tid == 0) {
            umma::fence_after_sync();
            issue_dgrad(sbase, kBYc, kOffWc2, 16, 64, tmem + kTOut);
            issue_wgrad(sbase, kBH2, kBYc, 16, tmem + kTWc2t, first);
            umma::commit(bar);
        }
        failed = !layer_done(bar, phase);
        if (!failed) masked_row_to_d(smem, my_lanes + kTOut, kBH2, r);
        if ((failed = layer_handoff(failed))) break;
        // colour layer 1: dH1 = dH2 W1; dW1 += dH2^T H1
        if (tid == 0) {
            umma::fence_after_sync();
            issue_dgrad(sbase, kBD, kOffWc1, 64, 64, tmem + kTOut);
            issue_wgrad(sbase, kBD, kBH1, 64, tmem + kTWc1, first);
            umma::commit(bar);
        }
        failed = !layer_done(bar, phase);
        if (!failed) masked_row_to_d(smem, my_lanes + kTOut, kBH1, r);
        if ((failed = layer_handoff(failed))) break;
        // colour layer 0: dXc = dH1 W0; dW0 += dH1^T Xc; d density output = dXc[:, 0:16] (+ d sigma in column 0)
        if (tid == 0) {
            umma::fence_after_sync();
            issue_dgrad(sbase, kBD, kOffWc0, 64, 32, tmem + kTOut);
            issue_wgrad(sbase, kBD, kBXc, 32, tmem + kTWc0, first);
            umma::commit(bar);
        }
        failed = !layer_done(bar, phase);
        if (!failed) {
            float v[16];
            umma::tmem_ld16(my_lanes + kTOut, v);
            v[0] += d4.x;
            uint32_t w[4];
#pragma unroll
            for (uint32_t j = 0; j < 2u; ++j) {
#pragma unroll
                for (uint32_t q = 0; q < 4u; ++q) w[q] = pack_h2(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
                put_chunk(smem, kBYd, r, j, 16u, w);
            }
        }
        if ((failed = layer_handoff(failed))) break;
        // density layer 1: dHd = dYd Wd1; dWd1^T += Hd^T dYd
        if (tid == 0) {
            umma::fence_after_sync();
            issue_dgrad(sbase, kBYd, kOffWd1, 16, 64, tmem + kTOut);
            issue_wgrad(sbase, kBHd, kBYd, 16, tmem + kTWd1t, first);
            umma::commit(bar);
        }
        failed = !layer_done(bar, phase);
        if (!failed) masked_row_to_d(smem, my_lanes + kTOut, kBHd, r);
        if ((failed = layer_handoff(failed))) break;
        // density layer 0: dX = dHd Wd0 (feature gradients); dWd0 += dHd^T X0
        if (tid == 0) {
            umma::fence_after_sync();
            issue_dgrad(sbase, kBD, kOffWd0, 64, 32, tmem + kTOut);
            issue_wgrad(sbase, kBD, kBX0, 32, tmem + kTWd0, first);
            umma::commit(bar);
        }
        failed = !layer_done(bar, phase);
        if (!failed) {
            float v[32];
            umma::tmem_ld32(my_lanes + kTOut, v);
            if (live) {
#pragma unroll
                for (uint32_t q = 0; q < 4u; ++q)
                    dfeat[4ull * g + q] = make_uint4(pack_h2(v[8 * q], v[8 * q + 1]), pack_h2(v[8 * q + 2], v[8 * q + 3]),
                                                     pack_h2(v[8 * q + 4], v[8 * q + 5]), pack_h2(v[8 * q + 6], v[8 * q + 7]));
            }
        }
        if ((failed = layer_handoff(failed))) break;
        first = false;
    }
    // This CTA's weight gradients (zero when it had no tile).  Every MMA has
    // completed: each tile ends with a wait on its last commit.
    float* out = partials + static_cast<unsigned long long>(blockIdx.x) * kMlpParams;
    if (!failed) {
        const bool mine = lane < 16u;
        const uint32_t row = 16u * warp + lane;  // M = 64 accumulator row held by this lane
        if (first) {
            for (uint32_t i = tid; i < kMlpParams; i += kTcThreads) out[i] = 0.0f;
        } else {
            store_wgrad<32>(my_lanes + kTWd0, out, kMlpD0, row, false, mine);
            store_wgrad<16>(my_lanes + kTWd1t, out, kMlpD1, row, true, mine);
            store_wgrad<32>(my_lanes + kTWc0, out, kMlpC0, row, false, mine);
            store_wgrad<64>(my_lanes + kTWc1, out, kMlpC1, row, false, mine);
            store_wgrad<16>(my_lanes + kTWc2t, out, kMlpC2, row, true, mine);
        }
    }
    if (failed && tid == 0) atomicOr(error, 1u);
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, kBwdTcCols);
}

uint32_t g_tc_blocks = 0, g_bwd_tc_blocks = 0;

}  // namespace

uint32_t g_tc_api_per[2] = {0, 0};

// Persistent grid of a tensor-memory kernel: resident CTAs per SM from its
// shared memory, registers and threads, capped so that their tensor-memory
// allocations (512 columns per SM) always fit.
template <class K>
cudaError_t tc_grid(K kernel, uint32_t smem_bytes, uint32_t cols, uint32_t* blocks, uint32_t* api_per) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, smem_sm = 0, reserved = 0, per_api = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_api, kernel, kTcThreads, smem_bytes)) != cudaSuccess) return e;
    if (api_per) *api_per = static_cast<uint32_t>(per_api);
    const uint32_t by_smem = static_cast<uint32_t>(smem_sm) / (smem_bytes + static_cast<uint32_t>(reserved) + fa.sharedSizeBytes);
    const uint32_t regs = (static_cast<uint32_t>(fa.numRegs) + 7u) & ~7u;
    const uint32_t by_regs = 65536u / (regs * kTcThreads);
    const uint32_t by_threads = 2048u / kTcThreads;
    uint32_t per = by_smem < by_regs ? by_smem : by_regs;
    per = per < by_threads ? per : by_threads;
    per = per < 512u / cols ? per : 512u / cols;
    *blocks = static_cast<uint32_t>(sms) * (per < 1u ? 1u : per);
    return cudaSuccess;
}

cudaError_t mlp_tc_init() {
    if (g_tc_blocks && g_bwd_tc_blocks) return cudaSuccess;
    uint32_t b0 = 0, b1 = 0;
    cudaError_t e = tc_grid(k_mlp_forward_tc<kTcRowsMlp>, kTcSmem, kTcCols, &b0, &g_tc_api_per[0]);
    if (e != cudaSuccess) return e;
    if ((e = tc_grid(k_mlp_forward_tc<kTcRowsTrain>, kTcSmem, kTcCols, &b1, nullptr)) != cudaSuccess) return e;
    g_tc_blocks = b0 < b1 ? b0 : b1;
    if ((e = tc_grid(k_mlp_backward_tc<kTcRowsMlp>, kBwdTcSmem, kBwdTcCols, &b0, &g_tc_api_per[1])) != cudaSuccess) return e;
    if ((e = tc_grid(k_mlp_backward_tc<kTcRowsTrain>, kBwdTcSmem, kBwdTcCols, &b1, nullptr)) != cudaSuccess) return e;
    g_bwd_tc_blocks = b0 < b1 ? b0 : b1;
    return cudaSuccess;
}

void mlp_tc_info(uint32_t out[4]) {
    if (mlp_tc_init() != cudaSuccess) {
        out[0] = out[1] = out[2] = out[3] = 0u;
        return;
    }
    out[0] = g_tc_blocks;
    out[1] = g_bwd_tc_blocks;
    out[2] = g_tc_api_per[0];
    out[3] = g_tc_api_per[1];
}

uint32_t mlp_backward_tc_blocks() { return mlp_tc_init() == cudaSuccess ? g_bwd_tc_blocks : 0u; }

cudaError_t launch_mlp_backward_tc(const void* mlp, const void* rows, int train_rows, const float* dirs, const float* dout,
                                   const uint32_t* n_device, uint32_t n, void* dfeat, float* partials, uint32_t blocks,
                                   uint32_t* error, cudaStream_t s) {
    cudaError_t e = mlp_tc_init();
    if (e != cudaSuccess) return e;
    if (blocks == 0u || blocks > g_bwd_tc_blocks) return cudaErrorInvalidValue;
    auto kernel = train_rows ? k_mlp_backward_tc<kTcRowsTrain> : k_mlp_backward_tc<kTcRowsMlp>;
    kernel<<<blocks, kTcThreads, kBwdTcSmem, s>>>(static_cast<const __half*>(mlp), static_cast<const uint4*>(rows), dirs,
                                                   reinterpret_cast<const float4*>(dout), n_device, n, static_cast<uint4*>(dfeat),
                                                   partials, error);
    return cudaGetLastError();
}

cudaError_t launch_mlp_forward_tc(const void* mlp, const void* feat, const float* dirs, uint32_t n, float* raw, uint32_t* error,
                                  cudaStream_t s) {
    if (n == 0u) return cudaSuccess;
    cudaError_t e = mlp_tc_init();
    if (e != cudaSuccess) return e;
    const uint32_t tiles = (n + kTcRows - 1u) / kTcRows;
    const uint32_t blocks = tiles < g_tc_blocks ? tiles : g_tc_blocks;
    k_mlp_forward_tc<kTcRowsMlp><<<blocks, kTcThreads, kTcSmem, s>>>(static_cast<const __half*>(mlp), static_cast<const uint4*>(feat),
                                                                      dirs, nullptr, n, reinterpret_cast<float4*>(raw), error);
    return cudaGetLastError();
}

cudaError_t launch_mlp_forward_tc_train(const void* mlp, const void* rows, const uint32_t* n_device, float* raw, uint32_t* error,
                                        cudaStream_t s) {
    cudaError_t e = mlp_tc_init();
    if (e != cudaSuccess) return e;
    k_mlp_forward_tc<kTcRowsTrain><<<g_tc_blocks, kTcThreads, kTcSmem, s>>>(
        static_cast<const __half*>(mlp), static_cast<const uint4*>(rows), nullptr, n_device, 0u, reinterpret_cast<float4*>(raw), error);
    return cudaGetLastError();
}

}  // namespace nb
