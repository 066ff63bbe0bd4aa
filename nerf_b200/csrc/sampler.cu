// sampler.cu -- training-ray sampler with deterministic compaction.
//
// Ray generation, AABB clipping and the cone-angle march follow the
// reference sampler (backend-cuda.cu:422-533): one camera per step, pixel
// from the hashed RNG, samples at step midpoints kept where the occupancy
// bitfield is set.  Instead of the reference's two atomic counters (whose
// order is nondeterministic), compaction is an ordered prefix sum:
//   pass 1 (k_sample_count): march each ray, record which steps hit occupied
//     cells in 32-step bit words, count samples; per-block totals.
//   pass 2 (k_sample_write): each block sums the totals of the blocks before
//     it, scans its own rays, and re-walks the step recurrence (no occupancy
//     lookups, only the recorded bits) to write samples at their final
//     offsets.  Rays are kept in ray order while the running total stays
//     within the per-step capacity.
// All float arithmetic that decides which steps are kept uses explicit
// rounding intrinsics, so the CPU oracle reproduces per-ray counts and
// offsets bit for bit.  (The reference normalises with the approximate
// rsqrtf; this path uses a correctly rounded 1/sqrt.)
#include "kernels.h"
#include "ray.cuh"

namespace nb {
namespace {

constexpr uint32_t kBgSalt0 = 0x1B873593u, kBgSalt1 = 0x5BD1E995u, kBgSalt2 = 0x27D4EB2Fu;

__device__ __forceinline__ uint32_t ray_seed(uint32_t frame, uint32_t global_ray) {
    return frame * 1315423911u ^ global_ray * 9781u;
}

__device__ __forceinline__ AabbConsts aabb_of(const TrainConsts& tc) {
    AabbConsts b;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        b.mn[k] = tc.aabb_min[k];
        b.mx[k] = tc.aabb_max[k];
        b.size[k] = tc.aabb_size[k];
    }
    return b;
}

// Training ray of a step: pixel from the hashed RNG (reference
// backend-cuda.cu:438-441), then the camera ray and its AABB chord.
__device__ __forceinline__ bool make_ray(const TrainConsts& tc, const AabbConsts& b, const float* cam, uint32_t seed, Ray& r,
                                         float& px, float& py) {
    px = __fmul_rn(rand01(seed ^ 0xA511E9B3u), static_cast<float>(tc.width));
    py = __fmul_rn(rand01(seed ^ 0x63D83595u), static_cast<float>(tc.height));
    if (!camera_ray(cam, tc.fx, tc.fy, tc.cx, tc.cy, static_cast<float>(tc.height), px, py, r)) return false;
    return clip_aabb(b, r);
}

// Block-wide exclusive scan of two counters (128 threads).
__device__ __forceinline__ void block_scan2(uint32_t a, uint32_t b, uint32_t& ea, uint32_t& eb) {
    __shared__ uint32_t wa[kSamplerBlock / 32], wb[kSamplerBlock / 32];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t ia = a, ib = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t xa = __shfl_up_sync(0xffffffffu, ia, o);
        const uint32_t xb = __shfl_up_sync(0xffffffffu, ib, o);
        if (lane >= static_cast<uint32_t>(o)) {
            ia += xa;
            ib += xb;
        }
    }
    if (lane == 31u) {
        wa[warp] = ia;
        wb[warp] = ib;
    }
    __syncthreads();
    uint32_t pa = 0u, pb = 0u;
    for (uint32_t w = 0; w < warp; ++w) {
        pa += wa[w];
        pb += wb[w];
    }
    ea = pa + ia - a;
    eb = pb + ib - b;
}

__global__ void __launch_bounds__(kSamplerBlock) k_sample_count(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    __shared__ float cam[16];
    const uint32_t frame = a.state->frame_index;
    const uint32_t n_rays = a.state->n_rays;
    if (threadIdx.x < 12u) cam[threadIdx.x] = a.cams[16ull * train_camera(frame, tc.n_images) + threadIdx.x];
    __syncthreads();
    const uint32_t r = blockIdx.x * kSamplerBlock + threadIdx.x;
    uint32_t count = 0u;
    if (r < n_rays && r < tc.max_rays) {
        const AabbConsts box = aabb_of(tc);
        Ray ray;
        float px, py;
        if (make_ray(tc, box, cam, ray_seed(frame, tc.dp_rank * tc.rays_per_batch + r), ray, px, py)) {
            const float dt_min = __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(tc.max_steps));
            float t = ray.tn;
            uint32_t i = 0u, word = 0u;
            while (t < ray.tf && i < tc.max_steps) {
                const float dt = march_dt(t, ray.tf, dt_min, tc.cone);
                float p[3];
                ray_point(ray, march_mid(t, dt), p);
                if (occupied(a.bitfield, tc.grid_res, box, p)) {
                    word |= 1u << (i & 31u);
                    ++count;
                }
                if ((i & 31u) == 31u) {
                    a.masks[(i >> 5) * tc.max_rays + r] = word;
                    word = 0u;
                }
                t = __fadd_rn(t, dt);
                ++i;
            }
            if ((i & 31u) != 0u) a.masks[(i >> 5) * tc.max_rays + r] = word;
        }
    }
    if (r < tc.max_rays) a.ray_counts[r] = count;
    const uint32_t s = warp_sum_u32(count), act = warp_sum_u32(count > 0u ? 1u : 0u);
    __shared__ uint32_t ws[kSamplerBlock / 32], wa[kSamplerBlock / 32];
    if ((threadIdx.x & 31u) == 0u) {
        ws[threadIdx.x >> 5] = s;
        wa[threadIdx.x >> 5] = act;
    }
    __syncthreads();
    if (threadIdx.x == 0u) {
        uint32_t bs = 0u, ba = 0u;
        for (uint32_t w = 0; w < kSamplerBlock / 32; ++w) {
            bs += ws[w];
            ba += wa[w];
        }
        a.block_samples[blockIdx.x] = bs;
        a.block_active[blockIdx.x] = ba;
    }
}

__global__ void __launch_bounds__(kSamplerBlock) k_sample_write(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    __shared__ float cam[16];
    __shared__ uint32_t pre_s, pre_a, tot_s, tot_a;
    const uint32_t frame = a.state->frame_index;
    const uint32_t camera = train_camera(frame, tc.n_images);
    if (threadIdx.x < 12u) cam[threadIdx.x] = a.cams[16ull * camera + threadIdx.x];
    if (threadIdx.x < 32u) {
        uint32_t ps = 0u, pa = 0u, ts = 0u, ta = 0u;
        for (uint32_t j = threadIdx.x; j < gridDim.x; j += 32u) {
            const uint32_t bs = a.block_samples[j], ba = a.block_active[j];
            ts += bs;
            ta += ba;
            if (j < blockIdx.x) {
                ps += bs;
                pa += ba;
            }
        }
        ps = warp_sum_u32(ps);
        pa = warp_sum_u32(pa);
        ts = warp_sum_u32(ts);
        ta = warp_sum_u32(ta);
        if (threadIdx.x == 0u) {
            pre_s = ps;
            pre_a = pa;
            tot_s = ts;
            tot_a = ta;
        }
    }
    const uint32_t r = blockIdx.x * kSamplerBlock + threadIdx.x;
    const uint32_t count = r < tc.max_rays ? a.ray_counts[r] : 0u;
    uint32_t ex_s, ex_a;
    block_scan2(count, count > 0u ? 1u : 0u, ex_s, ex_a);  // contains __syncthreads
    const uint32_t excl = pre_s + ex_s, incl = excl + count;
    const uint32_t slot = pre_a + ex_a;
    const uint32_t cap = tc.sample_cap;
    if (tot_s <= cap) {
        if (blockIdx.x == 0u && threadIdx.x == 0u) {
            a.state->n_samples = tot_s;
            a.state->n_active = tot_a;
            a.state->n_marched_active = tot_a;
        }
    } else if (count > 0u && excl <= cap && incl > cap) {
        a.state->n_samples = excl;
        a.state->n_active = slot;
        a.state->n_marched_active = tot_a;
    }
    if (count == 0u || incl > cap) return;

    const AabbConsts box = aabb_of(tc);
    Ray ray;
    float rpx = 0.0f, rpy = 0.0f;
    const uint32_t gr = tc.dp_rank * tc.rays_per_batch + r;
    const uint32_t seed = ray_seed(frame, gr);
    make_ray(tc, box, cam, seed, ray, rpx, rpy);
    a.ray_index[slot] = r;
    // Re-walk the step recurrence; the pass-1 bits say which steps to keep.
    const float dt_min = __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(tc.max_steps));
    float t = ray.tn;
    uint32_t i = 0u, out = excl, word = 0u;
    while (t < ray.tf && i < tc.max_steps && out < incl) {
        if ((i & 31u) == 0u) word = a.masks[(i >> 5) * tc.max_rays + r];
        const float dt = march_dt(t, ray.tf, dt_min, tc.cone);
        if ((word >> (i & 31u)) & 1u) {
            float p[3];
            ray_point(ray, march_mid(t, dt), p);
            a.pos_dt[out] = make_float4(p[0], p[1], p[2], dt);
            a.sample_ray[out] = slot;
            ++out;
        }
        t = __fadd_rn(t, dt);
        ++i;
    }
    // Ground truth: bilinear RGBA8 fetch at the unflipped pixel position,
    // composited on the ray's background (reference backend-cuda.cu:471-499).
    float bg[3] = {1.0f, 1.0f, 1.0f};
    if (tc.background == 1u) {
        bg[0] = rand01(seed ^ kBgSalt0);
        bg[1] = rand01(seed ^ kBgSalt1);
        bg[2] = rand01(seed ^ kBgSalt2);
    }
    const float pxc = fmaxf(0.0f, fminf(rpx, __fsub_rn(static_cast<float>(tc.width), 1.0f)));
    const float pyc = fmaxf(0.0f, fminf(rpy, __fsub_rn(static_cast<float>(tc.height), 1.0f)));
    const int x0 = static_cast<int>(floorf(pxc)), y0 = static_cast<int>(floorf(pyc));
    const int x1 = min(x0 + 1, static_cast<int>(tc.width) - 1), y1 = min(y0 + 1, static_cast<int>(tc.height) - 1);
    const float tx = __fsub_rn(pxc, static_cast<float>(x0)), ty = __fsub_rn(pyc, static_cast<float>(y0));
    const uint32_t* img = reinterpret_cast<const uint32_t*>(a.images) + static_cast<unsigned long long>(camera) * tc.width * tc.height;
    const uint32_t q00 = __ldg(img + static_cast<uint32_t>(y0) * tc.width + x0);
    const uint32_t q10 = __ldg(img + static_cast<uint32_t>(y0) * tc.width + x1);
    const uint32_t q01 = __ldg(img + static_cast<uint32_t>(y1) * tc.width + x0);
    const uint32_t q11 = __ldg(img + static_cast<uint32_t>(y1) * tc.width + x1);
    const float inv255 = 1.0f / 255.0f;
    const float omtx = __fsub_rn(1.0f, tx), omty = __fsub_rn(1.0f, ty);
    float v[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        const float s00 = __fmul_rn(static_cast<float>((q00 >> (8 * ch)) & 255u), inv255);
        const float s10 = __fmul_rn(static_cast<float>((q10 >> (8 * ch)) & 255u), inv255);
        const float s01 = __fmul_rn(static_cast<float>((q01 >> (8 * ch)) & 255u), inv255);
        const float s11 = __fmul_rn(static_cast<float>((q11 >> (8 * ch)) & 255u), inv255);
        const float ta = __fmaf_rn(s10, tx, __fmul_rn(s00, omtx));
        const float tb = __fmaf_rn(s11, tx, __fmul_rn(s01, omtx));
        v[ch] = __fmaf_rn(tb, ty, __fmul_rn(ta, omty));
    }
    RayRecord rec;
    rec.dir[0] = ray.d[0];
    rec.dir[1] = ray.d[1];
    rec.dir[2] = ray.d[2];
    rec.begin = excl;
    const float oma = __fsub_rn(1.0f, v[3]);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) rec.gt[ch] = __fmaf_rn(v[ch], v[3], __fmul_rn(bg[ch], oma));
    rec.gt[3] = v[3];
    rec.bg[0] = bg[0];
    rec.bg[1] = bg[1];
    rec.bg[2] = bg[2];
    rec.count = count;
    a.rays[slot] = rec;
}

}  // namespace

cudaError_t launch_sampler(const SamplerArgs& a, cudaStream_t s) {
    const uint32_t blocks = (a.tc.max_rays + kSamplerBlock - 1u) / kSamplerBlock;
    k_sample_count<<<blocks, kSamplerBlock, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_sample_write<<<blocks, kSamplerBlock, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
