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

// The next 32 steps of a ray's march.  Every lane runs the same step
// recurrence (t is warp-uniform, no divergence) and keeps the step whose
// index within the chunk equals its lane.  Returns the number of valid steps.
__device__ __forceinline__ uint32_t march_chunk(const Ray& ray, float dt_min, float cone, uint32_t max_steps, float& t,
                                                uint32_t& i, uint32_t lane, float& my_mid, float& my_dt) {
    uint32_t nv = 0u;
#pragma unroll 4
    for (uint32_t j = 0; j < 32u; ++j) {
        if (!(t < ray.tf && i < max_steps)) break;
        const float dt = march_dt(t, ray.tf, dt_min, cone);
        if (j == lane) {
            my_mid = march_mid(t, dt);
            my_dt = dt;
        }
        t = __fadd_rn(t, dt);
        ++i;
        ++nv;
    }
    return nv;
}

// Pass 1: one warp per ray.  Lane j tests step 32c+j of chunk c; the
// ballot of the 32 tests is the chunk's bit word.
__global__ void __launch_bounds__(kSamplerBlock) k_sample_count(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    __shared__ float cam[16];
    const uint32_t frame = a.state->frame_index;
    const uint32_t n_rays = a.state->n_rays;
    if (threadIdx.x < 12u) cam[threadIdx.x] = a.cams[16ull * train_camera(frame, tc.n_images) + threadIdx.x];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t r = blockIdx.x * (kSamplerBlock / 32u) + (threadIdx.x >> 5);
    if (r >= tc.max_rays) return;
    uint32_t count = 0u;
    if (r < n_rays) {
        const AabbConsts box = aabb_of(tc);
        Ray ray;
        float px, py;
        if (make_ray(tc, box, cam, ray_seed(frame, tc.dp_rank * tc.rays_per_batch + r), ray, px, py)) {
            const float dt_min = __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(tc.max_steps));
            float t = ray.tn;
            uint32_t i = 0u;
            // Software pipeline: the bitfield words of chunk c are loaded while
            // the step recurrence of chunk c+1 runs.
            float t_cur = t, mid = 0.0f, dt = 0.0f;
            uint32_t nv_cur = march_chunk(ray, dt_min, tc.cone, tc.max_steps, t, i, lane, mid, dt);
            uint32_t bit_cur = 0u, w = 0xFFFFFFFFu;
            if (lane < nv_cur) {
                float p[3];
                ray_point(ray, mid, p);
                w = occupancy_word(tc.grid_res, box, p, bit_cur);
            }
            uint32_t word_cur = w != 0xFFFFFFFFu ? __ldg(a.bitfield + w) : 0u;
            for (uint32_t c = 0;; ++c) {
                const float t_next = t;
                uint32_t nv_next = 0u, bit_next = 0u, word_next = 0u;
                if (nv_cur == 32u) {
                    nv_next = march_chunk(ray, dt_min, tc.cone, tc.max_steps, t, i, lane, mid, dt);
                    uint32_t wn = 0xFFFFFFFFu;
                    if (lane < nv_next) {
                        float p[3];
                        ray_point(ray, mid, p);
                        wn = occupancy_word(tc.grid_res, box, p, bit_next);
                    }
                    word_next = wn != 0xFFFFFFFFu ? __ldg(a.bitfield + wn) : 0u;
                }
                const bool occ = lane < nv_cur && ((word_cur >> bit_cur) & 1u);
                const uint32_t bits = __ballot_sync(0xffffffffu, occ);
                if (nv_cur > 0u && lane == 0u) {
                    a.masks[c * tc.max_rays + r] = bits;
                    if (bits) a.chunk_t[c * tc.max_rays + r] = t_cur;  // pass 2 resumes the march here
                }
                count += __popc(bits);
                if (nv_cur < 32u || nv_next == 0u) break;
                nv_cur = nv_next;
                bit_cur = bit_next;
                word_cur = word_next;
                t_cur = t_next;
            }
        }
    }
    if (lane == 0u) a.ray_counts[r] = count;
}

// Ordered compaction over all marched rays in one block: exclusive scans of
// sample counts and of the active flags; a ray is kept while its inclusive
// sample prefix stays within the capacity (kept rays are a prefix of the
// active rays, so a kept ray's slot is its active index).
constexpr uint32_t kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) k_sample_scan(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    const uint32_t n = min(a.state->n_rays, tc.max_rays);
    const uint32_t per = (n + kScanThreads - 1u) / kScanThreads;
    const uint32_t r0 = threadIdx.x * per, r1 = min(n, r0 + per);
    uint32_t ls = 0u, la = 0u;
    for (uint32_t r = r0; r < r1; ++r) {
        const uint32_t c = a.ray_counts[r];
        ls += c;
        la += c > 0u ? 1u : 0u;
    }
    __shared__ uint32_t ws[32], wa[32];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t is = ls, ia = la;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t xs = __shfl_up_sync(0xffffffffu, is, o), xa = __shfl_up_sync(0xffffffffu, ia, o);
        if (lane >= static_cast<uint32_t>(o)) {
            is += xs;
            ia += xa;
        }
    }
    if (lane == 31u) {
        ws[warp] = is;
        wa[warp] = ia;
    }
    __syncthreads();
    if (warp == 0u) {
        uint32_t vs = ws[lane], va = wa[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t xs = __shfl_up_sync(0xffffffffu, vs, o), xa = __shfl_up_sync(0xffffffffu, va, o);
            if (lane >= static_cast<uint32_t>(o)) {
                vs += xs;
                va += xa;
            }
        }
        ws[lane] = vs;  // inclusive over warps
        wa[lane] = va;
    }
    __syncthreads();
    uint32_t ps = is - ls + (warp ? ws[warp - 1u] : 0u);
    uint32_t pa = ia - la + (warp ? wa[warp - 1u] : 0u);
    const uint32_t tot_s = ws[31], tot_a = wa[31];
    const uint32_t cap = tc.sample_cap;
    for (uint32_t r = r0; r < r1; ++r) {
        const uint32_t c = a.ray_counts[r];
        const uint32_t incl = ps + c;
        const bool kept = c > 0u && incl <= cap;
        a.ray_offset[r] = ps;
        a.ray_slot[r] = kept ? pa : 0xFFFFFFFFu;
        if (c > 0u && ps <= cap && incl > cap) {  // the first ray past the capacity
            a.state->n_samples = ps;
            a.state->n_active = pa;
        }
        ps = incl;
        pa += c > 0u ? 1u : 0u;
    }
    if (threadIdx.x == 0u) {
        a.state->n_marched_active = tot_a;
        if (tot_s <= cap) {
            a.state->n_samples = tot_s;
            a.state->n_active = tot_a;
        }
    }
}

// Pass 2: one warp per kept ray.  Chunks without samples are skipped; a
// chunk with samples re-walks its 32 steps of the recurrence from the t that
// pass 1 recorded at its start, and lane j writes step 32c+j at its rank
// among the chunk's set bits.
__global__ void __launch_bounds__(kSamplerBlock) k_sample_write(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    __shared__ float cam[16];
    const uint32_t frame = a.state->frame_index;
    const uint32_t camera = train_camera(frame, tc.n_images);
    if (threadIdx.x < 12u) cam[threadIdx.x] = a.cams[16ull * camera + threadIdx.x];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t r = blockIdx.x * (kSamplerBlock / 32u) + (threadIdx.x >> 5);
    if (r >= min(a.state->n_rays, tc.max_rays)) return;
    const uint32_t count = a.ray_counts[r];
    if (count == 0u) return;
    const uint32_t slot = a.ray_slot[r];
    if (slot == 0xFFFFFFFFu) return;
    const uint32_t excl = a.ray_offset[r];

    const AabbConsts box = aabb_of(tc);
    Ray ray;
    float rpx = 0.0f, rpy = 0.0f;
    const uint32_t seed = ray_seed(frame, tc.dp_rank * tc.rays_per_batch + r);
    make_ray(tc, box, cam, seed, ray, rpx, rpy);
    const float dt_min = __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(tc.max_steps));
    uint32_t out = excl;
    const uint32_t end = excl + count;
    for (uint32_t c = 0; out < end; ++c) {
        const uint32_t bits = a.masks[c * tc.max_rays + r];
        if (bits == 0u) continue;
        float t = a.chunk_t[c * tc.max_rays + r];
        uint32_t i = 32u * c;
        float mid = 0.0f, dt = 0.0f;
        const uint32_t nv = march_chunk(ray, dt_min, tc.cone, tc.max_steps, t, i, lane, mid, dt);
        if (nv == 0u) break;
        if ((bits >> lane) & 1u) {
            float p[3];
            ray_point(ray, mid, p);
            const uint32_t o = out + __popc(bits & ((1u << lane) - 1u));
            a.pos_dt[o] = make_float4(p[0], p[1], p[2], dt);
            a.sample_ray[o] = slot;
        }
        out += __popc(bits);
    }
    if (lane != 0u) return;
    a.ray_index[slot] = r;
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
    const uint32_t rays_per_block = kSamplerBlock / 32u;
    const uint32_t blocks = (a.tc.max_rays + rays_per_block - 1u) / rays_per_block;
    k_sample_count<<<blocks, kSamplerBlock, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_sample_scan<<<1, kScanThreads, 0, s>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_sample_write<<<blocks, kSamplerBlock, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
