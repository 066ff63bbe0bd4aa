// sampler.cu -- training-ray sampler with deterministic compaction.
//
// Ray generation, AABB clipping and the cone-angle march follow the
// reference sampler (backend-cuda.cu:422-533): one camera per step, pixel
// from the hashed RNG, samples at step midpoints kept where the occupancy
// bitfield is set.  Instead of the reference's two atomic counters (whose
// order is nondeterministic), compaction is an ordered prefix sum, and the
// one serial part of the march -- the step recurrence t += dt(t) -- is
// separated from everything that can run in parallel:
//   k_march        one thread per ray: the ray, its chord and the step
//                  recurrence, writing t at the start of every 32-step chunk;
//   k_sample_bits  a 128-thread block per ray, thread k on steps 8k..8k+7
//                  from the stored start of their chunk, testing each
//                  midpoint against the bitfield, then storing t of every
//                  kept step in the ray's kept list (in step order) and the
//                  ray's count;
//   k_sample_scan  ordered exclusive scans of counts and active flags with
//                  the capacity cut;
//   k_sample_write a 128-thread block per kept ray: samples at their final
//                  offsets from the kept list, then the ray record with its
//                  ground-truth colour.
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
    return make_box(tc.aabb_min, tc.aabb_max, tc.aabb_size, tc.casc);
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

// Per-ray sample counts of the step of frame f.
__device__ __forceinline__ uint32_t* counts_of(const SamplerArgs& a, uint32_t frame) {
    return a.ray_counts + static_cast<unsigned long long>(frame & 1u) * a.tc.max_rays;
}

// Step recurrence of one ray per thread (reference backend-cuda.cu:455-468).
// The chain is serial by definition and is the whole cost of this kernel, so
// nothing else sits in its loop: it stores only t at the start of every
// 32-step chunk, and the bitfield tests and the sample writes re-run at most
// 31 steps of the same rounded recurrence from there (step_t), which gives
// the same t bit for bit.  Blocks are a single warp, so the few warps of a
// step spread over the SMs.
constexpr uint32_t kMarchBlock = 32;

__global__ void __launch_bounds__(kMarchBlock) k_march(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    __shared__ float cam[16];
    const uint32_t frame = a.state->frame_index;
    const uint32_t n_rays = min(a.state->n_rays, tc.max_rays);
    const uint32_t r0 = blockIdx.x * kMarchBlock;
    if (r0 >= n_rays) return;  // whole block
    const uint32_t lane = threadIdx.x;
    if (lane < 12u) cam[lane] = a.cams[16ull * train_camera(frame, tc.n_images) + lane];
    __syncwarp();
    const uint32_t r = r0 + lane;
    if (r >= n_rays) return;
    const AabbConsts box = aabb_of(tc);
    Ray ray{};
    RayGeom g{};
    bool live = make_ray(tc, box, cam, ray_seed(frame, tc.dp_rank * tc.rays_per_batch + r), ray, g.px, g.py);
    const float dt_min = live ? __fdiv_rn(__fsub_rn(ray.tf, ray.tn), static_cast<float>(tc.max_steps)) : 0.0f;
    // Below tf every dt is positive, and once t reaches tf it never drops
    // below it again (past tf, dt = tf - t is exact and brings t back to tf),
    // so the steps with t < tf are a prefix: 32 steps run without a per-step
    // exit test and are counted after.
    float* chunks = a.chunk_t + static_cast<unsigned long long>(r) * tc.mask_words;
    float t = ray.tn;
    uint32_t i = 0u;
    for (uint32_t base = 0; live; base += 32u) {
        chunks[base >> 5] = t;
        uint32_t nv = 0u;
#pragma unroll
        for (uint32_t j = 0; j < 32u; ++j) {
            nv += t < ray.tf ? 1u : 0u;
            t = __fadd_rn(t, march_dt(t, ray.tf, dt_min, tc.cone));
        }
        nv = min(nv, tc.max_steps - base);
        i = base + nv;
        live = nv == 32u && i < tc.max_steps;
    }
    g.tf = ray.tf;
    g.dt_min = dt_min;
    g.n_steps = i;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        g.o[k] = ray.o[k];
        g.d[k] = ray.d[k];
    }
    a.geom[r] = g;
}


// Bitfield tests: a grid-stride loop over rays, one 128-thread block each.
// Thread k takes steps 8k..8k+7 of each 1024-step group: from the stored start
// of their 32-step chunk it runs the march's own rounded recurrence to its
// first step and on through its eight (so every t is the march's, bit for
// bit), computes the eight occupancy cells and issues their bitfield loads
// together.  A block scan of the threads' kept counts places each thread's
// kept steps in the ray's kept list ([ray][max_steps], step order), which a
// second walk of its steps fills with their t.  The ray's sample count is the
// block's total.  (A warp per ray with a lane per chunk left the SMs idle
// three quarters of the time: too few warps, each with 32 serial lookups.)
constexpr uint32_t kBitsThreads = 128, kBitsSteps = 8;
__global__ void __launch_bounds__(kBitsThreads) k_sample_bits(const SamplerArgs a) {
    __shared__ uint32_t warp_total[kBitsThreads / 32u];
    const TrainConsts& tc = a.tc;
    const uint32_t n_rays = min(a.state->n_rays, tc.max_rays);
    uint32_t* counts = counts_of(a, a.state->frame_index);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const AabbConsts box = aabb_of(tc);
    for (uint32_t r = blockIdx.x; r < n_rays; r += gridDim.x) {
        const RayGeom g = a.geom[r];
        const float* ct = a.chunk_t + static_cast<unsigned long long>(r) * tc.mask_words;
        float* kt = a.kept_t + static_cast<unsigned long long>(r) * tc.max_steps;
        uint32_t kept = 0u;
        for (uint32_t s0 = 0; s0 < g.n_steps; s0 += kBitsThreads * kBitsSteps) {
            const uint32_t first = s0 + threadIdx.x * kBitsSteps;
            const uint32_t m = first < g.n_steps ? min(kBitsSteps, g.n_steps - first) : 0u;
            float t0 = 0.0f;
            uint32_t bits = 0u;
            if (m) {
                float t = ct[first >> 5];
                for (uint32_t j = first & 31u; j > 0u; --j) t = __fadd_rn(t, march_dt(t, g.tf, g.dt_min, tc.cone));
                t0 = t;
                uint32_t cell[kBitsSteps];
#pragma unroll
                for (uint32_t j = 0; j < kBitsSteps; ++j) {
                    const float dt = march_dt(t, g.tf, g.dt_min, tc.cone);
                    const float mid = march_mid(t, dt);
                    const float p[3] = {__fmaf_rn(mid, g.d[0], g.o[0]), __fmaf_rn(mid, g.d[1], g.o[1]),
                                        __fmaf_rn(mid, g.d[2], g.o[2])};
                    cell[j] = j < m ? occupancy_cell(tc.grid_res, box, p) : kNoCell;
                    t = __fadd_rn(t, dt);
                }
#pragma unroll
                for (uint32_t j = 0; j < kBitsSteps; ++j) bits |= cell_bit(a.bitfield, cell[j]) ? 1u << j : 0u;
            }
            // Exclusive scan of the kept counts in thread order.
            const uint32_t cnt = static_cast<uint32_t>(__popc(bits));
            uint32_t incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl += x;
            }
            if (lane == 31u) warp_total[warp] = incl;
            __syncthreads();
            uint32_t before = 0u, total = 0u;
#pragma unroll
            for (uint32_t w = 0; w < kBitsThreads / 32u; ++w) {
                const uint32_t v = warp_total[w];
                before += w < warp ? v : 0u;
                total += v;
            }
            __syncthreads();  // warp_total is rewritten by the next group
            uint32_t out = kept + before + incl - cnt;
            float t = t0;
            for (uint32_t left = bits; left;) {
                const float dt = march_dt(t, g.tf, g.dt_min, tc.cone);
                if (left & 1u) kt[out++] = t;
                left >>= 1;
                t = __fadd_rn(t, dt);
            }
            kept += total;
        }
        if (threadIdx.x == 0u) counts[r] = kept;
    }
}

// Ordered compaction over all marched rays in one block: exclusive scans of
// sample counts and of the active flags; a ray is kept while its inclusive
// sample prefix stays within the capacity (kept rays are a prefix of the
// active rays, so a kept ray's slot is its active index).
constexpr uint32_t kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) k_sample_scan(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    const uint32_t n = min(a.state->n_rays, tc.max_rays);
    const uint32_t frame = a.state->frame_index;
    const uint32_t* counts = counts_of(a, frame);
    const uint32_t per = (n + kScanThreads - 1u) / kScanThreads;
    const uint32_t r0 = threadIdx.x * per, r1 = min(n, r0 + per);
    uint32_t ls = 0u, la = 0u;
    for (uint32_t r = r0; r < r1; ++r) {
        const uint32_t c = counts[r];
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
        const uint32_t c = counts[r];
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
        a.state->counts_parity = frame & 1u;
        a.state->n_marched_active = tot_a;
        if (tot_s <= cap) {
            a.state->n_samples = tot_s;
            a.state->n_active = tot_a;
        }
    }
}

// Bilinear footprint of a ray's ground-truth fetch at the unflipped pixel
// position (reference backend-cuda.cu:471-499): texel k (k = 0..3) is
// (x0 or x1 for bit 0 of k, y0 or y1 for bit 1).
struct Footprint {
    unsigned long long texel[4];
    float tx, ty;
};

__device__ __forceinline__ Footprint footprint(const TrainConsts& tc, const RayGeom& g, uint32_t camera) {
    const float pxc = fmaxf(0.0f, fminf(g.px, __fsub_rn(static_cast<float>(tc.width), 1.0f)));
    const float pyc = fmaxf(0.0f, fminf(g.py, __fsub_rn(static_cast<float>(tc.height), 1.0f)));
    const int x0 = static_cast<int>(floorf(pxc)), y0 = static_cast<int>(floorf(pyc));
    const int x1 = min(x0 + 1, static_cast<int>(tc.width) - 1), y1 = min(y0 + 1, static_cast<int>(tc.height) - 1);
    const unsigned long long base = static_cast<unsigned long long>(camera) * tc.width * tc.height;
    Footprint f;
    f.texel[0] = base + static_cast<uint32_t>(y0) * tc.width + x0;
    f.texel[1] = base + static_cast<uint32_t>(y0) * tc.width + x1;
    f.texel[2] = base + static_cast<uint32_t>(y1) * tc.width + x0;
    f.texel[3] = base + static_cast<uint32_t>(y1) * tc.width + x1;
    f.tx = __fsub_rn(pxc, static_cast<float>(x0));
    f.ty = __fsub_rn(pyc, static_cast<float>(y0));
    return f;
}

// Ray record of a kept ray: direction, sample range, background and the
// ground truth -- the bilinear blend of the footprint's texels q00, q10, q01,
// q11, composited on the ray's background.
__device__ __forceinline__ void write_record(const SamplerArgs& a, const RayGeom& g, uint32_t r, uint32_t slot, uint32_t excl,
                                             uint32_t count, uint32_t frame, const Footprint& f, uint32_t q00, uint32_t q10,
                                             uint32_t q01, uint32_t q11) {
    const TrainConsts& tc = a.tc;
    const uint32_t seed = ray_seed(frame, tc.dp_rank * tc.rays_per_batch + r);
    a.ray_index[slot] = r;
    float bg[3] = {1.0f, 1.0f, 1.0f};
    if (tc.background == 1u) {
        bg[0] = rand01(seed ^ kBgSalt0);
        bg[1] = rand01(seed ^ kBgSalt1);
        bg[2] = rand01(seed ^ kBgSalt2);
    }
    const float tx = f.tx, ty = f.ty;
    const float inv255 = 1.0f / 255.0f;
    const float omtx = __fsub_rn(1.0f, tx), omty = __fsub_rn(1.0f, ty);
    float v[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        const float s00 = __fmul_rn(static_cast<float>((q00 >> (8 * ch)) & 255u), inv255);
        const float s10 = __fmul_rn(static_cast<float>((q10 >> (8 * ch)) & 255u), inv255);
        const float s01 = __fmul_rn(static_cast<float>((q01 >> (8 * ch)) & 255u), inv255);
        const float s11 = __fmul_rn(static_cast<float>((q11 >> (8 * ch)) & 255u), inv255);
        const float ta = __fmaf_rn(s00, omtx, __fmul_rn(s10, tx));
        const float tb = __fmaf_rn(s01, omtx, __fmul_rn(s11, tx));
        v[ch] = __fmaf_rn(ta, omty, __fmul_rn(tb, ty));
    }
    RayRecord rec;
    rec.dir[0] = g.d[0];
    rec.dir[1] = g.d[1];
    rec.dir[2] = g.d[2];
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

// One 128-thread block per kept ray (grid-stride): thread k writes samples
// k, k+128, ... of the ray at their final offsets, each from its t in the
// ray's kept list (midpoint position and dt as the march defines them);
// threads 0-3 fetch the ray record's four ground-truth texels first.
constexpr uint32_t kWriteThreads = 128;
__global__ void __launch_bounds__(kWriteThreads) k_sample_write(const SamplerArgs a) {
    const TrainConsts& tc = a.tc;
    const uint32_t frame = a.state->frame_index;
    const uint32_t camera = train_camera(frame, tc.n_images);
    const uint32_t n_rays = min(a.state->n_rays, tc.max_rays);
    const uint32_t tid = threadIdx.x;
    const uint32_t* counts = counts_of(a, frame);
    for (uint32_t r = blockIdx.x; r < n_rays; r += gridDim.x) {
        const uint32_t count = counts[r], slot = a.ray_slot[r], excl = a.ray_offset[r];
        if (count == 0u || slot == 0xFFFFFFFFu) continue;
        const RayGeom g = a.geom[r];
        Footprint f{};
        uint32_t texel = 0u;
        if (tid < 4u) {
            f = footprint(tc, g, camera);
            const unsigned long long ti = (tid & 2u) ? ((tid & 1u) ? f.texel[3] : f.texel[2]) : ((tid & 1u) ? f.texel[1] : f.texel[0]);
            texel = __ldg(reinterpret_cast<const uint32_t*>(a.images) + ti);
        }
        const float* kt = a.kept_t + static_cast<unsigned long long>(r) * tc.max_steps;
        for (uint32_t si = tid; si < count; si += kWriteThreads) {
            const float t = kt[si];
            const float dt = march_dt(t, g.tf, g.dt_min, tc.cone);
            const float mid = march_mid(t, dt);
            a.pos_dt[excl + si] = make_float4(__fmaf_rn(mid, g.d[0], g.o[0]), __fmaf_rn(mid, g.d[1], g.o[1]),
                                              __fmaf_rn(mid, g.d[2], g.o[2]), dt);
            a.sample_ray[excl + si] = slot;
        }
        if (tid < 32u) {  // warp 0
            const uint32_t q00 = __shfl_sync(0xffffffffu, texel, 0), q10 = __shfl_sync(0xffffffffu, texel, 1);
            const uint32_t q01 = __shfl_sync(0xffffffffu, texel, 2), q11 = __shfl_sync(0xffffffffu, texel, 3);
            if (tid == 0u) write_record(a, g, r, slot, excl, count, frame, f, q00, q10, q01, q11);
        }
    }
}

}  // namespace

cudaError_t launch_march(const SamplerArgs& a, cudaStream_t s) {
    k_march<<<(a.tc.max_rays + kMarchBlock - 1u) / kMarchBlock, kMarchBlock, 0, s>>>(a);
    return cudaGetLastError();
}

namespace {
cudaError_t sm_blocks(uint32_t per_sm, uint32_t* blocks) {  // grid-stride kernels: blocks per SM x SMs
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    *blocks = static_cast<uint32_t>(sms) * per_sm;
    return cudaSuccess;
}
}  // namespace

// 16 resident blocks of 128 threads per SM: every SM takes rays from the start.
cudaError_t launch_sample_bits(const SamplerArgs& a, cudaStream_t s) {
    uint32_t blocks = 0;
    cudaError_t e = sm_blocks(16u, &blocks);
    if (e != cudaSuccess) return e;
    k_sample_bits<<<blocks, kBitsThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_sample_scan(const SamplerArgs& a, cudaStream_t s) {
    k_sample_scan<<<1, kScanThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_sample_write(const SamplerArgs& a, cudaStream_t s) {
    uint32_t blocks = 0;
    cudaError_t e = sm_blocks(16u, &blocks);
    if (e != cudaSuccess) return e;
    k_sample_write<<<blocks, kWriteThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_sampler(const SamplerArgs& a, cudaStream_t s) {
    cudaError_t e = launch_sample_bits(a, s);
    if (e == cudaSuccess) e = launch_sample_scan(a, s);
    if (e == cudaSuccess) e = launch_sample_write(a, s);
    return e;
}

}  // namespace nb
