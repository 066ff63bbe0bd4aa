// optimizer.cu -- end of a training step.
//
//   k_wgrad_reduce  sums the per-CTA MLP weight-gradient partials of the
//                   backward kernel (deterministic order); on one GPU the
//                   statistics kernel does this in its first blocks.
//   k_grad_stats    sum of squares and non-finite flag over all gradients
//                   (fp16 hash-table part, fp32 MLP part); the last block to
//                   finish derives the step statistics, the update guard,
//                   the clip scale, the learning-rate decay and the bias
//                   corrections, and commits the step (reference
//                   backend-cuda.cu:1451-1536: grad stats, finalize, Adam
//                   scalars and commit, folded into one launch).
//   k_adam          Adam on fp32 masters with the fp16 mirror, one pass over
//                   the flat parameter vector, 4 parameters per thread; the
//                   hash-table gradients are cleared behind it for the next
//                   step (reference backend-cuda.cu:1537-1554).
#include "common.cuh"
#include "kernels.h"

namespace nb {
namespace {

// Weight gradients from the backward's per-CTA partials ([c][kMlpParams]):
// a 256-thread block sums the partials of 32 consecutive parameters (one per
// lane).  Warp w adds rows c of the w-th eighth of the partials in order,
// reading one 128-byte line per row, with 32 rows' loads issued before their
// adds; the eight warp sums are then added in warp order.  Every block takes
// one memory round trip per 32 rows of its eighth, and the fixed order makes
// the result deterministic.  Returns the sum in warp 0 (lane = parameter).
constexpr uint32_t kWgradParamsPerBlock = 32;
constexpr uint32_t kWgradBlocks = kMlpParams / kWgradParamsPerBlock;
static_assert(kMlpParams % kWgradParamsPerBlock == 0, "whole blocks of weight gradients");

__device__ __forceinline__ float wgrad_block_sum(const float* __restrict__ partials, uint32_t n, uint32_t block) {
    __shared__ float ws[8][32];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t per = (n + 7u) / 8u;
    const uint32_t c0 = min(n, warp * per), c1 = min(n, c0 + per);
    const float* p = partials + block * kWgradParamsPerBlock + lane;
    float s = 0.0f;
    uint32_t c = c0;
    // Rows in batches of 32 with every load in flight before the adds; the
    // last, partial batch the same way (rows past c1 add an exact zero), so a
    // warp takes one memory round trip per batch.
    for (; c < c1; c += 32u) {
        float v[32];
#pragma unroll
        for (uint32_t k = 0; k < 32u; ++k)
            v[k] = c + k < c1 ? __ldcs(p + static_cast<unsigned long long>(c + k) * kMlpParams) : 0.0f;
#pragma unroll
        for (uint32_t k = 0; k < 32u; ++k) s += v[k];
    }
    ws[warp][lane] = s;
    __syncthreads();
    float g = 0.0f;
    if (warp == 0u) {
        g = ws[0][lane];
#pragma unroll
        for (uint32_t w = 1; w < 8u; ++w) g += ws[w][lane];
    }
    return g;
}

__global__ void __launch_bounds__(256) k_wgrad_reduce(const float* __restrict__ partials, uint32_t n_partials, float* mlp_grad) {
    const float g = wgrad_block_sum(partials, n_partials, blockIdx.x);
    if (threadIdx.x < 32u) mlp_grad[blockIdx.x * kWgradParamsPerBlock + threadIdx.x] = g;
}

__device__ __forceinline__ void adam_scalars(const TrainConsts& tc, float grad_norm, uint32_t nonfinite, uint32_t step,
                                             AdamScalars& o) {
    const bool skip = nonfinite != 0u || !isfinite(grad_norm) || grad_norm > tc.guard;
    o.learning_rate = 0.0f;
    o.grad_scale = 1.0f;
    o.inv_bias_correction1 = 1.0f;
    o.inv_bias_correction2 = 1.0f;
    if (!skip) {
        const float decay = static_cast<float>(tc.lr_decay_ksteps) * 1000.0f;
        o.learning_rate = decay > 0.0f ? tc.lr * powf(0.1f, static_cast<float>(step) / decay) : tc.lr;
        o.grad_scale = grad_norm > tc.clip && grad_norm > 0.0f ? tc.clip / grad_norm : 1.0f;
        o.inv_bias_correction1 = 1.0f / (1.0f - powf(tc.beta1, static_cast<float>(step)));
        o.inv_bias_correction2 = 1.0f / (1.0f - powf(tc.beta2, static_cast<float>(step)));
    }
    o.inv_loss_scale = 1.0f / tc.loss_scale;
    o.skip_update = skip ? 1u : 0u;
}

__global__ void __launch_bounds__(256) k_grad_stats(const OptimArgs a) {
    uint64_t n_chunks = a.n_params / 8u;
    const uint64_t grid_chunks = a.n_grid / 8u;
    const uint4* gg = static_cast<const uint4*>(a.grid_grad);
    float sum = 0.0f;
    uint32_t bad = 0u;
    // Data-parallel peer mode: the grid part was reduced by k_dp_reduce_grads.
    uint64_t q0 = a.dp_peer ? grid_chunks : 0u;
    uint64_t first = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    if (a.fuse_wgrad) {
        // The first blocks sum the backward's per-CTA weight-gradient partials
        // (fixed order) and take the MLP part of the statistics; the others
        // take the hash-table part.
        if (blockIdx.x < kWgradBlocks) {
            const float g = wgrad_block_sum(a.partials, a.n_partials, blockIdx.x);
            if (threadIdx.x < 32u) {
                a.mlp_grad[blockIdx.x * kWgradParamsPerBlock + threadIdx.x] = g;
                if (!isfinite(g)) bad = 1u;
                else sum = g * g;
            }
            n_chunks = 0u;
        } else {
            n_chunks = grid_chunks;
            first = static_cast<uint64_t>(blockIdx.x - kWgradBlocks) * blockDim.x + threadIdx.x;
            stride = static_cast<uint64_t>(gridDim.x - kWgradBlocks) * blockDim.x;
        }
    }
    // Hash-table part: four 16-byte loads in flight per thread before their
    // sums (the loop is a chain of memory round trips otherwise); the same
    // chunks in the same order as one at a time.
    uint64_t q = q0 + first;
    const uint64_t grid_end = n_chunks < grid_chunks ? n_chunks : grid_chunks;
    for (; q + 3u * stride < grid_end; q += 4u * stride) {
        uint4 u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = gg[q + j * stride];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = unpack_h2(w[k]);
                if (!isfinite(f.x)) bad = 1u;
                else sum = fmaf(f.x, f.x, sum);
                if (!isfinite(f.y)) bad = 1u;
                else sum = fmaf(f.y, f.y, sum);
            }
        }
    }
    for (; q < n_chunks; q += stride) {
        float v[8];
        if (q < grid_chunks) {
            const uint4 u = gg[q];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = unpack_h2(w[k]);
                v[2 * k] = f.x;
                v[2 * k + 1] = f.y;
            }
        } else {
            const float4* mg = reinterpret_cast<const float4*>(a.mlp_in + 8u * (q - grid_chunks));
            const float4 x = mg[0], y = mg[1];
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
            v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (!isfinite(v[k])) bad = 1u;
            else sum = fmaf(v[k], v[k], sum);
        }
    }
    __shared__ float ps[8];
    __shared__ uint32_t pb[8];
    __shared__ bool last;
    const float ws = warp_sum(sum);
    const uint32_t wb = __any_sync(0xffffffffu, bad != 0u) ? 1u : 0u;
    if ((threadIdx.x & 31u) == 0u) {
        ps[threadIdx.x >> 5] = ws;
        pb[threadIdx.x >> 5] = wb;
    }
    __syncthreads();
    if (threadIdx.x == 0u) {
        float bs = 0.0f;
        uint32_t bb = 0u;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) {
            bs += ps[w];
            bb |= pb[w];
        }
        if (bs != 0.0f) atomicAdd(&a.state->grad_sumsq, bs);
        if (bb) atomicOr(&a.state->nonfinite, 1u);
        __threadfence();
        last = atomicAdd(&a.state->done_blocks, 1u) == gridDim.x - 1u;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0u) return;
    __threadfence();
    DeviceState* st = a.state;
    const TrainConsts& tc = a.tc;
    float sumsq = atomicAdd(&st->grad_sumsq, 0.0f);
    uint32_t nonfinite = atomicOr(&st->nonfinite, 0u);
    if (a.dp_peer) {  // every rank's owned range, in rank order (the same sum on every rank)
        const volatile DpSync* me = a.dp.sync[a.dp.rank];
        for (uint32_t r = 0; r < a.dp.world; ++r) {
            sumsq += me->partials[r][0];
            nonfinite |= me->partials[r][1] > 0.0f ? 1u : 0u;
        }
    }
    const float loss = *reinterpret_cast<volatile const float*>(a.mlp_in + kMlpGradLoss);
    const float grad_norm = sqrtf(fmaxf(0.0f, sumsq)) / tc.loss_scale;
    const uint32_t has_nonfinite = (nonfinite != 0u || !isfinite(loss) || !isfinite(grad_norm)) ? 1u : 0u;
    const uint32_t frame = st->frame_index;
    const uint32_t step = frame + 1u;
    st->stats.loss = loss;
    st->stats.grad_norm = grad_norm;
    st->stats.has_nonfinite = has_nonfinite;
    st->stats.completed_steps = step;
    st->stats.last_train_camera = train_camera(frame, tc.n_images);
    if (a.stats_host) {  // the host reads the statistics without a copy
        volatile StatsBlock* h = a.stats_host;
        h->loss = loss;
        h->grad_norm = grad_norm;
        h->has_nonfinite = has_nonfinite;
        h->completed_steps = step;
        h->last_train_camera = train_camera(frame, tc.n_images);
        __threadfence_system();
    }
    AdamScalars sc;
    adam_scalars(tc, grad_norm, has_nonfinite, step, sc);
    st->adam = sc;
    const uint32_t samples = st->n_samples, rays = st->n_rays;
    st->last_samples = samples;
    st->last_active = st->n_active;
    st->last_rays = rays;
    st->total_samples += samples;
    st->total_rays += rays;
    if (tc.target_samples != 0u) {
        // Data parallel: every rank marches the same number of rays, sized from
        // the samples of all ranks against the target of all ranks, so that no
        // rank's batch drifts from the others' and the barriers wait less.
        unsigned long long tot = samples, tgt = tc.target_samples;
        if (a.world > 1u) {
            tot = static_cast<unsigned long long>(*reinterpret_cast<volatile const float*>(a.mlp_in + kMlpGradSamples));
            tgt *= a.world;
        }
        unsigned long long next = tot == 0u ? 2ull * rays : static_cast<unsigned long long>(rays) * tgt / tot;
        next = next < 128ull ? 128ull : next;
        next = next > tc.max_rays ? tc.max_rays : next;
        st->n_rays = static_cast<uint32_t>(next);
    }
    st->frame_index = step;
    st->grad_sumsq = 0.0f;
    st->nonfinite = 0u;
    st->done_blocks = 0u;
    a.mlp_grad[kMlpGradLoss] = 0.0f;
}

// Adam state of 4 consecutive parameters: loss-scaled gradients, master
// weights and moments.  Masters and moments are touched once per step: they
// are streamed (evict-first) so that they do not push the hash table out of
// L2.
struct Chunk {
    float g[4];
    float4 w, m, v;
};

__device__ __forceinline__ void load_chunk(const OptimArgs& a, uint64_t q, uint64_t grid_chunks, Chunk& c) {
    if (a.dp_peer && q < grid_chunks) {  // summed gradients of the owned range
        const float4 x = reinterpret_cast<const float4*>(a.dp.gsum)[q - a.dp.lo / 4u];
        c.g[0] = x.x;
        c.g[1] = x.y;
        c.g[2] = x.z;
        c.g[3] = x.w;
    } else if (q < grid_chunks) {
        const uint2 u = static_cast<const uint2*>(a.grid_grad)[q];
        const float2 f0 = unpack_h2(u.x), f1 = unpack_h2(u.y);
        c.g[0] = f0.x;
        c.g[1] = f0.y;
        c.g[2] = f1.x;
        c.g[3] = f1.y;
    } else {
        const float4 x = reinterpret_cast<const float4*>(a.mlp_in)[q - grid_chunks];
        c.g[0] = x.x;
        c.g[1] = x.y;
        c.g[2] = x.z;
        c.g[3] = x.w;
    }
    c.w = __ldcs(reinterpret_cast<const float4*>(a.master) + q);
    c.m = __ldcs(reinterpret_cast<const float4*>(a.m) + q);
    c.v = __ldcs(reinterpret_cast<const float4*>(a.v) + q);
}

__device__ __forceinline__ void adam_chunk(const OptimArgs& a, uint64_t q, uint64_t grid_chunks, Chunk& c, const AdamScalars& s) {
    if (q < grid_chunks && !a.dp_peer) static_cast<uint2*>(a.grid_grad)[q] = make_uint2(0u, 0u);  // cleared for the next step
    if (s.skip_update) return;
    float* w = reinterpret_cast<float*>(&c.w);
    float* mm = reinterpret_cast<float*>(&c.m);
    float* vv = reinterpret_cast<float*>(&c.v);
    const float b1 = a.tc.beta1, b2 = a.tc.beta2;
    const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float gk = __fmul_rn(__fmul_rn(c.g[k], s.inv_loss_scale), s.grad_scale);
        // b*m + (1-b)*g with the first product fused, as the reference's
        // compiler contracts it (backend-cuda.cu:1546-1547).
        const float mi = __fmaf_rn(b1, mm[k], __fmul_rn(omb1, gk));
        const float vi = __fmaf_rn(b2, vv[k], __fmul_rn(__fmul_rn(omb2, gk), gk));
        const float num = __fmul_rn(s.learning_rate, __fmul_rn(mi, s.inv_bias_correction1));
        const float den = __fadd_rn(__fsqrt_rn(__fmul_rn(vi, s.inv_bias_correction2)), a.tc.eps);
        w[k] = __fsub_rn(w[k], __fdiv_rn(num, den));
        mm[k] = mi;
        vv[k] = vi;
    }
    __stcs(reinterpret_cast<float4*>(a.master) + q, c.w);
    __stcs(reinterpret_cast<float4*>(a.m) + q, c.m);
    __stcs(reinterpret_cast<float4*>(a.v) + q, c.v);
    const uint2 h = make_uint2(pack_h2(w[0], w[1]), pack_h2(w[2], w[3]));
    if (a.dp_peer && q < grid_chunks) {
        for (uint32_t r = 0; r < a.dp.world; ++r) reinterpret_cast<uint2*>(a.dp.p16[r])[q] = h;  // every rank's mirror
    } else {
        reinterpret_cast<uint2*>(a.params16)[q] = h;
    }
}

// Grid-stride pass over 4-parameter chunks of the flat vector (hash part
// first).  The loads of the next chunk are issued before the current one is
// updated, and the first chunk's loads before the step scalars are read, so
// each thread keeps two chunks of loads in flight.
// Chunk k of the pass: the whole flat vector, or (data-parallel peer mode)
// the owned grid range followed by the MLP part.
__device__ __forceinline__ uint64_t adam_chunk_index(const OptimArgs& a, uint64_t k, uint64_t grid_chunks) {
    if (!a.dp_peer) return k;
    const uint64_t lo = a.dp.lo / 4u, own = (a.dp.hi - a.dp.lo) / 4u;
    return k < own ? lo + k : grid_chunks + (k - own);
}

__global__ void __launch_bounds__(256) k_adam(const OptimArgs a, const AdamScalars* __restrict__ sp, const AdamScalars direct) {
    const uint64_t grid_chunks = a.n_grid / 4u;
    const uint64_t n_chunks = a.dp_peer ? (a.dp.hi - a.dp.lo) / 4u + (a.n_params - a.n_grid) / 4u : a.n_params / 4u;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint64_t k = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= n_chunks) return;
    Chunk cur;
    uint64_t q = adam_chunk_index(a, k, grid_chunks);
    load_chunk(a, q, grid_chunks, cur);
    const AdamScalars s = sp ? *sp : direct;
    for (;;) {
        const uint64_t kn = k + stride;
        Chunk nxt;
        const bool more = kn < n_chunks;
        const uint64_t qn = more ? adam_chunk_index(a, kn, grid_chunks) : 0u;
        if (more) load_chunk(a, qn, grid_chunks, nxt);
        adam_chunk(a, q, grid_chunks, cur, s);
        if (!more) break;
        cur = nxt;
        k = kn;
        q = qn;
    }
}

// Data-parallel peer mode: every rank's gradients of the owned range, 8 per
// thread (16-byte loads over NVLink), summed in fp32 in rank order; every
// rank's MLP gradients and loss, summed in rank order into mlp_sum.  The last
// block publishes the owned range's sum of squares to every rank.
__global__ void __launch_bounds__(256) k_dp_reduce_grads(const OptimArgs a) {
    const uint64_t lo8 = a.dp.lo / 8u, hi8 = a.dp.hi / 8u;
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = tid; i < kMlpGradSlots / 4u; i += stride) {
        float4 x[kMaxDpWorld];
#pragma unroll
        for (uint32_t r = 0; r < kMaxDpWorld; ++r)  // all loads in flight before the sum
            x[r] = r < a.dp.world ? __ldcv(reinterpret_cast<const float4*>(a.dp.mlp[r]) + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 s4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (uint32_t r = 0; r < kMaxDpWorld; ++r) {
            if (r >= a.dp.world) break;
            s4.x += x[r].x;
            s4.y += x[r].y;
            s4.z += x[r].z;
            s4.w += x[r].w;
        }
        reinterpret_cast<float4*>(a.dp.mlp_sum)[i] = s4;
    }
    float sum = 0.0f;
    uint32_t bad = 0u;
    for (uint64_t q = lo8 + tid; q < hi8; q += stride) {
        uint4 u[kMaxDpWorld];
#pragma unroll
        for (uint32_t r = 0; r < kMaxDpWorld; ++r)  // all loads in flight before the sum
            u[r] = r < a.dp.world ? __ldcv(static_cast<const uint4*>(a.dp.grad[r]) + q) : make_uint4(0u, 0u, 0u, 0u);
        float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (uint32_t r = 0; r < kMaxDpWorld; ++r) {
            if (r >= a.dp.world) break;
            const uint32_t w[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = unpack_h2(w[k]);
                v[2 * k] += f.x;
                v[2 * k + 1] += f.y;
            }
        }
        float4* dst = reinterpret_cast<float4*>(a.dp.gsum + (q - lo8) * 8u);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (!isfinite(v[k])) bad = 1u;
            else sum = fmaf(v[k], v[k], sum);
        }
    }
    __shared__ float ps[8];
    __shared__ uint32_t pb[8];
    __shared__ bool last;
    const float ws = warp_sum(sum);
    const uint32_t wb = __any_sync(0xffffffffu, bad != 0u) ? 1u : 0u;
    if ((threadIdx.x & 31u) == 0u) {
        ps[threadIdx.x >> 5] = ws;
        pb[threadIdx.x >> 5] = wb;
    }
    __syncthreads();
    DpSync* me = a.dp.sync[a.dp.rank];
    if (threadIdx.x == 0u) {
        float bs = 0.0f;
        uint32_t bb = 0u;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) {
            bs += ps[w];
            bb |= pb[w];
        }
        if (bs != 0.0f) atomicAdd(&me->sum, bs);
        if (bb) atomicOr(&me->bad, 1u);
        __threadfence();
        last = atomicAdd(&me->done, 1u) == gridDim.x - 1u;
    }
    __syncthreads();
    if (!last || threadIdx.x >= a.dp.world) return;
    __threadfence();
    const float total = atomicAdd(&me->sum, 0.0f);
    const float flag = atomicOr(&me->bad, 0u) ? 1.0f : 0.0f;
    DpSync* dst = a.dp.sync[threadIdx.x];  // every rank's slot for this rank
    dst->partials[a.dp.rank][0] = total;
    dst->partials[a.dp.rank][1] = flag;
    __syncwarp(0xffffffffu >> (32u - a.dp.world));
    if (threadIdx.x == 0u) {
        me->sum = 0.0f;
        me->bad = 0u;
        me->done = 0u;
    }
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(32) k_dp_barrier(const DpPeers d) {
    __shared__ uint32_t epoch;
    DpSync* me = d.sync[d.rank];
    if (threadIdx.x == 0u) {
        epoch = me->epoch + 1u;
        me->epoch = epoch;
    }
    __syncthreads();
    const uint32_t t = threadIdx.x;
    if (t < d.world) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(&d.sync[t]->flags[d.rank]), "r"(epoch) : "memory");
        const uint64_t t0 = global_ns();
        for (;;) {
            uint32_t seen;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(seen) : "l"(&me->flags[t]) : "memory");
            if (static_cast<int32_t>(seen - epoch) >= 0) break;
            if (global_ns() - t0 > d.timeout_ns) {  // give up, report, go on
                atomicExch(&me->error, 1u);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    __threadfence_system();
}

__global__ void k_f32_to_f16(const float* __restrict__ src, __half* __restrict__ dst, uint64_t n) {
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

// dst[i] = scale * (draw i of a splitmix64 stream from state0), the draw a
// uniform in [-1, 1) from its top 24 bits.  splitmix64's state advances by a
// constant per draw, so draw i is a function of i alone and the fill runs one
// thread per value, bit-identical to drawing the stream in order.
__global__ void k_splitmix_fill(float* __restrict__ dst, uint64_t n, uint64_t state0, float scale) {
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        uint64_t z = state0 + (i + 1u) * 0x9e3779b97f4a7c15ull;
        z = (z ^ (z >> 30u)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27u)) * 0x94d049bb133111ebull;
        z ^= z >> 31u;
        const float u24 = static_cast<float>(static_cast<uint32_t>(z >> 32u) >> 8u);
        const float unit = __fsub_rn(__fmul_rn(__fmul_rn(u24, 1.0f / 16777216.0f), 2.0f), 1.0f);
        dst[i] = __fmul_rn(unit, scale);
    }
}

uint32_t g_sms = 0;
uint32_t sm_count() {
    if (g_sms == 0u) {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_sms = static_cast<uint32_t>(sms);
    }
    return g_sms;
}

}  // namespace

// Blocks of the statistics kernel's parameter part: as many as are resident
// beside the weight-gradient blocks (fused form), so that the whole grid is
// one wave -- a second wave of a few blocks would take as long as the first.
uint32_t grad_stats_blocks(uint64_t n_params, bool fused) {
    static const int per_sm = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_grad_stats, 256, 0) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = 4;
        }
        return n;
    }();
    const uint64_t chunks = n_params / 8u;
    const uint64_t want = (chunks + 255u) / 256u;
    const uint64_t resident = static_cast<uint64_t>(per_sm) * sm_count();
    uint64_t cap = resident;
    if (fused) cap = resident >= kWgradBlocks + sm_count() ? resident - kWgradBlocks : sm_count();
    return static_cast<uint32_t>(want < cap ? (want == 0 ? 1 : want) : cap);
}

cudaError_t launch_wgrad_reduce(const OptimArgs& a, cudaStream_t s) {
    k_wgrad_reduce<<<kWgradBlocks, 256, 0, s>>>(a.partials, a.n_partials, a.mlp_grad);
    return cudaGetLastError();
}
cudaError_t launch_grad_stats(const OptimArgs& a, cudaStream_t s) {
    if (a.fuse_wgrad && (a.dp_peer || a.n_partials == 0u)) return cudaErrorInvalidValue;
    k_grad_stats<<<a.stats_blocks + (a.fuse_wgrad ? kWgradBlocks : 0u), 256, 0, s>>>(a);
    return cudaGetLastError();
}
cudaError_t launch_dp_reduce_grads(const OptimArgs& a, cudaStream_t s) {
    if (!a.dp_peer || a.dp.world == 0u || a.dp.world > kMaxDpWorld) return cudaErrorInvalidValue;
    k_dp_reduce_grads<<<4u * sm_count(), 256, 0, s>>>(a);
    return cudaGetLastError();
}
cudaError_t launch_dp_barrier(const DpPeers& d, cudaStream_t s) {
    if (d.world == 0u || d.world > kMaxDpWorld || d.rank >= d.world) return cudaErrorInvalidValue;
    k_dp_barrier<<<1, 32, 0, s>>>(d);
    return cudaGetLastError();
}
cudaError_t launch_adam(const OptimArgs& a, cudaStream_t s) {
    const uint64_t chunks = a.dp_peer ? (a.dp.hi - a.dp.lo) / 4u + (a.n_params - a.n_grid) / 4u : a.n_params / 4u;
    uint64_t blocks = (chunks + 255u) / 256u;
    const uint64_t cap = 4ull * sm_count();  // 4 resident blocks per SM, grid-stride beyond
    if (blocks > cap) blocks = cap;
    if (blocks == 0u) blocks = 1u;
    k_adam<<<static_cast<uint32_t>(blocks), 256, 0, s>>>(a, a.state ? &a.state->adam : nullptr, a.direct_scalars);
    return cudaGetLastError();
}
cudaError_t launch_f32_to_f16(const float* src, void* dst, uint64_t n, cudaStream_t s) {
    if (n == 0u) return cudaSuccess;
    uint64_t blocks = (n + 255u) / 256u;
    if (blocks > 4096u) blocks = 4096u;
    k_f32_to_f16<<<static_cast<uint32_t>(blocks), 256, 0, s>>>(src, static_cast<__half*>(dst), n);
    return cudaGetLastError();
}
cudaError_t launch_splitmix_fill(float* dst, uint64_t n, uint64_t state0, float scale, cudaStream_t s) {
    if (n == 0u) return cudaSuccess;
    const uint64_t want = (n + 255u) / 256u, cap = 8ull * sm_count();
    k_splitmix_fill<<<static_cast<uint32_t>(want < cap ? want : cap), 256, 0, s>>>(dst, n, state0, scale);
    return cudaGetLastError();
}

}  // namespace nb
