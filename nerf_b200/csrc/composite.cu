// composite.cu -- front-to-back volume compositing with the alpha-weighted
// MSE of the reference and its analytic backward, fused in one kernel
// (reference backend-cuda.cu:1095-1182; density activation exp instead of
// softplus, a per-ray background instead of white, optional early ray
// termination).
//
// Per ray with samples i (raw density x_i, raw colour r_i, step dt_i):
//   sigma_i = exp(x_i), a_i = 1 - exp(-sigma_i dt_i), c_i = sigmoid(r_i)
//   T_0 = 1, T_{i+1} = T_i (1 - a_i); the ray stops before the first sample
//   with T_i < stop (stop > 0); C = sum T_i a_i c_i + T_end bg
//   loss = w |C - gt|^2 with w = 0.1 + 0.9 alpha_gt, g = 2 w (C - gt) inv_norm
//   dL/da_i = g . (T_i c_i - S_i / max(1e-6, 1 - a_i)),
//   S_i = T_end bg + sum_{j>i} T_j a_j c_j
//   dL/dx_i = dL/da_i dt_i exp(-sigma_i dt_i) exp(clamp(x_i, -15, 15))
//   dL/dr_i = T_i a_i g c_i (1 - c_i)
// Outputs are multiplied by the loss scale.
//
// One warp per ray, 32 consecutive samples per chunk (coalesced float4
// loads).  Forward: T_i from an inclusive product scan of (1 - a) across the
// warp times the carried transmittance; the early-termination cut is the
// first lane with T_i < stop (T is non-increasing, so a ballot finds it).
// T_i is parked in dout[i].x.  Backward: chunks from the last used one down,
// S_i from a reverse (suffix) sum scan plus the carried suffix of later
// chunks.  Summation order differs from the sequential CPU oracle, hence the
// tolerance of the parity test.
#include "common.cuh"
#include "kernels.h"

namespace nb {
namespace {

constexpr uint32_t kWarps = 8;

__device__ __forceinline__ float sigmoidf(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

__global__ void __launch_bounds__(kWarps * 32) k_composite(const CompositeArgs a) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    // Data parallel: this rank's sample count rides with the loss in the
    // exchanged MLP-gradient buffer, so every rank sizes its next batch from
    // the same global count (exact in fp32 below 2^24).
    if (!a.direct && a.dp_world > 1u && blockIdx.x == 0u && threadIdx.x == 0u)
        a.loss_slot[kMlpGradSamples - kMlpGradLoss] = static_cast<float>(a.state->n_samples);
    uint32_t n;
    float inv_norm;
    if (a.direct) {
        n = a.n_rays;
        inv_norm = a.inv_norm;
    } else {
        n = a.state->n_active;
        inv_norm = n == 0u ? 0.0f : __fdiv_rn(1.0f, __fmul_rn(static_cast<float>(n), static_cast<float>(a.dp_world)));
    }
    // Warp per ray, grid-stride over the rays: the grid is sized to the SMs
    // (one wave), not to the ray capacity, so the capacity's thousands of idle
    // blocks are never scheduled.
    float loss_sum = 0.0f;
    for (uint32_t k = blockIdx.x * kWarps + warp; k < n; k += gridDim.x * kWarps) {
        float loss = 0.0f;
        const RayRecord ray = a.rays[k];
        const uint32_t b = ray.begin, count = ray.count;
        const float stop = a.stop_transmittance;
        float T = 1.0f;
        float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f;
        uint32_t used = count;
        // Each chunk's loads are issued one chunk ahead.
        float4 r_next = make_float4(0.f, 0.f, 0.f, 0.f);
        float dt_next = 0.0f;
        if (lane < count) {
            r_next = a.raw[b + lane];
            dt_next = a.pos_dt[b + lane].w;
        }
        for (uint32_t base = 0; base < count; base += 32u) {
            const uint32_t i = base + lane;
            const bool valid = i < count;
            const float4 r = r_next;
            const float dt = fmaxf(0.0f, dt_next);
            if (i + 32u < count) {
                r_next = a.raw[b + i + 32u];
                dt_next = a.pos_dt[b + i + 32u].w;
            }
            const float al = valid ? __fsub_rn(1.0f, expf(-__fmul_rn(expf(r.x), dt))) : 0.0f;
            const float om = __fsub_rn(1.0f, al);
            float P = om;  // inclusive product of (1 - a) over lanes <= this one
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float x = __shfl_up_sync(0xffffffffu, P, o);
                if (lane >= static_cast<uint32_t>(o)) P = __fmul_rn(P, x);
            }
            float ex = __shfl_up_sync(0xffffffffu, P, 1);
            if (lane == 0u) ex = 1.0f;
            const float Ti = __fmul_rn(T, ex);
            const bool use = valid && !(stop > 0.0f && Ti < stop);
            const uint32_t use_mask = __ballot_sync(0xffffffffu, use);
            if (use) {
                a.dout[b + i].x = Ti;
                const float w = __fmul_rn(Ti, al);
                acc0 = __fmaf_rn(w, sigmoidf(r.y), acc0);
                acc1 = __fmaf_rn(w, sigmoidf(r.z), acc1);
                acc2 = __fmaf_rn(w, sigmoidf(r.w), acc2);
            }
            const uint32_t n_use = __popc(use_mask);
            const uint32_t n_valid = min(32u, count - base);
            if (n_use < n_valid) {  // termination inside this chunk: T_end is T of the first unused sample
                used = base + n_use;
                T = __shfl_sync(0xffffffffu, Ti, n_use);
                break;
            }
            T = __fmul_rn(T, __shfl_sync(0xffffffffu, P, 31));
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        acc2 = warp_sum(acc2);
        if (count > 0u) {
            const float ga = fminf(1.0f, fmaxf(0.0f, ray.gt[3]));
            const float ray_w = __fadd_rn(0.1f, __fmul_rn(0.9f, ga));
            const float d0 = __fsub_rn(__fadd_rn(acc0, __fmul_rn(T, ray.bg[0])), ray.gt[0]);
            const float d1 = __fsub_rn(__fadd_rn(acc1, __fmul_rn(T, ray.bg[1])), ray.gt[1]);
            const float d2 = __fsub_rn(__fadd_rn(acc2, __fmul_rn(T, ray.bg[2])), ray.gt[2]);
            loss = __fmul_rn(__fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)), __fmul_rn(d2, d2)), ray_w);
            const float two_w = __fmul_rn(2.0f, ray_w);
            const float g0 = __fmul_rn(__fmul_rn(two_w, d0), inv_norm);
            const float g1 = __fmul_rn(__fmul_rn(two_w, d1), inv_norm);
            const float g2 = __fmul_rn(__fmul_rn(two_w, d2), inv_norm);
            float s0 = __fmul_rn(T, ray.bg[0]), s1 = __fmul_rn(T, ray.bg[1]), s2 = __fmul_rn(T, ray.bg[2]);
            const float ls = a.loss_scale;
            if (used > 0u) {
                // Chunks from the last used one down, loads one chunk ahead.
                const int last = static_cast<int>((used - 1u) & ~31u);
                float4 rn = make_float4(0.f, 0.f, 0.f, 0.f);
                float dtn = 0.0f, tn = 0.0f;
                if (static_cast<uint32_t>(last) + lane < used) {
                    rn = a.raw[b + last + lane];
                    dtn = a.pos_dt[b + last + lane].w;
                    tn = a.dout[b + last + lane].x;
                }
                for (int base = last; base >= 0; base -= 32) {
                    const uint32_t i = static_cast<uint32_t>(base) + lane;
                    const bool valid = i < used;
                    const float4 r = rn;
                    const float dt = fmaxf(0.0f, dtn), trans = tn;
                    if (base >= 32) {  // every lane of an earlier chunk is below used
                        rn = a.raw[b + i - 32u];
                        dtn = a.pos_dt[b + i - 32u].w;
                        tn = a.dout[b + i - 32u].x;
                    }
                    const float e = expf(-__fmul_rn(expf(r.x), dt));
                    const float al = __fsub_rn(1.0f, e);
                    const float om = fmaxf(1e-6f, __fsub_rn(1.0f, al));
                    const float w = valid ? __fmul_rn(trans, al) : 0.0f;
                    const float c0 = sigmoidf(r.y), c1 = sigmoidf(r.z), c2 = sigmoidf(r.w);
                    const float wc0 = __fmul_rn(w, c0), wc1 = __fmul_rn(w, c1), wc2 = __fmul_rn(w, c2);
                    // inclusive suffix sums over lanes >= this one
                    float q0 = wc0, q1 = wc1, q2 = wc2;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const float x0 = __shfl_down_sync(0xffffffffu, q0, o);
                        const float x1 = __shfl_down_sync(0xffffffffu, q1, o);
                        const float x2 = __shfl_down_sync(0xffffffffu, q2, o);
                        if (lane + o < 32u) {
                            q0 = __fadd_rn(q0, x0);
                            q1 = __fadd_rn(q1, x1);
                            q2 = __fadd_rn(q2, x2);
                        }
                    }
                    float e0 = __shfl_down_sync(0xffffffffu, q0, 1);
                    float e1 = __shfl_down_sync(0xffffffffu, q1, 1);
                    float e2 = __shfl_down_sync(0xffffffffu, q2, 1);
                    if (lane == 31u) e0 = e1 = e2 = 0.0f;
                    const float S0 = __fadd_rn(s0, e0), S1 = __fadd_rn(s1, e1), S2 = __fadd_rn(s2, e2);
                    if (valid) {
                        float dL_da = __fmul_rn(g0, __fsub_rn(__fmul_rn(trans, c0), __fdiv_rn(S0, om)));
                        dL_da = __fadd_rn(dL_da, __fmul_rn(g1, __fsub_rn(__fmul_rn(trans, c1), __fdiv_rn(S1, om))));
                        dL_da = __fadd_rn(dL_da, __fmul_rn(g2, __fsub_rn(__fmul_rn(trans, c2), __fdiv_rn(S2, om))));
                        const float xcl = fminf(15.0f, fmaxf(-15.0f, r.x));
                        float4 o;
                        o.x = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(dL_da, dt), e), expf(xcl)));
                        o.y = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g0), c0), __fsub_rn(1.0f, c0)));
                        o.z = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g1), c1), __fsub_rn(1.0f, c1)));
                        o.w = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g2), c2), __fsub_rn(1.0f, c2)));
                        a.dout[b + i] = o;
                    }
                    s0 = __fadd_rn(s0, __shfl_sync(0xffffffffu, q0, 0));
                    s1 = __fadd_rn(s1, __shfl_sync(0xffffffffu, q1, 0));
                    s2 = __fadd_rn(s2, __shfl_sync(0xffffffffu, q2, 0));
                }
            }
            for (uint32_t i = used + lane; i < count; i += 32u) a.dout[b + i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (lane == 0u) {
            if (a.ray_loss) a.ray_loss[k] = loss;
            if (a.ray_used) a.ray_used[k] = used;
        }
        loss_sum += loss;
    }
    // Block sum of the ray losses (lane 0 of each warp holds its rays'), normalised, added to the loss slot.
    __shared__ float part[kWarps];
    if (lane == 0u) part[warp] = loss_sum;
    __syncthreads();
    if (threadIdx.x == 0u) {
        float bs = 0.0f;
        for (uint32_t w = 0; w < kWarps; ++w) bs += part[w];
        if (bs != 0.0f && a.loss_slot) atomicAdd(a.loss_slot, bs * inv_norm);
    }
}

}  // namespace

cudaError_t launch_composite(const CompositeArgs& a, cudaStream_t s) {
    const uint32_t rays = a.direct ? a.n_rays : a.max_rays;
    if (rays == 0u) return cudaSuccess;
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    const uint32_t want = (rays + kWarps - 1u) / kWarps, cap = 8u * static_cast<uint32_t>(sms);
    k_composite<<<want < cap ? want : cap, kWarps * 32u, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
