// composite.cu -- front-to-back volume compositing with the alpha-weighted
// MSE of the reference and its analytic backward, fused in one pass per ray
// (reference backend-cuda.cu:1095-1182; density activation exp instead of
// softplus, a per-ray background instead of white, and optional early ray
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
// Outputs are multiplied by the loss scale.  T_i is parked in dout[i].x by
// the forward sweep and read back by the backward sweep.
#include "common.cuh"
#include "kernels.h"

namespace nb {
namespace {

__device__ __forceinline__ float sigmoidf(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

__global__ void __launch_bounds__(256) k_composite(const CompositeArgs a) {
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t n;
    float inv_norm;
    if (a.direct) {
        n = a.n_rays;
        inv_norm = a.inv_norm;
    } else {
        n = a.state->n_active;
        inv_norm = n == 0u ? 0.0f : __fdiv_rn(1.0f, __fmul_rn(static_cast<float>(n), static_cast<float>(a.dp_world)));
    }
    float loss = 0.0f;
    if (k < n) {
        const RayRecord ray = a.rays[k];
        const uint32_t b = ray.begin, count = ray.count;
        const float stop = a.stop_transmittance;
        float T = 1.0f;
        float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f;
        uint32_t used = count;
        for (uint32_t i = 0; i < count; ++i) {
            if (stop > 0.0f && T < stop) {
                used = i;
                break;
            }
            const float4 r = a.raw[b + i];
            const float dt = fmaxf(0.0f, a.pos_dt[b + i].w);
            const float sigma = expf(r.x);
            const float al = __fsub_rn(1.0f, expf(-__fmul_rn(sigma, dt)));
            const float w = __fmul_rn(T, al);
            acc0 = __fadd_rn(acc0, __fmul_rn(w, sigmoidf(r.y)));
            acc1 = __fadd_rn(acc1, __fmul_rn(w, sigmoidf(r.z)));
            acc2 = __fadd_rn(acc2, __fmul_rn(w, sigmoidf(r.w)));
            a.dout[b + i].x = T;
            T = __fmul_rn(T, __fsub_rn(1.0f, al));
        }
        if (count > 0u) {
            const float ga = fminf(1.0f, fmaxf(0.0f, ray.gt[3]));
            const float ray_w = __fadd_rn(0.1f, __fmul_rn(0.9f, ga));
            const float p0 = __fadd_rn(acc0, __fmul_rn(T, ray.bg[0]));
            const float p1 = __fadd_rn(acc1, __fmul_rn(T, ray.bg[1]));
            const float p2 = __fadd_rn(acc2, __fmul_rn(T, ray.bg[2]));
            const float d0 = __fsub_rn(p0, ray.gt[0]), d1 = __fsub_rn(p1, ray.gt[1]), d2 = __fsub_rn(p2, ray.gt[2]);
            loss = __fmul_rn(__fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)), __fmul_rn(d2, d2)), ray_w);
            const float two_w = __fmul_rn(2.0f, ray_w);
            const float g0 = __fmul_rn(__fmul_rn(two_w, d0), inv_norm);
            const float g1 = __fmul_rn(__fmul_rn(two_w, d1), inv_norm);
            const float g2 = __fmul_rn(__fmul_rn(two_w, d2), inv_norm);
            float s0 = __fmul_rn(T, ray.bg[0]), s1 = __fmul_rn(T, ray.bg[1]), s2 = __fmul_rn(T, ray.bg[2]);
            const float ls = a.loss_scale;
            for (int i = static_cast<int>(used) - 1; i >= 0; --i) {
                const uint32_t s = b + static_cast<uint32_t>(i);
                const float4 r = a.raw[s];
                const float dt = fmaxf(0.0f, a.pos_dt[s].w);
                const float sigma = expf(r.x);
                const float e = expf(-__fmul_rn(sigma, dt));
                const float al = __fsub_rn(1.0f, e);
                const float om = fmaxf(1e-6f, __fsub_rn(1.0f, al));
                const float trans = a.dout[s].x;
                const float w = __fmul_rn(trans, al);
                const float c0 = sigmoidf(r.y), c1 = sigmoidf(r.z), c2 = sigmoidf(r.w);
                float dL_da = __fmul_rn(g0, __fsub_rn(__fmul_rn(trans, c0), __fdiv_rn(s0, om)));
                dL_da = __fadd_rn(dL_da, __fmul_rn(g1, __fsub_rn(__fmul_rn(trans, c1), __fdiv_rn(s1, om))));
                dL_da = __fadd_rn(dL_da, __fmul_rn(g2, __fsub_rn(__fmul_rn(trans, c2), __fdiv_rn(s2, om))));
                const float xcl = fminf(15.0f, fmaxf(-15.0f, r.x));
                const float dx = __fmul_rn(__fmul_rn(__fmul_rn(dL_da, dt), e), expf(xcl));
                float4 o;
                o.x = __fmul_rn(ls, dx);
                o.y = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g0), c0), __fsub_rn(1.0f, c0)));
                o.z = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g1), c1), __fsub_rn(1.0f, c1)));
                o.w = __fmul_rn(ls, __fmul_rn(__fmul_rn(__fmul_rn(w, g2), c2), __fsub_rn(1.0f, c2)));
                a.dout[s] = o;
                s0 = __fadd_rn(s0, __fmul_rn(w, c0));
                s1 = __fadd_rn(s1, __fmul_rn(w, c1));
                s2 = __fadd_rn(s2, __fmul_rn(w, c2));
            }
            for (uint32_t i = used; i < count; ++i) a.dout[b + i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (a.ray_loss) a.ray_loss[k] = loss;
        if (a.ray_used) a.ray_used[k] = used;
    }
    // Block sum of the ray losses, normalised and added to the loss slot.
    __shared__ float part[8];
    const float ws = warp_sum(loss);
    if ((threadIdx.x & 31u) == 0u) part[threadIdx.x >> 5] = ws;
    __syncthreads();
    if (threadIdx.x == 0u) {
        float bs = 0.0f;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) bs += part[w];
        if (bs != 0.0f && a.loss_slot) atomicAdd(a.loss_slot, bs * inv_norm);
    }
}

}  // namespace

cudaError_t launch_composite(const CompositeArgs& a, cudaStream_t s) {
    const uint32_t rays = a.direct ? a.n_rays : a.max_rays;
    if (rays == 0u) return cudaSuccess;
    k_composite<<<(rays + 255u) / 256u, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace nb
