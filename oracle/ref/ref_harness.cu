// ref_harness.cu -- test-only launcher for the reference backend's own
// kernels, used to pin the CPU oracle (tests/golden/make_ref_goldens.py runs
// it on a GPU and commits the outputs as golden fixtures).
//
// The reference translation unit (backend-cuda.cu, compiled where it lies
// through a generated copy with one host-only line disabled, see Makefile) is
// included whole; this file only adds extern "C" entry points that launch
// its kernels on caller-provided device buffers, with the reference's own
// launch shapes:
//   sampler      k_sample_rays_flat          backend-cuda.cu:422-533 (128 threads, :644)
//   loss         k_ray_march_mse_grad        backend-cuda.cu:1095-1182 (256 threads)
//   step state   k_begin_training_step       backend-cuda.cu:1479-1488
//   Adam         k_prepare_adam_step_scalars backend-cuda.cu:1513-1536
//                k_adam_step_half            backend-cuda.cu:1537-1554
//   occupancy    k_update_occupancy_density / _bitfield, k_build_occ_inputs,
//                k_update_density_from_sigma, k_rebuild_occ_from_density
//                                            backend-cuda.cu:1555-1634
//   hashing      nerf::sampler hash_u32 / rand01 (:321-332), nerf::runtime
//                hash_u32 (:1439-1446)
// and two timing loops around the reference's own public entry points
// (nerf_train_step :2405-2420, nerf_inference :2436-2466), which give the
// reference-backend baseline of the training and render throughput.
//
// NERF_REF_PARITY builds a second variant in which the reference's
// approximate rsqrtf (used once, for the ray direction, :384) is replaced by
// a correctly rounded 1/sqrt: the sampler then computes exactly the
// arithmetic the oracle defines, so sample counts and positions can be
// compared bit for bit.  The stock variant is the reference as shipped.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cublas_v2.h>
#include <mma.h>

#include <cstdint>

#ifdef NERF_REF_PARITY
__device__ __forceinline__ float nerf_ref_rsqrt_correctly_rounded(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }
#define rsqrtf(x) nerf_ref_rsqrt_correctly_rounded(x)
#endif

#include "backend-cuda.patched.cu"

#ifdef NERF_REF_PARITY
#undef rsqrtf
#endif

namespace {

__global__ void k_ref_hash(const std::uint32_t* in, std::uint32_t* out_sampler, std::uint32_t* out_runtime, float* out_rand,
                           std::uint32_t n) {
    const std::uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out_sampler[i] = nerf::sampler::hash_u32(in[i]);
    out_runtime[i] = nerf::runtime::hash_u32(in[i]);
    out_rand[i] = nerf::sampler::rand01(in[i]);
}

int status(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }

// Adds one step's compacted sample count and kept ray count to acc[0], acc[1]
// (the reference exports no sample counter; this reads its SampleBatchState).
__global__ void k_ref_count_batch(const nerf::sampler::SampleBatchState* batch, unsigned long long* acc) {
    acc[0] += batch->sample_step_count;
    acc[1] += batch->active_ray_count;
}

nerf::runtime::TrainRuntime* ref_runtime(void* context) {
    auto* ctx = static_cast<nerf::runtime::ContextStorage*>(context);
    if (!ctx || !ctx->cuda_context) return nullptr;
    return ctx->cuda_context->train_runtime.get();
}

}  // namespace

extern "C" {

// Sizes of the reference's structs, for the caller's buffer allocation:
// SampleRay, SampleStep, SampleBatchState, TrainingDeviceState, AdamStepScalars.
void ref_struct_sizes(std::uint32_t out[5]) {
    out[0] = sizeof(nerf::sampler::SampleRay);
    out[1] = sizeof(nerf::sampler::SampleStep);
    out[2] = sizeof(nerf::sampler::SampleBatchState);
    out[3] = sizeof(nerf::runtime::TrainingDeviceState);
    out[4] = sizeof(nerf::network::AdamStepScalars);
}

int ref_hash(const std::uint32_t* d_in, std::uint32_t* d_sampler, std::uint32_t* d_runtime, float* d_rand, std::uint32_t n) {
    if (n == 0u) return 0;
    k_ref_hash<<<(n + 255u) / 256u, 256u>>>(d_in, d_sampler, d_runtime, d_rand, n);
    return status(cudaDeviceSynchronize());
}

// k_begin_training_step for one frame: writes {camera, occupancy mode} to out (host).
int ref_begin_step(std::uint32_t frame, std::uint32_t camera_count, std::uint32_t warmup, std::uint32_t interval,
                   void* d_state, std::uint32_t out[2]) {
    nerf::runtime::TrainingDeviceState st{};
    st.frame_index = frame;
    cudaError_t e = cudaMemcpy(d_state, &st, sizeof(st), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return status(e);
    nerf::runtime::k_begin_training_step<<<1, 1>>>(static_cast<nerf::runtime::TrainingDeviceState*>(d_state), camera_count,
                                                   warmup, interval);
    if ((e = cudaMemcpy(&st, d_state, sizeof(st), cudaMemcpyDeviceToHost)) != cudaSuccess) return status(e);
    out[0] = st.train_camera_idx;
    out[1] = st.occupancy_mode;
    return 0;
}

// k_sample_rays_flat with the step state {frame, camera}.  d_rays holds
// rays_per_batch SampleRay, d_steps rays_per_batch * max_steps SampleStep,
// d_batch one SampleBatchState; d_state one TrainingDeviceState.
int ref_sample_rays(std::uint32_t frame, std::uint32_t camera, void* d_state, const float* d_cams, const std::uint8_t* d_images,
                    std::uint32_t width, std::uint32_t height, float fx, float fy, float cx, float cy,
                    std::uint32_t rays_per_batch, std::uint32_t max_steps, const float aabb[6], const std::uint32_t* d_bitfield,
                    std::uint32_t grid_res, void* d_rays, void* d_steps, void* d_batch) {
    if (max_steps == 0u || max_steps > 256u) return -1;  // the reference's per-thread arrays hold 256 steps
    nerf::runtime::TrainingDeviceState st{};
    st.frame_index = frame;
    st.train_camera_idx = camera;
    cudaError_t e = cudaMemcpy(d_state, &st, sizeof(st), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return status(e);
    if ((e = cudaMemset(d_batch, 0, sizeof(nerf::sampler::SampleBatchState))) != cudaSuccess) return status(e);
    const float3 mn = make_float3(aabb[0], aabb[1], aabb[2]), mx = make_float3(aabb[3], aabb[4], aabb[5]);
    nerf::sampler::k_sample_rays_flat<<<(rays_per_batch + 127u) / 128u, 128u>>>(
        static_cast<const nerf::runtime::TrainingDeviceState*>(d_state), d_cams, d_images, width, height, fx, fy, cx, cy,
        rays_per_batch, max_steps, mn, mx, d_bitfield, grid_res, static_cast<nerf::sampler::SampleRay*>(d_rays),
        static_cast<nerf::sampler::SampleStep*>(d_steps), static_cast<nerf::sampler::SampleBatchState*>(d_batch));
    return status(cudaDeviceSynchronize());
}

// k_ray_march_mse_grad over the rays of a SampleBatchState (raw_rgb S x 3,
// raw_sigma S, trans_tmp S, loss_sum 1 float, zeroed here).
int ref_ray_march_mse_grad(const float* d_raw_rgb, const float* d_raw_sigma, const void* d_steps, const void* d_rays,
                           const void* d_batch, std::uint32_t max_ray_count, float* d_draw_rgb, float* d_draw_sigma,
                           float* d_trans, float* d_loss_sum) {
    cudaError_t e = cudaMemset(d_loss_sum, 0, sizeof(float));
    if (e != cudaSuccess) return status(e);
    if (max_ray_count == 0u) return 0;
    nerf::network::k_ray_march_mse_grad<<<(max_ray_count + 255u) / 256u, 256u>>>(
        d_raw_rgb, d_raw_sigma, static_cast<const nerf::sampler::SampleStep*>(d_steps),
        static_cast<const nerf::sampler::SampleRay*>(d_rays), static_cast<const nerf::sampler::SampleBatchState*>(d_batch),
        max_ray_count, d_draw_rgb, d_draw_sigma, d_trans, d_loss_sum);
    return status(cudaDeviceSynchronize());
}

// k_prepare_adam_step_scalars (state: optimizer_step, stats.grad_norm,
// stats.has_nonfinite) then k_adam_step_half.  scalars_out (host) receives
// the six AdamStepScalars fields as floats (skip_update as 0/1).
int ref_adam(float* d_p32, void* d_p16, const void* d_g16, float* d_m, float* d_v, std::uint32_t n, float beta1, float beta2,
             float eps, std::uint32_t optimizer_step, float grad_norm, std::uint32_t has_nonfinite, float lr,
             std::uint32_t lr_decay_ksteps, float clip, float guard, float loss_scale, void* d_state, void* d_scalars,
             float scalars_out[6]) {
    nerf::runtime::TrainingDeviceState st{};
    st.optimizer_step = optimizer_step;
    st.stats.grad_norm = grad_norm;
    st.stats.has_nonfinite = has_nonfinite;
    cudaError_t e = cudaMemcpy(d_state, &st, sizeof(st), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return status(e);
    auto* sc = static_cast<nerf::network::AdamStepScalars*>(d_scalars);
    nerf::runtime::k_prepare_adam_step_scalars<<<1, 1>>>(static_cast<const nerf::runtime::TrainingDeviceState*>(d_state), lr,
                                                         beta1, beta2, lr_decay_ksteps, clip, guard, loss_scale, sc);
    if (n != 0u)
        nerf::runtime::k_adam_step_half<<<(n + 255u) / 256u, 256u>>>(d_p32, static_cast<__half*>(d_p16),
                                                                     static_cast<const __half*>(d_g16), d_m, d_v, n, beta1,
                                                                     beta2, eps, sc);
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return status(e);
    nerf::network::AdamStepScalars h{};
    if ((e = cudaMemcpy(&h, sc, sizeof(h), cudaMemcpyDeviceToHost)) != cudaSuccess) return status(e);
    scalars_out[0] = h.learning_rate;
    scalars_out[1] = h.grad_scale;
    scalars_out[2] = h.inv_bias_correction1;
    scalars_out[3] = h.inv_bias_correction2;
    scalars_out[4] = h.inv_loss_scale;
    scalars_out[5] = static_cast<float>(h.skip_update);
    return 0;
}

// One occupancy update of the reference (backend-cuda.cu:2267-2291) for
// {frame, mode}: density decay / init, bitfield reset / init, query inputs
// (update_count rows of 7 floats) for the round-robin cells, density
// max-update from raw sigma (update_count values), bitfield rebuild.
int ref_occupancy(std::uint32_t frame, std::uint32_t mode, void* d_state, float* d_density, std::uint32_t* d_bitfield,
                  std::uint32_t grid_res, std::uint32_t update_count, const float aabb[6], float decay, float threshold,
                  const float* d_raw_sigma, float* d_inputs) {
    nerf::runtime::TrainingDeviceState st{};
    st.frame_index = frame;
    st.occupancy_mode = mode;
    cudaError_t e = cudaMemcpy(d_state, &st, sizeof(st), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return status(e);
    auto* s = static_cast<const nerf::runtime::TrainingDeviceState*>(d_state);
    const std::uint32_t cells = grid_res * grid_res * grid_res, words = (cells + 31u) / 32u;
    const float3 mn = make_float3(aabb[0], aabb[1], aabb[2]), mx = make_float3(aabb[3], aabb[4], aabb[5]);
    nerf::runtime::k_update_occupancy_density<<<(cells + 255u) / 256u, 256u>>>(d_density, cells, decay, s);
    nerf::runtime::k_update_occupancy_bitfield<<<(words + 255u) / 256u, 256u>>>(d_bitfield, words, s);
    if (update_count != 0u) {
        nerf::runtime::k_build_occ_inputs<<<(update_count + 255u) / 256u, 256u>>>(s, update_count, update_count, cells, grid_res,
                                                                                   mn, mx, d_inputs);
        nerf::runtime::k_update_density_from_sigma<<<(update_count + 255u) / 256u, 256u>>>(d_density, d_raw_sigma, s,
                                                                                             update_count, cells);
    }
    nerf::runtime::k_rebuild_occ_from_density<<<(cells + 255u) / 256u, 256u>>>(d_density, s, cells, threshold, d_bitfield);
    return status(cudaDeviceSynchronize());
}

// The last CUDA runtime error of the calling thread (cudaGetLastError: the
// reference's entry points report a failed runtime call only as a status),
// its name copied into name[len].
int ref_last_cuda_error(char* name, std::uint32_t len) {
    const cudaError_t e = cudaGetLastError();
    if (name && len) {
        const char* s = cudaGetErrorName(e);
        std::uint32_t i = 0;
        for (; s && s[i] && i + 1 < len; ++i) name[i] = s[i];
        name[i] = 0;
    }
    return static_cast<int>(e);
}

// The reference's own training step, timed: `steps` calls of its
// nerf_train_step (one graph launch each on the context's stream) between two
// CUDA events on that stream.  After every step a one-thread kernel adds the
// step's compacted sample and kept-ray counts to a device accumulator, so
// samples/s covers exactly the timed steps (about 2 us per step of the timed
// region is this counter).  out: {samples, rays}; *ms: device time.
int ref_train_timed(void* context, std::uint32_t steps, float* ms, std::uint64_t out[2]) {
    nerf::runtime::TrainRuntime* rt = ref_runtime(context);
    if (!rt || !rt->training_configured || !ms || !out) return -1;
    auto* ctx = static_cast<nerf::runtime::ContextStorage*>(context);
    const auto* batch = reinterpret_cast<const nerf::sampler::SampleBatchState*>(ctx->sample_batch_state.ptr);
    unsigned long long* acc = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaMalloc(&acc, 2 * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemsetAsync(acc, 0, 2 * sizeof(unsigned long long), rt->stream);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventRecord(e0, rt->stream);
    int rc = 0;
    for (std::uint32_t i = 0; e == cudaSuccess && rc == 0 && i < steps; ++i) {
        rc = static_cast<int>(nerf_train_step(context));
        if (rc == 0) {
            k_ref_count_batch<<<1, 1, 0, rt->stream>>>(batch, acc);
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess && rc == 0) e = cudaEventRecord(e1, rt->stream);
    if (e == cudaSuccess && rc == 0) e = cudaEventSynchronize(e1);
    if (e == cudaSuccess && rc == 0) e = cudaEventElapsedTime(ms, e0, e1);
    unsigned long long h[2] = {0, 0};
    if (e == cudaSuccess && rc == 0) e = cudaMemcpy(h, acc, sizeof(h), cudaMemcpyDeviceToHost);
    out[0] = h[0];
    out[1] = h[1];
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (acc) cudaFree(acc);
    return rc != 0 ? 1000 + rc : status(e);
}

// The reference's nerf_inference of dataset camera `camera_idx` at
// `samples_per_ray` uniform samples, timed with CUDA events on the context's
// stream (dst NULL: the image stays in the context's device buffer).
int ref_inference_timed(void* context, std::uint32_t camera_idx, std::uint32_t samples_per_ray, float* ms) {
    nerf::runtime::TrainRuntime* rt = ref_runtime(context);
    if (!rt || !ms) return -1;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventRecord(e0, rt->stream);
    int rc = 0;
    if (e == cudaSuccess) {
        NerfInferenceRequest req{camera_idx, samples_per_ray, NERF_MEMORY_CUDA_DEVICE, nullptr, 0};
        rc = static_cast<int>(nerf_inference(context, &req, nullptr));
    }
    if (e == cudaSuccess && rc == 0) e = cudaEventRecord(e1, rt->stream);
    if (e == cudaSuccess && rc == 0) e = cudaEventSynchronize(e1);
    if (e == cudaSuccess && rc == 0) e = cudaEventElapsedTime(ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    return rc != 0 ? 1000 + rc : status(e);
}

}  // extern "C"
