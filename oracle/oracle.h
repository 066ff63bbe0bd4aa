/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A scalar C++ restatement, on the host, of the NeRF train/render hot path
 * that libnerf_b200.so runs on the GPU.  It exists to check the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference leg load liboracle.so.  Nothing in the product links it.
 *
 * Two kinds of semantics live here:
 *  - restated from the reference backend (Xayah-Graphics/NeRF
 *    backend-cuda.cu): step/camera hash, pixel RNG, ray generation, AABB
 *    clipping, cone-angle marching against the occupancy bitfield, ground
 *    truth bilinear fetch, occupancy decay/max/threshold, alpha-weighted MSE
 *    with its analytic backward, gradient statistics + update guard, Adam with
 *    fp32 masters, splitmix Xavier initialisation.  Each function cites the
 *    reference line it follows.  These are pinned against the reference's own
 *    kernels run on a B200 (tests/golden/ref_*.json, made by
 *    tests/golden/make_ref_goldens.py through oracle/_ref).
 *  - defined here because the reference has no such code (it uses a frequency
 *    encoding and 128-wide MLPs): the multiresolution hash grid, degree-4
 *    spherical harmonics, the 32->64->16 / 32->64->64->16 MLPs and the
 *    trunc_exp density activation.  For these the oracle IS the definition
 *    (parity unpinned by the reference); the formulas follow the published
 *    instant-ngp method (Mueller et al., SIGGRAPH 2022).
 *
 * Sign/ordering conventions that the CUDA path must reproduce bit-exactly on
 * integer outputs (hash indices, bitfield, per-ray sample counts, offsets)
 * are spelled out at each function in oracle_core.cpp.
 */
#ifndef NERF_ORACLE_H
#define NERF_ORACLE_H

#include <stdint.h>
#include "../include/nerf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- integer primitives (reference backend-cuda.cu:321-332, 1439-1446, 1479-1488) ---- */
uint32_t oracle_hash_u32(uint32_t x);
float oracle_rand01(uint32_t seed);
uint32_t oracle_train_camera(uint32_t frame_index, uint32_t image_count);
uint32_t oracle_occupancy_mode(uint32_t frame_index, uint32_t warmup_steps, uint32_t update_interval);

/* ---- initialisation (reference backend-cuda.cu:1810-1847) ---- */
/* Fills n_matrices fan_out x fan_in matrices back to back with the splitmix
 * uniform Xavier draw of the reference, stream seeded from (seed_a, seed_b). */
void oracle_splitmix_xavier(uint64_t seed_a, uint64_t seed_b, const uint32_t* fan_in, const uint32_t* fan_out,
                            uint32_t n_matrices, float* out);
/* Uniform(-scale, scale) draws from the same generator. */
void oracle_splitmix_uniform(uint64_t seed_a, uint64_t seed_b, uint64_t count, float scale, float* out);

/* ---- hash grid ---- */
#define ORACLE_MAX_LEVELS 32
typedef struct OracleGridLayout {
    uint32_t n_levels;
    uint32_t log2_hashmap_size;
    uint32_t base_resolution;
    uint32_t max_resolution;
    float scale[ORACLE_MAX_LEVELS];
    uint32_t resolution[ORACLE_MAX_LEVELS]; /* vertices per axis */
    uint32_t dense[ORACLE_MAX_LEVELS];
    uint32_t offset[ORACLE_MAX_LEVELS + 1]; /* in entries (2 fp16 features each) */
} OracleGridLayout;
int oracle_grid_layout(uint32_t n_levels, uint32_t log2_hashmap_size, uint32_t base_resolution, uint32_t max_resolution,
                       OracleGridLayout* out);
/* idx/w: n x L x 8 corner entry indices (absolute, offset included) and weights. */
void oracle_grid_corners(const OracleGridLayout* g, const float* pos_unit, uint32_t n, uint32_t* idx, float* w);
/* params: fp16 bits, entries x 2.  feat: fp16 bits, n x 2L. */
void oracle_grid_forward(const OracleGridLayout* g, const uint16_t* params, const float* pos_unit, uint32_t n,
                         uint16_t* feat);
/* dfeat: fp32 n x 2L; grad accumulated (+=) in double, entries x 2. */
void oracle_grid_backward(const OracleGridLayout* g, const float* pos_unit, const float* dfeat, uint32_t n, double* grad);

/* ---- direction encoding ---- */
void oracle_sh4(const float* dirs, uint32_t n, float* out16);

/* ---- MLPs (fp16 operands, fp32 accumulation) ---- */
#define ORACLE_MLP_PARAMS 10240u
/* mlp: fp16 bits, 10240 values laid out as
 *   density W0 [64][32] | density W1 [16][64] | colour W0 [64][32] | colour W1 [64][64] | colour W2 [16][64]
 * feat: fp16 bits n x 32; dirs n x 3 (unit); out n x 4 (raw sigma, raw r, g, b). */
void oracle_mlp_forward(const uint16_t* mlp, const uint16_t* feat, const float* dirs, uint32_t n, float* out);
/* dout n x 4 (loss-scaled d raw sigma, d raw rgb); dfeat n x 32 out (fp32);
 * wgrad 10240 accumulated (+=) in double. */
void oracle_mlp_backward(const uint16_t* mlp, const uint16_t* feat, const float* dirs, const float* dout, uint32_t n,
                         float* dfeat, double* wgrad);

/* ---- compositing + loss (reference backend-cuda.cu:1095-1182) ---- */
/* raw: S x 4 per sample (raw sigma, raw rgb); dt: S; rays: begin[r], count[r];
 * gt: R x 4 (composited rgb, alpha); bg: R x 3.  Writes dout S x 4
 * (loss_scale * dL/draw), loss per ray, and the number of samples used per
 * ray (early termination). */
void oracle_composite(const float* raw, const float* dt, const uint32_t* begin, const uint32_t* count, uint32_t n_rays,
                      const float* gt, const float* bg, float inv_norm, float loss_scale, float stop_transmittance,
                      float* dout, float* ray_loss, uint32_t* used, float* rgb_out);

/* ---- Adam (reference backend-cuda.cu:1513-1554) ---- */
typedef struct OracleAdamScalars {
    float learning_rate;
    float grad_scale;
    float inv_bias_correction1;
    float inv_bias_correction2;
    float inv_loss_scale;
    uint32_t skip_update;
} OracleAdamScalars;
void oracle_adam_scalars(float grad_norm, uint32_t has_nonfinite, uint32_t optimizer_step, const NerfHyperParams* hp,
                         OracleAdamScalars* out);
void oracle_adam(float* master, uint16_t* param16, const float* grad, float* m, float* v, uint64_t n, float beta1,
                 float beta2, float eps, const OracleAdamScalars* s);

/* ---- occupancy maintenance (reference backend-cuda.cu:1555-1634) ---- */
/* mode: 0 none, 1 warm-up init, 2 refresh; sigma: densities of the update window. */
void oracle_occupancy_update(float* density, uint32_t* bitfield, const float* sigma, uint32_t cell_count,
                             uint32_t update_count, uint32_t frame_index, uint32_t mode, float decay, float threshold);

/* ---- CPU emulation of the whole backend (same C ABI semantics) ---- */
typedef struct OracleOptions {
    uint32_t n_levels;
    uint32_t log2_hashmap_size;
    uint32_t base_resolution;
    uint32_t max_resolution;
    float hash_init_scale;
    uint32_t background;              /* 0 white, 1 random per ray */
    float stop_transmittance;         /* 0 disables early termination */
    uint32_t target_samples_per_step; /* 0: fixed rays_per_batch */
    uint32_t max_samples_per_step;    /* 0: rays * steps */
    uint32_t dp_rank;
    uint32_t dp_world;
    uint32_t n_threads;
    uint32_t n_cascades;              /* occupancy cascades (0 or 1: the configured AABB only) */
} OracleOptions;

typedef struct OracleBatchInfo {
    uint32_t rays;        /* rays marched this step */
    uint32_t active_rays; /* rays kept with >= 1 sample */
    uint32_t samples;     /* compacted samples kept */
    uint32_t camera;
} OracleBatchInfo;

void* oracle_ctx_create(const NerfCreateDesc* desc, const OracleOptions* opt);
void oracle_ctx_destroy(void* ctx);
int oracle_ctx_configure(void* ctx, const NerfTrainingConfig* cfg);
int oracle_ctx_step(void* ctx);
/* Split form of a step for data-parallel emulation: compute gradients,
 * then (after the caller sums grads over ranks) apply the update. */
int oracle_ctx_step_grads(void* ctx);
int oracle_ctx_step_apply(void* ctx);
int oracle_ctx_stats(void* ctx, NerfTrainStats* out);
int oracle_ctx_batch_info(void* ctx, OracleBatchInfo* out);
uint64_t oracle_ctx_param_count(void* ctx, uint64_t* n_grid, uint64_t* n_mlp);
/* All pointers optional (NULL skips). Arrays are the full flat parameter vector. */
int oracle_ctx_get_params(void* ctx, float* master, uint16_t* p16, float* m, float* v, float* grad);
int oracle_ctx_set_params(void* ctx, const float* master);
int oracle_ctx_set_grads(void* ctx, const float* grad, float loss_sum, uint32_t active_rays);
// Data parallel with a per-step sample target: the compacted samples of all
// ranks in the pending step (call between step_grads and step_apply); the
// next ray count then follows the global count against world x target.
int oracle_ctx_set_global_samples(void* ctx, uint64_t samples);
/* World positions (x, y, z) of the update_count cells queried by an
 * occupancy refresh at this frame. */
void oracle_occupancy_cells(uint32_t frame, uint32_t update_count, uint32_t cell_count, uint32_t grid_res, const float* mn,
                            const float* mx, float* out_xyz);
/* Loss sum (already normalised) and kept rays of the pending step. */
int oracle_ctx_get_loss(void* ctx, float* loss_sum, uint32_t* active_rays);
int oracle_ctx_get_occupancy(void* ctx, float* density, uint32_t* bitfield);
int oracle_ctx_set_occupancy(void* ctx, const float* density, const uint32_t* bitfield);
int oracle_ctx_set_frame(void* ctx, uint32_t frame_index);
/* Last batch: per-ray (rays marched) counts; per kept ray begin/count/gt/bg/dir;
 * per sample pos+dt.  Any pointer may be NULL. */
int oracle_ctx_get_batch(void* ctx, uint32_t* ray_counts, uint32_t* ray_index, uint32_t* ray_begin,
                         uint32_t* ray_count, float* ray_gt, float* ray_bg, float* ray_dir, float* sample_pos_dt);
/* Render one view with the given 3x4 camera-to-world matrix (row-major rows of
 * the 4x4); writes packed RGBA8 (alpha 255) and per-pixel sample counts. */
int oracle_ctx_render(void* ctx, const float* c2w12, uint32_t width, uint32_t height, float fx, float fy, float cx,
                      float cy, uint32_t max_steps, float stop_transmittance, uint32_t* rgba, uint32_t* samples_per_pixel,
                      uint32_t pixel_begin, uint32_t pixel_end);

#ifdef __cplusplus
}
#endif

#endif
