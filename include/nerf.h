/*
 * nerf.h -- C ABI of the NeRF train/render backend.
 *
 * This header declares the drop-in boundary that the B200 backend
 * (libnerf_b200.so) implements.  Every type and function here keeps the
 * name, field order, field type and meaning of the reference interface
 * (Xayah-Graphics/NeRF nerf.h), because callers such as the reference's
 * benchmark.cpp are compiled against that layout.  The text of this file is
 * our own; the per-item citations name the reference line each declaration
 * stands in for.
 *
 * Error convention (reference backend-cuda.cu:1993-2592):
 *   NERF_STATUS_INVALID_USAGE  null argument or size/limit violation
 *   NERF_STATUS_STATE_ERROR    call out of order (no scene, not configured)
 *   NERF_STATUS_IO_ERROR       checkpoint file could not be read or written
 *   NERF_STATUS_CUDA_ERROR     a CUDA call failed
 *   NERF_STATUS_FAILURE        allocation or initialisation failed
 * No C++ exception crosses this boundary.
 */
#ifndef NERF_H
#define NERF_H

#include <stdint.h>

/* Symbol visibility (reference nerf.h:6-22). */
#if defined(_WIN32) || defined(__CYGWIN__)
#  if defined(NERF_BUILD_SHARED) && defined(NERF_BUILD_EXPORTS)
#    define NERF_API __declspec(dllexport)
#  elif defined(NERF_BUILD_SHARED)
#    define NERF_API __declspec(dllimport)
#  else
#    define NERF_API
#  endif
#elif defined(__GNUC__) || defined(__clang__)
#  if defined(NERF_BUILD_SHARED)
#    define NERF_API __attribute__((visibility("default")))
#  else
#    define NERF_API
#  endif
#else
#  define NERF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Result code of every entry point (reference nerf.h:29). */
typedef enum NerfStatus {
    NERF_STATUS_OK            = 0,
    NERF_STATUS_INVALID_USAGE = 1,
    NERF_STATUS_STATE_ERROR   = 2,
    NERF_STATUS_IO_ERROR      = 3,
    NERF_STATUS_CUDA_ERROR    = 4,
    NERF_STATUS_FAILURE       = 5
} NerfStatus;

/*
 * Scene + capacity description given at context creation
 * (reference nerf.h:31-56).  Images are image_count tightly packed RGBA8
 * frames of image_width x image_height; cameras are image_count row-major
 * 4x4 camera-to-world matrices (camera looks down -Z, +Y up).  Both arrays
 * are copied to the device; the caller may free them after the call.
 */
typedef struct NerfCreateDesc {
    uint32_t occupancy_grid_res;     /* cells per axis of the occupancy grid   */
    uint32_t max_sample_steps;       /* capacity of the compacted sample stream */
    uint32_t max_batch_rays;         /* capacity of rays per training batch     */
    uint64_t arena_alignment_bytes;  /* power of two; sub-buffer alignment      */

    const uint8_t* images_rgba8;
    uint64_t images_bytes;

    const float* cameras_4x4_packed;
    uint64_t cameras_bytes;

    uint32_t image_count;
    uint32_t image_width;
    uint32_t image_height;

    float fx;
    float fy;
    float cx;
    float cy;
} NerfCreateDesc;

/* reference nerf.h:57-58 */
NERF_API NerfStatus nerf_create_context(const NerfCreateDesc* desc, void** out_context);
NERF_API NerfStatus nerf_destroy_context(void* context);

/* Optimiser settings (reference nerf.h:60-69). */
typedef struct NerfHyperParams {
    float learning_rate;
    float adam_beta1;
    float adam_beta2;
    float adam_eps;
    float grad_clip_norm;          /* global-norm clip threshold              */
    float update_guard_grad_norm;  /* skip the update above this grad norm   */
    float loss_scale;              /* static loss scale of the fp16 gradients */
    uint32_t lr_decay_ksteps;      /* lr *= 0.1 every lr_decay_ksteps*1000    */
} NerfHyperParams;

/* Occupancy-grid maintenance (reference nerf.h:70-76). */
typedef struct NerfOccupancyParams {
    float decay;
    float threshold;
    uint32_t cells_per_update;
    uint32_t update_interval;
    uint32_t warmup_steps;
} NerfOccupancyParams;

/* Training configuration (reference nerf.h:77-88). */
typedef struct NerfTrainingConfig {
    float aabb_min_x;
    float aabb_min_y;
    float aabb_min_z;
    float aabb_max_x;
    float aabb_max_y;
    float aabb_max_z;
    NerfHyperParams hyper_params;
    NerfOccupancyParams occupancy_params;
    uint32_t rays_per_batch;
    uint32_t max_sample_steps_per_ray;
} NerfTrainingConfig;

/* reference nerf.h:89-90 */
NERF_API NerfStatus nerf_configure_training(void* context, const NerfTrainingConfig* config);
NERF_API NerfStatus nerf_train_step(void* context);

/* Statistics of the last completed step (reference nerf.h:92-98). */
typedef struct NerfTrainStats {
    float loss;
    float grad_norm;
    uint32_t has_nonfinite;
    uint32_t completed_steps;
    uint32_t last_train_camera;
} NerfTrainStats;

/* reference nerf.h:99 */
NERF_API NerfStatus nerf_read_train_stats(void* context, NerfTrainStats* out_stats);

/* Where nerf_inference writes its RGBA8 image (reference nerf.h:101). */
typedef enum NerfMemoryKind { NERF_MEMORY_HOST = 1, NERF_MEMORY_CUDA_DEVICE = 2 } NerfMemoryKind;

/* Render request for one dataset camera (reference nerf.h:102-108). */
typedef struct NerfInferenceRequest {
    uint32_t camera_idx;
    uint32_t samples_per_ray;
    uint32_t memory_kind;
    void* dst_rgba8;
    uint64_t dst_bytes;
} NerfInferenceRequest;

/* Description of the rendered image (reference nerf.h:109-116). */
typedef struct NerfInferenceInfo {
    uint64_t capacity_bytes;
    uint64_t valid_bytes;
    uint32_t row_stride_bytes;
    uint32_t width;
    uint32_t height;
    uint32_t generation;
} NerfInferenceInfo;

/* reference nerf.h:117 */
NERF_API NerfStatus nerf_inference(void* context, const NerfInferenceRequest* request, NerfInferenceInfo* out_info);

/* Checkpoint file (reference nerf.h:119-121). */
typedef struct NerfCheckpointFileDesc {
    const char* path_utf8;
} NerfCheckpointFileDesc;

/* reference nerf.h:122-123 */
NERF_API NerfStatus nerf_save_network_weights(void* context, const NerfCheckpointFileDesc* desc);
NERF_API NerfStatus nerf_load_network_weights(void* context, const NerfCheckpointFileDesc* desc);

#ifdef __cplusplus
}
#endif

#endif /* NERF_H */
