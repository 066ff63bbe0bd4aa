/*
 * nerf_b200.h -- additive exports of libnerf_b200.so.
 *
 * None of these change the nerf.h ABI; a caller that only knows nerf.h (the
 * reference's benchmark.cpp) never sees them.  They expose what the fixed
 * ABI cannot carry:
 *   - model / training options (hash-grid size, background, early
 *     termination, per-step sample target), also settable by environment
 *     variables read by nerf_create_context;
 *   - counters of the compacted sample stream (the train samples/s metric);
 *   - parameter / occupancy / batch read-back used by the parity tests;
 *   - one-process-per-GPU data-parallel training over NCCL;
 *   - rendering of arbitrary poses, optionally sharded by image tile;
 *   - kernel-level entry points (device pointers, caller's stream) used by
 *     the parity tests and the per-kernel microbenchmarks.
 * The reference has no counterpart for any of these except where a comment
 * names one.
 */
#ifndef NERF_B200_H
#define NERF_B200_H

#include <stdint.h>

#include "nerf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- options */
typedef struct NerfB200Options {
    uint32_t n_levels;                /* hash-grid levels; the fused field needs 16      */
    uint32_t log2_hashmap_size;       /* T = 2^log2 entries per hashed level             */
    uint32_t base_resolution;         /* N_min                                           */
    uint32_t max_resolution;          /* N_max                                           */
    float hash_init_scale;            /* hash entries drawn U(-s, s)                     */
    uint32_t background;              /* 0 white (reference), 1 random colour per ray    */
    float stop_transmittance;         /* training: stop a ray once T < this; 0 disables  */
    float render_stop_transmittance;  /* nerf_inference: same for rendering              */
    uint32_t target_samples_per_step; /* 0: fixed rays_per_batch; else adapt ray count   */
    uint32_t max_samples_per_step;    /* 0: rays_per_batch * max_sample_steps_per_ray    */
    uint32_t n_cascades;              /* occupancy cascades (1..8): cascade k covers the
                                         configured AABB scaled by 2^k about its centre,
                                         each with grid_res^3 cells; rays march the
                                         outermost box, positions are normalised in it */
} NerfB200Options;

/* Defaults, then overrides from NERF_B200_* environment variables
 * (LOG2_HASHMAP_SIZE, BASE_RESOLUTION, MAX_RESOLUTION, BACKGROUND, STOP_T,
 * RENDER_STOP_T, TARGET_SAMPLES, MAX_SAMPLES, CASCADES). */
NERF_API void nerf_b200_default_options(NerfB200Options* out);
/* nerf_create_context with explicit options (nerf_create_context uses the defaults). */
NERF_API NerfStatus nerf_b200_create_context(const NerfCreateDesc* desc, const NerfB200Options* options, void** out_context);

/* --------------------------------------------------------------- counters */
typedef struct NerfB200Counters {
    uint32_t frame_index;          /* steps completed                                  */
    uint32_t rays;                 /* rays marched in the last step                    */
    uint32_t active_rays;          /* rays kept (>= 1 sample, within capacity)         */
    uint32_t samples;              /* compacted samples trained on in the last step    */
    uint32_t marched_active_rays;  /* rays with >= 1 sample before the capacity cut    */
    uint32_t next_rays;            /* rays the next step will march                    */
    uint64_t total_samples;        /* since configure                                  */
    uint64_t total_rays;
    uint32_t kernels_per_step;     /* this library's kernel launches in one training step */
    uint32_t dp_peer;              /* 1: data-parallel exchange over peer memory          */
} NerfB200Counters;
NERF_API NerfStatus nerf_b200_read_counters(void* context, NerfB200Counters* out);

/* ------------------------------------------------------------ profiling */
/* The context's CUDA stream (every context call is ordered on it). */
NERF_API NerfStatus nerf_b200_context_stream(void* context, void** stream);
/* One training step launched kernel by kernel instead of as the captured
 * graph, with CUDA events between launches.  Segments: occupancy query,
 * occupancy update, sampler bitfield tests, compaction scan, sample writes,
 * field forward, composite, MLP backward, hash-table gradient scatter,
 * weight-gradient reduce (folded into the statistics on one GPU), gradient
 * exchange (0 on one GPU), gradient statistics, the next step's ray march,
 * Adam. */
#define NERF_B200_STEP_KERNELS 14
typedef struct NerfB200StepProfile {
    float milliseconds[NERF_B200_STEP_KERNELS];
    float total_milliseconds;
} NerfB200StepProfile;
NERF_API NerfStatus nerf_b200_train_step_profiled(void* context, NerfB200StepProfile* out);

/* ------------------------------------------------------------- hash grid */
#define NERF_B200_MAX_LEVELS 32
typedef struct NerfB200GridLayout {
    uint32_t n_levels;
    uint32_t log2_hashmap_size;
    uint32_t base_resolution;
    uint32_t max_resolution;
    float scale[NERF_B200_MAX_LEVELS];
    uint32_t resolution[NERF_B200_MAX_LEVELS]; /* vertices per axis                 */
    uint32_t dense[NERF_B200_MAX_LEVELS];
    uint32_t offset[NERF_B200_MAX_LEVELS + 1]; /* entry offsets; [n_levels] = total */
} NerfB200GridLayout;
NERF_API NerfStatus nerf_b200_grid_layout(uint32_t n_levels, uint32_t log2_hashmap_size, uint32_t base_resolution,
                                          uint32_t max_resolution, NerfB200GridLayout* out);
NERF_API NerfStatus nerf_b200_context_grid_layout(void* context, NerfB200GridLayout* out);

/* ------------------------------------------------- parameters and state */
/* Flat parameter vector: hash-grid entries x 2 features, then the 10240 MLP
 * weights (density W0 64x32, W1 16x64, colour W0 64x32, W1 64x64, W2 16x64,
 * each [out][in] row-major). */
NERF_API NerfStatus nerf_b200_param_counts(void* context, uint64_t* n_grid, uint64_t* n_mlp);
/* Host buffers of n_grid + n_mlp elements; NULL skips. */
NERF_API NerfStatus nerf_b200_read_params(void* context, float* master, uint16_t* params_f16, float* adam_m, float* adam_v);
NERF_API NerfStatus nerf_b200_write_params(void* context, const float* master);
/* Training-state checkpoint for an exact resume (extends the reference's
 * weights-only nerf_save_network_weights, backend-cuda.cu:2466-2592, whose
 * load resets the optimiser and occupancy): fp32 masters, both Adam moments,
 * occupancy densities and bitfield, and the step state (frame, next ray
 * count, counters, last statistics), in the same container (u64 header
 * length, JSON header, raw tensors).  Both need a configured context
 * (NERF_STATUS_STATE_ERROR otherwise); load fails with NERF_STATUS_IO_ERROR
 * when the file is missing, malformed, or sized for another hash grid or
 * occupancy grid.  After a load the next nerf_train_step samples exactly the
 * rays the saved run would have sampled. */
NERF_API NerfStatus nerf_b200_save_training_state(void* context, const char* path_utf8);
NERF_API NerfStatus nerf_b200_load_training_state(void* context, const char* path_utf8);
/* density: n_cascades * grid_res^3 floats; bitfield: ceil(that / 32) words; NULL skips. */
NERF_API NerfStatus nerf_b200_read_occupancy(void* context, float* density, uint32_t* bitfield);
NERF_API NerfStatus nerf_b200_write_occupancy(void* context, const float* density, const uint32_t* bitfield);
NERF_API NerfStatus nerf_b200_set_frame_index(void* context, uint32_t frame_index);

/* Last training batch.  ray_counts: samples of every marched ray (rays);
 * ray_index / ray_records: kept rays (active_rays); sample_pos_dt (x,y,z,dt)
 * and sample_ray: kept samples.  NULL skips. */
typedef struct NerfB200RayRecord {
    float dir[3];
    uint32_t begin;
    float gt[4];   /* ground truth composited on bg, ground-truth alpha */
    float bg[3];
    uint32_t count;
} NerfB200RayRecord;
NERF_API NerfStatus nerf_b200_read_batch(void* context, uint32_t* ray_counts, uint32_t* ray_index,
                                         NerfB200RayRecord* ray_records, float* sample_pos_dt, uint32_t* sample_ray);

/* ------------------------------------------------------- data parallel */
/* One process per GPU.  Rank 0 creates the id, every rank passes it to
 * nerf_b200_dp_init before nerf_configure_training; the training step then
 * sums gradients and the loss over ranks with NCCL.  Rank r marches global
 * ray indices r*rays_per_batch + i, so N ranks train on the union of N
 * disjoint batches. */
#define NERF_B200_DP_ID_BYTES 128
NERF_API NerfStatus nerf_b200_dp_unique_id(uint8_t out_id[NERF_B200_DP_ID_BYTES]);
NERF_API NerfStatus nerf_b200_dp_init(void* context, uint32_t rank, uint32_t world_size,
                                      const uint8_t id[NERF_B200_DP_ID_BYTES]);
/* Peer mode without NCCL: every rank exports its handle (the CUDA IPC
 * handle of its model memory plus the sizes all ranks must share), the caller
 * gathers the world's handles in rank order with any host-side exchange it
 * already has (a torch.distributed all-gather, an MPI all-gather, a file), and
 * every rank passes the gathered array (world x NERF_B200_DP_HANDLE_BYTES) to
 * nerf_b200_dp_init_peers before nerf_configure_training.  The step is the
 * same peer-mode step as after nerf_b200_dp_init, but no communicator is
 * created, so setting up a job costs a few IPC mappings instead of an NCCL
 * initialisation.  Errors: INVALID_USAGE for a handle of another layout or
 * world > 64; STATE_ERROR when the context is already data parallel; FAILURE
 * when a peer's memory cannot be mapped (then nothing is mapped and the
 * context stays single-GPU: the caller must not train the ranks apart). */
#define NERF_B200_DP_HANDLE_BYTES 128
NERF_API NerfStatus nerf_b200_dp_peer_handle(void* context, uint8_t out[NERF_B200_DP_HANDLE_BYTES]);
NERF_API NerfStatus nerf_b200_dp_init_peers(void* context, uint32_t rank, uint32_t world_size, const uint8_t* handles);
/* The failure path of a stalled rank, on one GPU.  In peer mode every wait
 * of the step's barriers is bounded (NERF_B200_DP_TIMEOUT_MS, read by
 * nerf_b200_dp_init; default 5000): a rank whose peer stops stepping gives up
 * the wait, records the error, finishes its step, and nerf_read_train_stats
 * returns NERF_STATUS_CUDA_ERROR from then on (the replicas are no longer in
 * step).  This call runs the same barrier kernel on a configured
 * single-GPU context (NERF_STATUS_STATE_ERROR otherwise) as rank 0 of two,
 * against a second rank whose flag is never written, with a wait limit of
 * timeout_us microseconds; asynchronous on the context's stream.  No
 * counterpart in the reference, which has no multi-GPU path; its own failure
 * report is the non-finite flag of the step statistics
 * (backend-cuda.cu:1495-1508). */
NERF_API NerfStatus nerf_b200_dp_barrier_test(void* context, uint32_t timeout_us);

/* ------------------------------------------------------------- rendering */
/* Render an arbitrary pose (row-major 3x4 camera-to-world, camera looks down
 * -Z).  tile_size > 0 shards the image into tile_size^2 tiles dealt
 * round-robin over tile_world ranks; this call renders the tiles of
 * tile_rank and leaves other pixels untouched. */
typedef struct NerfB200RenderRequest {
    const float* c2w_3x4;
    uint32_t width;
    uint32_t height;
    float fx, fy, cx, cy;
    uint32_t max_steps;          /* marching resolution along the AABB chord */
    float stop_transmittance;    /* < 0: context default */
    uint32_t tile_size;
    uint32_t tile_rank;
    uint32_t tile_world;
    uint32_t memory_kind;        /* NerfMemoryKind of dst_rgba8 */
    void* dst_rgba8;             /* width*height*4 bytes, or NULL to keep on device */
    uint64_t dst_bytes;
} NerfB200RenderRequest;
typedef struct NerfB200RenderInfo {
    uint64_t rays;               /* pixels rendered by this call      */
    uint64_t samples;            /* field evaluations of this call    */
    float milliseconds;          /* device time of the render kernel  */
} NerfB200RenderInfo;
NERF_API NerfStatus nerf_b200_render(void* context, const NerfB200RenderRequest* request, NerfB200RenderInfo* info);
/* Device pointer of the context's last render output (width*height RGBA8). */
NERF_API NerfStatus nerf_b200_render_output(void* context, const void** device_rgba8);

/* ------------------------------------------------------ synthetic scenes */
/* Seeded procedural scenes and their exact ground-truth renders (host code),
 * standing in for the Blender datasets: kind 0 = spheres of constant colour,
 * kind 1 = spheres and boxes with value-noise albedo, kind 2 = an
 * unbounded-style scene (n_primitives spheres and boxes standing on a ground
 * slab over [-12, 12]^2, centres within +-extent, inside a sky shell of radii
 * 12 to 12.5, value-noise albedo).  Writes n_views RGBA8 images (NULL:
 * cameras only), row-major 4x4 camera-to-world matrices and (fx, fy, cx, cy).
 * camera_mode: 0 sphere, 1 upper hemisphere, 2 circular orbit of orbit_views
 * views at orbit_elevation (radians), 3 ring of orbit_views cameras of the
 * given radius at height orbit_elevation looking outward (even views) and
 * inward (odd views). */
typedef struct NerfB200SceneDesc {
    uint32_t kind;
    uint32_t seed;
    uint32_t n_primitives;
    float density;
    float extent;        /* primitive centres uniform in [-extent, extent]^3 */
    float size_min;      /* sphere radius / box edge drawn uniform in [size_min, size_max] */
    float size_max;
    uint32_t n_views;
    uint32_t width;
    uint32_t height;
    float fov;           /* horizontal field of view, radians */
    float radius;        /* camera distance from the origin */
    uint32_t camera_mode;
    float orbit_elevation;
    uint32_t orbit_views;
    uint32_t view_offset; /* index of the first view (held-out sets use another offset) */
    uint32_t n_threads;   /* 0: all host threads */
} NerfB200SceneDesc;
NERF_API NerfStatus nerf_b200_scene_render(const NerfB200SceneDesc* desc, uint8_t* images_rgba8, float* cameras_4x4,
                                           float* intrinsics4);

/* ------------------------------------------------------------ datasets */
/* The reference's dataset format (its driver's loader, benchmark.cpp:148-303):
 * a Blender "transforms" JSON (camera_angle_x; frames with file_path and a
 * row-major 4x4 transform_matrix) next to 8-bit PNG images.  path is the JSON
 * file or its directory (then transforms_train.json); a file_path without an
 * extension gets ".png".  PNG: 8-bit grey, grey + alpha, RGB, RGBA or palette,
 * not interlaced, decoded to RGBA8.  Errors: NERF_STATUS_IO_ERROR for missing or
 * malformed files, NERF_STATUS_INVALID_USAGE for null arguments, a buffer too
 * small, or images of different sizes.  No counterpart in the reference
 * library: its driver does this with nlohmann::json and stb_image. */
typedef struct NerfB200BlenderInfo {
    uint32_t image_count;
    uint32_t width;
    uint32_t height;
    float camera_angle_x;
} NerfB200BlenderInfo;
NERF_API NerfStatus nerf_b200_blender_probe(const char* path, NerfB200BlenderInfo* out);
/* Decodes every image on n_threads threads (0: all host threads) into
 * images_rgba8 ([n][H][W][4], e.g. pinned memory for nerf_create_context) and
 * writes the cameras and (fx, fy, cx, cy) = ((W/2) / tan(angle/2), same,
 * (W-1)/2, (H-1)/2).  remap = 1 applies the reference driver's convention
 * (world axes (x, -z, y) -> (x, y, z), translation * 0.33 + 0.5: the scene in
 * [0,1]^3); remap = 0 keeps the file's matrices. */
NERF_API NerfStatus nerf_b200_blender_load(const char* path, uint32_t remap, uint32_t n_threads, uint8_t* images_rgba8,
                                           uint64_t images_bytes, float* cameras_4x4, float* intrinsics4);
/* Writes dir/transforms_train.json and dir/train/r_<i>.png (RGBA8). */
NERF_API NerfStatus nerf_b200_blender_write(const char* dir, const uint8_t* images_rgba8, const float* cameras_4x4, uint32_t n,
                                            uint32_t width, uint32_t height, float camera_angle_x, uint32_t n_threads);
/* One PNG: read into rgba8 (bytes capacity; NULL rgba8 only reports the size),
 * or write RGBA8 (filter 0, deflate stored blocks). */
NERF_API NerfStatus nerf_b200_png_read(const char* path, uint8_t* rgba8, uint64_t bytes, uint32_t* width, uint32_t* height);
NERF_API NerfStatus nerf_b200_png_write(const char* path, const uint8_t* rgba8, uint32_t width, uint32_t height);

/* ------------------------------------- kernel-level entry points (tests) */
/* All pointers are device pointers; stream is a cudaStream_t (NULL = legacy
 * default stream).  Calls are asynchronous.  Parameter and gradient tables
 * (params_f16, grad_f16, grid_grad_f16, mlp_params_f16) start on a 16-byte
 * boundary: they are read and reduced in 16-byte blocks, and a misaligned
 * table is refused with NERF_STATUS_INVALID_USAGE. */
NERF_API NerfStatus nerf_b200_grid_forward(const NerfB200GridLayout* layout, const float* pos_unit, uint32_t n,
                                           const void* params_f16, void* feat_f16, void* stream);
NERF_API NerfStatus nerf_b200_grid_backward(const NerfB200GridLayout* layout, const float* pos_unit, uint32_t n,
                                            const void* dfeat_f16, void* grad_f16, void* stream);
/* Fused field on n samples: params_f16 is the flat vector of `layout`
 * (16 levels).  feat_f16 (n x 32) receives the hash features, raw (n x 4)
 * the raw density and colour. */
NERF_API NerfStatus nerf_b200_field_forward(const NerfB200GridLayout* layout, const void* params_f16, const float* pos_unit,
                                            const float* dirs, uint32_t n, void* feat_f16, float* raw, void* stream);
/* Backward of the fused field for loss-scaled d raw (n x 4).  Adds the hash
 * gradient into grid_grad_f16 and writes the 10240 MLP weight gradients to
 * mlp_grad.  partials must hold nerf_b200_field_backward_partial_floats()
 * floats. */
NERF_API uint64_t nerf_b200_field_backward_partial_floats(void);
NERF_API NerfStatus nerf_b200_field_backward(const NerfB200GridLayout* layout, const void* params_f16, const float* pos_unit,
                                             const float* dirs, uint32_t n, const void* feat_f16, const float* dout,
                                             void* grid_grad_f16, float* partials, float* mlp_grad, void* stream);
/* The two MLPs of the fused field alone, on given hash features (the
 * encode skipped; used to measure the MLPs against the tensor-pipe roofline).
 * mlp_params_f16: the 10240 MLP weights (the tail of the flat parameter
 * vector); feat_f16: n x 32 fp16 features; dirs: n x 3 unit directions.
 * Forward writes raw (n x 4).  Backward takes loss-scaled d raw (n x 4),
 * writes the feature gradients dfeat_f16 (n x 32 fp16) and the 10240 weight
 * gradients (partials as in nerf_b200_field_backward). */
NERF_API NerfStatus nerf_b200_mlp_forward(const void* mlp_params_f16, const void* feat_f16, const float* dirs, uint32_t n,
                                          float* raw, void* stream);
/* nerf_b200_mlp_forward on the 5th-generation tensor cores (tcgen05.mma with
 * tensor-memory accumulators, 128-row tiles).  error_word: one device uint32;
 * bit 0 is set when a CTA's MMAs did not complete within a second (the CTA
 * then stops; its rows of raw are not written). */
NERF_API NerfStatus nerf_b200_mlp_forward_tc(const void* mlp_params_f16, const void* feat_f16, const float* dirs, uint32_t n,
                                             float* raw, uint32_t* error_word, void* stream);
/* nerf_b200_mlp_backward on tcgen05: per 128-row tile the forward is
 * recomputed, each backward layer's input-gradient MMA and weight-gradient MMA
 * read the same shared-memory operands, and the weight gradients accumulate
 * in tensor memory across the CTA's tiles.  Same outputs and partials contract
 * as nerf_b200_mlp_backward; error_word as in nerf_b200_mlp_forward_tc. */
/* Launch geometry of the tensor-core MLP kernels: out[0] / out[1] persistent
 * grid of the forward / backward (CTAs), out[2] / out[3] the CUDA runtime's
 * occupancy answer for them (CTAs per SM). */
NERF_API NerfStatus nerf_b200_mlp_tc_info(uint32_t out[4]);
NERF_API NerfStatus nerf_b200_mlp_backward_tc(const void* mlp_params_f16, const void* feat_f16, const float* dirs, uint32_t n,
                                              const float* dout, void* dfeat_f16, float* partials, float* mlp_grad,
                                              uint32_t* error_word, void* stream);
NERF_API NerfStatus nerf_b200_mlp_backward(const void* mlp_params_f16, const void* feat_f16, const float* dirs, uint32_t n,
                                           const float* dout, void* dfeat_f16, float* partials, float* mlp_grad,
                                           void* stream);
/* Allocation-free nerf_b200_field_backward (no counterpart in the reference).
 * For callers that cannot allocate device memory -- a plugin inside a host
 * application that owns the device memory budget, or code where a cudaMalloc
 * would synchronise the device at the wrong moment.  The weight-gradient
 * scratch lives in a static device array of
 * nerf_b200_field_backward_noalloc_max_rows() x 10240 floats (13.1 MB, held
 * by every GPU that loads the library until exit); the call fails with
 * NERF_STATUS_INVALID_USAGE when this GPU needs more rows, that is when
 * nerf_b200_field_backward_partial_floats() / 10240 exceeds
 * nerf_b200_field_backward_noalloc_max_rows(), or when n exceeds 2^31-1.
 * The first call on a device looks up the array's device address; make it
 * before any stream capture.  The address is kept for the process: after a
 * cudaDeviceReset of that device do not call this entry point again.  Calls
 * share the array: calls that overlap on the GPU race.  Other arguments as
 * in nerf_b200_field_backward. */
NERF_API uint32_t nerf_b200_field_backward_noalloc_max_rows(void);
NERF_API NerfStatus nerf_b200_field_backward_noalloc(const NerfB200GridLayout* layout, const void* params_f16,
                                                     const float* pos_unit, const float* dirs, uint32_t n,
                                                     const void* feat_f16, const float* dout, void* grid_grad_f16,
                                                     float* mlp_grad, void* stream);
/* Compositing + alpha-weighted MSE forward and backward over n_rays rays
 * (ray records as in nerf_b200_read_batch), raw (S x 4), pos_dt (S x 4, only
 * .w = dt is read).  Writes loss_scale * dL/draw to dout, per-ray loss and
 * samples used (optional), and adds sum(loss) * inv_norm to *loss_sum. */
NERF_API NerfStatus nerf_b200_composite(const NerfB200RayRecord* rays, uint32_t n_rays, const float* raw,
                                        const float* pos_dt, float inv_norm, float loss_scale, float stop_transmittance,
                                        float* dout, float* ray_loss, uint32_t* ray_used, float* loss_sum, void* stream);
/* One Adam step over the flat parameter vector with explicit scalars
 * (learning_rate, grad_scale, inv_bias_correction1, inv_bias_correction2,
 * inv_loss_scale, skip).  Grid gradients are zeroed after use. */
NERF_API NerfStatus nerf_b200_adam(float* master, void* params_f16, void* grid_grad_f16, const float* mlp_grad, float* adam_m,
                                   float* adam_v, uint64_t n_grid, uint64_t n_params, const float scalars[5], uint32_t skip,
                                   float beta1, float beta2, float eps, void* stream);
/* Occupancy maintenance of one step with an explicit mode (0 none, 1
 * warm-up init, 2 refresh) and frame; sigma holds the update window's
 * densities. */
NERF_API NerfStatus nerf_b200_occupancy_update(float* density, uint32_t* bitfield, const float* sigma, uint32_t cell_count,
                                               uint32_t update_count, uint32_t frame_index, uint32_t mode, float decay,
                                               float threshold, void* stream);

#ifdef __cplusplus
}
#endif

#endif
