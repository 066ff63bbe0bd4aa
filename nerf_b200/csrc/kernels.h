// kernels.h -- launch interface of the sm_100a kernels (internal to libnerf_b200).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "types.h"

namespace nb {

struct alignas(16) LevelTable {
    // scale, res, dense, offset per level (LevelParams layout)
    float scale[kMaxLevels];
    uint32_t res[kMaxLevels];
    uint32_t dense[kMaxLevels];
    uint32_t offset[kMaxLevels];
    uint32_t n_levels;
    uint32_t hash_mask;
};
LevelTable make_level_table(const GridLayout& g);

// ---- standalone hash-grid encoder (unit-cube points, any level count) ----
cudaError_t launch_grid_forward(const LevelTable& lt, const float* pos_unit, uint32_t n, const void* params,
                                void* feat, cudaStream_t s);
cudaError_t launch_grid_backward(const LevelTable& lt, const float* pos_unit, uint32_t n, const void* dfeat_f16,
                                 void* grad_f16, cudaStream_t s);

// ---- fused field (hash grid L=16 + density/colour MLPs) ----
// kFieldMlp: the MLPs alone on given hash features (feat holds n x 32 fp16
// input rows; forward writes raw, backward writes dfeat and weight gradients).
enum FieldMode : int { kFieldTrain = 0, kFieldOccupancy = 1, kFieldDirect = 2, kFieldMlp = 3 };
struct FieldArgs {
    LevelTable lt;
    const void* params16;   // flat fp16 parameters (grid entries, then MLP)
    uint32_t mlp_offset;    // index of the first MLP parameter
    uint32_t n_direct;      // rows for kFieldDirect
    DeviceState* state;
    // training rows
    const float4* pos_dt;
    const uint32_t* sample_ray;
    const RayRecord* rays;
    float aabb_min[3], aabb_max[3], aabb_size[3];  // marching box (positions are normalised in it)
    CascadeBox casc;
    // occupancy rows
    uint32_t grid_res, cell_count, update_count, warmup_steps, update_interval;
    float* occ_sigma;
    // direct rows
    const float* pos_unit;
    const float* dirs;
    // outputs / inputs
    void* feat;            // training: 112-byte rows (features, SH, unit position); direct: fp16 n x 32
    float4* raw;           // forward: raw sigma, raw rgb
    const float4* dout;    // backward: loss-scaled d raw
    void* grid_grad;       // backward: fp16 entries x 2 (reduction target)
    float* partials;       // backward: [grid][kMlpParams] per-CTA weight gradients
    void* dfeat;           // training backward: fp16 n x 32 feature gradients for the scatter kernel
};
cudaError_t launch_field_forward(const FieldArgs& a, int mode, uint32_t grid_blocks, cudaStream_t s);
// Training and MLP modes: the MLP backward writing dfeat (the training step
// then launches the hash-table scatter, launch_grid_scatter).  Direct mode:
// one fused kernel (MLP backward + scatter).
cudaError_t launch_field_backward(const FieldArgs& a, int mode, uint32_t grid_blocks, cudaStream_t s);
// Training forward without the MLPs: hash encode + SH of a.state->n_samples
// rows into the 112-byte training rows a.feat (launch_mlp_forward_tc_train
// then evaluates the MLPs).
cudaError_t launch_field_encode(const FieldArgs& a, cudaStream_t s);
// The hash-table scatter of the training backward alone (feature gradients
// in a.dfeat, positions in the training rows a.feat, a.state->n_samples rows).
cudaError_t launch_grid_scatter(const FieldArgs& a, cudaStream_t s);
uint32_t field_forward_blocks();
uint32_t field_backward_blocks();
cudaError_t field_init_attributes();
// field_init_attributes() once per device, under a lock (context.cu).
cudaError_t ensure_attributes();

// ---- the field MLPs on tcgen05 (mlp_tc.cu) ----
// Forward of the MLPs on given features (n x 32 fp16) and directions, raw
// (n x 4) out; *error gets bit 0 when a CTA's MMAs did not complete in time.
cudaError_t launch_mlp_forward_tc(const void* mlp, const void* feat, const float* dirs, uint32_t n, float* raw, uint32_t* error,
                                  cudaStream_t s);
// Forward over the 112-byte training rows of the field forward (n read from
// *n_device), raw (n x 4) out.
cudaError_t launch_mlp_forward_tc_train(const void* mlp, const void* rows, const uint32_t* n_device, float* raw, uint32_t* error,
                                        cudaStream_t s);
// Backward of the MLPs over n rows (or *n_device when non-null): rows are
// 64-byte feature rows with dirs (train_rows = 0) or the 112-byte training
// rows of the forward (train_rows = 1, SH taken from the row); dout is the
// loss-scaled d raw (n x 4).  Writes dfeat (n x 32 fp16) and one row of
// kMlpParams weight gradients per CTA into partials; blocks is at most
// mlp_backward_tc_blocks() (persistent CTAs, tile t to CTA t mod blocks).
cudaError_t launch_mlp_backward_tc(const void* mlp, const void* rows, int train_rows, const float* dirs, const float* dout,
                                   const uint32_t* n_device, uint32_t n, void* dfeat, float* partials, uint32_t blocks,
                                   uint32_t* error, cudaStream_t s);
uint32_t mlp_backward_tc_blocks();
// Persistent grids of the forward / backward tensor-core MLP kernels and the
// runtime's occupancy answer for each (CTAs per SM).
void mlp_tc_info(uint32_t out[4]);

// ---- sampler ----
// Geometry of a marched training ray (48 bytes).
struct alignas(16) RayGeom {
    float o[3], d[3];
    float tf, dt_min;
    float px, py;       // pixel position of the ray
    uint32_t n_steps;   // steps of the march (0 when the ray misses the box)
    uint32_t pad;
};
struct SamplerArgs {
    TrainConsts tc;
    DeviceState* state;
    const float* cams;
    const uint8_t* images;
    const uint32_t* bitfield;
    uint32_t* ray_counts;     // [2][max_rays], half (frame & 1) belongs to the step of that frame
    float* kept_t;            // [max_rays][max_steps] t of the ray's kept steps, in step order
    float* chunk_t;           // [max_rays][mask_words] t at the start of each 32-step chunk
    RayGeom* geom;            // [max_rays]
    uint32_t* ray_offset;     // [max_rays] exclusive sample prefix
    uint32_t* ray_slot;       // [max_rays] compacted index, or ~0 when not kept
    RayRecord* rays;          // [max_rays] compacted
    float4* pos_dt;           // [sample_cap]
    uint32_t* sample_ray;     // [sample_cap]
    uint32_t* ray_index;      // [max_rays] compacted -> marched ray index
};
// Step recurrence of every ray of the step whose frame is in the state.  A
// step's march only depends on the frame and the ray count, so the training
// step ends with the next step's march.
cudaError_t launch_march(const SamplerArgs& a, cudaStream_t s);
// Bitfield tests, compaction scan and sample writes (after launch_march),
// one launch each or all three in order.
cudaError_t launch_sample_bits(const SamplerArgs& a, cudaStream_t s);
cudaError_t launch_sample_scan(const SamplerArgs& a, cudaStream_t s);
cudaError_t launch_sample_write(const SamplerArgs& a, cudaStream_t s);
cudaError_t launch_sampler(const SamplerArgs& a, cudaStream_t s);

// ---- compositing + loss ----
struct CompositeArgs {
    const RayRecord* rays;
    const float4* raw;
    const float4* pos_dt;
    float4* dout;
    DeviceState* state;
    float* loss_slot;     // MLP-gradient buffer slot of the loss sum
    uint32_t max_rays;
    uint32_t dp_world;
    float loss_scale;
    float stop_transmittance;
    // direct mode (tests): explicit ray count and normaliser
    int direct;
    uint32_t n_rays;
    float inv_norm;
    float* ray_loss;      // optional per-ray loss
    uint32_t* ray_used;   // optional per-ray samples used
};
cudaError_t launch_composite(const CompositeArgs& a, cudaStream_t s);

// ---- occupancy ----
struct OccupancyArgs {
    DeviceState* state;
    float* density;
    uint32_t* bitfield;
    const float* occ_sigma;
    uint32_t cell_count, update_count, warmup_steps, update_interval;
    float decay, threshold;
    int direct;             // 1: use `mode` and `frame` below instead of the device state
    uint32_t mode, frame;
};
cudaError_t launch_occupancy_update(const OccupancyArgs& a, cudaStream_t s);

// ---- optimiser ----
// Data-parallel step over peer memory (one process per GPU, the model arenas
// of all ranks mapped into every rank): each rank owns the grid parameters
// [lo, hi); it sums every rank's gradients of that range, runs Adam on it and
// writes the fp16 parameters into every rank's mirror.
constexpr uint32_t kMaxDpWorld = kMaxDpRanks;
struct DpPeers {
    uint32_t world, rank;
    uint64_t lo, hi;                    // owned grid-parameter range (multiples of 8)
    const void* grad[kMaxDpWorld];      // every rank's fp16 grid gradients (own included)
    const float* mlp[kMaxDpWorld];      // every rank's fp32 MLP gradients + loss slot
    void* p16[kMaxDpWorld];             // every rank's fp16 parameter mirror
    DpSync* sync[kMaxDpWorld];          // every rank's synchronisation words
    float* gsum;                        // [hi - lo] summed gradients of the owned range
    float* mlp_sum;                     // [kMlpGradSlots] summed MLP gradients and loss
    uint64_t timeout_ns;                // a barrier wait gives up after this long (DpSync::error)
};
struct OptimArgs {
    TrainConsts tc;
    DeviceState* state;
    float* master;
    void* params16;
    void* grid_grad;         // fp16 [n_grid]
    float* mlp_grad;         // fp32 [kMlpGradSlots]
    float* m;
    float* v;
    const float* partials;
    uint32_t n_partials;
    uint64_t n_grid;         // grid parameters (multiple of 16)
    uint64_t n_params;       // grid + MLP
    uint32_t stats_blocks;
    AdamScalars direct_scalars;  // used when state is null (kernel-level entry point)
    uint32_t dp_peer;            // 1: gradients summed over the ranks by k_dp_reduce_grads (DpPeers)
    DpPeers dp;
    const float* mlp_in;         // MLP gradients + loss read by statistics and Adam (mlp_grad, or dp.mlp_sum)
    uint32_t fuse_wgrad;         // statistics kernel also reduces the weight-gradient partials (single GPU)
    StatsBlock* stats_host;      // mapped pinned host mirror of the step statistics, or null
    uint32_t world;              // data-parallel ranks (1: one GPU)
};
cudaError_t launch_wgrad_reduce(const OptimArgs& a, cudaStream_t s);
cudaError_t launch_grad_stats(const OptimArgs& a, cudaStream_t s);
cudaError_t launch_adam(const OptimArgs& a, cudaStream_t s);
uint32_t grad_stats_blocks(uint64_t n_params, bool fused);
cudaError_t launch_f32_to_f16(const float* src, void* dst, uint64_t n, cudaStream_t s);
// dst[i] = scale * draw i of the splitmix64 stream whose state is state0 before
// the first draw (a uniform in [-1, 1) from the top 24 bits of each draw).
cudaError_t launch_splitmix_fill(float* dst, uint64_t n, uint64_t state0, float scale, cudaStream_t s);
// Sum of every rank's grid gradients over the owned range into dp.gsum and of
// every rank's MLP gradients into dp.mlp_sum; the owned range's sum of squares
// and non-finite flag go to every rank's DpSync::partials.
cudaError_t launch_dp_reduce_grads(const OptimArgs& a, cudaStream_t s);
// Barrier of all ranks over their DpSync words: each rank announces a new
// epoch to every rank and waits (at most d.timeout_ns, then DpSync::error) until
// every rank has announced it.  Writes made before it (by this rank's earlier
// kernels, to any rank's memory) are visible to every rank after it.
cudaError_t launch_dp_barrier(const DpPeers& d, cudaStream_t s);

// ---- render ----
struct RenderArgs {
    LevelTable lt;
    const void* params16;
    uint32_t mlp_offset;
    const uint32_t* bitfield;
    uint32_t grid_res;
    float aabb_min[3], aabb_max[3], aabb_size[3];  // marching box
    CascadeBox casc;
    float c2w[12];
    uint32_t width, height;
    float fx, fy, cx, cy;
    uint32_t max_steps;
    float stop_transmittance;
    uint32_t tile, tile_rank, tile_world;  // 0 tile: whole image on this rank
    uint32_t* rgba;             // width*height packed RGBA8
    uint32_t* spp;              // optional samples per pixel
    uint32_t* work_counter;     // device counter for dynamic pixel scheduling
    unsigned long long* total_samples;  // optional
};
cudaError_t launch_render(const RenderArgs& a, cudaStream_t s);
cudaError_t render_init_attributes();

}  // namespace nb
