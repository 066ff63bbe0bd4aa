// types.h -- layouts shared by host code and kernels of libnerf_b200.
#pragma once
#include <cstdint>

namespace nb {

constexpr uint32_t kMaxLevels = 32;
constexpr uint32_t kFeatPerLevel = 2;

// Multiresolution hash-grid layout (field-for-field the NerfB200GridLayout of
// include/nerf_b200.h).  See grid_layout() in context.cu for the rule.
struct GridLayout {
    uint32_t n_levels;
    uint32_t log2_hashmap_size;
    uint32_t base_resolution;
    uint32_t max_resolution;
    float scale[kMaxLevels];
    uint32_t resolution[kMaxLevels];
    uint32_t dense[kMaxLevels];
    uint32_t offset[kMaxLevels + 1];
};

// Flat MLP parameters (fp16, [out][in] row-major per matrix), stored right
// after the hash-grid entries in the flat parameter vector.
constexpr uint32_t kMlpD0 = 0;                 // density  W0 64 x 32
constexpr uint32_t kMlpD1 = kMlpD0 + 64 * 32;  // density  W1 16 x 64
constexpr uint32_t kMlpC0 = kMlpD1 + 16 * 64;  // colour   W0 64 x 32
constexpr uint32_t kMlpC1 = kMlpC0 + 64 * 32;  // colour   W1 64 x 64
constexpr uint32_t kMlpC2 = kMlpC1 + 64 * 64;  // colour   W2 16 x 64 (rows 0..2 used)
constexpr uint32_t kMlpParams = kMlpC2 + 16 * 64;  // 10240
// The fp32 MLP-gradient buffer carries extra scalars after the weights so
// that one data-parallel all-reduce sums them with the gradients.
constexpr uint32_t kMlpGradLoss = kMlpParams;      // sum of normalised ray losses
constexpr uint32_t kMlpGradSamples = kMlpParams + 1;  // this step's compacted samples (summed over the ranks)
constexpr uint32_t kMlpGradSlots = kMlpParams + 8;

constexpr uint32_t kOccNone = 0, kOccWarmupInit = 1, kOccRefresh = 2;

// One compacted training ray (48 B).
struct alignas(16) RayRecord {
    float dir[3];
    uint32_t begin;  // first sample in the compacted stream
    float gt[4];     // ground truth composited on bg, and ground-truth alpha
    float bg[3];
    uint32_t count;  // samples of this ray
};
static_assert(sizeof(RayRecord) == 48, "RayRecord layout");

struct AdamScalars {
    float learning_rate;
    float grad_scale;
    float inv_bias_correction1;
    float inv_bias_correction2;
    float inv_loss_scale;
    uint32_t skip_update;
};

// Training statistics returned by nerf_read_train_stats (NerfTrainStats layout).
struct StatsBlock {
    float loss;
    float grad_norm;
    uint32_t has_nonfinite;
    uint32_t completed_steps;
    uint32_t last_train_camera;
};

// Device-resident step state.  Every kernel of a step derives what it needs
// from frame_index, so the captured step graph needs no host input.
struct DeviceState {
    uint32_t frame_index;
    uint32_t n_rays;      // rays marched this step
    uint32_t n_samples;   // compacted samples kept this step
    uint32_t n_active;    // compacted rays kept this step
    uint32_t n_marched_active;  // rays with >= 1 sample before the capacity cut
    uint32_t done_blocks; // completion counter of the statistics kernel
    uint32_t nonfinite;
    float grad_sumsq;
    AdamScalars adam;
    StatsBlock stats;
    uint32_t last_samples;
    uint32_t last_active;
    uint32_t last_rays;
    uint32_t counts_parity;  // which half of the per-ray count buffer the last step used
    unsigned long long total_samples;
    unsigned long long total_rays;
    uint32_t mlp_error;   // a tensor-core MLP kernel's MMAs did not complete in time
};

// Data-parallel peer mode: synchronisation words of one rank, in its model
// arena (mapped by every rank).  Zeroed at creation, never reset afterwards:
// barrier epochs only grow.
constexpr uint32_t kMaxDpRanks = 8;
struct DpSync {
    uint32_t flags[kMaxDpRanks];        // flags[q]: last barrier epoch rank q announced to this rank
    float partials[kMaxDpRanks][2];     // partials[q]: rank q's owned-range sum of squares, non-finite flag
    uint32_t epoch;                     // this rank's last barrier epoch
    uint32_t done;                      // last-block counter of the gradient reduction
    uint32_t error;                     // a barrier wait ran out of time
    uint32_t bad;                       // non-finite flag of the gradient reduction in progress
    float sum;                          // sum of squares of the gradient reduction in progress
    uint32_t pad[3];
};

// Per-step constants of the training graph, passed by value to kernels.
// Occupancy cascades: cascade k covers centre c +- half h * 2^k; cascade 0 is
// the configured AABB (min bmn, size bsize).  One cascade: the marching box
// is that AABB.
struct CascadeBox {
    float bmn[3], bsize[3], c[3], h[3];
    uint32_t cascades;
};

struct TrainConsts {
    // scene
    uint32_t n_images, width, height, pad_;
    float fx, fy, cx, cy;
    float aabb_min[3], aabb_max[3], aabb_size[3];  // marching box (outermost cascade)
    CascadeBox casc;
    float cone;
    // sampler
    uint32_t max_rays;
    uint32_t max_steps;
    uint32_t mask_words;     // 32-step words per ray
    uint32_t sample_cap;
    uint32_t rays_per_batch; // nominal batch (rank ray-index stride)
    uint32_t dp_rank, dp_world;
    uint32_t background;     // 0 white, 1 random
    uint32_t target_samples;
    // occupancy
    uint32_t grid_res, cell_count, update_count, warmup_steps, update_interval;
    float occ_decay, occ_threshold;
    // loss / optimiser
    float loss_scale, stop_transmittance;
    float lr, beta1, beta2, eps, clip, guard;
    uint32_t lr_decay_ksteps;
};

}  // namespace nb
