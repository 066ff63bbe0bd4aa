// oracle_internal.h -- TEST INFRASTRUCTURE ONLY (see oracle.h).
#pragma once
#include <cstdint>
#include <cstring>

#include "oracle.h"

namespace oracle {

constexpr uint32_t kMaxLevels = 32;
constexpr uint32_t kOccNone = 0, kOccWarmupInit = 1, kOccRefresh = 2;

// Flat MLP parameter layout (fp16 values, [out][in] row-major per matrix).
constexpr uint32_t kMlpD0 = 0;                 // density  64 x 32
constexpr uint32_t kMlpD1 = kMlpD0 + 64 * 32;  // density  16 x 64
constexpr uint32_t kMlpC0 = kMlpD1 + 16 * 64;  // colour   64 x 32
constexpr uint32_t kMlpC1 = kMlpC0 + 64 * 32;  // colour   64 x 64
constexpr uint32_t kMlpC2 = kMlpC1 + 64 * 64;  // colour   16 x 64 (rows 0..2 used)
constexpr uint32_t kMlpParams = kMlpC2 + 16 * 64;
static_assert(kMlpParams == ORACLE_MLP_PARAMS, "mlp size");

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

struct AdamScalars {
    float learning_rate;
    float grad_scale;
    float inv_bias_correction1;
    float inv_bias_correction2;
    float inv_loss_scale;
    uint32_t skip_update;
};

// Forward activations of one sample, kept for its backward.
struct MlpTrace {
    float xd[32];  // hash features (fp16 values)
    float hd[64];  // density hidden (fp16 values)
    float xc[32];  // colour input: density outputs + SH (fp16 values)
    float h1[64];
    float h2[64];
};

using f16 = _Float16;
inline float h2f(uint16_t b) {
    f16 h;
    std::memcpy(&h, &b, 2);
    return static_cast<float>(h);
}
inline uint16_t f2h(float x) {
    f16 h = static_cast<f16>(x);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}
inline float rh(float x) { return static_cast<float>(static_cast<f16>(x)); }

uint32_t hash_u32(uint32_t x);
float rand01(uint32_t seed);
uint32_t train_camera(uint32_t frame_index, uint32_t image_count);
uint32_t occupancy_mode(uint32_t frame_index, uint32_t warmup_steps, uint32_t update_interval);
void splitmix_xavier(uint64_t seed_a, uint64_t seed_b, const uint32_t* fan_in, const uint32_t* fan_out, uint32_t n,
                     float* out);
void splitmix_uniform(uint64_t seed_a, uint64_t seed_b, uint64_t count, float scale, float* out);
int grid_layout(uint32_t L, uint32_t log2T, uint32_t base, uint32_t maxres, GridLayout* g);
void grid_level_corners(const GridLayout& g, uint32_t l, const float p_unit[3], uint32_t idx[8], float w[8]);
void grid_forward_point(const GridLayout& g, const uint16_t* params, const float p_unit[3], uint16_t* feat);
void grid_backward_point(const GridLayout& g, const float p_unit[3], const float* dfeat, double* grad, uint32_t l_begin,
                         uint32_t l_step);
void sh4(const float d[3], float o[16]);
void mlp_forward_row(const float* W, const uint16_t* feat16, const float dir[3], MlpTrace* t, float out[4]);
void mlp_backward_row(const float* W, const MlpTrace& t, const float dout[4], float dfeat[32], double* gW);
float density_activation(float x);
float density_activation_grad(float x);
float sigmoid(float x);
float composite_ray(const float* raw, const float* dt, uint32_t count, const float gt[4], const float bg[3], float inv_norm,
                    float loss_scale, float stop_T, float* dout, uint32_t* used_out, float rgb_out[3]);
void adam_scalars(float grad_norm, uint32_t has_nonfinite, uint32_t step, const NerfHyperParams& hp, AdamScalars* s);
void adam_range(float* master, uint16_t* p16, const float* grad, float* m, float* v, uint64_t begin, uint64_t end,
                float beta1, float beta2, float eps, const AdamScalars& s);

}  // namespace oracle
