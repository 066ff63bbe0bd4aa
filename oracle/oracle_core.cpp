// oracle_core.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Scalar restatement of the per-sample / per-ray numerics.  Compiled with
// -ffp-contract=off so that every float operation rounds exactly where it is
// written; where the CUDA path uses a fused multiply-add the oracle calls
// std::fmaf at the same place.  Half precision uses the compiler's _Float16
// (IEEE binary16, round-to-nearest-even conversions).
#include "oracle_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace oracle {

// ---------------------------------------------------------------------------
// Integer primitives
// ---------------------------------------------------------------------------

// 32-bit avalanche hash of the reference sampler/runtime
// (reference backend-cuda.cu:321-328 and :1439-1446, identical bodies).
uint32_t hash_u32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Uniform [0,1) from the low 24 bits of the hash (reference backend-cuda.cu:329-332).
float rand01(uint32_t seed) {
    const uint32_t h = hash_u32(seed);
    return static_cast<float>(h & 0x00FFFFFFu) / static_cast<float>(0x01000000u);
}

// Camera of a training step (reference backend-cuda.cu:1482).
uint32_t train_camera(uint32_t frame_index, uint32_t image_count) {
    return hash_u32(frame_index * 747796405u + 2891336453u) % image_count;
}

// Occupancy action of a step (reference backend-cuda.cu:1483-1487):
// warmup-init on step 0, nothing during the rest of warmup, then a refresh
// every update_interval steps.
uint32_t occupancy_mode(uint32_t frame_index, uint32_t warmup_steps, uint32_t update_interval) {
    if (frame_index < warmup_steps) return frame_index == 0u ? kOccWarmupInit : kOccNone;
    return (update_interval != 0u && frame_index % update_interval == 0u) ? kOccRefresh : kOccNone;
}

// ---------------------------------------------------------------------------
// splitmix64 Xavier initialisation (reference backend-cuda.cu:1810-1847)
// ---------------------------------------------------------------------------

static uint64_t splitmix_seed(uint64_t a, uint64_t b) {
    // The reference writes `a + G ^ b * M`; C++ precedence makes it (a + G) ^ (b * M).
    return (a + 0x9e3779b97f4a7c15ull) ^ (b * 0xbf58476d1ce4e5b9ull);
}

static float splitmix_next_unit(uint64_t& state) {
    state += 0x9e3779b97f4a7c15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30u)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27u)) * 0x94d049bb133111ebull;
    z ^= z >> 31u;
    // 24 random bits mapped to [-1, 1): every step below is exact in fp32.
    return static_cast<float>(static_cast<uint32_t>(z >> 32u) >> 8u) * (1.0f / 16777216.0f) * 2.0f - 1.0f;
}

void splitmix_xavier(uint64_t seed_a, uint64_t seed_b, const uint32_t* fan_in, const uint32_t* fan_out, uint32_t n,
                     float* out) {
    uint64_t state = splitmix_seed(seed_a, seed_b);
    uint64_t off = 0;
    for (uint32_t m = 0; m < n; ++m) {
        const float scale = std::sqrt(6.0f / static_cast<float>(fan_in[m] + fan_out[m]));
        const uint64_t count = static_cast<uint64_t>(fan_in[m]) * fan_out[m];
        for (uint64_t i = 0; i < count; ++i) out[off + i] = splitmix_next_unit(state) * scale;
        off += count;
    }
}

void splitmix_uniform(uint64_t seed_a, uint64_t seed_b, uint64_t count, float scale, float* out) {
    uint64_t state = splitmix_seed(seed_a, seed_b);
    for (uint64_t i = 0; i < count; ++i) out[i] = splitmix_next_unit(state) * scale;
}

// ---------------------------------------------------------------------------
// Multiresolution hash grid (defined here; instant-ngp method)
//
// Level l has scale s_l = float(N_min * b^l - 1) with b = (N_max/N_min)^(1/(L-1)),
// evaluated in double on the host and rounded once to float.  A unit-cube
// point p (clamped to [0,1]) maps to u = fma(p, s_l, 0.5) per axis; the cell
// corner is i = floor(u) clamped to [0, R_l-2] and the fraction f = u - floor(u).
// R_l = ceil(s_l) + 2 vertices per axis cover every corner i+1.  A level is
// dense when R_l^3 <= T (entry = x + R(y + R z)) and hashed otherwise
// (entry = (x ^ y*2654435761 ^ z*805459861) & (T-1)).  Level sizes are
// R_l^3 rounded up to 8 entries (dense) or T (hashed), stored back to back.
// Corner c uses bit 0 for x, bit 1 for y, bit 2 for z; its weight is
// ((wx*wy)*wz) with w = f for the upper and 1-f for the lower vertex.  The
// forward feature is the fma chain acc = fma(w_c, param_c, acc) over c = 0..7
// from acc = 0, rounded once to fp16.
// ---------------------------------------------------------------------------

int grid_layout(uint32_t L, uint32_t log2T, uint32_t base, uint32_t maxres, GridLayout* g) {
    if (L == 0u || L > kMaxLevels || log2T < 4u || log2T > 26u || base < 2u || maxres < base) return 1;
    std::memset(g, 0, sizeof(*g));
    g->n_levels = L;
    g->log2_hashmap_size = log2T;
    g->base_resolution = base;
    g->max_resolution = maxres;
    const double log2b = L > 1u ? std::log2(static_cast<double>(maxres) / static_cast<double>(base)) / (L - 1u) : 0.0;
    const uint64_t T = 1ull << log2T;
    uint64_t off = 0;
    for (uint32_t l = 0; l < L; ++l) {
        const double s = std::exp2(l * log2b) * static_cast<double>(base) - 1.0;
        const float sf = static_cast<float>(s);
        const uint32_t R = static_cast<uint32_t>(std::ceil(static_cast<double>(sf))) + 2u;
        const uint64_t R3 = static_cast<uint64_t>(R) * R * R;
        const bool dense = R3 <= T;
        const uint64_t size = dense ? (R3 + 7u) / 8u * 8u : T;
        g->scale[l] = sf;
        g->resolution[l] = R;
        g->dense[l] = dense ? 1u : 0u;
        g->offset[l] = static_cast<uint32_t>(off);
        off += size;
        if (off >= (1ull << 31)) return 2;
    }
    g->offset[L] = static_cast<uint32_t>(off);
    return 0;
}

static inline float clamp01(float x) { return std::min(1.0f, std::max(0.0f, x)); }

void grid_level_corners(const GridLayout& g, uint32_t l, const float p_unit[3], uint32_t idx[8], float w[8]) {
    const float s = g.scale[l];
    const uint32_t R = g.resolution[l];
    const uint32_t mask = (1u << g.log2_hashmap_size) - 1u;
    uint32_t i[3];
    float f[3];
    for (int d = 0; d < 3; ++d) {
        const float u = std::fmaf(clamp01(p_unit[d]), s, 0.5f);
        const float fl = std::floor(u);
        f[d] = u - fl;
        int32_t ii = static_cast<int32_t>(fl);
        ii = std::max(0, std::min(static_cast<int32_t>(R) - 2, ii));
        i[d] = static_cast<uint32_t>(ii);
    }
    for (uint32_t c = 0; c < 8u; ++c) {
        const uint32_t cx = i[0] + (c & 1u), cy = i[1] + ((c >> 1) & 1u), cz = i[2] + ((c >> 2) & 1u);
        uint32_t e;
        if (g.dense[l]) e = cx + R * (cy + R * cz);
        else e = (cx ^ (cy * 2654435761u) ^ (cz * 805459861u)) & mask;
        idx[c] = g.offset[l] + e;
        const float wx = (c & 1u) ? f[0] : 1.0f - f[0];
        const float wy = (c & 2u) ? f[1] : 1.0f - f[1];
        const float wz = (c & 4u) ? f[2] : 1.0f - f[2];
        w[c] = (wx * wy) * wz;
    }
}

void grid_forward_point(const GridLayout& g, const uint16_t* params, const float p_unit[3], uint16_t* feat) {
    for (uint32_t l = 0; l < g.n_levels; ++l) {
        uint32_t idx[8];
        float w[8];
        grid_level_corners(g, l, p_unit, idx, w);
        float a0 = 0.0f, a1 = 0.0f;
        for (int c = 0; c < 8; ++c) {
            a0 = std::fmaf(w[c], h2f(params[2u * idx[c] + 0u]), a0);
            a1 = std::fmaf(w[c], h2f(params[2u * idx[c] + 1u]), a1);
        }
        feat[2u * l + 0u] = f2h(a0);
        feat[2u * l + 1u] = f2h(a1);
    }
}

void grid_backward_point(const GridLayout& g, const float p_unit[3], const float* dfeat, double* grad, uint32_t l_begin,
                         uint32_t l_step) {
    for (uint32_t l = l_begin; l < g.n_levels; l += l_step) {
        uint32_t idx[8];
        float w[8];
        grid_level_corners(g, l, p_unit, idx, w);
        for (int c = 0; c < 8; ++c) {
            grad[2u * idx[c] + 0u] += static_cast<double>(w[c]) * dfeat[2u * l + 0u];
            grad[2u * idx[c] + 1u] += static_cast<double>(w[c]) * dfeat[2u * l + 1u];
        }
    }
}

// ---------------------------------------------------------------------------
// Real spherical harmonics, bands 0..3 (16 coefficients) of a unit direction.
// Standard orthonormal real basis with the Condon-Shortley phase.
// ---------------------------------------------------------------------------
void sh4(const float d[3], float o[16]) {
    const float x = d[0], y = d[1], z = d[2];
    const float xy = x * y, xz = x * z, yz = y * z, x2 = x * x, y2 = y * y, z2 = z * z;
    o[0] = 0.28209479177387814f;
    o[1] = -0.48860251190291987f * y;
    o[2] = 0.48860251190291987f * z;
    o[3] = -0.48860251190291987f * x;
    o[4] = 1.0925484305920792f * xy;
    o[5] = -1.0925484305920792f * yz;
    o[6] = 0.94617469575755997f * z2 - 0.31539156525251999f;
    o[7] = -1.0925484305920792f * xz;
    o[8] = 0.54627421529603959f * x2 - 0.54627421529603959f * y2;
    o[9] = 0.59004358992664352f * y * (-3.0f * x2 + y2);
    o[10] = 2.8906114426405538f * xy * z;
    o[11] = 0.45704579946446572f * y * (1.0f - 5.0f * z2);
    o[12] = 0.3731763325901154f * z * (5.0f * z2 - 3.0f);
    o[13] = 0.45704579946446572f * x * (1.0f - 5.0f * z2);
    o[14] = 1.4453057213202769f * z * (x2 - y2);
    o[15] = 0.59004358992664352f * x * (-x2 + 3.0f * y2);
}

// ---------------------------------------------------------------------------
// MLPs.  Operands of every matrix product are fp16, products are summed in
// fp32 (the tensor-core contract); ReLU outputs are rounded to fp16 because
// they feed the next product.  The ReLU derivative is taken from the fp16
// activation (H > 0), as the CUDA path does.
// ---------------------------------------------------------------------------

void mlp_forward_row(const float* W, const uint16_t* feat16, const float dir[3], MlpTrace* t, float out[4]) {
    const float* Wd0 = W + kMlpD0;
    const float* Wd1 = W + kMlpD1;
    const float* Wc0 = W + kMlpC0;
    const float* Wc1 = W + kMlpC1;
    const float* Wc2 = W + kMlpC2;
    for (int k = 0; k < 32; ++k) t->xd[k] = h2f(feat16[k]);
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int k = 0; k < 32; ++k) s += Wd0[j * 32 + k] * t->xd[k];
        t->hd[j] = rh(std::max(s, 0.0f));
    }
    float yd[16];
    for (int o = 0; o < 16; ++o) {
        float s = 0.0f;
        for (int j = 0; j < 64; ++j) s += Wd1[o * 64 + j] * t->hd[j];
        yd[o] = s;
    }
    float sh[16];
    sh4(dir, sh);
    for (int k = 0; k < 16; ++k) t->xc[k] = rh(yd[k]);
    for (int k = 0; k < 16; ++k) t->xc[16 + k] = rh(sh[k]);
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int k = 0; k < 32; ++k) s += Wc0[j * 32 + k] * t->xc[k];
        t->h1[j] = rh(std::max(s, 0.0f));
    }
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int k = 0; k < 64; ++k) s += Wc1[j * 64 + k] * t->h1[k];
        t->h2[j] = rh(std::max(s, 0.0f));
    }
    float yc[3];
    for (int o = 0; o < 3; ++o) {
        float s = 0.0f;
        for (int j = 0; j < 64; ++j) s += Wc2[o * 64 + j] * t->h2[j];
        yc[o] = s;
    }
    out[0] = yd[0];
    out[1] = yc[0];
    out[2] = yc[1];
    out[3] = yc[2];
}

void mlp_backward_row(const float* W, const MlpTrace& t, const float dout[4], float dfeat[32], double* gW) {
    const float* Wd0 = W + kMlpD0;
    const float* Wd1 = W + kMlpD1;
    const float* Wc0 = W + kMlpC0;
    const float* Wc1 = W + kMlpC1;
    const float* Wc2 = W + kMlpC2;
    float dyc[16] = {};
    for (int o = 0; o < 3; ++o) dyc[o] = rh(dout[1 + o]);
    float dh2[64], dh1[64], dyd[16], dhd[64];
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int o = 0; o < 16; ++o) s += Wc2[o * 64 + j] * dyc[o];
        dh2[j] = t.h2[j] > 0.0f ? rh(s) : 0.0f;
    }
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int i = 0; i < 64; ++i) s += Wc1[i * 64 + j] * dh2[i];
        dh1[j] = t.h1[j] > 0.0f ? rh(s) : 0.0f;
    }
    for (int k = 0; k < 16; ++k) {
        float s = 0.0f;
        for (int j = 0; j < 64; ++j) s += Wc0[j * 32 + k] * dh1[j];
        dyd[k] = rh(s + (k == 0 ? dout[0] : 0.0f));
    }
    for (int j = 0; j < 64; ++j) {
        float s = 0.0f;
        for (int o = 0; o < 16; ++o) s += Wd1[o * 64 + j] * dyd[o];
        dhd[j] = t.hd[j] > 0.0f ? rh(s) : 0.0f;
    }
    for (int k = 0; k < 32; ++k) {
        float s = 0.0f;
        for (int j = 0; j < 64; ++j) s += Wd0[j * 32 + k] * dhd[j];
        dfeat[k] = s;
    }
    if (!gW) return;
    for (int j = 0; j < 64; ++j)
        for (int k = 0; k < 32; ++k) gW[kMlpD0 + j * 32 + k] += static_cast<double>(dhd[j]) * t.xd[k];
    for (int o = 0; o < 16; ++o)
        for (int j = 0; j < 64; ++j) gW[kMlpD1 + o * 64 + j] += static_cast<double>(dyd[o]) * t.hd[j];
    for (int j = 0; j < 64; ++j)
        for (int k = 0; k < 32; ++k) gW[kMlpC0 + j * 32 + k] += static_cast<double>(dh1[j]) * t.xc[k];
    for (int i = 0; i < 64; ++i)
        for (int j = 0; j < 64; ++j) gW[kMlpC1 + i * 64 + j] += static_cast<double>(dh2[i]) * t.h1[j];
    for (int o = 0; o < 3; ++o)
        for (int j = 0; j < 64; ++j) gW[kMlpC2 + o * 64 + j] += static_cast<double>(dyc[o]) * t.h2[j];
}

// ---------------------------------------------------------------------------
// Activations
// ---------------------------------------------------------------------------

// trunc_exp: sigma = exp(x); d sigma / dx = exp(clamp(x, -15, 15)).
float density_activation(float x) { return std::exp(x); }
float density_activation_grad(float x) { return std::exp(std::min(15.0f, std::max(-15.0f, x))); }
float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// ---------------------------------------------------------------------------
// Compositing + alpha-weighted MSE, forward and backward for one ray
// (reference backend-cuda.cu:1095-1182).  The reference composites on white;
// here the background colour is a per-ray input (white reproduces the
// reference).  With stop_T > 0 the ray stops before the first sample whose
// incoming transmittance is below stop_T; later samples get no gradient.
// ---------------------------------------------------------------------------
float composite_ray(const float* raw, const float* dt, uint32_t count, const float gt[4], const float bg[3],
                    float inv_norm, float loss_scale, float stop_T, float* dout, uint32_t* used_out, float rgb_out[3]) {
    // A ray without samples carries no loss (reference backend-cuda.cu:1103).
    if (count == 0u) {
        if (used_out) *used_out = 0u;
        if (rgb_out)
            for (int ch = 0; ch < 3; ++ch) rgb_out[ch] = bg[ch];
        return 0.0f;
    }
    float T = 1.0f;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    uint32_t used = count;
    // Per-sample forward state kept for the backward sweep.
    float* Ti = dout;  // reuse dout as scratch for T_i in slot 0 until the backward overwrites it
    for (uint32_t i = 0; i < count; ++i) {
        if (stop_T > 0.0f && T < stop_T) {
            used = i;
            break;
        }
        const float sigma = density_activation(raw[4 * i + 0]);
        const float a = 1.0f - std::exp(-(sigma * std::max(0.0f, dt[i])));
        const float w = T * a;
        for (int ch = 0; ch < 3; ++ch) acc[ch] += w * sigmoid(raw[4 * i + 1 + ch]);
        Ti[4 * i + 0] = T;
        T *= 1.0f - a;
    }
    float pred[3], g[3];
    const float ga = std::min(1.0f, std::max(0.0f, gt[3]));
    const float ray_w = 0.1f + 0.9f * ga;
    float loss = 0.0f;
    for (int ch = 0; ch < 3; ++ch) {
        pred[ch] = acc[ch] + T * bg[ch];
        const float d = pred[ch] - gt[ch];
        loss += d * d;
        g[ch] = 2.0f * ray_w * d * inv_norm;
    }
    loss *= ray_w;
    if (rgb_out)
        for (int ch = 0; ch < 3; ++ch) rgb_out[ch] = pred[ch];
    float suffix[3] = {T * bg[0], T * bg[1], T * bg[2]};
    for (int64_t i = static_cast<int64_t>(used) - 1; i >= 0; --i) {
        const float x = raw[4 * i + 0];
        const float sigma = density_activation(x);
        const float dti = std::max(0.0f, dt[i]);
        const float e = std::exp(-(sigma * dti));
        const float a = 1.0f - e;
        const float one_minus_a = std::max(1e-6f, 1.0f - a);
        const float trans = Ti[4 * i + 0];
        const float w = trans * a;
        float c[3];
        for (int ch = 0; ch < 3; ++ch) c[ch] = sigmoid(raw[4 * i + 1 + ch]);
        float dL_da = 0.0f;
        for (int ch = 0; ch < 3; ++ch) dL_da += g[ch] * (trans * c[ch] - suffix[ch] / one_minus_a);
        dout[4 * i + 0] = loss_scale * (dL_da * dti * e * density_activation_grad(x));
        for (int ch = 0; ch < 3; ++ch) {
            dout[4 * i + 1 + ch] = loss_scale * (w * g[ch] * c[ch] * (1.0f - c[ch]));
            suffix[ch] += w * c[ch];
        }
    }
    for (uint32_t i = used; i < count; ++i)
        for (int k = 0; k < 4; ++k) dout[4 * i + k] = 0.0f;
    if (used_out) *used_out = used;
    return loss;
}

// ---------------------------------------------------------------------------
// Adam (reference backend-cuda.cu:1513-1554)
// ---------------------------------------------------------------------------
void adam_scalars(float grad_norm, uint32_t has_nonfinite, uint32_t step, const NerfHyperParams& hp, AdamScalars* s) {
    const bool skip = has_nonfinite != 0u || !std::isfinite(grad_norm) || grad_norm > hp.update_guard_grad_norm;
    float lr = 0.0f, gs = 1.0f, b1 = 1.0f, b2 = 1.0f;
    if (!skip) {
        const float decay = static_cast<float>(hp.lr_decay_ksteps) * 1000.0f;
        lr = decay > 0.0f ? hp.learning_rate * std::pow(0.1f, static_cast<float>(step) / decay) : hp.learning_rate;
        gs = grad_norm > hp.grad_clip_norm && grad_norm > 0.0f ? hp.grad_clip_norm / grad_norm : 1.0f;
        b1 = 1.0f / (1.0f - std::pow(hp.adam_beta1, static_cast<float>(step)));
        b2 = 1.0f / (1.0f - std::pow(hp.adam_beta2, static_cast<float>(step)));
    }
    s->learning_rate = lr;
    s->grad_scale = gs;
    s->inv_bias_correction1 = b1;
    s->inv_bias_correction2 = b2;
    s->inv_loss_scale = 1.0f / hp.loss_scale;
    s->skip_update = skip ? 1u : 0u;
}

void adam_range(float* master, uint16_t* p16, const float* grad, float* m, float* v, uint64_t begin, uint64_t end,
                float beta1, float beta2, float eps, const AdamScalars& s) {
    if (s.skip_update) return;
    for (uint64_t i = begin; i < end; ++i) {
        const float g = grad[i] * s.inv_loss_scale * s.grad_scale;
        // b*m + (1-b)*g with the first product fused, as the reference's
        // compiler contracts it (backend-cuda.cu:1546-1547).
        const float mi = std::fmaf(beta1, m[i], (1.0f - beta1) * g);
        const float vi = std::fmaf(beta2, v[i], (1.0f - beta2) * g * g);
        const float step = s.learning_rate * (mi * s.inv_bias_correction1) / (std::sqrt(vi * s.inv_bias_correction2) + eps);
        const float w = master[i] - step;
        m[i] = mi;
        v[i] = vi;
        master[i] = w;
        p16[i] = f2h(w);
    }
}

}  // namespace oracle

// ---------------------------------------------------------------------------
// C entry points for the numerics
// ---------------------------------------------------------------------------
using namespace oracle;

extern "C" {

uint32_t oracle_hash_u32(uint32_t x) { return hash_u32(x); }
float oracle_rand01(uint32_t seed) { return rand01(seed); }
uint32_t oracle_train_camera(uint32_t f, uint32_t n) { return train_camera(f, n); }
uint32_t oracle_occupancy_mode(uint32_t f, uint32_t w, uint32_t i) { return occupancy_mode(f, w, i); }

void oracle_splitmix_xavier(uint64_t a, uint64_t b, const uint32_t* fi, const uint32_t* fo, uint32_t n, float* out) {
    splitmix_xavier(a, b, fi, fo, n, out);
}
void oracle_splitmix_uniform(uint64_t a, uint64_t b, uint64_t count, float scale, float* out) {
    splitmix_uniform(a, b, count, scale, out);
}

int oracle_grid_layout(uint32_t L, uint32_t log2T, uint32_t base, uint32_t maxres, OracleGridLayout* out) {
    static_assert(sizeof(OracleGridLayout) == sizeof(GridLayout), "layout mirror");
    return grid_layout(L, log2T, base, maxres, reinterpret_cast<GridLayout*>(out));
}

void oracle_grid_corners(const OracleGridLayout* g, const float* pos, uint32_t n, uint32_t* idx, float* w) {
    const GridLayout& gl = *reinterpret_cast<const GridLayout*>(g);
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t l = 0; l < gl.n_levels; ++l)
            grid_level_corners(gl, l, pos + 3u * i, idx + (static_cast<uint64_t>(i) * gl.n_levels + l) * 8u,
                               w + (static_cast<uint64_t>(i) * gl.n_levels + l) * 8u);
}

void oracle_grid_forward(const OracleGridLayout* g, const uint16_t* params, const float* pos, uint32_t n, uint16_t* feat) {
    const GridLayout& gl = *reinterpret_cast<const GridLayout*>(g);
    for (uint32_t i = 0; i < n; ++i) grid_forward_point(gl, params, pos + 3u * i, feat + 2ull * gl.n_levels * i);
}

void oracle_grid_backward(const OracleGridLayout* g, const float* pos, const float* dfeat, uint32_t n, double* grad) {
    const GridLayout& gl = *reinterpret_cast<const GridLayout*>(g);
    for (uint32_t i = 0; i < n; ++i) grid_backward_point(gl, pos + 3u * i, dfeat + 2ull * gl.n_levels * i, grad, 0, 1);
}

void oracle_sh4(const float* dirs, uint32_t n, float* out) {
    for (uint32_t i = 0; i < n; ++i) sh4(dirs + 3u * i, out + 16u * i);
}

void oracle_mlp_forward(const uint16_t* mlp, const uint16_t* feat, const float* dirs, uint32_t n, float* out) {
    float W[kMlpParams];
    for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(mlp[i]);
    for (uint32_t i = 0; i < n; ++i) {
        MlpTrace t;
        mlp_forward_row(W, feat + 32u * i, dirs + 3u * i, &t, out + 4u * i);
    }
}

void oracle_mlp_backward(const uint16_t* mlp, const uint16_t* feat, const float* dirs, const float* dout, uint32_t n,
                         float* dfeat, double* wgrad) {
    float W[kMlpParams];
    for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(mlp[i]);
    for (uint32_t i = 0; i < n; ++i) {
        MlpTrace t;
        float out[4];
        mlp_forward_row(W, feat + 32u * i, dirs + 3u * i, &t, out);
        mlp_backward_row(W, t, dout + 4u * i, dfeat + 32u * i, wgrad);
    }
}

void oracle_composite(const float* raw, const float* dt, const uint32_t* begin, const uint32_t* count, uint32_t n_rays,
                      const float* gt, const float* bg, float inv_norm, float loss_scale, float stop_T, float* dout,
                      float* ray_loss, uint32_t* used, float* rgb_out) {
    for (uint32_t r = 0; r < n_rays; ++r) {
        const uint32_t b = begin[r];
        const float l = composite_ray(raw + 4ull * b, dt + b, count[r], gt + 4u * r, bg + 3u * r, inv_norm, loss_scale,
                                      stop_T, dout + 4ull * b, used ? used + r : nullptr, rgb_out ? rgb_out + 3u * r : nullptr);
        if (ray_loss) ray_loss[r] = l;
    }
}

void oracle_adam_scalars(float grad_norm, uint32_t has_nonfinite, uint32_t step, const NerfHyperParams* hp,
                         OracleAdamScalars* out) {
    static_assert(sizeof(OracleAdamScalars) == sizeof(AdamScalars), "mirror");
    adam_scalars(grad_norm, has_nonfinite, step, *hp, reinterpret_cast<AdamScalars*>(out));
}

void oracle_adam(float* master, uint16_t* p16, const float* grad, float* m, float* v, uint64_t n, float b1, float b2,
                 float eps, const OracleAdamScalars* s) {
    adam_range(master, p16, grad, m, v, 0, n, b1, b2, eps, *reinterpret_cast<const AdamScalars*>(s));
}

}  // extern "C"
