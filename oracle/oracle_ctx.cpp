// oracle_ctx.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// CPU emulation of the backend behind the nerf.h ABI: training-ray sampler,
// occupancy maintenance, one training step, and rendering.  The CUDA path
// must produce bit-identical per-ray sample counts, compaction offsets and
// occupancy bitfields (given the same density grid), and floating-point
// values within the tolerances written in tests/.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "oracle_internal.h"

namespace oracle {
namespace {

template <class F>
void parallel_for(uint64_t n, uint32_t threads, F&& fn) {
    if (threads <= 1u || n < 2u * threads) {
        fn(uint64_t{0}, n, 0u);
        return;
    }
    std::vector<std::thread> pool;
    const uint64_t chunk = (n + threads - 1u) / threads;
    for (uint32_t t = 0; t < threads; ++t) {
        const uint64_t b = t * chunk, e = std::min<uint64_t>(n, b + chunk);
        if (b >= e) break;
        pool.emplace_back([=, &fn] { fn(b, e, t); });
    }
    for (auto& th : pool) th.join();
}

// Per-ray background salts for the random-background mode.
constexpr uint32_t kBgSalt[3] = {0x1B873593u, 0x5BD1E995u, 0x27D4EB2Fu};

struct Ray {
    float o[3], d[3];
    float tn, tf;
    float px, py;  // continuous pixel coordinates (py not flipped)
};

// Pinhole ray through a continuous pixel position (reference
// backend-cuda.cu:373-390).  dir_cam = ((px-cx)/fx, (H-1-py-cy)/fy, -1);
// world dir = R * dir_cam as fma(r2, z, fma(r1, y, r0*x)); the reference
// normalises with the approximate rsqrtf, here 1/sqrt(len2) is correctly
// rounded so that host and device agree to the bit.
bool ray_dir(const float* cam, float fx, float fy, float cx, float cy, float px, float pyf, float d[3]) {
    const float dcx = (px - cx) / fx;
    const float dcy = (pyf - cy) / fy;
    const float dcz = -1.0f;
    // a*b + c*d + e*f evaluated as fma(e, f, fma(a, b, c*d)): the contraction
    // the reference's compiler applies (pinned against its kernel outputs).
    for (int k = 0; k < 3; ++k) d[k] = std::fmaf(cam[4 * k + 2], dcz, std::fmaf(cam[4 * k + 0], dcx, cam[4 * k + 1] * dcy));
    const float len2 = std::fmaf(d[2], d[2], std::fmaf(d[0], d[0], d[1] * d[1]));
    if (len2 <= 1e-16f) return false;
    const float inv = 1.0f / std::sqrt(len2);
    for (int k = 0; k < 3; ++k) d[k] = d[k] * inv;
    return true;
}

// Slab test clamped to t >= 0 (reference backend-cuda.cu:391-408).
bool intersect_aabb(const float o[3], const float d[3], const float mn[3], const float mx[3], float* tn, float* tf) {
    float tmin[3], tmax[3];
    for (int k = 0; k < 3; ++k) {
        const float inv = std::fabs(d[k]) > 1e-8f ? 1.0f / d[k] : (d[k] >= 0.0f ? 1e8f : -1e8f);
        const float t0 = (mn[k] - o[k]) * inv;
        const float t1 = (mx[k] - o[k]) * inv;
        tmin[k] = std::fmin(t0, t1);
        tmax[k] = std::fmax(t0, t1);
    }
    float t_near = std::fmax(std::fmax(tmin[0], tmin[1]), tmin[2]);
    const float t_far = std::fmin(std::fmin(tmax[0], tmax[1]), tmax[2]);
    if (!(t_near <= t_far && t_far > 0.0f)) return false;
    if (t_near < 0.0f) t_near = 0.0f;
    *tn = t_near;
    *tf = t_far;
    return true;
}

// Marching box and occupancy cascades: cascade k covers centre c +- half h *
// 2^k (cascade 0: the configured AABB bmn, bsize); rays are clipped to the
// outermost cascade (mn, mx, size), which with one cascade is that AABB.
struct Box {
    float mn[3], mx[3], size[3];
    float bmn[3], bsize[3], c[3], h[3];
    uint32_t K = 1;
};
Box make_box(const float amin[3], const float amax[3], uint32_t K) {
    Box b;
    b.K = K;
    for (int k = 0; k < 3; ++k) {
        b.bmn[k] = amin[k];
        b.bsize[k] = amax[k] - amin[k];
        b.c[k] = (amin[k] + amax[k]) * 0.5f;
        b.h[k] = b.bsize[k] * 0.5f;
        b.mn[k] = amin[k];
        b.mx[k] = amax[k];
    }
    if (K > 1u) {
        const float s = std::ldexp(1.0f, static_cast<int>(K) - 1);
        for (int k = 0; k < 3; ++k) {
            const float hs = b.h[k] * s;
            b.mn[k] = b.c[k] - hs;
            b.mx[k] = b.c[k] + hs;
        }
    }
    for (int k = 0; k < 3; ++k) b.size[k] = b.mx[k] - b.mn[k];
    return b;
}
// Cascade of p: 0 inside the configured AABB, else ceil(log2 m) with
// m = max_k |p_k - c_k| / h_k (from m = f 2^e, f in [0.5, 1)).
uint32_t cascade_of(const Box& b, const float p[3]) {
    float m = 0.0f;
    for (int k = 0; k < 3; ++k) m = std::fmax(m, std::fabs(p[k] - b.c[k]) / b.h[k]);
    if (!(m > 1.0f)) return 0u;
    int e = 0;
    const float f = std::frexp(m, &e);
    return static_cast<uint32_t>(f == 0.5f ? e - 1 : e);
}

// Bitfield lookup of the cell holding p (reference backend-cuda.cu:338-351),
// in the R^3 grid of p's cascade (cascade after cascade in the bitfield).
bool occupied(const uint32_t* bits, uint32_t R, const Box& b, const float p[3]) {
    float rel[3];
    uint32_t mip = 0;
    if (b.K <= 1u) {
        for (int k = 0; k < 3; ++k) rel[k] = (p[k] - b.mn[k]) / b.size[k];
    } else {
        mip = cascade_of(b, p);
        if (mip >= b.K) return false;
        const float s = std::ldexp(1.0f, static_cast<int>(mip));
        for (int k = 0; k < 3; ++k) {
            const float lo = mip == 0u ? b.bmn[k] : b.c[k] - b.h[k] * s;
            rel[k] = (p[k] - lo) / (b.bsize[k] * s);
        }
    }
    for (int k = 0; k < 3; ++k)
        if (rel[k] < 0.0f || rel[k] >= 1.0f) return false;
    uint32_t ix[3];
    for (int k = 0; k < 3; ++k) ix[k] = std::min(R - 1u, static_cast<uint32_t>(rel[k] * static_cast<float>(R)));
    const uint32_t idx = mip * R * R * R + ix[0] + ix[1] * R + ix[2] * R * R;
    return ((bits[idx >> 5] >> (idx & 31u)) & 1u) != 0u;
}

float cone_angle(float fx, float fy) {
    const float ix = fx > 0.0f ? 1.0f / fx : 0.0f;
    const float iy = fy > 0.0f ? 1.0f / fy : 0.0f;
    return 0.5f * (ix + iy);
}

// Cone-angle march (reference backend-cuda.cu:450-470):
//   dt = min(max(dt_min, t*cone), t_far - t), t_mid = t + dt/2, p = fma(t_mid, d, o),
//   keep the step when p's cell is occupied, t += dt, at most max_steps steps.
template <class F>
uint32_t march(const Ray& r, uint32_t max_steps, float cone, const Box& box, uint32_t R, const uint32_t* bits, F&& on_sample) {
    const float dt_min = (r.tf - r.tn) / static_cast<float>(max_steps);
    float t = r.tn;
    uint32_t i = 0, count = 0;
    while (t < r.tf && i < max_steps) {
        const float dt = std::fmin(std::fmax(dt_min, t * cone), r.tf - t);
        const float t_mid = t + 0.5f * dt;
        float p[3];
        for (int k = 0; k < 3; ++k) p[k] = std::fmaf(t_mid, r.d[k], r.o[k]);
        if (occupied(bits, R, box, p)) {
            on_sample(i, t_mid, dt, p);
            ++count;
        }
        t += dt;
        ++i;
    }
    return count;
}

}  // namespace

struct Ctx {
    // scene (copied at create, reference backend-cuda.cu:1928-1990)
    uint32_t n_images = 0, W = 0, H = 0;
    float fx = 0, fy = 0, cx = 0, cy = 0;
    std::vector<uint8_t> images;
    std::vector<float> cams;
    uint32_t grid_res = 0, max_sample_steps = 0, max_batch_rays = 0;
    OracleOptions opt{};
    GridLayout grid{};
    uint64_t n_grid = 0, n_params = 0;
    std::vector<float> master, m, v, grad;
    std::vector<uint16_t> p16;
    std::vector<float> density;
    std::vector<uint32_t> bits;
    // configuration
    bool configured = false;
    NerfTrainingConfig cfg{};
    float mn[3] = {0, 0, 0}, mx[3] = {1, 1, 1}, size[3] = {1, 1, 1};  // marching box
    Box box = make_box(mn, mx, 1);
    uint32_t cell_count = 0, update_count = 0, cap = 0;
    // step state
    uint32_t frame = 0, n_rays = 0;
    NerfTrainStats stats{};
    double loss_sum = 0.0;
    // Data parallel: the compacted samples of all ranks in this step (set by
    // the caller with the summed gradients; 0: this rank's own count).
    uint64_t global_samples = 0;
    uint32_t active = 0;
    bool grads_pending = false;
    // last batch
    std::vector<uint32_t> ray_counts;
    std::vector<uint32_t> k_index, k_begin, k_count;
    std::vector<float> k_gt, k_bg, k_dir;
    std::vector<float> s_pos;  // x y z dt
    std::vector<uint32_t> s_ray;
    OracleBatchInfo info{};

    void init_params();
    void occupancy_step(uint32_t mode);
    void sample_batch(uint32_t camera);
    void forward_backward();
    void apply_update();
    float density_at(const float p_world[3]) const;
    void to_unit(const float p[3], float u[3]) const {
        for (int k = 0; k < 3; ++k) u[k] = std::min(1.0f, std::max(0.0f, (p[k] - mn[k]) / size[k]));
    }
};

void Ctx::init_params() {
    n_grid = 2ull * grid.offset[grid.n_levels];
    n_params = n_grid + kMlpParams;
    master.assign(n_params, 0.0f);
    // Hash table: U(-s, s) from its own splitmix stream.
    splitmix_uniform(0x2468ull, 0x1357ull, n_grid, opt.hash_init_scale, master.data());
    // MLPs: the reference's Xavier draw and stream seeds, applied to the
    // 64-wide shapes (reference backend-cuda.cu:1810-1847).
    const uint32_t dfi[2] = {32, 64}, dfo[2] = {64, 16};
    splitmix_xavier(0x1234ull, 0x5678ull, dfi, dfo, 2, master.data() + n_grid + kMlpD0);
    const uint32_t cfi[3] = {32, 64, 64}, cfo[3] = {64, 64, 16};
    splitmix_xavier(0x9abcull, 0xdef0ull, cfi, cfo, 3, master.data() + n_grid + kMlpC0);
    p16.resize(n_params);
    for (uint64_t i = 0; i < n_params; ++i) p16[i] = f2h(master[i]);
    m.assign(n_params, 0.0f);
    v.assign(n_params, 0.0f);
    grad.assign(n_params, 0.0f);
}

float Ctx::density_at(const float p[3]) const {
    float u[3];
    to_unit(p, u);
    uint16_t feat[64];
    grid_forward_point(grid, p16.data(), u, feat);
    float W[kMlpParams];
    for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(p16[n_grid + i]);
    MlpTrace t;
    float out[4];
    const float dir[3] = {0.0f, 0.0f, 1.0f};
    mlp_forward_row(W, feat, dir, &t, out);
    return density_activation(out[0]);
}

// Occupancy maintenance of one step given the query window's densities
// (reference backend-cuda.cu:1555-1634 and the call order at :2267-2291):
// warm-up init sets every cell to 1 and every bit; refresh decays every
// cell, folds max(cell, sigma_k) over the window cells (start + k) mod C with
// start = frame * update_count mod C, and rebuilds every bit as cell > threshold.
void occupancy_apply(float* density, uint32_t* bits, const float* sig, uint32_t cell_count, uint32_t update_count,
                     uint32_t frame, uint32_t mode, float decay, float threshold) {
    const uint32_t words = (cell_count + 31u) / 32u;
    if (mode == kOccWarmupInit) {
        std::fill(density, density + cell_count, 1.0f);
        std::fill(bits, bits + words, 0xFFFFFFFFu);
        return;
    }
    if (mode != kOccRefresh) return;
    for (uint32_t c = 0; c < cell_count; ++c) density[c] *= decay;
    std::fill(bits, bits + words, 0u);
    const uint32_t start = static_cast<uint32_t>(static_cast<uint64_t>(frame) * update_count % cell_count);
    for (uint32_t k = 0; k < update_count; ++k) {
        const uint32_t cell = static_cast<uint32_t>((static_cast<uint64_t>(start) + k) % cell_count);
        density[cell] = std::fmax(density[cell], sig[k]);
    }
    for (uint32_t c = 0; c < cell_count; ++c)
        if (density[c] > threshold) bits[c >> 5] |= 1u << (c & 31u);
}

// World position of the k-th queried cell of an occupancy refresh: cells
// are visited round-robin from frame * update_count mod C, the query point is
// the cell centre (reference backend-cuda.cu:1575-1616).
// With cascades the cells run cascade after cascade, each centre in its
// cascade's box.
void occupancy_cell_center(uint32_t frame, uint32_t k, uint32_t update_count, uint32_t cell_count, uint32_t R, const Box& b,
                           float c[3]) {
    const uint32_t start = static_cast<uint32_t>(static_cast<uint64_t>(frame) * update_count % cell_count);
    const uint32_t q = static_cast<uint32_t>((static_cast<uint64_t>(start) + k) % cell_count);
    const uint32_t mip = q / (R * R * R), cell = q - mip * R * R * R;
    const uint32_t z = cell / (R * R), rem = cell - z * R * R, y = rem / R, x = rem - y * R;
    const uint32_t ci[3] = {x, y, z};
    const float s = std::ldexp(1.0f, static_cast<int>(mip));
    for (int d = 0; d < 3; ++d) {
        const float lo = mip == 0u ? b.bmn[d] : b.c[d] - b.h[d] * s;
        const float step = (b.bsize[d] * s) / static_cast<float>(R);
        c[d] = std::fmaf(static_cast<float>(ci[d]) + 0.5f, step, lo);
    }
}

// Densities of the query window: cell centres through the hash grid and the
// density MLP, sigma = exp(raw).
void Ctx::occupancy_step(uint32_t mode) {
    std::vector<float> sig;
    if (mode == kOccRefresh) {
        sig.resize(update_count);
        float W[kMlpParams];
        for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(p16[n_grid + i]);
        parallel_for(update_count, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
            for (uint64_t k = b; k < e; ++k) {
                float c[3];
                occupancy_cell_center(frame, static_cast<uint32_t>(k), update_count, cell_count, grid_res, box, c);
                float u[3];
                to_unit(c, u);
                uint16_t feat[64];
                grid_forward_point(grid, p16.data(), u, feat);
                MlpTrace t;
                float out[4];
                const float dir[3] = {0.0f, 0.0f, 1.0f};
                mlp_forward_row(W, feat, dir, &t, out);
                sig[k] = density_activation(out[0]);
            }
        });
    }
    occupancy_apply(density.data(), bits.data(), sig.data(), cell_count, update_count, frame, mode,
                    cfg.occupancy_params.decay, cfg.occupancy_params.threshold);
}

// Training-ray sampler (reference backend-cuda.cu:422-533) with the
// deterministic compaction of this backend: rays are kept in ray order while
// the running sample total stays within the per-step capacity; rays without
// samples are dropped from the active list.
void Ctx::sample_batch(uint32_t camera) {
    const uint32_t n = n_rays;
    const float* cam = cams.data() + 16ull * camera;
    const uint8_t* img = images.data() + static_cast<uint64_t>(camera) * W * H * 4u;
    const float cone = cone_angle(fx, fy);
    const uint32_t max_steps = cfg.max_sample_steps_per_ray;
    ray_counts.assign(n, 0u);
    std::vector<Ray> rays(n);
    std::vector<uint8_t> ok(n, 0);
    parallel_for(n, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        for (uint64_t r = b; r < e; ++r) {
            const uint32_t gr = opt.dp_rank * cfg.rays_per_batch + static_cast<uint32_t>(r);
            const uint32_t seed = frame * 1315423911u ^ gr * 9781u;
            Ray ray{};
            ray.px = rand01(seed ^ 0xA511E9B3u) * static_cast<float>(W);
            ray.py = rand01(seed ^ 0x63D83595u) * static_cast<float>(H);
            const float pyf = static_cast<float>(H) - 1.0f - ray.py;
            for (int k = 0; k < 3; ++k) ray.o[k] = cam[4 * k + 3];
            if (!ray_dir(cam, fx, fy, cx, cy, ray.px, pyf, ray.d)) continue;
            if (!intersect_aabb(ray.o, ray.d, box.mn, box.mx, &ray.tn, &ray.tf)) continue;
            if (!(ray.tf - ray.tn > 0.0f)) continue;
            rays[r] = ray;
            ok[r] = 1;
            ray_counts[r] = march(ray, max_steps, cone, box, grid_res, bits.data(),
                                  [](uint32_t, float, float, const float*) {});
        }
    });
    // Ordered compaction.
    k_index.clear();
    k_begin.clear();
    k_count.clear();
    uint64_t total = 0;
    for (uint32_t r = 0; r < n; ++r) {
        const uint32_t c = ray_counts[r];
        if (c == 0u) continue;
        if (total + c > cap) break;
        k_index.push_back(r);
        k_begin.push_back(static_cast<uint32_t>(total));
        k_count.push_back(c);
        total += c;
    }
    const uint32_t nk = static_cast<uint32_t>(k_index.size());
    s_pos.assign(4ull * total, 0.0f);
    s_ray.assign(total, 0u);
    k_gt.assign(4ull * nk, 0.0f);
    k_bg.assign(3ull * nk, 1.0f);
    k_dir.assign(3ull * nk, 0.0f);
    parallel_for(nk, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        for (uint64_t k = b; k < e; ++k) {
            const uint32_t r = k_index[k];
            const Ray& ray = rays[r];
            uint32_t s = k_begin[k];
            march(ray, max_steps, cone, box, grid_res, bits.data(),
                  [&](uint32_t, float, float dt, const float* p) {
                      s_pos[4ull * s + 0] = p[0];
                      s_pos[4ull * s + 1] = p[1];
                      s_pos[4ull * s + 2] = p[2];
                      s_pos[4ull * s + 3] = dt;
                      s_ray[s] = static_cast<uint32_t>(k);
                      ++s;
                  });
            // Ground truth: bilinear RGBA8 fetch at the unflipped pixel
            // position, composited on the ray's background (reference
            // backend-cuda.cu:471-499).
            const uint32_t gr = opt.dp_rank * cfg.rays_per_batch + r;
            const uint32_t seed = frame * 1315423911u ^ gr * 9781u;
            float bg[3] = {1.0f, 1.0f, 1.0f};
            if (opt.background == 1u)
                for (int ch = 0; ch < 3; ++ch) bg[ch] = rand01(seed ^ kBgSalt[ch]);
            const float pxc = std::fmax(0.0f, std::fmin(ray.px, static_cast<float>(W) - 1.0f));
            const float pyc = std::fmax(0.0f, std::fmin(ray.py, static_cast<float>(H) - 1.0f));
            const int x0 = static_cast<int>(std::floor(pxc)), y0 = static_cast<int>(std::floor(pyc));
            const int x1 = std::min(x0 + 1, static_cast<int>(W) - 1), y1 = std::min(y0 + 1, static_cast<int>(H) - 1);
            const float tx = pxc - static_cast<float>(x0), ty = pyc - static_cast<float>(y0);
            const float inv255 = 1.0f / 255.0f;
            auto px = [&](int x, int y, int ch) { return static_cast<float>(img[(static_cast<uint64_t>(y) * W + x) * 4u + ch]) * inv255; };
            float v[4];
            for (int ch = 0; ch < 4; ++ch) {
                const float a = std::fmaf(px(x0, y0, ch), 1.0f - tx, px(x1, y0, ch) * tx);
                const float bb = std::fmaf(px(x0, y1, ch), 1.0f - tx, px(x1, y1, ch) * tx);
                v[ch] = std::fmaf(a, 1.0f - ty, bb * ty);
            }
            for (int ch = 0; ch < 3; ++ch) k_gt[4 * k + ch] = std::fmaf(v[ch], v[3], bg[ch] * (1.0f - v[3]));
            k_gt[4 * k + 3] = v[3];
            for (int ch = 0; ch < 3; ++ch) k_bg[3 * k + ch] = bg[ch];
            for (int ch = 0; ch < 3; ++ch) k_dir[3 * k + ch] = ray.d[ch];
        }
    });
    info.rays = n;
    info.active_rays = nk;
    info.samples = static_cast<uint32_t>(total);
}

// Field forward, composite + loss, field backward for the last batch.
void Ctx::forward_backward() {
    const uint64_t S = s_ray.size();
    const uint32_t nk = static_cast<uint32_t>(k_index.size());
    const uint32_t L = grid.n_levels;
    float W[kMlpParams];
    for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(p16[n_grid + i]);
    std::vector<uint16_t> feat(S * 2ull * L);
    std::vector<float> raw(4 * S), dt(S), dout(4 * S);
    parallel_for(S, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        for (uint64_t s = b; s < e; ++s) {
            float u[3];
            to_unit(&s_pos[4 * s], u);
            grid_forward_point(grid, p16.data(), u, &feat[s * 2ull * L]);
            MlpTrace t;
            mlp_forward_row(W, &feat[s * 2ull * L], &k_dir[3ull * s_ray[s]], &t, &raw[4 * s]);
            dt[s] = s_pos[4 * s + 3];
        }
    });
    active = nk;
    const uint32_t world = std::max(1u, opt.dp_world);
    const float inv_norm = nk == 0u ? 0.0f : 1.0f / (static_cast<float>(nk) * static_cast<float>(world));
    std::vector<float> ray_loss(nk, 0.0f);
    parallel_for(nk, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        for (uint64_t k = b; k < e; ++k) {
            const uint32_t s0 = k_begin[k];
            ray_loss[k] = composite_ray(&raw[4ull * s0], &dt[s0], k_count[k], &k_gt[4 * k], &k_bg[3 * k], inv_norm,
                                        cfg.hyper_params.loss_scale, opt.stop_transmittance, &dout[4ull * s0], nullptr, nullptr);
        }
    });
    double lsum = 0.0;
    for (float l : ray_loss) lsum += l;
    loss_sum = lsum * inv_norm;
    // Backward: MLP per sample (wgrad per thread), then the hash scatter split by level.
    std::vector<float> dfeat(S * 2ull * L);
    const uint32_t nt = std::max(1u, opt.n_threads);
    std::vector<std::vector<double>> gw(nt, std::vector<double>(kMlpParams, 0.0));
    parallel_for(S, nt, [&](uint64_t b, uint64_t e, uint32_t tid) {
        for (uint64_t s = b; s < e; ++s) {
            MlpTrace t;
            float out[4];
            mlp_forward_row(W, &feat[s * 2ull * L], &k_dir[3ull * s_ray[s]], &t, out);
            mlp_backward_row(W, t, &dout[4 * s], &dfeat[s * 2ull * L], gw[tid].data());
        }
    });
    std::vector<double> gg(n_grid, 0.0);
    parallel_for(L, nt, [&](uint64_t lb, uint64_t le, uint32_t) {
        for (uint64_t s = 0; s < S; ++s) {
            float u[3];
            to_unit(&s_pos[4 * s], u);
            for (uint64_t l = lb; l < le; ++l)
                grid_backward_point(grid, u, &dfeat[s * 2ull * L], gg.data(), static_cast<uint32_t>(l), L);
        }
    });
    for (uint64_t i = 0; i < n_grid; ++i) grad[i] = static_cast<float>(gg[i]);
    for (uint32_t i = 0; i < kMlpParams; ++i) {
        double a = 0.0;
        for (uint32_t t = 0; t < nt; ++t) a += gw[t][i];
        grad[n_grid + i] = static_cast<float>(a);
    }
}

// Statistics, update guard, clip, Adam, step commit (reference
// backend-cuda.cu:1451-1554 and the graph tail at :2360-2380).
void Ctx::apply_update() {
    double sumsq = 0.0;
    uint32_t nonfinite = 0;
    for (uint64_t i = 0; i < n_params; ++i) {
        const float g = grad[i];
        if (!std::isfinite(g)) {
            nonfinite = 1;
            continue;
        }
        sumsq += static_cast<double>(g) * g;
    }
    const float loss = static_cast<float>(loss_sum);
    const float grad_norm = std::sqrt(static_cast<float>(sumsq)) / cfg.hyper_params.loss_scale;
    const uint32_t has_nonfinite = (nonfinite || !std::isfinite(loss) || !std::isfinite(grad_norm)) ? 1u : 0u;
    const uint32_t opt_step = frame + 1u;
    stats.loss = loss;
    stats.grad_norm = grad_norm;
    stats.has_nonfinite = has_nonfinite;
    stats.completed_steps = frame + 1u;
    stats.last_train_camera = train_camera(frame, n_images);
    AdamScalars s;
    adam_scalars(grad_norm, has_nonfinite, opt_step, cfg.hyper_params, &s);
    parallel_for(n_params, opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        adam_range(master.data(), p16.data(), grad.data(), m.data(), v.data(), b, e, cfg.hyper_params.adam_beta1,
                   cfg.hyper_params.adam_beta2, cfg.hyper_params.adam_eps, s);
    });
    // Next step's ray count when a per-step sample target is set.
    // Data parallel: every rank sizes its next batch from the samples of all
    // ranks against the target of all ranks, so all ranks march the same count.
    if (opt.target_samples_per_step != 0u) {
        uint64_t samples = info.samples, target = opt.target_samples_per_step;
        if (opt.dp_world > 1u && global_samples != 0u) {
            samples = global_samples;
            target *= opt.dp_world;
        }
        uint64_t next = samples == 0u ? 2ull * n_rays : static_cast<uint64_t>(n_rays) * target / samples;
        next = std::max<uint64_t>(128u, std::min<uint64_t>(next, max_batch_rays));
        n_rays = static_cast<uint32_t>(next);
    }
    ++frame;
    grads_pending = false;
    global_samples = 0;
}

}  // namespace oracle

using namespace oracle;

extern "C" {

void* oracle_ctx_create(const NerfCreateDesc* desc, const OracleOptions* opt) {
    if (!desc || !opt) return nullptr;
    Ctx* c = new (std::nothrow) Ctx();
    if (!c) return nullptr;
    c->opt = *opt;
    if (c->opt.n_threads == 0u) c->opt.n_threads = 1u;
    if (c->opt.dp_world == 0u) c->opt.dp_world = 1u;
    if (grid_layout(opt->n_levels, opt->log2_hashmap_size, opt->base_resolution, opt->max_resolution, &c->grid) != 0) {
        delete c;
        return nullptr;
    }
    c->n_images = desc->image_count;
    c->W = desc->image_width;
    c->H = desc->image_height;
    c->fx = desc->fx;
    c->fy = desc->fy;
    c->cx = desc->cx;
    c->cy = desc->cy;
    c->images.assign(desc->images_rgba8, desc->images_rgba8 + desc->images_bytes);
    c->cams.assign(desc->cameras_4x4_packed, desc->cameras_4x4_packed + desc->cameras_bytes / sizeof(float));
    c->grid_res = desc->occupancy_grid_res;
    c->max_sample_steps = desc->max_sample_steps;
    c->max_batch_rays = desc->max_batch_rays;
    if (c->opt.n_cascades == 0u) c->opt.n_cascades = 1u;
    c->cell_count = c->grid_res * c->grid_res * c->grid_res * c->opt.n_cascades;
    c->density.assign(c->cell_count, 0.0f);
    c->bits.assign((c->cell_count + 31u) / 32u, 0u);
    c->init_params();
    return c;
}

void oracle_ctx_destroy(void* ctx) { delete static_cast<Ctx*>(ctx); }

int oracle_ctx_configure(void* ctx, const NerfTrainingConfig* cfg) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !cfg) return NERF_STATUS_INVALID_USAGE;
    if (cfg->rays_per_batch == 0u || cfg->max_sample_steps_per_ray == 0u) return NERF_STATUS_INVALID_USAGE;
    if (cfg->occupancy_params.update_interval == 0u || c->n_images == 0u) return NERF_STATUS_INVALID_USAGE;
    if (cfg->rays_per_batch > c->max_batch_rays) return NERF_STATUS_INVALID_USAGE;
    c->cfg = *cfg;
    c->mn[0] = cfg->aabb_min_x;
    c->mn[1] = cfg->aabb_min_y;
    c->mn[2] = cfg->aabb_min_z;
    c->mx[0] = cfg->aabb_max_x;
    c->mx[1] = cfg->aabb_max_y;
    c->mx[2] = cfg->aabb_max_z;
    c->box = make_box(c->mn, c->mx, c->opt.n_cascades);
    for (int k = 0; k < 3; ++k) {  // the marching box: the outermost cascade
        c->mn[k] = c->box.mn[k];
        c->mx[k] = c->box.mx[k];
        c->size[k] = c->box.size[k];
    }
    c->update_count = std::min(cfg->occupancy_params.cells_per_update, c->cell_count);
    const uint64_t want = c->opt.max_samples_per_step
                              ? c->opt.max_samples_per_step
                              : static_cast<uint64_t>(cfg->rays_per_batch) * cfg->max_sample_steps_per_ray;
    c->cap = static_cast<uint32_t>(std::min<uint64_t>(want, c->max_sample_steps));
    c->frame = 0;
    c->n_rays = cfg->rays_per_batch;
    std::fill(c->density.begin(), c->density.end(), 0.0f);
    std::fill(c->bits.begin(), c->bits.end(), 0u);
    std::fill(c->m.begin(), c->m.end(), 0.0f);
    std::fill(c->v.begin(), c->v.end(), 0.0f);
    std::fill(c->grad.begin(), c->grad.end(), 0.0f);
    c->stats = NerfTrainStats{};
    c->configured = true;
    return NERF_STATUS_OK;
}

int oracle_ctx_step_grads(void* ctx) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !c->configured) return NERF_STATUS_STATE_ERROR;
    const uint32_t camera = train_camera(c->frame, c->n_images);
    c->info.camera = camera;
    c->occupancy_step(occupancy_mode(c->frame, c->cfg.occupancy_params.warmup_steps, c->cfg.occupancy_params.update_interval));
    c->sample_batch(camera);
    c->forward_backward();
    c->grads_pending = true;
    return NERF_STATUS_OK;
}

int oracle_ctx_step_apply(void* ctx) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !c->grads_pending) return NERF_STATUS_STATE_ERROR;
    c->apply_update();
    return NERF_STATUS_OK;
}

int oracle_ctx_step(void* ctx) {
    const int s = oracle_ctx_step_grads(ctx);
    if (s != NERF_STATUS_OK) return s;
    return oracle_ctx_step_apply(ctx);
}

int oracle_ctx_stats(void* ctx, NerfTrainStats* out) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !out) return NERF_STATUS_INVALID_USAGE;
    *out = c->stats;
    return NERF_STATUS_OK;
}

int oracle_ctx_batch_info(void* ctx, OracleBatchInfo* out) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !out) return NERF_STATUS_INVALID_USAGE;
    *out = c->info;
    return NERF_STATUS_OK;
}

uint64_t oracle_ctx_param_count(void* ctx, uint64_t* n_grid, uint64_t* n_mlp) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (n_grid) *n_grid = c->n_grid;
    if (n_mlp) *n_mlp = kMlpParams;
    return c->n_params;
}

int oracle_ctx_get_params(void* ctx, float* master, uint16_t* p16, float* m, float* v, float* grad) {
    Ctx* c = static_cast<Ctx*>(ctx);
    const size_t n = c->n_params;
    if (master) std::memcpy(master, c->master.data(), n * 4);
    if (p16) std::memcpy(p16, c->p16.data(), n * 2);
    if (m) std::memcpy(m, c->m.data(), n * 4);
    if (v) std::memcpy(v, c->v.data(), n * 4);
    if (grad) std::memcpy(grad, c->grad.data(), n * 4);
    return NERF_STATUS_OK;
}

int oracle_ctx_set_params(void* ctx, const float* master) {
    Ctx* c = static_cast<Ctx*>(ctx);
    std::memcpy(c->master.data(), master, c->n_params * 4);
    for (uint64_t i = 0; i < c->n_params; ++i) c->p16[i] = f2h(c->master[i]);
    return NERF_STATUS_OK;
}

int oracle_ctx_set_grads(void* ctx, const float* grad, float loss_sum, uint32_t active_rays) {
    Ctx* c = static_cast<Ctx*>(ctx);
    std::memcpy(c->grad.data(), grad, c->n_params * 4);
    c->loss_sum = loss_sum;
    c->active = active_rays;
    return NERF_STATUS_OK;
}

int oracle_ctx_set_global_samples(void* ctx, uint64_t samples) {
    static_cast<Ctx*>(ctx)->global_samples = samples;
    return NERF_STATUS_OK;
}

void oracle_occupancy_cells(uint32_t frame, uint32_t update_count, uint32_t cell_count, uint32_t grid_res, const float* mn,
                            const float* mx, float* out_xyz) {
    const Box b = make_box(mn, mx, 1u);
    for (uint32_t k = 0; k < update_count; ++k) occupancy_cell_center(frame, k, update_count, cell_count, grid_res, b, out_xyz + 3ull * k);
}

int oracle_ctx_get_loss(void* ctx, float* loss_sum, uint32_t* active_rays) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (loss_sum) *loss_sum = static_cast<float>(c->loss_sum);
    if (active_rays) *active_rays = c->active;
    return NERF_STATUS_OK;
}

int oracle_ctx_get_occupancy(void* ctx, float* density, uint32_t* bitfield) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (density) std::memcpy(density, c->density.data(), c->density.size() * 4);
    if (bitfield) std::memcpy(bitfield, c->bits.data(), c->bits.size() * 4);
    return NERF_STATUS_OK;
}

int oracle_ctx_set_occupancy(void* ctx, const float* density, const uint32_t* bitfield) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (density) std::memcpy(c->density.data(), density, c->density.size() * 4);
    if (bitfield) std::memcpy(c->bits.data(), bitfield, c->bits.size() * 4);
    return NERF_STATUS_OK;
}

void oracle_occupancy_update(float* density, uint32_t* bits, const float* sigma, uint32_t cell_count,
                             uint32_t update_count, uint32_t frame, uint32_t mode, float decay, float threshold) {
    occupancy_apply(density, bits, sigma, cell_count, update_count, frame, mode, decay, threshold);
}

int oracle_ctx_set_frame(void* ctx, uint32_t frame_index) {
    static_cast<Ctx*>(ctx)->frame = frame_index;
    return NERF_STATUS_OK;
}

int oracle_ctx_get_batch(void* ctx, uint32_t* ray_counts, uint32_t* ray_index, uint32_t* ray_begin, uint32_t* ray_count,
                         float* ray_gt, float* ray_bg, float* ray_dir, float* sample_pos_dt) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (ray_counts) std::memcpy(ray_counts, c->ray_counts.data(), c->ray_counts.size() * 4);
    if (ray_index) std::memcpy(ray_index, c->k_index.data(), c->k_index.size() * 4);
    if (ray_begin) std::memcpy(ray_begin, c->k_begin.data(), c->k_begin.size() * 4);
    if (ray_count) std::memcpy(ray_count, c->k_count.data(), c->k_count.size() * 4);
    if (ray_gt) std::memcpy(ray_gt, c->k_gt.data(), c->k_gt.size() * 4);
    if (ray_bg) std::memcpy(ray_bg, c->k_bg.data(), c->k_bg.size() * 4);
    if (ray_dir) std::memcpy(ray_dir, c->k_dir.data(), c->k_dir.size() * 4);
    if (sample_pos_dt) std::memcpy(sample_pos_dt, c->s_pos.data(), c->s_pos.size() * 4);
    return NERF_STATUS_OK;
}

// Rendering: pixel-centre rays, the training march (dt_min = range/max_steps,
// cone-angle growth, occupied cells only), front-to-back compositing on white
// with early termination, RGBA8 by round-to-nearest of clamp(c)*255
// (reference backend-cuda.cu:534-635 for ray set-up and pixel packing).
int oracle_ctx_render(void* ctx, const float* c2w12, uint32_t width, uint32_t height, float fx, float fy, float cx, float cy,
                      uint32_t max_steps, float stop_T, uint32_t* rgba, uint32_t* spp, uint32_t pixel_begin,
                      uint32_t pixel_end) {
    Ctx* c = static_cast<Ctx*>(ctx);
    if (!c || !c2w12 || !rgba || max_steps == 0u) return NERF_STATUS_INVALID_USAGE;
    float cam[16];
    std::memcpy(cam, c2w12, 12 * sizeof(float));
    cam[12] = cam[13] = cam[14] = 0.0f;
    cam[15] = 1.0f;
    float W[kMlpParams];
    for (uint32_t i = 0; i < kMlpParams; ++i) W[i] = h2f(c->p16[c->n_grid + i]);
    const float cone = cone_angle(fx, fy);
    const uint32_t total = width * height;
    pixel_end = std::min(pixel_end, total);
    parallel_for(pixel_end > pixel_begin ? pixel_end - pixel_begin : 0u, c->opt.n_threads, [&](uint64_t b, uint64_t e, uint32_t) {
        for (uint64_t q = b; q < e; ++q) {
            const uint32_t pix = pixel_begin + static_cast<uint32_t>(q);
            const uint32_t x = pix % width, y = pix / width;
            Ray ray{};
            ray.px = static_cast<float>(x) + 0.5f;
            ray.py = static_cast<float>(y) + 0.5f;
            const float pyf = static_cast<float>(height) - 1.0f - ray.py;
            for (int k = 0; k < 3; ++k) ray.o[k] = cam[4 * k + 3];
            float T = 1.0f, acc[3] = {0.0f, 0.0f, 0.0f};
            uint32_t n = 0;
            const bool hit = ray_dir(cam, fx, fy, cx, cy, ray.px, pyf, ray.d) &&
                             intersect_aabb(ray.o, ray.d, c->mn, c->mx, &ray.tn, &ray.tf) && (ray.tf - ray.tn > 0.0f);
            if (hit) {
                bool stopped = false;
                march(ray, max_steps, cone, c->box, c->grid_res, c->bits.data(),
                      [&](uint32_t, float, float dt, const float* p) {
                          if (stopped) return;
                          if (stop_T > 0.0f && T < stop_T) {
                              stopped = true;
                              return;
                          }
                          float u[3];
                          c->to_unit(p, u);
                          uint16_t feat[64];
                          grid_forward_point(c->grid, c->p16.data(), u, feat);
                          MlpTrace t;
                          float out[4];
                          mlp_forward_row(W, feat, ray.d, &t, out);
                          const float a = 1.0f - std::exp(-(density_activation(out[0]) * std::max(0.0f, dt)));
                          const float w = T * a;
                          for (int ch = 0; ch < 3; ++ch) acc[ch] += w * sigmoid(out[1 + ch]);
                          T *= 1.0f - a;
                          ++n;
                      });
            }
            uint32_t px8[3];
            for (int ch = 0; ch < 3; ++ch) {
                const float v = std::fmin(1.0f, std::fmax(0.0f, acc[ch] + T));
                px8[ch] = static_cast<uint32_t>(std::nearbyint(v * 255.0f));
            }
            rgba[pix] = (255u << 24) | (px8[2] << 16) | (px8[1] << 8) | px8[0];
            if (spp) spp[pix] = n;
        }
    });
    return NERF_STATUS_OK;
}

}  // extern "C"
