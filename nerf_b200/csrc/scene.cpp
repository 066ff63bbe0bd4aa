// scene.cpp -- procedural scenes and their ground-truth renders.
//
// The reference trains on the Blender nerf_synthetic scenes, which are not
// available here; its benchmark configurations are stood in for by seeded
// analytic scenes rendered on the host:
//   kind 0: spheres of constant density and colour (smoke configuration)
//   kind 1: spheres and axis-aligned boxes of constant density whose albedo
//           is 3-octave value noise (bounded training configuration)
//   kind 2: an unbounded-style scene: spheres and boxes standing on a ground
//           slab, inside a sky shell (radii 12 to 12.5), all with
//           value-noise albedo (large-scene configuration; the shell's density
//           is constant, so the renders stay exact)
// Density is piecewise constant along a ray, so the renderer integrates it
// exactly: the ray is cut at every primitive boundary, each segment has
// opacity 1 - exp(-sigma * length) and colour (kind 0) the density-weighted
// primitive colour or (kind 1) the albedo at the centre of the segment's
// first optical depth.  Images are RGBA8 with alpha = 1 - transmittance and
// colour un-premultiplied (the nerf_synthetic convention).  Texel (x, y) is
// rendered along the camera ray at continuous pixel (x, y), the position the
// training sampler assigns to that texel.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/nerf_b200.h"

// The exported name.  The CPU oracle's library compiles this same file under
// another name (oracle_scene_render), so that a process which must not load
// libnerf_b200.so -- the benchmark's reference arm -- renders the identical
// datasets.
#ifndef NB_SCENE_ENTRY
#define NB_SCENE_ENTRY nerf_b200_scene_render
#endif

namespace {

uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) : s(mix64(seed)) {}
    double uniform() {
        s = mix64(s);
        return static_cast<double>(s >> 11) * (1.0 / 9007199254740992.0);
    }
    double range(double a, double b) { return a + (b - a) * uniform(); }
};

struct Prim {
    int box;           // 0 sphere, 1 box, 2 spherical shell (r to r2)
    double c[3];
    double r;          // sphere radius, box half-size (all axes unless hs is set), shell inner radius
    double rgb[3];
    double hs[3] = {0, 0, 0};  // box half-sizes per axis (when non-zero)
    double r2 = 0.0;           // shell outer radius
};

struct Scene {
    int kind;
    uint32_t seed;
    double density;
    std::vector<Prim> prims;
};

double value_lattice(uint32_t seed, int x, int y, int z, int ch) {
    uint64_t h = mix64((static_cast<uint64_t>(seed) << 32) ^ (static_cast<uint64_t>(static_cast<uint32_t>(x)) * 73856093ull) ^
                       (static_cast<uint64_t>(static_cast<uint32_t>(y)) * 19349663ull) ^
                       (static_cast<uint64_t>(static_cast<uint32_t>(z)) * 83492791ull) ^ (static_cast<uint64_t>(ch) << 60));
    return static_cast<double>(h >> 11) * (1.0 / 9007199254740992.0);
}
double smooth(double t) { return t * t * (3.0 - 2.0 * t); }
double value_noise(uint32_t seed, const double p[3], int ch) {
    const int ix = static_cast<int>(std::floor(p[0])), iy = static_cast<int>(std::floor(p[1])), iz = static_cast<int>(std::floor(p[2]));
    const double fx = smooth(p[0] - ix), fy = smooth(p[1] - iy), fz = smooth(p[2] - iz);
    double acc = 0.0;
    for (int c = 0; c < 8; ++c) {
        const int dx = c & 1, dy = (c >> 1) & 1, dz = (c >> 2) & 1;
        const double w = (dx ? fx : 1 - fx) * (dy ? fy : 1 - fy) * (dz ? fz : 1 - fz);
        acc += w * value_lattice(seed, ix + dx, iy + dy, iz + dz, ch);
    }
    return acc;
}
// 3 octaves at base frequency 2 per unit, persistence 0.5; albedo in [0.1, 0.95].
void albedo(uint32_t seed, const double p[3], double out[3]) {
    for (int ch = 0; ch < 3; ++ch) {
        double v = 0.0, amp = 1.0, norm = 0.0, f = 2.0;
        for (int o = 0; o < 3; ++o) {
            const double q[3] = {p[0] * f, p[1] * f, p[2] * f};
            v += amp * value_noise(seed + 101u * o, q, ch);
            norm += amp;
            amp *= 0.5;
            f *= 2.0;
        }
        out[ch] = 0.1 + 0.85 * (v / norm);
    }
}

bool ray_sphere(const double c[3], double r, const double o[3], const double d[3], double& t0, double& t1) {
    double oc[3] = {o[0] - c[0], o[1] - c[1], o[2] - c[2]};
    const double b = oc[0] * d[0] + oc[1] * d[1] + oc[2] * d[2];
    const double cc = oc[0] * oc[0] + oc[1] * oc[1] + oc[2] * oc[2] - r * r;
    const double disc = b * b - cc;
    if (disc <= 0.0) return false;
    const double s = std::sqrt(disc);
    t0 = -b - s;
    t1 = -b + s;
    return true;
}

bool ray_prim(const Prim& pr, const double o[3], const double d[3], double& t0, double& t1) {
    if (pr.box == 2) {  // shell seen from inside its inner sphere: from the inner exit to the outer exit
        double a0, a1, b0, b1;
        if (!ray_sphere(pr.c, pr.r, o, d, a0, a1) || !ray_sphere(pr.c, pr.r2, o, d, b0, b1)) return false;
        t0 = std::max(a1, 0.0);
        t1 = b1;
        return t1 > t0;
    }
    if (!pr.box) {
        double oc[3] = {o[0] - pr.c[0], o[1] - pr.c[1], o[2] - pr.c[2]};
        const double b = oc[0] * d[0] + oc[1] * d[1] + oc[2] * d[2];
        const double cc = oc[0] * oc[0] + oc[1] * oc[1] + oc[2] * oc[2] - pr.r * pr.r;
        const double disc = b * b - cc;
        if (disc <= 0.0) return false;
        const double s = std::sqrt(disc);
        t0 = -b - s;
        t1 = -b + s;
    } else {
        t0 = -1e30;
        t1 = 1e30;
        for (int k = 0; k < 3; ++k) {
            const double h = pr.hs[k] > 0.0 ? pr.hs[k] : pr.r;
            const double lo = pr.c[k] - h, hi = pr.c[k] + h;
            if (std::fabs(d[k]) < 1e-12) {
                if (o[k] < lo || o[k] > hi) return false;
                continue;
            }
            double a = (lo - o[k]) / d[k], b = (hi - o[k]) / d[k];
            if (a > b) std::swap(a, b);
            t0 = std::max(t0, a);
            t1 = std::min(t1, b);
        }
        if (t0 >= t1) return false;
    }
    t0 = std::max(t0, 0.0);
    return t1 > t0;
}

// Exact integration of the piecewise-constant density along a ray.
void render_ray(const Scene& sc, const double o[3], const double d[3], double rgb[3], double& alpha) {
    struct Ev {
        double t;
        int prim, enter;
    };
    Ev evs[256];
    int ne = 0;
    for (size_t i = 0; i < sc.prims.size() && ne + 2 <= 256; ++i) {
        double t0, t1;
        if (!ray_prim(sc.prims[i], o, d, t0, t1)) continue;
        evs[ne++] = {t0, static_cast<int>(i), 1};
        evs[ne++] = {t1, static_cast<int>(i), 0};
    }
    std::sort(evs, evs + ne, [](const Ev& a, const Ev& b) { return a.t < b.t; });
    double T = 1.0, acc[3] = {0, 0, 0};
    int inside[64] = {};
    int n_in = 0;
    for (int e = 0; e + 1 < ne; ++e) {
        if (evs[e].enter) {
            ++n_in;
            inside[evs[e].prim & 63]++;
        } else {
            --n_in;
            inside[evs[e].prim & 63]--;
        }
        const double ta = evs[e].t, tb = evs[e + 1].t;
        if (n_in <= 0 || tb <= ta) continue;
        const double sigma = sc.density * n_in;
        const double a = 1.0 - std::exp(-sigma * (tb - ta));
        double c[3] = {0, 0, 0};
        if (sc.kind == 0) {
            for (size_t i = 0; i < sc.prims.size(); ++i)
                if (inside[i & 63] > 0)
                    for (int k = 0; k < 3; ++k) c[k] += sc.prims[i].rgb[k] / n_in;
        } else {
            const double tm = ta + 0.5 * std::min(tb - ta, 1.0 / sigma);
            const double p[3] = {o[0] + tm * d[0], o[1] + tm * d[1], o[2] + tm * d[2]};
            albedo(sc.seed, p, c);
        }
        for (int k = 0; k < 3; ++k) acc[k] += T * a * c[k];
        T *= 1.0 - a;
        if (T < 1e-6) break;
    }
    alpha = 1.0 - T;
    for (int k = 0; k < 3; ++k) rgb[k] = alpha > 1e-9 ? acc[k] / alpha : 0.0;
}

Scene make_scene(const NerfB200SceneDesc& s) {
    Scene sc;
    sc.kind = static_cast<int>(s.kind);
    sc.seed = s.seed;
    sc.density = s.density;
    Rng rng(0x5eed0000ull + s.seed);
    if (s.kind == 2u) {
        // Ground slab z in [-0.1, 0] over [-12, 12]^2, primitives standing on it
        // with centres uniform in [-extent, extent]^2, the sky shell around all.
        Prim ground{};
        ground.box = 1;
        ground.c[0] = ground.c[1] = 0.0;
        ground.c[2] = -0.05;
        ground.hs[0] = ground.hs[1] = 12.0;
        ground.hs[2] = 0.05;
        sc.prims.push_back(ground);
        const uint32_t n = std::min<uint32_t>(s.n_primitives, 60u);
        for (uint32_t i = 0; i < n; ++i) {
            Prim p{};
            p.box = static_cast<int>(i & 1u);
            const double size = rng.range(s.size_min, s.size_max);
            p.r = p.box ? 0.5 * size : size;
            p.c[0] = rng.range(-s.extent, s.extent);
            p.c[1] = rng.range(-s.extent, s.extent);
            p.c[2] = p.r;
            sc.prims.push_back(p);
        }
        Prim sky{};
        sky.box = 2;
        sky.r = 12.0;
        sky.r2 = 12.5;
        sc.prims.push_back(sky);
        return sc;
    }
    const uint32_t n = std::min<uint32_t>(s.n_primitives, 64u);
    for (uint32_t i = 0; i < n; ++i) {
        Prim p{};
        p.box = (s.kind == 1 && (i & 1u)) ? 1 : 0;
        for (int k = 0; k < 3; ++k) p.c[k] = rng.range(-s.extent, s.extent);
        const double size = rng.range(s.size_min, s.size_max);
        p.r = p.box ? 0.5 * size : size;
        for (int k = 0; k < 3; ++k) p.rgb[k] = rng.uniform();
        sc.prims.push_back(p);
    }
    return sc;
}

void look_at(const double eye[3], float* m) {
    double f[3] = {-eye[0], -eye[1], -eye[2]};
    double n = std::sqrt(f[0] * f[0] + f[1] * f[1] + f[2] * f[2]);
    for (double& x : f) x /= n;
    const double z[3] = {-f[0], -f[1], -f[2]};
    double up[3] = {0, 0, 1};
    if (std::fabs(z[2]) > 0.999) up[0] = 1, up[2] = 0;
    double x[3] = {up[1] * z[2] - up[2] * z[1], up[2] * z[0] - up[0] * z[2], up[0] * z[1] - up[1] * z[0]};
    n = std::sqrt(x[0] * x[0] + x[1] * x[1] + x[2] * x[2]);
    for (double& v : x) v /= n;
    const double y[3] = {z[1] * x[2] - z[2] * x[1], z[2] * x[0] - z[0] * x[2], z[0] * x[1] - z[1] * x[0]};
    for (int r = 0; r < 3; ++r) {
        m[4 * r + 0] = static_cast<float>(x[r]);
        m[4 * r + 1] = static_cast<float>(y[r]);
        m[4 * r + 2] = static_cast<float>(z[r]);
        m[4 * r + 3] = static_cast<float>(eye[r]);
    }
    m[12] = m[13] = m[14] = 0.0f;
    m[15] = 1.0f;
}

// Camera of mode 3: on a ring of the given radius at height orbit_elevation
// (a length here), looking outward (even views) or inward (odd views) along
// the horizontal; returns false for the other modes.
bool ring_camera(const NerfB200SceneDesc& s, uint32_t view, float* m) {
    if (s.camera_mode != 3u) return false;
    const double az = 2.0 * M_PI * view / std::max<uint32_t>(1u, s.orbit_views);
    const double eye[3] = {s.radius * std::cos(az), s.radius * std::sin(az), s.orbit_elevation};
    const double sign = (view & 1u) ? -1.0 : 1.0;
    const double fwd[3] = {sign * std::cos(az), sign * std::sin(az), 0.0};
    const double z[3] = {-fwd[0], -fwd[1], -fwd[2]};  // camera looks down -z
    const double up[3] = {0, 0, 1};
    double x[3] = {up[1] * z[2] - up[2] * z[1], up[2] * z[0] - up[0] * z[2], up[0] * z[1] - up[1] * z[0]};
    const double n = std::sqrt(x[0] * x[0] + x[1] * x[1] + x[2] * x[2]);
    for (double& v : x) v /= n;
    const double y[3] = {z[1] * x[2] - z[2] * x[1], z[2] * x[0] - z[0] * x[2], z[0] * x[1] - z[1] * x[0]};
    for (int r = 0; r < 3; ++r) {
        m[4 * r + 0] = static_cast<float>(x[r]);
        m[4 * r + 1] = static_cast<float>(y[r]);
        m[4 * r + 2] = static_cast<float>(z[r]);
        m[4 * r + 3] = static_cast<float>(eye[r]);
    }
    m[12] = m[13] = m[14] = 0.0f;
    m[15] = 1.0f;
    return true;
}

void camera_eye(const NerfB200SceneDesc& s, uint32_t view, double eye[3]) {
    Rng rng((static_cast<uint64_t>(s.seed) << 20) ^ (0xCA3E00ull + view));
    double dir[3];
    if (s.camera_mode == 2u) {  // circular orbit at fixed elevation
        const double az = 2.0 * M_PI * view / std::max<uint32_t>(1u, s.orbit_views);
        const double el = s.orbit_elevation;
        dir[0] = std::cos(el) * std::cos(az);
        dir[1] = std::cos(el) * std::sin(az);
        dir[2] = std::sin(el);
    } else {
        for (;;) {
            for (double& x : dir) x = rng.range(-1.0, 1.0);
            const double n2 = dir[0] * dir[0] + dir[1] * dir[1] + dir[2] * dir[2];
            if (n2 < 1e-4 || n2 > 1.0) continue;
            const double n = std::sqrt(n2);
            for (double& x : dir) x /= n;
            if (s.camera_mode == 1u && dir[2] < 0.05) continue;  // upper hemisphere
            break;
        }
    }
    for (int k = 0; k < 3; ++k) eye[k] = s.radius * dir[k];
}

}  // namespace

extern "C" {

NERF_API NerfStatus NB_SCENE_ENTRY(const NerfB200SceneDesc* s, uint8_t* images, float* cams, float* intrinsics) {
    if (!s || !cams || !intrinsics || s->width == 0u || s->height == 0u || !(s->fov > 0.0f)) return NERF_STATUS_INVALID_USAGE;
    const Scene sc = make_scene(*s);
    const uint32_t W = s->width, H = s->height;
    const double fx = 0.5 * W / std::tan(0.5 * s->fov);
    const double cxp = 0.5 * (W - 1.0), cyp = 0.5 * (H - 1.0);
    intrinsics[0] = static_cast<float>(fx);
    intrinsics[1] = static_cast<float>(fx);
    intrinsics[2] = static_cast<float>(cxp);
    intrinsics[3] = static_cast<float>(cyp);
    for (uint32_t v = 0; v < s->n_views; ++v) {
        if (ring_camera(*s, s->view_offset + v, cams + 16ull * v)) continue;
        double eye[3];
        camera_eye(*s, s->view_offset + v, eye);
        look_at(eye, cams + 16ull * v);
    }
    if (!images) return NERF_STATUS_OK;
    const uint64_t total = static_cast<uint64_t>(s->n_views) * H;
    uint32_t nt = s->n_threads ? s->n_threads : std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> pool;
    for (uint32_t t = 0; t < nt; ++t) {
        pool.emplace_back([&, t] {
            for (uint64_t row = t; row < total; row += nt) {
                const uint32_t v = static_cast<uint32_t>(row / H), y = static_cast<uint32_t>(row % H);
                const float* m = cams + 16ull * v;
                for (uint32_t x = 0; x < W; ++x) {
                    const double dc[3] = {(x - cxp) / fx, ((H - 1.0 - y) - cyp) / fx, -1.0};
                    double d[3];
                    for (int k = 0; k < 3; ++k) d[k] = m[4 * k] * dc[0] + m[4 * k + 1] * dc[1] + m[4 * k + 2] * dc[2];
                    const double n = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
                    for (double& q : d) q /= n;
                    const double o[3] = {m[3], m[7], m[11]};
                    double rgb[3], a;
                    render_ray(sc, o, d, rgb, a);
                    uint8_t* px = images + ((static_cast<uint64_t>(v) * H + y) * W + x) * 4u;
                    for (int k = 0; k < 3; ++k) px[k] = static_cast<uint8_t>(std::lround(std::min(1.0, std::max(0.0, rgb[k])) * 255.0));
                    px[3] = static_cast<uint8_t>(std::lround(std::min(1.0, std::max(0.0, a)) * 255.0));
                }
            }
        });
    }
    for (auto& th : pool) th.join();
    return NERF_STATUS_OK;
}

}  // extern "C"
