// ray.cuh -- pinhole rays, AABB chords, the cone-angle step and the
// occupancy-bitfield lookup shared by the training sampler and the renderer.
// Every operation has an explicit rounding intrinsic so the CPU oracle
// reproduces the step sequence, and therefore the set of kept samples,
// bit for bit.
#pragma once
#include "common.cuh"

namespace nb {

struct Ray {
    float o[3], d[3];
    float tn, tf;
};

// Marching box and occupancy cascades.  mn / mx / size: the box rays are
// clipped to and positions are normalised in -- the outermost cascade.
// Cascade k (k < cascades) covers centre +- half * 2^k; cascade 0 is the
// configured AABB (bmn, bsize), and with one cascade the marching box is that
// AABB itself.
struct AabbConsts {
    float mn[3], mx[3], size[3];
    float bmn[3], bsize[3], c[3], h[3];
    uint32_t cascades;
};

// 2^k as a float (exact, k < 127).
NB_DEV float pow2f(uint32_t k) { return __int_as_float(static_cast<int>((127u + k) << 23)); }

NB_DEV AabbConsts make_box(const float mn[3], const float mx[3], const float size[3], const CascadeBox& cb) {
    AabbConsts b;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        b.mn[k] = mn[k];
        b.mx[k] = mx[k];
        b.size[k] = size[k];
        b.bmn[k] = cb.bmn[k];
        b.bsize[k] = cb.bsize[k];
        b.c[k] = cb.c[k];
        b.h[k] = cb.h[k];
    }
    b.cascades = cb.cascades;
    return b;
}

// Cascade of a point: 0 inside the configured AABB, else ceil(log2(m)) for
// m = max_k |p_k - centre_k| / half_k (m = f 2^e with f in [0.5, 1): e, or
// e - 1 when m is a power of two); cascades or more when outside them all.
NB_DEV uint32_t cascade_of(const AabbConsts& b, const float p[3]) {
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 3; ++k) m = fmaxf(m, __fdiv_rn(fabsf(__fsub_rn(p[k], b.c[k])), b.h[k]));
    if (!(m > 1.0f)) return 0u;
    int e = 0;
    const float f = frexpf(m, &e);
    return static_cast<uint32_t>(f == 0.5f ? e - 1 : e);
}

// Camera ray through continuous pixel (px, py); py is measured from the top
// row and flipped to H-1-py (reference backend-cuda.cu:373-390, 438-441).
// cam: rows 0..2 of a row-major 4x4 camera-to-world matrix.  The direction is
// normalised with a correctly rounded 1/sqrt.  Sums of products a*b + c*d
// (+ e*f) are evaluated as fma(e, f, fma(a, b, c*d)), the contraction the
// reference's compiler applies to the same expressions.
NB_DEV bool camera_ray(const float* cam, float fx, float fy, float cx, float cy, float height, float px, float py, Ray& r) {
    const float pyf = __fsub_rn(__fsub_rn(height, 1.0f), py);
    r.o[0] = cam[3];
    r.o[1] = cam[7];
    r.o[2] = cam[11];
    const float dcx = __fdiv_rn(__fsub_rn(px, cx), fx);
    const float dcy = __fdiv_rn(__fsub_rn(pyf, cy), fy);
#pragma unroll
    for (int k = 0; k < 3; ++k)
        r.d[k] = __fmaf_rn(cam[4 * k + 2], -1.0f, __fmaf_rn(cam[4 * k + 0], dcx, __fmul_rn(cam[4 * k + 1], dcy)));
    const float len2 = __fmaf_rn(r.d[2], r.d[2], __fmaf_rn(r.d[0], r.d[0], __fmul_rn(r.d[1], r.d[1])));
    if (len2 <= 1e-16f) return false;
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(len2));
#pragma unroll
    for (int k = 0; k < 3; ++k) r.d[k] = __fmul_rn(r.d[k], inv);
    return true;
}

// Slab test clamped to t >= 0 (reference backend-cuda.cu:391-408); also
// requires a non-empty chord.
NB_DEV bool clip_aabb(const AabbConsts& b, Ray& r) {
    float tmin[3], tmax[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float inv_d = fabsf(r.d[k]) > 1e-8f ? __fdiv_rn(1.0f, r.d[k]) : (r.d[k] >= 0.0f ? 1e8f : -1e8f);
        const float t0 = __fmul_rn(__fsub_rn(b.mn[k], r.o[k]), inv_d);
        const float t1 = __fmul_rn(__fsub_rn(b.mx[k], r.o[k]), inv_d);
        tmin[k] = fminf(t0, t1);
        tmax[k] = fmaxf(t0, t1);
    }
    float tn = fmaxf(fmaxf(tmin[0], tmin[1]), tmin[2]);
    const float tf = fminf(fminf(tmax[0], tmax[1]), tmax[2]);
    if (!(tn <= tf && tf > 0.0f)) return false;
    if (tn < 0.0f) tn = 0.0f;
    r.tn = tn;
    r.tf = tf;
    return __fsub_rn(tf, tn) > 0.0f;
}

// Index of the occupancy cell holding p (reference backend-cuda.cu:338-351)
// in the bitfield (the R^3 grids of the cascades, one after another), or
// kNoCell when p lies outside every cascade.
constexpr uint32_t kNoCell = 0xFFFFFFFFu;
NB_DEV uint32_t occupancy_cell(uint32_t R, const AabbConsts& b, const float p[3]) {
    float rel[3];
    uint32_t mip = 0u;
    if (b.cascades <= 1u) {
#pragma unroll
        for (int k = 0; k < 3; ++k) rel[k] = __fdiv_rn(__fsub_rn(p[k], b.mn[k]), b.size[k]);
    } else {
        mip = cascade_of(b, p);
        if (mip >= b.cascades) return kNoCell;
        const float s = pow2f(mip);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float lo = mip == 0u ? b.bmn[k] : __fsub_rn(b.c[k], __fmul_rn(b.h[k], s));
            rel[k] = __fdiv_rn(__fsub_rn(p[k], lo), __fmul_rn(b.bsize[k], s));
        }
    }
    if (rel[0] < 0.0f || rel[0] >= 1.0f || rel[1] < 0.0f || rel[1] >= 1.0f || rel[2] < 0.0f || rel[2] >= 1.0f) return kNoCell;
    const float Rf = static_cast<float>(R);
    const uint32_t ix = min(R - 1u, static_cast<uint32_t>(__fmul_rn(rel[0], Rf)));
    const uint32_t iy = min(R - 1u, static_cast<uint32_t>(__fmul_rn(rel[1], Rf)));
    const uint32_t iz = min(R - 1u, static_cast<uint32_t>(__fmul_rn(rel[2], Rf)));
    return mip * R * R * R + ix + iy * R + iz * R * R;
}

NB_DEV bool cell_bit(const uint32_t* __restrict__ bits, uint32_t cell) {
    return cell != kNoCell && ((__ldg(bits + (cell >> 5)) >> (cell & 31u)) & 1u) != 0u;
}

// Occupancy bit of the cell holding p.
NB_DEV bool occupied(const uint32_t* __restrict__ bits, uint32_t R, const AabbConsts& b, const float p[3]) {
    return cell_bit(bits, occupancy_cell(R, b, p));
}

// One step of the cone-angle march (reference backend-cuda.cu:455-468):
// dt = min(max(dt_min, t*cone), t_far - t), midpoint t + dt/2.
NB_DEV float march_dt(float t, float tf, float dt_min, float cone) {
    return fminf(fmaxf(dt_min, __fmul_rn(t, cone)), __fsub_rn(tf, t));
}
NB_DEV float march_mid(float t, float dt) { return __fadd_rn(t, __fmul_rn(0.5f, dt)); }
NB_DEV void ray_point(const Ray& r, float t, float p[3]) {
#pragma unroll
    for (int k = 0; k < 3; ++k) p[k] = __fmaf_rn(t, r.d[k], r.o[k]);
}
NB_DEV float cone_angle(float fx, float fy) {
    const float ix = fx > 0.0f ? __fdiv_rn(1.0f, fx) : 0.0f;
    const float iy = fy > 0.0f ? __fdiv_rn(1.0f, fy) : 0.0f;
    return __fmul_rn(0.5f, __fadd_rn(ix, iy));
}

}  // namespace nb
