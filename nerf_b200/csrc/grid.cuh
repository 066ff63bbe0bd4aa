// grid.cuh -- multiresolution hash-grid corner math, gather and scatter.
//
// Level l has scale s_l, R_l vertices per axis, and a dense or hashed table
// starting at entry offset_l (see grid_layout() in context.cu).  A unit-cube
// point p maps to u = fma(clamp01(p), s_l, 0.5) per axis, the cell corner
// i = clamp(floor(u), 0, R_l - 2) and the fraction f = u - floor(u).  Corner c
// (bit 0 = x, bit 1 = y, bit 2 = z) has weight ((wx*wy)*wz), w = f or 1-f,
// and entry x + R(y + Rz) on dense levels or
// (x ^ y*2654435761 ^ z*805459861) & (T-1) on hashed levels.  Each entry holds
// two fp16 features; the forward value is fma-accumulated over c = 0..7 from
// zero and rounded once to fp16.  Every operation is written with an explicit
// rounding intrinsic so that the CPU oracle reproduces indices, weights and
// forward features bit for bit.
#pragma once
#include "common.cuh"

namespace nb {

struct alignas(16) LevelParams {
    float scale;
    uint32_t res;
    uint32_t dense;
    uint32_t offset;
};

NB_DEV float clamp01(float x) { return fminf(1.0f, fmaxf(0.0f, x)); }

// Cell corner i and fractions f of p on one level.
NB_DEV void level_cell(const float p[3], const LevelParams lp, uint32_t i[3], float f[3]) {
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        const float u = __fmaf_rn(clamp01(p[d]), lp.scale, 0.5f);
        const float fl = floorf(u);
        f[d] = __fsub_rn(u, fl);
        int ii = static_cast<int>(fl);
        ii = max(0, min(static_cast<int>(lp.res) - 2, ii));
        i[d] = static_cast<uint32_t>(ii);
    }
}
// Table entries of all 8 corners of cell i.  The dense / hashed choice is
// one branch (uniform across a warp when the warp works on one level), and
// the per-axis terms are shared between corners: (y+1)*p = y*p + p mod 2^32.
NB_DEV void corner_entries(const uint32_t i[3], const LevelParams lp, uint32_t hash_mask, uint32_t idx[8]) {
    if (lp.dense) {
        const uint32_t R = lp.res, RR = R * R;
        const uint32_t b = lp.offset + i[0] + R * (i[1] + R * i[2]);
        idx[0] = b;
        idx[1] = b + 1u;
        idx[2] = b + R;
        idx[3] = b + R + 1u;
        idx[4] = b + RR;
        idx[5] = b + RR + 1u;
        idx[6] = b + RR + R;
        idx[7] = b + RR + R + 1u;
    } else {
        const uint32_t x0 = i[0], x1 = i[0] + 1u;
        const uint32_t y0 = i[1] * 2654435761u, y1 = y0 + 2654435761u;
        const uint32_t z0 = i[2] * 805459861u, z1 = z0 + 805459861u;
        const uint32_t yz[4] = {y0 ^ z0, y1 ^ z0, y0 ^ z1, y1 ^ z1};
#pragma unroll
        for (uint32_t k = 0; k < 4u; ++k) {
            idx[2 * k] = lp.offset + ((x0 ^ yz[k]) & hash_mask);
            idx[2 * k + 1] = lp.offset + ((x1 ^ yz[k]) & hash_mask);
        }
    }
}
// Trilinear weight of corner c, ((wx*wy)*wz) with the x-y products shared.
NB_DEV void corner_weights(const float f[3], float w[8]) {
    const float g0[3] = {__fsub_rn(1.0f, f[0]), __fsub_rn(1.0f, f[1]), __fsub_rn(1.0f, f[2])};
    const float xy[4] = {__fmul_rn(g0[0], g0[1]), __fmul_rn(f[0], g0[1]), __fmul_rn(g0[0], f[1]), __fmul_rn(f[0], f[1])};
#pragma unroll
    for (uint32_t c = 0; c < 8u; ++c) w[c] = __fmul_rn(xy[c & 3u], (c & 4u) ? f[2] : g0[2]);
}

NB_DEV void level_corners(const float p[3], const LevelParams lp, uint32_t hash_mask, uint32_t idx[8], float w[8]) {
    uint32_t i[3];
    float f[3];
    level_cell(p, lp, i, f);
    corner_entries(i, lp, hash_mask, idx);
    corner_weights(f, w);
}

// Corners c and c|1 differ only in x.  When their entries form an aligned
// pair (indices differing in bit 0 only: always on hashed levels for even x,
// on dense levels for an even first index) both are fetched with one 8-byte
// load.  Level offsets are multiples of 8 entries, so absolute and
// level-relative alignment agree.
NB_DEV void gather_pair(const uint32_t* __restrict__ P, uint32_t ea, uint32_t eb, uint32_t& va, uint32_t& vb) {
    if ((ea ^ eb) == 1u) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(P + (ea & ~1u)));
        va = (ea & 1u) ? v.y : v.x;
        vb = (ea & 1u) ? v.x : v.y;
    } else {
        va = __ldg(P + ea);
        vb = __ldg(P + eb);
    }
}
// Reduction of corners c and c|1: when both entries lie in one aligned
// 4-entry block (x and x+1 differ only in their two low bits -- 3 cases in
// 4, on dense and hashed levels alike) one 16-byte .v4 reduction carries both,
// adding zero to the block's other two entries.  L2 reductions cost per
// operation, not per byte, so this saves one operation.
NB_DEV void red_pair(uint32_t* G, uint32_t ea, uint32_t eb, uint32_t va, uint32_t vb) {
    if ((ea ^ eb) < 4u) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (uint32_t k = 0; k < 4u; ++k) w[k] = k == (ea & 3u) ? va : (k == (eb & 3u) ? vb : 0u);
        asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};\n" ::"l"(G + (ea & ~3u)), "r"(w[0]), "r"(w[1]),
                     "r"(w[2]), "r"(w[3])
                     : "memory");
    } else {
        red_add_f16x2(G + ea, va);
        red_add_f16x2(G + eb, vb);
    }
}

NB_DEV void gather8(const uint32_t* __restrict__ P, const uint32_t idx[8], uint32_t v[8]) {
#pragma unroll
    for (int c = 0; c < 8; c += 2) gather_pair(P, idx[c], idx[c + 1], v[c], v[c + 1]);
}

NB_DEV uint32_t interpolate(const uint32_t v[8], const float w[8]) {
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float2 f = unpack_h2(v[c]);
        a0 = __fmaf_rn(w[c], f.x, a0);
        a1 = __fmaf_rn(w[c], f.y, a1);
    }
    return pack_h2(a0, a1);
}

// Interpolated feature pair of one level (packed f16x2).  params: one
// uint32 (two fp16 features) per entry.
NB_DEV uint32_t level_forward(const uint32_t* __restrict__ params, const float p[3], const LevelParams lp, uint32_t hash_mask) {
    uint32_t idx[8], v[8];
    float w[8];
    level_corners(p, lp, hash_mask, idx, w);
    gather8(params, idx, v);
    return interpolate(v, w);
}

// Two (point, level) tasks with all their gathers issued before any is used.
NB_DEV void level_forward2(const uint32_t* __restrict__ params, const float pa[3], const LevelParams la, const float pb[3],
                           const LevelParams lb, uint32_t hash_mask, uint32_t& ra, uint32_t& rb) {
    uint32_t ia[8], ib[8], va[8], vb[8];
    float wa[8], wb[8];
    level_corners(pa, la, hash_mask, ia, wa);
    level_corners(pb, lb, hash_mask, ib, wb);
    gather8(params, ia, va);
    gather8(params, ib, vb);
    ra = interpolate(va, wa);
    rb = interpolate(vb, wb);
}

// A (point, level) lookup split in two so that many lookups' loads can be in
// flight at once: gather_level issues the four corner-pair loads and keeps
// only what the interpolation needs (the loaded words, the cell fractions and
// which aligned pairs came back swapped); finish_level interpolates exactly as
// level_forward does (same weights, same fma order, one fp16 rounding).
struct LevelGather {
    uint2 v[4];      // corners (2k, 2k+1)
    float f[3];
    uint32_t swap;   // bit k: pair k was loaded as one aligned word pair in swapped order
};
NB_DEV void gather_level(const uint32_t* __restrict__ P, const float p[3], const LevelParams lp, uint32_t hash_mask,
                         bool live, LevelGather& g) {
    uint32_t i[3], idx[8];
    level_cell(p, lp, i, g.f);
    corner_entries(i, lp, hash_mask, idx);
    g.swap = 0u;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) {
        const uint32_t ea = idx[2 * k], eb = idx[2 * k + 1];
        if (!live) {  // a dead row loads nothing
            g.v[k] = make_uint2(0u, 0u);
        } else if ((ea ^ eb) == 1u) {
            g.v[k] = __ldg(reinterpret_cast<const uint2*>(P + (ea & ~1u)));
            g.swap |= (ea & 1u) << k;
        } else {
            g.v[k].x = __ldg(P + ea);
            g.v[k].y = __ldg(P + eb);
        }
    }
}
NB_DEV uint32_t finish_level(const LevelGather& g) {
    float w[8];
    corner_weights(g.f, w);
    uint32_t v[8];
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) {
        const bool s = (g.swap >> k) & 1u;
        v[2 * k] = s ? g.v[k].y : g.v[k].x;
        v[2 * k + 1] = s ? g.v[k].x : g.v[k].y;
    }
    return interpolate(v, w);
}

struct LevelGatherWide {
    uint4 q[4];    // pair k: the aligned 16-byte block holding corners 2k and 2k+1, or those two corners in .x, .y
    float f[3];
    uint32_t sel;  // pair k: bits 4k..4k+1 = word of corner 2k in q[k], bits 4k+2..4k+3 = word of corner 2k+1
};
// The same lookup with 16-byte loads.  The x-neighbours of a pair share their
// aligned 16-byte block whenever their entries differ in the two low bits
// only: always for x even (entries e and e ^ 1 on hashed levels, e and e + 1
// on dense ones) and for half of the odd x; then the pair is one 16-byte load,
// which touches one sector where two 4-byte loads would touch it twice.  It
// holds twice the registers per lookup: the renderer gains from it (fewer
// sectors per pixel), the training forward, whose warps share more sectors
// and need more lookups in flight, does not.  The table must start on a
// 16-byte boundary.
NB_DEV void gather_level(const uint32_t* __restrict__ P, const float p[3], const LevelParams lp, uint32_t hash_mask,
                         bool live, LevelGatherWide& g) {
    uint32_t i[3], idx[8];
    level_cell(p, lp, i, g.f);
    corner_entries(i, lp, hash_mask, idx);
    g.sel = 0u;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) {
        const uint32_t ea = idx[2 * k], eb = idx[2 * k + 1];
        if (!live) {  // a dead row loads nothing
            g.q[k] = make_uint4(0u, 0u, 0u, 0u);
            g.sel |= 4u << (4u * k);
        } else if (((ea ^ eb) >> 2) == 0u) {
            g.q[k] = __ldg(reinterpret_cast<const uint4*>(P + (ea & ~3u)));
            g.sel |= ((ea & 3u) | ((eb & 3u) << 2)) << (4u * k);
        } else {
            g.q[k] = make_uint4(__ldg(P + ea), __ldg(P + eb), 0u, 0u);
            g.sel |= 4u << (4u * k);
        }
    }
}
NB_DEV uint32_t pick_word(const uint4 q, uint32_t w) {
    return (w & 2u) ? ((w & 1u) ? q.w : q.z) : ((w & 1u) ? q.y : q.x);
}
NB_DEV uint32_t finish_level(const LevelGatherWide& g) {
    float w[8];
    corner_weights(g.f, w);
    uint32_t v[8];
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) {
        v[2 * k] = pick_word(g.q[k], (g.sel >> (4u * k)) & 3u);
        v[2 * k + 1] = pick_word(g.q[k], (g.sel >> (4u * k + 2u)) & 3u);
    }
    return interpolate(v, w);
}

// Scatter of one level's feature gradient (d0, d1) to the eight corner
// entries with fp16x2 reductions performed at L2.
NB_DEV void level_backward(uint32_t* grad, const float p[3], const LevelParams lp, uint32_t hash_mask, float d0, float d1) {
    uint32_t idx[8];
    float w[8];
    level_corners(p, lp, hash_mask, idx, w);
#pragma unroll
    for (int c = 0; c < 8; c += 2)
        red_pair(grad, idx[c], idx[c + 1], pack_h2(w[c] * d0, w[c] * d1), pack_h2(w[c + 1] * d0, w[c + 1] * d1));
}

}  // namespace nb
