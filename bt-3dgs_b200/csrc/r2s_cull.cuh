// Exact pixel-range culling of a 2D splat inside one tile (host and device).
//
// A splat passes the rasterizer's cut-off at pixel offset (u, v) from its
// mean when
//     s(u, v) = a u^2 / 2 + b u v + c v^2 / 2  <=  S,   S = ln(|w mu| / 1e-5)
// ((a, b, c) the conic; csrc/RasterizeToPixelsFwd.cu:159-179 skips every
// pixel with alpha = w mu exp(-s) below 1e-5).  The tile kernels first bound
// a record by its axis-aligned culling box (the extents of the whole ellipse
// s <= S).  Inside a tile that box is loose: the ellipse crosses the strip of
// the tile's columns over fewer rows than its full height when it is tilted
// or only grazes the tile.  strip_range() narrows the rows (or, with the
// roles swapped, the columns) to the projection of
//     {s <= S'}  ∩  {uL <= u <= uR}
// on the walked axis, an interval because both sets are convex.  Its upper
// end is the ellipse's top point (v = V, u = -b V / a) when that point lies
// in the strip, else the upper root of s(u0, v) = S' on the strip edge u0
// nearer to it; the lower end mirrors it.  S' widens S so that every pixel
// the float32 kernels count stays inside the range (relative 2e-4 plus 1e-6
// times the conditioning a c / det for the rounding of the three-term sum,
// absolute 2e-4 for the approximate log2 of the threshold); the interval
// gets a further margin of 1e-2 px plus 1e-5 of the magnitudes that enter
// the root (and of the offsets) for the rounding of the root itself.
// Culling only drops pixels the cut-off rejects, so the sums it feeds are
// unchanged.
//
// Voxels (brick_rows): the 3D splat passes where s(u, v, w) = d^T P d / 2
// <= S with S = ln(|w| / 1e-6) (csrc/VoxelizeToVoxelsFwd.cu:182-214).  In the
// slice w = dz the quadratic in (u, v) has the 2x2 block M = [[a, b], [b, d]]
// of the conic P = [[a, b, c], [b, d, e], [c, e, f]], its centre shifted by
// -M^-1 (c dz, e dz) and its minimum raised by dz^2 det(P) / (2 det(M)); each
// slice keeps the rows of that ellipse's bounding box (and none when the box
// misses the x range), with S first widened by the 3D conditioning
// a d f / det(P) and the slice's level then by strip_range's 2D margins.
#pragma once

#include <math.h>
#include <stdint.h>

#ifdef __CUDACC__
#define R2S_HD __host__ __device__ __forceinline__
#else
#define R2S_HD inline
#endif

namespace r2s {

constexpr float kCullLn2 = 0.69314718055994531f;

// Quantities of a 2D splat that both strip passes of tile_cull share.
struct StripConic {
    float a, b, c;     // conic
    float det, Sm;     // a c - b^2, widened level
    float inv_a, inv_c, inv_det;
    bool exact;        // false: degenerate or ill-conditioned, keep the box
};

R2S_HD StripConic strip_conic(float a, float b, float c, float S) {
    StripConic k;
    k.a = a;
    k.b = b;
    k.c = c;
    k.det = a * c - b * b;
    k.exact = a > 0.f && c > 0.f && k.det > 0.f && S >= 0.f && S < 1e30f;
    k.inv_det = 1.0f / k.det;
    const float cond = (a * c) * k.inv_det;
    k.exact = k.exact && cond < 1e6f;
    k.Sm = S * (1.0f + 2e-4f + 1e-6f * cond) + 2e-4f;
    k.inv_a = 1.0f / a;
    k.inv_c = 1.0f / c;
    return k;
}

// Narrows the tile-local index range [lo, hi] of the walked axis v.  v0 is
// the offset v of index 0 (pixel centre minus mean), [uL, uR] the offsets of
// the first and last pixel centre of the strip on the other axis; (a, c) are
// the conic's u and v coefficients (k.a / k.c, or swapped with their
// reciprocals for the column pass).  Leaves the range as it is for a
// degenerate or ill-conditioned conic, non-finite offsets or an already empty
// range; empties it (lo > hi) when no pixel of the strip can pass.
R2S_HD void strip_range(const StripConic& k, float a, float c, float inv_a, float inv_c, float uL,
                        float uR, float v0, int& lo, int& hi) {
    if (lo > hi || !k.exact || !(uL <= uR) || !(fabsf(v0) < 1e30f)) return;
    const float b = k.b, det = k.det, Sm = k.Sm;
    const float V = sqrtf(2.0f * Sm * (a * k.inv_det));
    const float ut = -b * V * inv_a;  // u of the top point; the bottom point sits at -ut
    float vhi, vlo, mhi, mlo;
    if (ut >= uL && ut <= uR) {
        vhi = V;
        mhi = V;
    } else {
        const float u0 = ut < uL ? uL : uR;
        const float disc = 2.0f * c * Sm - det * u0 * u0;
        if (!(disc >= 0.f)) {
            lo = 1;
            hi = 0;
            return;
        }
        const float r = sqrtf(disc);
        vhi = (r - b * u0) * inv_c;
        mhi = (fabsf(b * u0) + r) * inv_c;
    }
    if (-ut >= uL && -ut <= uR) {
        vlo = -V;
        mlo = V;
    } else {
        const float u0 = -ut < uL ? uL : uR;
        const float disc = 2.0f * c * Sm - det * u0 * u0;
        if (!(disc >= 0.f)) {
            lo = 1;
            hi = 0;
            return;
        }
        const float r = sqrtf(disc);
        vlo = (-r - b * u0) * inv_c;
        mlo = (fabsf(b * u0) + r) * inv_c;
    }
    // index i has offset v0 + i: keep i in [vlo - m - v0, vhi + m - v0]; the
    // margin also covers the rounding of offsets the caller shifted
    const float mag = fabsf(v0) + fmaxf(fabsf(uL), fabsf(uR));
    const float flo = (vlo - (1e-2f + 1e-5f * (mlo + mag))) - v0;
    const float fhi = (vhi + (1e-2f + 1e-5f * (mhi + mag))) - v0;
    if (!(flo <= fhi)) return;  // rounding or NaN: keep the range
    const float flo_c = fminf(fmaxf(flo, (float)lo), (float)hi + 1.0f);
    const float fhi_c = fmaxf(fminf(fhi, (float)hi), (float)lo - 1.0f);
    lo = (int)ceilf(flo_c);
    hi = (int)floorf(fhi_c);
}

// Narrows a record's culling box [c_lo, c_hi] x [r_lo, r_hi] inside the tile
// with origin (X0, Y0): first the rows over the box's column strip, then the
// columns over the narrowed row strip.  s_thr is the cut-off in log2 units
// (log2(|w mu| 1e5)); (mx, my) the mean, (a, b, c) the conic.
R2S_HD void tile_cull(float mx, float my, float a, float b, float c, float s_thr, float X0,
                      float Y0, int& c_lo, int& c_hi, int& r_lo, int& r_hi) {
    if (c_lo > c_hi || r_lo > r_hi) return;
    const StripConic k = strip_conic(a, b, c, s_thr * kCullLn2);
    strip_range(k, k.a, k.c, k.inv_a, k.inv_c, (X0 + ((float)c_lo + 0.5f)) - mx,
                (X0 + ((float)c_hi + 0.5f)) - mx, (Y0 + 0.5f) - my, r_lo, r_hi);
    if (r_lo > r_hi) {
        c_lo = 1;
        c_hi = 0;
        return;
    }
    strip_range(k, k.c, k.a, k.inv_c, k.inv_a, (Y0 + ((float)r_lo + 0.5f)) - my,
                (Y0 + ((float)r_hi + 0.5f)) - my, (X0 + 0.5f) - mx, c_lo, c_hi);
    if (c_lo > c_hi) {
        r_lo = 1;
        r_hi = 0;
    }
}

// Row ranges of a 3D splat in the eight z-slices of an 8x8x8 brick with
// origin (X0, Y0, Z0), inside its culling box [xl, xh] x [yl, yh] x [zl, zh]:
// byte k of (tab_lo, tab_hi) (slices 0-3, 4-7) = first row | last row << 4,
// 0x0f for a slice with no row; [ezl, ezh] the slices with rows (ezl > ezh:
// none).  q = (P00, P01, P02, P11, P12, P22) = (a, b, c, d, e, f); s_thr the
// cut-off in log2 units (log2(|w| 1e6)).  Each slice is bounded by the
// axis-aligned box of its ellipse: centre (du, dv) = dz (ku, kv) from the
// mean, half-widths sqrt(2 S_z d / det M) and sqrt(2 S_z a / det M) at level
// S_z = S' - ks dz^2; a slice whose box misses the culling box's x or y range
// has no row.  Branch-free over the eight slices (one square root each); a
// degenerate or ill-conditioned conic keeps the box's rows in every slice.
R2S_HD void brick_rows(float mx, float my, float mz, const float q[6], float s_thr, float X0,
                       float Y0, float Z0, int xl, int xh, int yl, int yh, int zl, int zh,
                       uint32_t& tab_lo, uint32_t& tab_hi, int& ezl, int& ezh) {
    tab_lo = tab_hi = 0x0f0f0f0fu;
    ezl = 8;
    ezh = -1;
    if (xl > xh || yl > yh || zl > zh) return;
    const float a = q[0], b = q[1], c = q[2], d = q[3], e = q[4], f = q[5];
    const float S = s_thr * kCullLn2;
    const float x0 = (X0 + 0.5f) - mx, y0 = (Y0 + 0.5f) - my;  // offsets of voxel 0
    const float detM = a * d - b * b;
    const float det3 = f * detM - a * e * e + 2.0f * b * c * e - d * c * c;
    const float cond3 = (a * d * f) / det3, cond2 = (a * d) / detM;
    const bool exact = a > 0.f && d > 0.f && f > 0.f && detM > 0.f && det3 > 0.f && S >= 0.f &&
                       S < 1e30f && cond3 < 1e6f && cond2 < 1e6f && fabsf(x0) < 1e30f &&
                       fabsf(y0) < 1e30f && fabsf(mz) < 1e30f;
    // the 3D level with strip_range's margins on the 3D conditioning, then the
    // 2D widening of each slice's level
    const float Sm = S * (1.0f + 2e-4f + 1e-6f * cond3) + 2e-4f;
    const float rel2 = 1.0f + 2e-4f + 1e-6f * cond2;
    const float inv = 1.0f / detM;
    const float ku = -(d * c - b * e) * inv, kv = -(a * e - b * c) * inv, ks = 0.5f * det3 * inv;
    const float wu = sqrtf(2.0f * d * inv), wv = sqrtf(2.0f * a * inv);
    for (int k = 0; k < 8; ++k) {
        if (k < zl || k > zh) continue;
        int lo = yl, hi = yh;
        if (exact) {
            const float dz = (Z0 + ((float)k + 0.5f)) - mz;
            const float Sz = Sm - ks * dz * dz;
            const float r = sqrtf(fmaxf(Sz * rel2 + 2e-4f, 0.0f));
            const float cu = ku * dz, cv = kv * dz;
            const float hu = r * wu, hv = r * wv;
            // voxel i has offset x0 + i: keep i in [cu - hu - m - x0, cu + hu + m - x0]
            const float mu_ = 1e-2f + 1e-5f * (fabsf(cu) + hu + fabsf(x0));
            const float mv_ = 1e-2f + 1e-5f * (fabsf(cv) + hv + fabsf(y0));
            const float fxl = (cu - hu - mu_) - x0, fxh = (cu + hu + mu_) - x0;
            const float fyl = (cv - hv - mv_) - y0, fyh = (cv + hv + mv_) - y0;
            const bool hit = Sz >= 0.f && fxl <= (float)xh && fxh >= (float)xl;
            const int ylo = (int)ceilf(fminf(fmaxf(fyl, (float)yl), (float)yh + 1.0f));
            const int yhi = (int)floorf(fmaxf(fminf(fyh, (float)yh), (float)yl - 1.0f));
            lo = hit ? ylo : 1;
            hi = hit ? yhi : 0;
            if (!(fyl <= fyh)) lo = yl, hi = yh;  // NaN: keep the box
        }
        if (lo > hi) continue;
        const uint32_t byte = (uint32_t)lo | ((uint32_t)hi << 4);
        if (k < 4)
            tab_lo = (tab_lo & ~(0xffu << (8 * k))) | (byte << (8 * k));
        else
            tab_hi = (tab_hi & ~(0xffu << (8 * (k - 4)))) | (byte << (8 * (k - 4)));
        ezl = k < ezl ? k : ezl;
        ezh = k;
    }
}

}  // namespace r2s
