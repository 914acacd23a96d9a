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
// the root for the rounding of the root itself.  Culling only drops pixels
// the cut-off rejects, so the sums it feeds are unchanged.
#pragma once

#include <math.h>

#ifdef __CUDACC__
#define R2S_HD __host__ __device__ __forceinline__
#else
#define R2S_HD inline
#endif

namespace r2s {

constexpr float kCullLn2 = 0.69314718055994531f;

// Narrows the tile-local index range [lo, hi] of the walked axis v.  v0 is
// the offset v of index 0 (pixel centre minus mean), [uL, uR] the offsets of
// the first and last pixel centre of the strip on the other axis.  Leaves
// the range as it is for a degenerate or ill-conditioned conic, a negative
// or non-finite S, non-finite offsets or an already empty range; empties it
// (lo > hi) when no pixel of the strip can pass.
R2S_HD void strip_range(float a, float b, float c, float S, float uL, float uR, float v0, int& lo,
                        int& hi) {
    if (lo > hi || !(uL <= uR) || !(fabsf(v0) < 1e30f)) return;
    const float det = a * c - b * b;
    if (!(a > 0.f && c > 0.f && det > 0.f && S >= 0.f && S < 1e30f)) return;
    const float cond = (a * c) / det;
    if (!(cond < 1e6f)) return;
    const float Sm = S * (1.0f + 2e-4f + 1e-6f * cond) + 2e-4f;
    const float V = sqrtf(2.0f * Sm * (a / det));
    const float ut = -b * V / a;  // u of the top point; the bottom point sits at -ut
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
        vhi = (r - b * u0) / c;
        mhi = (fabsf(b * u0) + r) / c;
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
        vlo = (-r - b * u0) / c;
        mlo = (fabsf(b * u0) + r) / c;
    }
    // index i has offset v0 + i: keep i in [vlo - m - v0, vhi + m - v0]
    const float flo = (vlo - (1e-2f + 1e-5f * mlo)) - v0;
    const float fhi = (vhi + (1e-2f + 1e-5f * mhi)) - v0;
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
    const float S = s_thr * kCullLn2;
    strip_range(a, b, c, S, (X0 + ((float)c_lo + 0.5f)) - mx, (X0 + ((float)c_hi + 0.5f)) - mx,
                (Y0 + 0.5f) - my, r_lo, r_hi);
    if (r_lo > r_hi) {
        c_lo = 1;
        c_hi = 0;
        return;
    }
    strip_range(c, b, a, S, (Y0 + ((float)r_lo + 0.5f)) - my, (Y0 + ((float)r_hi + 0.5f)) - my,
                (X0 + 0.5f) - mx, c_lo, c_hi);
    if (c_lo > c_hi) {
        r_lo = 1;
        r_hi = 0;
    }
}

}  // namespace r2s
