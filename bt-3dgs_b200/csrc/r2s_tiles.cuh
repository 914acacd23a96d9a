// Tile / brick rectangles of splats.  These decide the integer binning
// outputs (tiles_per_gauss, keys, per-tile ranges), which must equal the
// reference's bit for bit, so the float expressions keep the reference's
// evaluation order (compiled with the same fast-math flags).  For float64
// inputs the reference evaluates them in double (OpType<double> = double,
// csrc/IsectTilesKernel.cu:66-67); the templates follow that.
#pragma once

#include "r2s_common.cuh"

namespace r2s {

__device__ __forceinline__ uint32_t sat_u32(float v) { return __float2uint_rz(v); }
__device__ __forceinline__ uint32_t sat_u32(double v) { return __double2uint_rz(v); }

// Clamp of a tile bound to [0, upper] (IsectTilesKernel.cu:30-40).
template <typename T>
__device__ __forceinline__ uint32_t clamp_tile(T v, uint32_t upper) {
    if (!isfinite(v) || v <= static_cast<T>(0)) return 0u;
    if (v >= static_cast<T>(upper)) return upper;
    return static_cast<uint32_t>(v);
}

// Tile rectangle of one (view, Gaussian) from its 2D mean and rectangular
// radii (IsectTilesKernel.cu:76-112): [floor((m - r)/T), ceil((m + r)/T))
// clamped to the grid, divisions performed as divisions.
template <typename T>
__device__ __forceinline__ Rect2 tile_rect_2d(T mx, T my, T rad_x, T rad_y, uint32_t tile,
                                              uint32_t ntx, uint32_t nty, int32_t& count) {
    Rect2 r{0u, 0u};
    count = 0;
    if (rad_x <= 0 || rad_y <= 0) return r;
    if (!isfinite(mx) || !isfinite(my)) return r;
    const T ts = static_cast<T>(tile);
    const T trx = rad_x / ts;
    const T try_ = rad_y / ts;
    const T tx = mx / ts;
    const T ty = my / ts;
    const uint32_t x0 = clamp_tile(floor(tx - trx), ntx);
    const uint32_t y0 = clamp_tile(floor(ty - try_), nty);
    const uint32_t x1 = clamp_tile(ceil(tx + trx), ntx);
    const uint32_t y1 = clamp_tile(ceil(ty + try_), nty);
    if (x1 <= x0 || y1 <= y0) return r;
    r.x = pack16(x0, x1);
    r.y = pack16(y0, y1);
    count = static_cast<int32_t>((y1 - y0) * (x1 - x0));
    return r;
}

// Brick rectangle of one Gaussian (IsectTiles3DKernel.cu:72-110): bounds go
// through the saturating float->uint conversion of the reference's
// static_cast (negative and NaN -> 0) and are clamped to the grid.  The
// reference's count is the product of the three unsigned extents, which is
// 0 whenever an extent is 0.
template <typename T>
__device__ __forceinline__ Rect3 tile_rect_3d(T mx, T my, T mz, T rx, T ry, T rz, uint32_t tile,
                                              uint32_t nt2, uint32_t nt1, uint32_t nt0,
                                              int32_t& count) {
    Rect3 r{0u, 0u, 0u, 0u};
    count = 0;
    if (rx <= 0 || ry <= 0 || rz <= 0) return r;
    const T ts = static_cast<T>(tile);
    const T trx = rx / ts;
    const T try_ = ry / ts;
    const T trz = rz / ts;
    const T tx = mx / ts;
    const T ty = my / ts;
    const T tz = mz / ts;
    const uint32_t x0 = min(sat_u32(floor(tx - trx)), nt2);
    const uint32_t y0 = min(sat_u32(floor(ty - try_)), nt1);
    const uint32_t z0 = min(sat_u32(floor(tz - trz)), nt0);
    const uint32_t x1 = min(sat_u32(ceil(tx + trx)), nt2);
    const uint32_t y1 = min(sat_u32(ceil(ty + try_)), nt1);
    const uint32_t z1 = min(sat_u32(ceil(tz + trz)), nt0);
    if (x1 <= x0 || y1 <= y0 || z1 <= z0) return r;
    r.x = pack16(x0, x1);
    r.y = pack16(y0, y1);
    r.z = pack16(z0, z1);
    count = static_cast<int32_t>((z1 - z0) * (y1 - y0) * (x1 - x0));
    return r;
}

}  // namespace r2s
