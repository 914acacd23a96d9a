// Host harness of the tile culling in r2s_cull.cuh (CPU tests only).
//
// For each case it narrows a box of a tile with tile_cull() and re-evaluates
// every pixel of the box with the float32 cut-off test of the 16x16 tile
// kernels, in both of their evaluation orders:
//   forward, and backward walking columns:  -s = dy (C dy + B dx) + (A dx) dx
//   backward walking rows:                  -s = dx (A dx + B dy) + (C dy) dy
// (A, B, C = -log2(e) (a/2, b, c/2)); a pixel passes when -s >= -s_thr, i.e.
// when the bits of -s compare as signed integers at most those of -s_thr.
// The threshold is loosened by 1e-5 (relative, at least 1e-5 absolute) to
// cover the approximate log2 of the device.  A pixel that passes outside the
// narrowed ranges is a violation.  Built with -ffp-contract=off: every fused
// multiply-add of the kernels is an explicit fmaf here.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "r2s_cull.cuh"

namespace {

constexpr float kLog2e = 1.4426950408889634f;

inline int32_t fbits(float x) {
    int32_t i;
    memcpy(&i, &x, 4);
    return i;
}

inline float s_threshold(float wmu) {
    const float a = fabsf(wmu) * 1e5f;
    return a >= 1.0f ? log2f(a) : -1.0f;
}

}  // namespace

// cases: [n][8] float = mx, my, a, b, c, wmu, X0, Y0 (tile origin)
// boxes: [n][6] int = c_lo, c_hi, r_lo, r_hi (starting box), cmax, rmax
// out:   [n][8] int = c_lo, c_hi, r_lo, r_hi after culling, violations,
//        passing rows (union over both orders), passing columns, passes
extern "C" int cull_probe(const float* cases, const int* boxes, int64_t n, int* out) {
    int64_t total_viol = 0;
    for (int64_t k = 0; k < n; ++k) {
        const float* q = cases + 8 * k;
        const int* bx = boxes + 6 * k;
        const float mx = q[0], my = q[1], a = q[2], b = q[3], c = q[4], wmu = q[5];
        const float X0 = q[6], Y0 = q[7];
        int c_lo = bx[0], c_hi = bx[1], r_lo = bx[2], r_hi = bx[3];
        const float s_thr = s_threshold(wmu);
        r2s::tile_cull(mx, my, a, b, c, s_thr, X0, Y0, c_lo, c_hi, r_lo, r_hi);
        const float loose = s_thr + fmaxf(1e-5f, 1e-5f * fabsf(s_thr));
        const int32_t thr_n = fbits(-loose);
        const float A = -0.5f * kLog2e * a, B = -kLog2e * b, C = -0.5f * kLog2e * c;
        int viol = 0, passes = 0;
        uint32_t rows = 0, cols = 0;
        for (int r = bx[2]; r <= bx[3] && r <= bx[5]; ++r) {
            for (int col = bx[0]; col <= bx[1] && col <= bx[4]; ++col) {
                const float dx = (X0 + ((float)col + 0.5f)) - mx;
                const float dy = (Y0 + ((float)r + 0.5f)) - my;
                const float fwd = fmaf(dy, fmaf(C, dy, B * dx), (A * dx) * dx);
                const float bwr = fmaf(dx, fmaf(A, dx, B * dy), (C * dy) * dy);
                const bool pass = fbits(fwd) <= thr_n || fbits(bwr) <= thr_n;
                if (!(s_thr >= 0.f) || !pass) continue;
                ++passes;
                rows |= 1u << r;
                cols |= 1u << col;
                if (r < r_lo || r > r_hi || col < c_lo || col > c_hi) ++viol;
            }
        }
        int* o = out + 8 * k;
        o[0] = c_lo;
        o[1] = c_hi;
        o[2] = r_lo;
        o[3] = r_hi;
        o[4] = viol;
        o[5] = __builtin_popcount(rows);
        o[6] = __builtin_popcount(cols);
        o[7] = passes;
        total_viol += viol;
    }
    return (int)(total_viol > 0x7fffffff ? 0x7fffffff : total_viol);
}

// 3D: cases [n][13] float = mx, my, mz, P00, P01, P02, P11, P12, P22, w, X0, Y0, Z0;
// boxes [n][6] int = xl, xh, yl, yh, zl, zh (starting box inside the 8^3 brick);
// out [n][4] int = violations, (z, y) rows holding a passing voxel, rows kept by
// brick_rows, passing voxels.  The voxel kernels' two evaluation orders:
//   forward:  -s = dx (A dx + (Cq dz + B dy)) + (dy (E dz + D dy) + (F dz) dz)
//   backward: -s = dx (A dx + (B dy + Cq dz)) + (dy (D dy + E dz) + (F dz) dz)
// with (A, B, Cq, D, E, F) = -log2(e) (a/2, b, c, d/2, e, f/2); threshold
// log2(|w| 1e6), loosened as in the 2D probe.
extern "C" int cull_probe3(const float* cases, const int* boxes, int64_t n, int* out) {
    int64_t total_viol = 0;
    for (int64_t k = 0; k < n; ++k) {
        const float* c = cases + 13 * k;
        const int* bx = boxes + 6 * k;
        const float mx = c[0], my = c[1], mz = c[2], w = c[9];
        const float q[6] = {c[3], c[4], c[5], c[6], c[7], c[8]};
        const float X0 = c[10], Y0 = c[11], Z0 = c[12];
        const float a1 = fabsf(w) * 1e6f;
        const float s_thr = a1 >= 1.0f ? log2f(a1) : -1.0f;
        uint32_t tlo, thi;
        int ezl, ezh;
        r2s::brick_rows(mx, my, mz, q, s_thr, X0, Y0, Z0, bx[0], bx[1], bx[2], bx[3], bx[4], bx[5],
                        tlo, thi, ezl, ezh);
        const float loose = s_thr + fmaxf(1e-5f, 1e-5f * fabsf(s_thr));
        const int32_t thr_n = fbits(-loose);
        const float A = -0.5f * kLog2e * q[0], B = -kLog2e * q[1], Cq = -kLog2e * q[2];
        const float D = -0.5f * kLog2e * q[3], E = -kLog2e * q[4], F = -0.5f * kLog2e * q[5];
        int viol = 0, passes = 0, rows = 0, kept = 0;
        for (int z = 0; z < 8; ++z) {
            const uint32_t byte = ((z < 4 ? tlo : thi) >> (8 * (z & 3))) & 0xffu;
            const int lo = byte & 15, hi = byte >> 4;
            if (lo <= hi) kept += hi - lo + 1;
            if (z < bx[4] || z > bx[5]) continue;
            const float dz = (Z0 + ((float)z + 0.5f)) - mz;
            for (int y = bx[2]; y <= bx[3]; ++y) {
                const float dy = (Y0 + ((float)y + 0.5f)) - my;
                bool row = false;
                for (int x = bx[0]; x <= bx[1]; ++x) {
                    const float dx = (X0 + ((float)x + 0.5f)) - mx;
                    const float fw = fmaf(dx, fmaf(A, dx, fmaf(Cq, dz, B * dy)),
                                          fmaf(dy, fmaf(E, dz, D * dy), (F * dz) * dz));
                    const float bw = fmaf(dx, fmaf(A, dx, fmaf(B, dy, Cq * dz)),
                                          fmaf(dy, fmaf(D, dy, E * dz), (F * dz) * dz));
                    const bool pass = fbits(fw) <= thr_n || fbits(bw) <= thr_n;
                    if (!(s_thr >= 0.f) || !pass) continue;
                    ++passes;
                    row = true;
                    if (y < lo || y > hi || z < ezl || z > ezh) ++viol;
                }
                rows += row;
            }
        }
        int* o = out + 4 * k;
        o[0] = viol;
        o[1] = rows;
        o[2] = kept;
        o[3] = passes;
        total_viol += viol;
    }
    return (int)(total_viol > 0x7fffffff ? 0x7fffffff : total_viol);
}
