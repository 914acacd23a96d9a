// Additive X-ray rasterization forward and backward.
//
// Forward (reference: csrc/RasterizeToPixelsFwd.cu:56-186): one CTA per
// (view, tile), one thread per pixel; the tile's sorted Gaussian list is
// staged through shared memory in batches.  Differences in how the work is
// done (the result is the same sum over the same contributing set):
//   * generic kernel: every staged Gaussian carries a bit mask of the warps
//     (pixel blocks of 8x4 for tile sizes divisible by 8) whose pixels can
//     reach the |alpha| >= 1e-5 cut-off; a warp only evaluates the Gaussians
//     of its mask bits (ballot + find-first-set);
//   * float32 16x16 kernel: every warp covers the whole tile for a quarter of
//     the list and evaluates only the 4-row groups that the Gaussian's
//     ellipse reaches inside the tile (r2s_cull.cuh narrows the culling box
//     to the rows where the ellipse crosses the tile's columns), with the
//     batch sorted by group range so that each range runs its own loop;
//     partial sums of the four warps are added at the end;
//   * float32 evaluates sigma*log2(e) with a pre-scaled conic and one ex2.
//
// Backward (reference: csrc/RasterizeToPixelsBwd.cu:76-265 "pixel" and
// 349-480 "primitive"): one CTA per (view, tile) with the tile's upstream
// gradient in shared memory.  The generic kernel gives each warp whole
// Gaussians and walks only the pixel rectangle that can contribute; the
// float32 16x16 kernel gives each thread one Gaussian record and walks the
// rows, or the columns when they are fewer, of its culling box narrowed to
// the ellipse inside the tile (the ranges that the forward of the same
// binning wrote to its culling table, 2 bytes per record, or its own
// tile_cull without one).  Per (Gaussian, tile) both reduce
// six moments of the contributing pixels,
//   S0 = sum v e,  Sx = sum v e dx,  Sy = sum v e dy,
//   Sxx = sum v e dx^2,  Sxy = sum v e dx dy,  Syy = sum v e dy^2
// (+ Ax, Ay = sum |v e (conic d)|_x,y for absgrad), with e = exp(-sigma) and
// d = pixel - mean, and adds them to a per-(view, Gaussian) record with two
// vector reductions.  Every reference gradient is a fixed linear map of
// these moments:
//   v_means2d = w mu (a Sx + b Sy, b Sx + c Sy)
//   v_conics  = -w mu (Sxx/2, Sxy, Syy/2)
//   v_opacity = mu S0,   v_mu = w S0,   v_means2d_abs = |w mu| (Ax, Ay)
#include <math_constants.h>

#include "r2s_common.cuh"
#include "r2s_cull.cuh"
#include "r2s_debug.cuh"
#include "r2s_cutoff.cuh"
#include "r2s_refexpr.cuh"

namespace r2s {

constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ __forceinline__ size_t al16(size_t x) { return (x + 15) & ~size_t(15); }
constexpr float kAlphaMin2D = 1e-5f;

// ---------------------------------------------------------------------------
// Culling extents (see cull_extent in r2s_preprocess.cu for the margins)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void conic_cull_extents(float a, float b, float c, float amp,
                                                   float thresh, float& ex, float& ey) {
    if (isnan(amp) || isnan(a) || isnan(b) || isnan(c)) {
        ex = ey = CUDART_INF_F;
        return;
    }
    const float aa = fabsf(amp);
    if (!(aa >= thresh)) {
        ex = ey = -1.0f;
        return;
    }
    const float det = a * c - b * b;
    if (!(a > 0.f && c > 0.f && det > 0.f)) {
        ex = ey = CUDART_INF_F;
        return;
    }
    const float cond = (a * c) / det;
    if (!isfinite(cond) || cond > 1e6f) {
        ex = ey = CUDART_INF_F;
        return;
    }
    const float s_cut = logf(aa / thresh) * 1.0001f + 1e-4f;
    const float rel = 1.0f + 1e-4f + 4e-7f * cond;
    ex = sqrtf(2.0f * s_cut * (c / det) * rel) * 1.0001f + 1e-3f;
    ey = sqrtf(2.0f * s_cut * (a / det) * rel) * 1.0001f + 1e-3f;
}

// Inclusive index range [lo, hi] of tile-local pixels whose centre lies within
// [m - e, m + e], clamped to [0, lim]; empty when lo > hi.
__device__ __forceinline__ void cull_range(float m, float e, float origin, int lim, int& lo,
                                           int& hi) {
    if (!(e >= 0.f)) {
        lo = 1;
        hi = 0;
        return;
    }
    if (!isfinite(m) || isinf(e)) {
        lo = 0;
        hi = lim;
        return;
    }
    const float flo = fmaxf(m - e - origin - 0.5f, 0.0f);
    const float fhi = fminf(m + e - origin - 0.5f, static_cast<float>(lim));
    if (flo > fhi) {
        lo = 1;
        hi = 0;
        return;
    }
    lo = static_cast<int>(ceilf(flo));
    hi = static_cast<int>(floorf(fhi));
}

// ---------------------------------------------------------------------------
// Pixel layout of a tile CTA
// ---------------------------------------------------------------------------
struct TileGeom {
    int T;        // tile edge
    int nthr;     // T*T threads
    bool blocked; // warps own 8x4 pixel blocks
    __device__ __forceinline__ void pixel(int tid, int& lx, int& ly) const {
        if (blocked) {
            const int w = tid >> 5, l = tid & 31, wx = T >> 3;
            lx = (w % wx) * 8 + (l & 7);
            ly = (w / wx) * 4 + (l >> 3);
        } else {
            ly = tid / T;
            lx = tid - ly * T;
        }
    }
    // bounding box of warp w's pixels, clipped to [0, cmax] x [0, rmax]
    __device__ __forceinline__ int4 warp_box(int w, int cmax, int rmax) const {
        int c0, c1, r0, r1;
        if (blocked) {
            const int wx = T >> 3;
            c0 = (w % wx) * 8;
            c1 = c0 + 7;
            r0 = (w / wx) * 4;
            r1 = r0 + 3;
        } else {
            const int first = w * 32, last = min(w * 32 + 31, nthr - 1);
            r0 = first / T;
            r1 = last / T;
            c0 = (r0 == r1) ? first - r0 * T : 0;
            c1 = (r0 == r1) ? last - r1 * T : T - 1;
        }
        c1 = min(c1, cmax);
        r1 = min(r1, rmax);
        return make_int4(c0, c1, r0, r1);
    }
};

__device__ __forceinline__ unsigned warp_lane_mask(int nthr, int warp) {
    const int n = nthr - warp * 32;
    return n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
}

template <typename S>
struct RasterSrc {
    const float4* splats;  // fused float32 records [C*N][2]
    const S* means2d;      // reference-layout inputs [C*N][2]
    const S* conics;       // [C*N][3]
    const S* opac;         // [C*N]
    const S* mus;          // [C*N]
};

template <typename S, bool SPLATS>
__device__ __forceinline__ void load_gauss(const RasterSrc<S>& src, int64_t g, S& mx, S& my, S& a,
                                           S& b, S& c, S& wmu, float& ex, float& ey) {
    if constexpr (SPLATS) {
        const float4 p = src.splats[2 * g];
        const float4 q = src.splats[2 * g + 1];
        mx = p.x;
        my = p.y;
        a = p.z;
        b = p.w;
        c = q.x;
        wmu = q.y;
        ex = q.z;
        ey = q.w;
    } else {
        mx = src.means2d[2 * g];
        my = src.means2d[2 * g + 1];
        a = src.conics[3 * g];
        b = src.conics[3 * g + 1];
        c = src.conics[3 * g + 2];
        wmu = src.opac[g] * src.mus[g];
        conic_cull_extents((float)a, (float)b, (float)c, (float)wmu, kAlphaMin2D, ex, ey);
    }
}

// ===========================================================================
// Forward
// ===========================================================================
template <typename S, bool SPLATS>
__global__ void raster_fwd_kernel(RasterSrc<S> src, const int32_t* __restrict__ offsets,
                                  const int32_t* __restrict__ flatten_ids, int64_t n_keys,
                                  int64_t n_isects, uint32_t W, uint32_t H, TileGeom geo,
                                  uint32_t ntx, uint32_t nty, S* __restrict__ image) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nthr = geo.nthr;
    const size_t arr = al16((size_t)nthr * sizeof(S));
    S* s_mx = reinterpret_cast<S*>(smem_raw);
    S* s_my = reinterpret_cast<S*>(smem_raw + arr);
    S* s_a = reinterpret_cast<S*>(smem_raw + 2 * arr);
    S* s_b = reinterpret_cast<S*>(smem_raw + 3 * arr);
    S* s_c = reinterpret_cast<S*>(smem_raw + 4 * arr);
    S* s_w = reinterpret_cast<S*>(smem_raw + 5 * arr);
    uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem_raw + 6 * arr);
    int4* s_box = reinterpret_cast<int4*>(smem_raw + 6 * arr + al16((size_t)nthr * 4));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = geo.T;
    const int64_t cam = blockIdx.z;
    const uint32_t tx = blockIdx.x, ty = blockIdx.y;
    const int64_t key = cam * (int64_t)ntx * nty + (int64_t)ty * ntx + tx;
    const int X0 = tx * T, Y0 = ty * T;
    const int cmax = min(T - 1, (int)W - 1 - X0), rmax = min(T - 1, (int)H - 1 - Y0);
    const int n_warps = (nthr + 31) >> 5;
    if (tid < n_warps) s_box[tid] = geo.warp_box(tid, cmax, rmax);

    int lx, ly;
    geo.pixel(tid, lx, ly);
    const bool inside = lx <= cmax && ly <= rmax;
    const S px = static_cast<S>(X0 + lx) + static_cast<S>(0.5);
    const S py = static_cast<S>(Y0 + ly) + static_cast<S>(0.5);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    const unsigned wmask = warp_lane_mask(nthr, warp);
    S acc = static_cast<S>(0);
    __syncthreads();

    for (int b0 = start; b0 < end; b0 += nthr) {
        const int n = min(nthr, end - b0);
        __syncthreads();
        if (tid < n) {
            const int64_t g = flatten_ids[b0 + tid];
            S mx, my, a, b, c, wmu;
            float ex, ey;
            load_gauss<S, SPLATS>(src, g, mx, my, a, b, c, wmu, ex, ey);
            int c_lo, c_hi, r_lo, r_hi;
            cull_range((float)mx, ex, (float)X0, cmax, c_lo, c_hi);
            cull_range((float)my, ey, (float)Y0, rmax, r_lo, r_hi);
            uint32_t m = 0;
            if (c_lo <= c_hi && r_lo <= r_hi) {
                for (int w = 0; w < n_warps; ++w) {
                    const int4 bx = s_box[w];
                    if (c_lo <= bx.y && c_hi >= bx.x && r_lo <= bx.w && r_hi >= bx.z) m |= 1u << w;
                }
            }
            s_mx[tid] = mx;
            s_my[tid] = my;
            if constexpr (std::is_same<S, float>::value) {
                s_a[tid] = 0.5f * kLog2e * a;
                s_b[tid] = kLog2e * b;
                s_c[tid] = 0.5f * kLog2e * c;
            } else {
                s_a[tid] = a;
                s_b[tid] = b;
                s_c[tid] = c;
            }
            s_w[tid] = wmu;
            s_mask[tid] = m;
        }
        __syncthreads();
        for (int c0 = 0; c0 < n; c0 += 32) {
            const int j = c0 + lane;
            unsigned bits = __ballot_sync(wmask, j < n && ((s_mask[j] >> warp) & 1u));
            while (bits) {
                const int t = c0 + __ffs(bits) - 1;
                bits &= bits - 1;
                const S dx = px - s_mx[t];
                const S dy = py - s_my[t];
                if constexpr (std::is_same<S, float>::value) {
                    const float u = fmaf(s_a[t], dx, s_b[t] * dy);
                    const float s = fmaf(dx, u, s_c[t] * dy * dy);
                    const float al = s_w[t] * exp2f(-s);
                    acc += (s < 0.f || fabsf(al) < kAlphaMin2D) ? 0.f : al;
                } else {
                    const S sig = static_cast<S>(0.5) * (s_a[t] * dx * dx + s_c[t] * dy * dy) +
                                  s_b[t] * dx * dy;
                    const S al = s_w[t] * expf_neg(sig);
                    const bool skip = sig < static_cast<S>(0) ||
                                      fabsf(static_cast<float>(al)) < static_cast<S>(1e-5);
                    acc += skip ? static_cast<S>(0) : al;
                }
            }
        }
    }
    if (inside) image[(cam * H + (Y0 + ly)) * (int64_t)W + X0 + lx] = acc;
}

// ===========================================================================
// Backward: sufficient statistics per (view, Gaussian)
// ===========================================================================
template <typename S>
__device__ __forceinline__ void stats_red(S* dst, const S v[8], bool with_abs) {
    if constexpr (std::is_same<S, float>::value) {
        red_add_v4(dst, v[0], v[1], v[2], v[3]);
        if (with_abs) red_add_v4(dst + 4, v[4], v[5], v[6], v[7]);
        else red_add_v2(dst + 4, v[4], v[5]);
    } else {
        const int n = with_abs ? 8 : 6;
        for (int k = 0; k < n; ++k) atomicAdd(dst + k, v[k]);
    }
}

template <typename S, bool SPLATS, int EXPMODE>
__global__ void raster_bwd_kernel(RasterSrc<S> src, const int32_t* __restrict__ offsets,
                                  const int32_t* __restrict__ flatten_ids, int64_t n_keys,
                                  int64_t n_isects, const S* __restrict__ v_image, uint32_t W,
                                  uint32_t H, int T, uint32_t ntx, uint32_t nty, int with_abs,
                                  S* __restrict__ stats) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nthr = blockDim.x;
    const int TP = T + 1;
    S* s_v = reinterpret_cast<S*>(smem_raw);
    S* s_mx = s_v + T * TP;
    S* s_my = s_mx + nthr;
    S* s_a = s_my + nthr;
    S* s_b = s_a + nthr;
    S* s_c = s_b + nthr;
    S* s_w = s_c + nthr;
    int32_t* s_g = reinterpret_cast<int32_t*>(s_w + nthr);
    uint32_t* s_box = reinterpret_cast<uint32_t*>(s_g + nthr);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_warps = nthr >> 5;
    const int64_t cam = blockIdx.z;
    const uint32_t tx = blockIdx.x, ty = blockIdx.y;
    const int64_t key = cam * (int64_t)ntx * nty + (int64_t)ty * ntx + tx;
    const int X0 = tx * T, Y0 = ty * T;
    const int cmax = min(T - 1, (int)W - 1 - X0), rmax = min(T - 1, (int)H - 1 - Y0);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (start >= end) return;

    const S* vcam = v_image + cam * (int64_t)H * W;
    for (int p = tid; p < T * T; p += nthr) {
        const int r = p / T, c = p - r * T;
        s_v[r * TP + c] = (c <= cmax && r <= rmax) ? vcam[(int64_t)(Y0 + r) * W + X0 + c]
                                                   : static_cast<S>(0);
    }

    for (int b0 = start; b0 < end; b0 += nthr) {
        const int n = min(nthr, end - b0);
        __syncthreads();
        if (tid < n) {
            const int64_t g = flatten_ids[b0 + tid];
            S mx, my, a, b, c, wmu;
            float ex, ey;
            load_gauss<S, SPLATS>(src, g, mx, my, a, b, c, wmu, ex, ey);
            int c_lo, c_hi, r_lo, r_hi;
            cull_range((float)mx, ex, (float)X0, cmax, c_lo, c_hi);
            cull_range((float)my, ey, (float)Y0, rmax, r_lo, r_hi);
            if (c_lo > c_hi || r_lo > r_hi) c_lo = 1, c_hi = 0, r_lo = 0, r_hi = 0;
            s_mx[tid] = mx;
            s_my[tid] = my;
            s_a[tid] = a;
            s_b[tid] = b;
            s_c[tid] = c;
            s_w[tid] = wmu;
            s_g[tid] = (int32_t)g;
            s_box[tid] = (uint32_t)c_lo | ((uint32_t)c_hi << 8) | ((uint32_t)r_lo << 16) |
                         ((uint32_t)r_hi << 24);
        }
        __syncthreads();
        for (int t = warp; t < n; t += n_warps) {
            const uint32_t bx = s_box[t];
            const int c_lo = bx & 0xff, c_hi = (bx >> 8) & 0xff;
            const int r_lo = (bx >> 16) & 0xff, r_hi = bx >> 24;
            if (c_lo > c_hi) continue;
            const int w = c_hi - c_lo + 1;
            const int npx = w * (r_hi - r_lo + 1);
            const float inv_w = 1.0f / (float)w;
            const S mx = s_mx[t], my = s_my[t], a = s_a[t], b = s_b[t], c = s_c[t], wmu = s_w[t];
            S acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int p = lane; p < npx; p += 32) {
                const int rr = __float2int_rz(((float)p + 0.5f) * inv_w);
                const int cc = p - rr * w;
                const int lx = c_lo + cc, ly = r_lo + rr;
                const S v = s_v[ly * TP + lx];
                const S dx = static_cast<S>(X0 + lx) + static_cast<S>(0.5) - mx;
                const S dy = static_cast<S>(Y0 + ly) + static_cast<S>(0.5) - my;
                S e;
                bool skip;
                if constexpr (std::is_same<S, float>::value) {
                    const float A = 0.5f * kLog2e * a, B = kLog2e * b, Cc = 0.5f * kLog2e * c;
                    const float u = fmaf(A, dx, B * dy);
                    const float s = fmaf(dx, u, Cc * dy * dy);
                    e = exp2f(-s);
                    skip = s < 0.f || fabsf(wmu * e) < kAlphaMin2D;
                } else {
                    const S sig = static_cast<S>(0.5) * (a * dx * dx + c * dy * dy) + b * dx * dy;
                    if constexpr (EXPMODE == 0) {
                        e = expf_neg(sig);
                        skip = sig < static_cast<S>(0) ||
                               fabsf(static_cast<float>(wmu * e)) < static_cast<S>(1e-5);
                    } else {
                        e = exp(-sig);
                        skip = sig < static_cast<S>(0) || fabs(wmu * e) < static_cast<S>(1e-5);
                    }
                }
                const S ve = skip ? static_cast<S>(0) : v * e;
                const S vx = ve * dx, vy = ve * dy;
                acc[0] += ve;
                acc[1] += vx;
                acc[2] += vy;
                acc[3] += vx * dx;
                acc[4] += vx * dy;
                acc[5] += vy * dy;
                if (with_abs) {
                    acc[6] += fabs(a * vx + b * vy);
                    acc[7] += fabs(b * vx + c * vy);
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = warp_sum(acc[k]);
            if (lane == 0) stats_red(stats + (int64_t)s_g[t] * 8, acc, with_abs != 0);
        }
    }
}

// Per-(view, Gaussian) gradients of the reference from the statistics.
template <typename S>
__global__ void raster_unpack_kernel(const S* __restrict__ stats, const S* __restrict__ conics,
                                     const S* __restrict__ opac, const S* __restrict__ mus,
                                     int64_t total, S* __restrict__ v_abs, S* __restrict__ v_m2,
                                     S* __restrict__ v_con, S* __restrict__ v_op,
                                     S* __restrict__ v_mu) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const S* st = stats + i * 8;
    const S S0 = st[0], Sx = st[1], Sy = st[2], Sxx = st[3], Sxy = st[4], Syy = st[5];
    const S a = conics[3 * i], b = conics[3 * i + 1], c = conics[3 * i + 2];
    const S w = opac[i], mu = mus[i];
    const S wm = w * mu;
    v_m2[2 * i] = wm * (a * Sx + b * Sy);
    v_m2[2 * i + 1] = wm * (b * Sx + c * Sy);
    v_con[3 * i] = -wm * static_cast<S>(0.5) * Sxx;
    v_con[3 * i + 1] = -wm * Sxy;
    v_con[3 * i + 2] = -wm * static_cast<S>(0.5) * Syy;
    v_op[i] = mu * S0;
    v_mu[i] = w * S0;
    if (v_abs) {
        v_abs[2 * i] = fabs(wm) * st[6];
        v_abs[2 * i + 1] = fabs(wm) * st[7];
    }
}

// ===========================================================================
// float32, 16x16 tiles: the fast kernels
// ===========================================================================
//
// Validity test.  The reference keeps a pair when sigma >= 0 and
// |w mu exp(-sigma)| >= 1e-5.  With s = sigma*log2(e) this is
// 0 <= s <= s_thr, s_thr = log2(|w mu| * 1e5); for non-negative floats the
// IEEE bit patterns are ordered like the values and every negative s (sign
// bit set) compares above s_thr as an unsigned integer, so one integer
// compare decides the pair.  In the forward, pairs within rounding of the
// alpha cut-off may be decided differently from the reference's float test
// (each such pair moves a pixel by at most ~1e-5); the 16x16 backward
// re-decides them exactly (r2s_cutoff.cuh).  The 16x16 forward evaluates -s with negated
// coefficients (exact: negation commutes with rounding) and compare the bits
// of -s as signed integers with INT_MIN + bits(s_thr); the one value decided
// differently from "0 <= s <= s_thr" is s = -0.0, which needs a conic that is
// not positive definite and a pixel centre on the mean, and counts as s < 0.

__device__ __forceinline__ bool s_valid(float s, uint32_t thr_bits) {
    return __float_as_uint(s) <= thr_bits;
}

// Culling ranges of one (record, tile) pair after tile_cull, 4 bits each:
// c_lo | c_hi << 4 | r_lo << 8 | r_hi << 12 (an empty range stays empty).
__device__ __forceinline__ uint16_t pack_cull(int c_lo, int c_hi, int r_lo, int r_hi) {
    return (uint16_t)((c_lo & 15) | ((c_hi & 15) << 4) | ((r_lo & 15) << 8) | ((r_hi & 15) << 12));
}
__device__ __forceinline__ void unpack_cull(uint16_t v, int& c_lo, int& c_hi, int& r_lo, int& r_hi) {
    c_lo = v & 15;
    c_hi = (v >> 4) & 15;
    r_lo = (v >> 8) & 15;
    r_hi = v >> 12;
}

constexpr int kFwd16Threads = 128;  // 4 warps, each covering the whole tile for a quarter of the list
constexpr int kFwd16Batch = 256;

// Forward of 16x16 tiles.  Every warp covers all 256 pixels of the tile (lane
// L: column L & 15, rows (L >> 4) + 2k), so a warp evaluates one record at a
// time with no per-warp work list.  A record reaches a contiguous range
// [g0, g1] of the four 4-row groups (its culling box narrowed to the ellipse,
// tile_cull); staging (two records per thread, batches of 256) sorts each
// batch by that range, one of ten patterns, with a deterministic counting
// sort (ballots, slot order) and stores each record at its slot, and the
// warps take every fourth record of each pattern's run through a loop
// compiled for that pattern: no per-record group tests, straight-line group
// bodies.  Each
// group is 2 pixels per lane in packed pairs.  The four warps' partial sums
// are added in shared memory at the end.  Nine resident CTAs per SM (56
// registers) measured fastest: 23.71 ms at config 2 against 24.14 ms for
// eight, 24.71 ms for ten and more for twelve or the compiler's own 63.
__global__ void __launch_bounds__(kFwd16Threads, 9)
raster_fwd16_kernel(const float4* __restrict__ splats, const int32_t* __restrict__ offsets,
                    const int32_t* __restrict__ flatten_ids, int64_t n_keys, int64_t n_isects,
                    int64_t n_splats, uint32_t W, uint32_t H, uint32_t ntx, uint32_t nty,
                    float* __restrict__ image, uint16_t* __restrict__ cull_out) {
    // staged records in pattern order
    __shared__ float4 s_p[kFwd16Batch];  // mx, my, A = a/2 log2e, B = b log2e
    __shared__ float4 s_q[kFwd16Batch];  // C = c/2 log2e, w*mu, s_thr, 0
    __shared__ float s_acc[kFwd16Threads / 32][256];
    __shared__ int s_wc[2 * kFwd16Threads / 32][11];  // per-(half, warp) pattern counts, then slots
    __shared__ int s_off[12];                     // first slot of each pattern's run

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t cam = blockIdx.z;
    const int X0 = blockIdx.x * 16, Y0 = blockIdx.y * 16;
    const int64_t key = cam * (int64_t)ntx * nty + (int64_t)blockIdx.y * ntx + blockIdx.x;
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (R2S_DBG_BAD(start >= 0 && start <= end && end <= n_isects, R2S_DBG_TILE_RANGE))
        return;  // uniform over the CTA
    const int cmax = min(15, (int)W - 1 - X0), rmax = min(15, (int)H - 1 - Y0);

    const int col = lane & 15, rb = lane >> 4;
    const float px = (float)(X0 + col) + 0.5f;
    float2 py[4];
#pragma unroll
    for (int g = 0; g < 4; ++g)
        py[g] = make_float2((float)(Y0 + 4 * g + rb) + 0.5f, (float)(Y0 + 4 * g + rb) + 2.5f);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};

    for (int b0 = start; b0 < end; b0 += kFwd16Batch) {
        const int n = min(kFwd16Batch, end - b0);
        __syncthreads();
        int pid[2] = {10, 10};  // row-group pattern of the records; 10: no pixel
        float4 sp[2], sq[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int ti = k * kFwd16Threads + tid;
            if (ti >= n) continue;
            const int64_t g = flatten_ids[b0 + ti];
            if (R2S_DBG_BAD(g >= 0 && g < n_splats, R2S_DBG_RECORD_ID)) continue;
            const float4 p = splats[2 * g];
            const float4 q = splats[2 * g + 1];
            int c_lo, c_hi, r_lo, r_hi;
            cull_range(p.x, q.z, (float)X0, cmax, c_lo, c_hi);
            cull_range(p.y, q.w, (float)Y0, rmax, r_lo, r_hi);
            const float s_thr = s_threshold(q.y);
            tile_cull(p.x, p.y, p.z, p.w, q.x, s_thr, (float)X0, (float)Y0, c_lo, c_hi, r_lo,
                      r_hi);
            if (c_lo <= c_hi && r_lo <= r_hi) {  // (g0, g1) -> 0..9, g0 <= g1
                const int g0 = r_lo >> 2, g1 = r_hi >> 2;
                pid[k] = g0 * 4 + g1 - (g0 * (g0 + 1)) / 2;
            }
            if (cull_out != nullptr) cull_out[b0 + ti] = pack_cull(c_lo, c_hi, r_lo, r_hi);
            // negated coefficients: the packed chain yields -s exactly, so ex2
            // takes it as is; the cut-off test compares the bits of -s as
            // signed integers against INT_MIN + bits(s_thr)
            sp[k] = make_float4(p.x, p.y, -0.5f * kLog2e * p.z, -kLog2e * p.w);
            sq[k] = make_float4(-0.5f * kLog2e * q.x, q.y,
                                __uint_as_float(__float_as_uint(s_thr) ^ 0x80000000u), 0.f);
        }
        {  // deterministic counting sort of the batch by pattern (ballots, slot order)
            const unsigned below = (1u << lane) - 1u;
            int rank[2] = {0, 0};
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
                for (int p = 0; p < 11; ++p) {
                    const unsigned bm = __ballot_sync(0xffffffffu, pid[k] == p);
                    if (pid[k] == p) rank[k] = __popc(bm & below);
                    if (lane == 0) s_wc[k * (kFwd16Threads / 32) + warp][p] = __popc(bm);
                }
            __syncthreads();
            if (tid == 0) {
                int run = 0;
                for (int p = 0; p < 11; ++p) {
                    s_off[p] = run;
                    for (int w = 0; w < 2 * kFwd16Threads / 32; ++w) {
                        const int c = s_wc[w][p];
                        s_wc[w][p] = run;
                        run += c;
                    }
                }
                s_off[11] = run;
            }
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if (pid[k] < 10) {
                    const int slot = s_wc[k * (kFwd16Threads / 32) + warp][pid[k]] + rank[k];
                    s_p[slot] = sp[k];
                    s_q[slot] = sq[k];
                }
        }
        __syncthreads();
        auto run = [&](auto c0, auto c1, int b, int e) {
            constexpr int G0 = decltype(c0)::value, G1 = decltype(c1)::value;
            for (int i = b + warp; i < e; i += kFwd16Threads / 32) {
                const float4 Q = s_q[i];
                const float4 P = s_p[i];
                const int thr_n = __float_as_int(Q.z);
                const float dx = px - P.x;
                const float xx = P.z * dx * dx;
                const float xy = P.w * dx;
                const float2 xx2 = make_float2(xx, xx), xy2 = make_float2(xy, xy);
                const float2 C2 = make_float2(Q.x, Q.x), nmy = make_float2(-P.y, -P.y);
#pragma unroll
                for (int g = G0; g <= G1; ++g) {
                    const float2 dy = fadd2(py[g], nmy);
                    const float2 sn = ffma2(dy, ffma2(C2, dy, xy2), xx2);  // -s
                    const float e0 = exp2f(sn.x), e1 = exp2f(sn.y);
                    if (__float_as_int(sn.x) <= thr_n) acc[2 * g] = fmaf(Q.y, e0, acc[2 * g]);
                    if (__float_as_int(sn.y) <= thr_n) acc[2 * g + 1] = fmaf(Q.y, e1, acc[2 * g + 1]);
                }
            }
        };
        using I0 = std::integral_constant<int, 0>;
        using I1 = std::integral_constant<int, 1>;
        using I2 = std::integral_constant<int, 2>;
        using I3 = std::integral_constant<int, 3>;
        run(I0{}, I0{}, s_off[0], s_off[1]);
        run(I0{}, I1{}, s_off[1], s_off[2]);
        run(I0{}, I2{}, s_off[2], s_off[3]);
        run(I0{}, I3{}, s_off[3], s_off[4]);
        run(I1{}, I1{}, s_off[4], s_off[5]);
        run(I1{}, I2{}, s_off[5], s_off[6]);
        run(I1{}, I3{}, s_off[6], s_off[7]);
        run(I2{}, I2{}, s_off[7], s_off[8]);
        run(I2{}, I3{}, s_off[8], s_off[9]);
        run(I3{}, I3{}, s_off[9], s_off[10]);
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        s_acc[warp][(4 * g + rb) * 16 + col] = acc[2 * g];
        s_acc[warp][(4 * g + rb + 2) * 16 + col] = acc[2 * g + 1];
    }
    __syncthreads();
    float* out = image + cam * (int64_t)H * W;
    for (int p = tid; p < 256; p += kFwd16Threads) {
        const int r = p >> 4, c = p & 15;
        const float v = (s_acc[0][p] + s_acc[1][p]) + (s_acc[2][p] + s_acc[3][p]);
        if (c <= cmax && r <= rmax &&
            !R2S_DBG_BAD(Y0 + r < (int)H && X0 + c < (int)W, R2S_DBG_PIXEL))
            out[(int64_t)(Y0 + r) * W + X0 + c] = v;
    }
}

constexpr int kBwd16Threads = 256;  // one (view, tile) per CTA, one Gaussian record per thread
constexpr int kBwd16Batch = 1024;   // records staged and sorted per batch (32 groups of 32)

// Backward statistics of 16x16 tiles, one Gaussian record per thread.
//
// The tile's upstream gradient sits in shared memory, row-major and
// column-major.  Staging narrows each record's culling box to the ellipse
// inside the tile (tile_cull, or the ranges the forward of the same binning
// wrote to its culling table) and picks the shorter axis to walk: a record
// with fewer columns than rows is stored transposed (x <-> y, a <-> c, its
// index flagged in the sign bit) and walks the columns of the column-major
// copy; its moments are swapped back at the end.  The CTA stages the tile's
// list in batches of 1024 records and orders each batch with a counting sort
// on the walked range (first, last index), so that each group of 32 lanes
// walks similar ranges: a warp executes the union of its lanes' ranges.  Warp w takes the sorted groups
// w, w+8, w+16, w+24, which spreads short and long row ranges evenly over the
// warps.  Per pixel: sigma from the column offset dx (exact per column) and
// the row terms B dy, C dy^2, one ex2, and packed updates of the per-column
// sums Col_c = sum_rows v e and the row sums sum_c v e, sum_c v e dx.  The
// moments follow without cancellation:
//   S0 = sum_c Col_c, Sx = sum_c Col_c dx_c, Sxx = sum_c Col_c dx_c^2,
//   Sy = sum_r dy_r R0_r, Syy = sum_r dy_r^2 R0_r, Sxy = sum_r dy_r R1_r.
// No cross-lane reduction is needed; each record adds its eight values with
// two vector reductions.
template <bool WITH_ABS>
__global__ void __launch_bounds__(kBwd16Threads)
raster_bwd16_kernel(const float4* __restrict__ splats, const int32_t* __restrict__ offsets,
                    const int32_t* __restrict__ flatten_ids, int64_t n_keys, int64_t n_isects,
                    int64_t n_splats, const float* __restrict__ v_image, uint32_t W, uint32_t H,
                    uint32_t ntx,
                    uint32_t nty, const uint16_t* __restrict__ cull_in,
                    float* __restrict__ stats) {
    // upstream gradient of the tile, row-major and (16 floats further, so
    // that the two copies sit in different banks) column-major
    __shared__ __align__(16) float s_vv[2 * 256 + 16];
    float* const s_v = s_vv;
    float* const s_vT = s_vv + 256 + 16;
    __shared__ float4 s_p[kBwd16Batch];
    __shared__ float4 s_q[kBwd16Batch];
    __shared__ int32_t s_g[kBwd16Batch];
    __shared__ uint8_t s_rows[kBwd16Batch];  // first row | last row << 4
    __shared__ uint16_t s_perm[kBwd16Batch];
    __shared__ int32_t s_cnt[257];
    __shared__ int32_t s_wsum[kBwd16Threads / 32];
    __shared__ uint16_t s_fix[kBwd16Batch];  // records with a pixel in the cut-off band
    __shared__ int s_nfix;
    __shared__ float s_fx[kBwd16Threads / 32][8];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t cam = blockIdx.z;
    const int X0 = blockIdx.x * 16, Y0 = blockIdx.y * 16;
    const int64_t key = cam * (int64_t)ntx * nty + (int64_t)blockIdx.y * ntx + blockIdx.x;
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (start >= end) return;
    if (R2S_DBG_BAD(start >= 0 && end <= n_isects, R2S_DBG_TILE_RANGE)) return;  // CTA-uniform
    const int cmax = min(15, (int)W - 1 - X0), rmax = min(15, (int)H - 1 - Y0);
    {
        const float* vc = v_image + cam * (int64_t)H * W;
        const int r = tid >> 4, c = tid & 15;
        const float v = (c <= cmax && r <= rmax) ? vc[(int64_t)(Y0 + r) * W + X0 + c] : 0.f;
        s_v[tid] = v;
        s_vT[c * 16 + r] = v;
    }
    const float X0f = (float)X0, Y0f = (float)Y0;

    for (int base = start; base < end; base += kBwd16Batch) {
        // stage the batch; bucket 256 holds records that reach no pixel
        s_cnt[tid] = 0;
        if (tid == 0) s_cnt[256] = 0, s_nfix = 0;
        __syncthreads();
        constexpr int kPer = kBwd16Batch / kBwd16Threads;
        int bucket[kPer], rank[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int idx = k * kBwd16Threads + tid;
            const int i = base + idx;
            int32_t g = 0;
            float4 p = make_float4(0.f, 0.f, 0.f, 0.f), q = p;
            int rows = 0x0f;  // empty: first row 15 > last row 0
            bucket[k] = 256;
            if (i < end && R2S_DBG_BAD(flatten_ids[i] >= 0 && flatten_ids[i] < n_splats,
                                        R2S_DBG_RECORD_ID)) {
                // checked build: an id outside the records stays unstaged
            } else if (i < end) {
                g = flatten_ids[i];
                p = splats[2 * (int64_t)g];
                q = splats[2 * (int64_t)g + 1];
                int c_lo, c_hi, r_lo, r_hi;
                if (cull_in != nullptr) {  // the forward's ranges for this record
                    unpack_cull(cull_in[i], c_lo, c_hi, r_lo, r_hi);
                } else {
                    cull_range(p.x, q.z, X0f, cmax, c_lo, c_hi);
                    cull_range(p.y, q.w, Y0f, rmax, r_lo, r_hi);
                    tile_cull(p.x, p.y, p.z, p.w, q.x, s_threshold(q.y), X0f, Y0f, c_lo, c_hi,
                              r_lo, r_hi);
                }
                if (c_lo <= c_hi && r_lo <= r_hi) {
                    // cut-off band of the record: a pixel near the cut-off lies
                    // inside the record's culling extents (q.z, q.w) and the tile
                    const float Dx = fminf(q.z, fmaxf(fabsf((X0f + 0.5f) - p.x),
                                                      fabsf((X0f + 15.5f) - p.x)));
                    const float Dy = fminf(q.w, fmaxf(fabsf((Y0f + 0.5f) - p.y),
                                                      fabsf((Y0f + 15.5f) - p.y)));
                    const float band = cutoff_band(p.z, p.w, q.x, s_threshold(q.y), Dx, Dy);
                    if (c_hi - c_lo < r_hi - r_lo) {
                        // fewer columns than rows: walk the columns, with the
                        // record transposed (x <-> y, a <-> c) and flagged in
                        // the sign bit of its index
                        const float a = p.z;
                        p = make_float4(p.y, p.x, q.x, p.w);
                        q = make_float4(a, q.y, q.w, q.z);
                        r_lo = c_lo;
                        r_hi = c_hi;
                        g = (int32_t)((uint32_t)g | 0x80000000u);
                    }
                    q.z = band;
                    bucket[k] = r_lo * 16 + r_hi;
                    rows = r_lo | (r_hi << 4);
                }
            }
            s_g[idx] = g;
            s_p[idx] = p;
            s_q[idx] = q;
            s_rows[idx] = (uint8_t)rows;
            rank[k] = atomicAdd(&s_cnt[bucket[k]], 1);
        }
        __syncthreads();
        {
            const int c = s_cnt[tid];
            const int incl = warp_inclusive_scan(c);
            if (lane == 31) s_wsum[warp] = incl;
            __syncthreads();
            int wbase = 0;
#pragma unroll
            for (int w = 0; w < kBwd16Threads / 32; ++w) wbase += w < warp ? s_wsum[w] : 0;
            s_cnt[tid] = wbase + incl - c;
            if (tid == kBwd16Threads - 1) s_cnt[256] = wbase + incl;  // after every live record
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            s_perm[s_cnt[bucket[k]] + rank[k]] = (uint16_t)(k * kBwd16Threads + tid);
        __syncthreads();
        const int n_groups = (min(kBwd16Batch, end - base) + 31) >> 5;

        for (int grp = warp; grp < n_groups; grp += kBwd16Threads / 32) {
            const int idx = s_perm[grp * 32 + lane];
            int r_lo = s_rows[idx] & 15, r_hi = s_rows[idx] >> 4;
            const bool live = r_lo <= r_hi;
            if (!live) r_lo = 16, r_hi = -1;
            const int row0 = __reduce_min_sync(0xffffffffu, r_lo);
            const int row1 = __reduce_max_sync(0xffffffffu, r_hi);
            if (row0 > row1) continue;  // warp-uniform
            const int32_t gi = s_g[idx];
            const bool tr = gi < 0;  // transposed record: walks columns
            const int64_t g = gi & 0x7fffffff;
            const float Uo = tr ? Y0f : X0f, Vo = tr ? X0f : Y0f;
            const float* const vb = tr ? s_vT : s_v;
            const float4 p = s_p[idx], q = s_q[idx];

            // negated coefficients; the packed chain yields z = s_thr - s (the
            // threshold enters the last FMA through the row term): a pixel is
            // kept when z >= 0 and lies in the cut-off band when |z| <= q.z
            // (tested once per record on the smallest |z| of the walk).  The
            // sums run over 2^z = 2^s_thr e^-sigma and are scaled back by
            // 2^-s_thr once per record.
            const float A = -0.5f * kLog2e * p.z, B = -kLog2e * p.w, Cc = -0.5f * kLog2e * q.x;
            const float s_thr = s_threshold(q.y);
            float z_min = CUDART_INF_F;
            const float2 A2 = make_float2(A, A);
            const float2 a2 = make_float2(p.z, p.z), b2 = make_float2(p.w, p.w);
            float2 dx[8], col[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                dx[j] = make_float2((Uo + (2 * j + 0.5f)) - p.x, (Uo + (2 * j + 1.5f)) - p.x);
                col[j] = make_float2(0.f, 0.f);
            }
            float Sy = 0.f, Syy = 0.f, Sxy = 0.f, Ax = 0.f, Ay = 0.f;
            for (int r = row0; r <= row1; ++r) {
                const bool rin = r >= r_lo && r <= r_hi;
                const float dy = (Vo + ((float)r + 0.5f)) - p.y;
                const float by = B * dy, cyy = fmaf(Cc * dy, dy, s_thr);
                const float2 by2 = make_float2(by, by), cyy2 = make_float2(cyy, cyy);
                const float bdy = p.w * dy, cdy = q.x * dy;
                const float2 bdy2 = make_float2(bdy, bdy), cdy2 = make_float2(cdy, cdy);
                const float4* vr = reinterpret_cast<const float4*>(vb + r * 16);
                float2 r0 = make_float2(0.f, 0.f), r1 = r0;
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 v4 = vr[j4];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int j = 2 * j4 + h;
                        const float2 v2 = h ? make_float2(v4.z, v4.w) : make_float2(v4.x, v4.y);
                        const float2 t = ffma2(A2, dx[j], by2);
                        const float2 z = ffma2(dx[j], t, cyy2);  // s_thr - s
                        float e0 = exp2f(z.x), e1 = exp2f(z.y);
                        z_min = fminf(z_min, fminf(fabsf(z.x), fabsf(z.y)));
                        e0 = (rin && z.x >= 0.f) ? e0 : 0.f;
                        e1 = (rin && z.y >= 0.f) ? e1 : 0.f;
                        const float2 ve = fmul2(v2, make_float2(e0, e1));
                        col[j] = fadd2(col[j], ve);
                        r0 = fadd2(r0, ve);
                        r1 = ffma2(ve, dx[j], r1);
                        if constexpr (WITH_ABS) {
                            const float2 qx = ffma2(a2, dx[j], bdy2);  // a dx + b dy
                            const float2 qy = ffma2(b2, dx[j], cdy2);  // b dx + c dy
                            Ax = fmaf(fabsf(ve.x), fabsf(qx.x), Ax);
                            Ax = fmaf(fabsf(ve.y), fabsf(qx.y), Ax);
                            Ay = fmaf(fabsf(ve.x), fabsf(qy.x), Ay);
                            Ay = fmaf(fabsf(ve.y), fabsf(qy.y), Ay);
                        }
                    }
                }
                const float R0 = r0.x + r0.y, R1 = r1.x + r1.y;
                Sy = fmaf(dy, R0, Sy);
                Syy = fmaf(dy * dy, R0, Syy);
                Sxy = fmaf(dy, R1, Sxy);
            }
            if (!live) continue;
            if (!(z_min > q.z)) s_fix[atomicAdd(&s_nfix, 1)] = (uint16_t)idx;  // also NaN
            float S0 = 0.f, Sx = 0.f, Sxx = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                S0 += col[j].x + col[j].y;
                const float2 cx = fmul2(col[j], dx[j]);
                Sx += cx.x + cx.y;
                Sxx = fmaf(cx.x, dx[j].x, Sxx);
                Sxx = fmaf(cx.y, dx[j].y, Sxx);
            }
            {  // 2^-s_thr: the sums back to e^-sigma
                const float k = exp2f(-s_thr);
                S0 *= k, Sx *= k, Sy *= k, Sxx *= k, Sxy *= k, Syy *= k, Ax *= k, Ay *= k;
            }
            if (tr) {  // back to image axes
                float t = Sx;
                Sx = Sy, Sy = t;
                t = Sxx;
                Sxx = Syy, Syy = t;
                t = Ax;
                Ax = Ay, Ay = t;
            }
            float* st = stats + g * 8;
            red_add_v4(st, S0, Sx, Sy, Sxx);
            if constexpr (WITH_ABS)
                red_add_v4(st + 4, Sxy, Syy, Ax, Ay);
            else
                red_add_v2(st + 4, Sxy, Syy);
        }
        __syncthreads();
        // records with a pixel in the cut-off band: every pixel of the walk
        // re-decided by the reference's own test, one pixel per thread; where
        // the decisions differ, the pixel's moments are added or taken back
        const int n_fix = s_nfix;
        for (int f = 0; f < n_fix; ++f) {
            const int idx = s_fix[f];
            const int32_t gi = s_g[idx];
            const bool tr = gi < 0;
            const float4 p = s_p[idx], q = s_q[idx];
            const int r_lo = s_rows[idx] & 15, r_hi = s_rows[idx] >> 4;
            const int rw = tid >> 4, cw = tid & 15;  // walked row and column
            // the main loop's fast decision, operation for operation
            const float Uo = tr ? Y0f : X0f, Vo = tr ? X0f : Y0f;
            const float A = -0.5f * kLog2e * p.z, B = -kLog2e * p.w, Cc = -0.5f * kLog2e * q.x;
            const float s_thr = s_threshold(q.y);
            const float dx = (Uo + ((float)cw + 0.5f)) - p.x;
            const float dy = (Vo + ((float)rw + 0.5f)) - p.y;
            const float by = B * dy, cyy = fmaf(Cc * dy, dy, s_thr);
            const float z = fmaf(dx, fmaf(A, dx, by), cyy);
            const bool fast = rw >= r_lo && rw <= r_hi && z >= 0.f;
            // the reference's decision, in image axes
            const int i = tr ? cw : rw, j = tr ? rw : cw;
            const bool inside = i <= rmax && j <= cmax;
            const float mx = tr ? p.y : p.x, my = tr ? p.x : p.y;
            const float ca = tr ? q.x : p.z, cc = tr ? p.z : q.x;
            // outside the band the sign of z is the reference's decision
            const bool exact =
                inside && (fabsf(z) > q.z ? z >= 0.f
                                          : ref_keep2d(ca, p.w, cc, q.y,
                                                       (X0f + ((float)j + 0.5f)) - mx,
                                                       (Y0f + ((float)i + 0.5f)) - my));
            const bool diff = inside && fast != exact;
            float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (diff) {
                const float sgn = exact ? 1.0f : -1.0f;
                const float ve = (tr ? s_vT : s_v)[rw * 16 + cw] * (exp2f(z) * exp2f(-s_thr));
                m[0] = sgn * ve;
                m[1] = sgn * ve * dx;
                m[2] = sgn * ve * dy;
                m[3] = sgn * ve * dx * dx;
                m[4] = sgn * ve * dx * dy;
                m[5] = sgn * ve * dy * dy;
                m[6] = sgn * fabsf(ve) * fabsf(fmaf(p.z, dx, p.w * dy));
                m[7] = sgn * fabsf(ve) * fabsf(fmaf(p.w, dx, q.x * dy));
                if (tr) {  // back to image axes
                    float t = m[1];
                    m[1] = m[2], m[2] = t;
                    t = m[3];
                    m[3] = m[5], m[5] = t;
                    t = m[6];
                    m[6] = m[7], m[7] = t;
                }
            }
            if (!__syncthreads_or(diff)) continue;  // CTA-uniform
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float v = warp_sum(m[k]);
                if (lane == 0) s_fx[warp][k] = v;
            }
            __syncthreads();
            // stats layout: S0, Sx, Sy, Sxx, Sxy, Syy (, Ax, Ay)
            if (tid < (WITH_ABS ? 8 : 6)) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kBwd16Threads / 32; ++w) v += s_fx[w][tid];
                atomicAdd(stats + (gi & 0x7fffffff) * (int64_t)8 + tid, v);
            }
        }
        __syncthreads();
    }
}

// Splat records from the reference-layout inputs (rasterizer wrappers).
__global__ void pack_splats_kernel(const float* __restrict__ means2d,
                                   const float* __restrict__ conics, const float* __restrict__ opac,
                                   const float* __restrict__ mus, int64_t total,
                                   float4* __restrict__ splats) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const float a = conics[3 * i], b = conics[3 * i + 1], c = conics[3 * i + 2];
    const float wmu = opac[i] * mus[i];
    float ex, ey;
    conic_cull_extents(a, b, c, wmu, kAlphaMin2D, ex, ey);
    splats[2 * i] = make_float4(means2d[2 * i], means2d[2 * i + 1], a, b);
    splats[2 * i + 1] = make_float4(c, wmu, ex, ey);
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
int check_tiles(int64_t C, uint32_t W, uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty) {
    R2S_REQUIRE(T > 0 && T * T <= 1024, "tile_size must be positive with tile_size**2 <= 1024");
    R2S_REQUIRE(ntx > 0 && nty > 0, "rasterize: tile grid must be non-empty");
    R2S_REQUIRE((uint64_t)ntx * T >= W && (uint64_t)nty * T >= H,
                "rasterize: tile grid does not cover the image");
    R2S_REQUIRE(C <= 65535 && nty <= 65535, "rasterize: too many views or tile rows for one launch");
    return R2S_OK;
}

int launch_raster_fwd16(const float4* splats, const int32_t* offsets, const int32_t* flatten_ids,
                        int64_t C, int64_t N, int64_t n_isects, uint32_t W, uint32_t H,
                        uint32_t ntx, uint32_t nty, float* image, cudaStream_t stream,
                        uint16_t* cull_out = nullptr) {
    const dim3 grid(ntx, nty, (unsigned)C);
    raster_fwd16_kernel<<<grid, kFwd16Threads, 0, stream>>>(
        splats, offsets, flatten_ids, C * (int64_t)ntx * nty, n_isects, C * N, W, H, ntx, nty,
        image, cull_out);
    return check_launch("rasterize_to_pixels_fwd");
}

int launch_raster_bwd16(const float4* splats, const int32_t* offsets, const int32_t* flatten_ids,
                        const float* v_image, int64_t C, int64_t N, int64_t n_isects, uint32_t W,
                        uint32_t H, uint32_t ntx, uint32_t nty, int with_abs, float* stats,
                        cudaStream_t stream, const uint16_t* cull_in = nullptr) {
    cudaMemsetAsync(stats, 0, (size_t)C * N * 8 * sizeof(float), stream);
    if (n_isects == 0) return check_launch("rasterize_to_pixels_bwd");
    const dim3 grid(ntx, nty, (unsigned)C);
    if (with_abs)
        raster_bwd16_kernel<true><<<grid, kBwd16Threads, 0, stream>>>(
            splats, offsets, flatten_ids, C * (int64_t)ntx * nty, n_isects, C * N, v_image, W, H,
            ntx, nty, cull_in, stats);
    else
        raster_bwd16_kernel<false><<<grid, kBwd16Threads, 0, stream>>>(
            splats, offsets, flatten_ids, C * (int64_t)ntx * nty, n_isects, C * N, v_image, W, H,
            ntx, nty, cull_in, stats);
    return check_launch("rasterize_to_pixels_bwd");
}

template <typename S, bool SPLATS>
int launch_raster_fwd(const RasterSrc<S>& src, const int32_t* offsets, const int32_t* flatten_ids,
                      int64_t C, int64_t n_isects, uint32_t W, uint32_t H, uint32_t T,
                      uint32_t ntx, uint32_t nty, S* image, cudaStream_t stream) {
    TileGeom geo;
    geo.T = (int)T;
    geo.nthr = (int)(T * T);
    geo.blocked = (T % 8) == 0;
    const int n_warps = (geo.nthr + 31) / 32;
    const size_t smem = 6 * al16((size_t)geo.nthr * sizeof(S)) + al16((size_t)geo.nthr * 4) +
                        (size_t)n_warps * 16;
    auto kern = raster_fwd_kernel<S, SPLATS>;
    if (int rc = set_dynamic_smem(kern, smem, "rasterize")) return rc;
    const dim3 grid(ntx, nty, (unsigned)C);
    kern<<<grid, geo.nthr, smem, stream>>>(src, offsets, flatten_ids, C * (int64_t)ntx * nty,
                                           n_isects, W, H, geo, ntx, nty, image);
    return check_launch("rasterize_to_pixels_fwd");
}

template <typename S, bool SPLATS, int EXPMODE>
int launch_raster_bwd(const RasterSrc<S>& src, const int32_t* offsets, const int32_t* flatten_ids,
                      const S* v_image, int64_t C, int64_t N, int64_t n_isects, uint32_t W,
                      uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty, int with_abs, S* stats,
                      cudaStream_t stream) {
    cudaMemsetAsync(stats, 0, (size_t)C * N * 8 * sizeof(S), stream);
    if (n_isects == 0) return check_launch("rasterize_to_pixels_bwd");
    // at least one warp; 4 warps for 16x16 tiles
    int nthr = (int)(T * T);
    nthr = nthr < 128 ? 128 : (nthr > 256 ? 256 : nthr);
    nthr = (nthr + 31) / 32 * 32;
    const size_t smem = (size_t)T * (T + 1) * sizeof(S) + (size_t)nthr * (6 * sizeof(S) + 8);
    auto kern = raster_bwd_kernel<S, SPLATS, EXPMODE>;
    if (int rc = set_dynamic_smem(kern, smem, "rasterize")) return rc;
    const dim3 grid(ntx, nty, (unsigned)C);
    kern<<<grid, nthr, smem, stream>>>(src, offsets, flatten_ids, C * (int64_t)ntx * nty, n_isects,
                                       v_image, W, H, (int)T, ntx, nty, with_abs, stats);
    return check_launch("rasterize_to_pixels_bwd");
}

}  // namespace r2s

using namespace r2s;

extern "C" int r2s_rasterize_to_pixels_fwd(int dtype, const void* means2d, const void* conics,
                                           const void* opacities, const void* mus,
                                           const int32_t* offsets, const int32_t* flatten_ids,
                                           int64_t C, int64_t N, int64_t n_isects, uint32_t W,
                                           uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty,
                                           void* splat_scratch, void* image,
                                           r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0 && n_isects >= 0, "rasterize_to_pixels_fwd: negative size");
    const size_t es = dtype == R2S_F64 ? 8 : 4;
    if (C == 0 || (int64_t)W * H == 0) return R2S_OK;
    if (N == 0 || n_isects == 0) {
        cudaMemsetAsync(image, 0, (size_t)C * W * H * es, stream);
        return check_launch("rasterize_to_pixels_fwd");
    }
    if (int rc = check_tiles(C, W, H, T, ntx, nty)) return rc;
    if (dtype == R2S_F32 && T == 16 && splat_scratch != nullptr) {
        pack_splats_kernel<<<grid_for(C * N), kThreads, 0, stream>>>(
            (const float*)means2d, (const float*)conics, (const float*)opacities,
            (const float*)mus, C * N, (float4*)splat_scratch);
        return launch_raster_fwd16((const float4*)splat_scratch, offsets, flatten_ids, C, N,
                                   n_isects, W, H, ntx, nty, (float*)image, stream);
    }
    return R2S_DTYPE_DISPATCH(dtype, "rasterize_to_pixels_fwd", [&] {
        RasterSrc<scalar_t> src{nullptr, (const scalar_t*)means2d, (const scalar_t*)conics,
                                (const scalar_t*)opacities, (const scalar_t*)mus};
        return launch_raster_fwd<scalar_t, false>(src, offsets, flatten_ids, C, n_isects, W, H, T,
                                                  ntx, nty, (scalar_t*)image, stream);
    });
}

extern "C" int r2s_rasterize_to_pixels_bwd(int dtype, int mode, const void* means2d,
                                           const void* conics, const void* opacities,
                                           const void* mus, const int32_t* offsets,
                                           const int32_t* flatten_ids, const void* v_image,
                                           int64_t C, int64_t N, int64_t n_isects, uint32_t W,
                                           uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty,
                                           void* splat_scratch, void* stats, void* v_abs,
                                           void* v_m2, void* v_con, void* v_op, void* v_mu,
                                           r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0 && n_isects >= 0, "rasterize_to_pixels_bwd: negative size");
    R2S_REQUIRE(mode == 0 || mode == 1, "rasterize_to_pixels_bwd: mode must be 0 or 1");
    const int64_t total = C * N;
    const size_t es = dtype == R2S_F64 ? 8 : 4;
    if (total == 0) return R2S_OK;
    if (n_isects == 0 || (int64_t)W * H == 0) {
        cudaMemsetAsync(v_m2, 0, total * 2 * es, stream);
        cudaMemsetAsync(v_con, 0, total * 3 * es, stream);
        cudaMemsetAsync(v_op, 0, total * es, stream);
        cudaMemsetAsync(v_mu, 0, total * es, stream);
        if (v_abs) cudaMemsetAsync(v_abs, 0, total * 2 * es, stream);
        return check_launch("rasterize_to_pixels_bwd");
    }
    if (int rc = check_tiles(C, W, H, T, ntx, nty)) return rc;
    return R2S_DTYPE_DISPATCH(dtype, "rasterize_to_pixels_bwd", [&] {
        RasterSrc<scalar_t> src{nullptr, (const scalar_t*)means2d, (const scalar_t*)conics,
                                (const scalar_t*)opacities, (const scalar_t*)mus};
        int rc;
        if (std::is_same<scalar_t, float>::value && T == 16 && splat_scratch != nullptr) {
            pack_splats_kernel<<<grid_for(total), kThreads, 0, stream>>>(
                (const float*)means2d, (const float*)conics, (const float*)opacities,
                (const float*)mus, total, (float4*)splat_scratch);
            rc = launch_raster_bwd16((const float4*)splat_scratch, offsets, flatten_ids,
                                     (const float*)v_image, C, N, n_isects, W, H, ntx, nty,
                                     v_abs != nullptr, (float*)stats, stream);
        } else rc = mode == 0
                     ? launch_raster_bwd<scalar_t, false, 0>(src, offsets, flatten_ids,
                                                             (const scalar_t*)v_image, C, N,
                                                             n_isects, W, H, T, ntx, nty,
                                                             v_abs != nullptr, (scalar_t*)stats,
                                                             stream)
                     : launch_raster_bwd<scalar_t, false, 1>(src, offsets, flatten_ids,
                                                             (const scalar_t*)v_image, C, N,
                                                             n_isects, W, H, T, ntx, nty,
                                                             v_abs != nullptr, (scalar_t*)stats,
                                                             stream);
        if (rc) return rc;
        raster_unpack_kernel<scalar_t><<<grid_for(total), kThreads, 0, stream>>>(
            (const scalar_t*)stats, (const scalar_t*)conics, (const scalar_t*)opacities,
            (const scalar_t*)mus, total, (scalar_t*)v_abs, (scalar_t*)v_m2, (scalar_t*)v_con,
            (scalar_t*)v_op, (scalar_t*)v_mu);
        return check_launch("rasterize_to_pixels_bwd");
    });
}

extern "C" int r2s_raster_splats_fwd_f32(const float* splats, const int32_t* offsets,
                                         const int32_t* flatten_ids, int64_t C, int64_t N,
                                         int64_t n_isects, uint32_t W, uint32_t H, uint32_t T,
                                         uint32_t ntx, uint32_t nty, float* image,
                                         uint16_t* cull_ranges, r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0 && n_isects >= 0, "raster_splats_fwd: negative size");
    R2S_REQUIRE(cull_ranges == nullptr || T == 16,
                "raster_splats_fwd: the culling table is built for 16-pixel tiles");
    if (C == 0 || (int64_t)W * H == 0) return R2S_OK;
    if (N == 0 || n_isects == 0) {
        cudaMemsetAsync(image, 0, (size_t)C * W * H * 4, stream);
        return check_launch("raster_splats_fwd");
    }
    if (int rc = check_tiles(C, W, H, T, ntx, nty)) return rc;
    if (T == 16)
        return launch_raster_fwd16((const float4*)splats, offsets, flatten_ids, C, N, n_isects, W,
                                   H, ntx, nty, image, stream, cull_ranges);
    RasterSrc<float> src{(const float4*)splats, nullptr, nullptr, nullptr, nullptr};
    return launch_raster_fwd<float, true>(src, offsets, flatten_ids, C, n_isects, W, H, T, ntx,
                                          nty, image, stream);
}

extern "C" int r2s_raster_splats_bwd_f32(const float* splats, const int32_t* offsets,
                                         const int32_t* flatten_ids, const float* v_image,
                                         int64_t C, int64_t N, int64_t n_isects, uint32_t W,
                                         uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty,
                                         int with_abs, const uint16_t* cull_ranges, float* stats,
                                         r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0 && n_isects >= 0, "raster_splats_bwd: negative size");
    R2S_REQUIRE(cull_ranges == nullptr || T == 16,
                "raster_splats_bwd: the culling table is built for 16-pixel tiles");
    if (C * N == 0) return R2S_OK;
    if ((int64_t)W * H == 0) {
        cudaMemsetAsync(stats, 0, (size_t)C * N * 32, stream);
        return check_launch("raster_splats_bwd");
    }
    if (int rc = check_tiles(C, W, H, T, ntx, nty)) return rc;
    if (T == 16)
        return launch_raster_bwd16((const float4*)splats, offsets, flatten_ids, v_image, C, N,
                                   n_isects, W, H, ntx, nty, with_abs, stats, stream, cull_ranges);
    RasterSrc<float> src{(const float4*)splats, nullptr, nullptr, nullptr, nullptr};
    return launch_raster_bwd<float, true, 0>(src, offsets, flatten_ids, v_image, C, N, n_isects, W,
                                             H, T, ntx, nty, with_abs, stats, stream);
}

// ===========================================================================
// Backward without caller scratch
// ===========================================================================
//
// Some host programs cannot give this library scratch memory: their device
// memory belongs to an allocator the plugin may not call (a fixed arena sized
// at start-up, or a framework that forbids cudaMalloc from inside its
// operators), and their binding passes only the operator's inputs and
// outputs.  For them the backward below keeps its scratch -- the
// per-(view, Gaussian) statistics and the packed splat records, 64 bytes per
// pair -- in one static device array of the library, so the call allocates
// nothing.  The array is part of the library's device image: every GPU that
// loads the library holds its 8 MiB until the process exits.
#include <cuda.h>
#include <mutex>

namespace r2s {
namespace {

constexpr int64_t kNoAllocMaxPairs = 131072;               // (view, Gaussian) pairs
constexpr size_t kNoAllocFloats = (size_t)kNoAllocMaxPairs * 16;  // 8 stats + 8 splat floats
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

// Driver entry points (taken through the runtime, so the library does not
// link libcuda): the current context and its process-unique id.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct NoAllocSlot {
    unsigned long long ctx_id;  // context the address belongs to (0: none yet)
    float* ptr;
};

std::mutex g_noalloc_mutex;
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices] = {};
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
bool g_ctx_fns_loaded = false;

int current_context_id(int dev, unsigned long long* id) {
    if (!g_ctx_fns_loaded) {
        g_ctx_fns_loaded = true;
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f);
    }
    if (g_ctx_get_current == nullptr || g_ctx_get_id == nullptr)
        return fail(R2S_ERR_CUDA, "noalloc: driver entry points cuCtxGetCurrent/cuCtxGetId missing");
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
        return fail(R2S_ERR_CUDA, "noalloc: no current CUDA context on device %d", dev);
    if (g_ctx_get_id(ctx, id) != CUDA_SUCCESS)
        return fail(R2S_ERR_CUDA, "noalloc: cuCtxGetId failed on device %d", dev);
    return R2S_OK;
}

// Device address of the static scratch on the current device.  The host-side
// name g_noalloc_scratch is only a stand-in for the symbol, so the address is
// looked up with cudaGetSymbolAddress while that device is current -- by the
// first call on each device -- and cached together with the id of the
// device's context.  A call from another context of the same ordinal (after
// cudaDeviceReset, or a context the caller made current) looks it up again,
// so a stale address is never used.
int noalloc_scratch(float** out) {
    int dev = -1;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess)
        return fail(R2S_ERR_CUDA, "noalloc: cudaGetDevice failed (%s)", cudaGetErrorString(err));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(R2S_ERR_UNSUPPORTED, "noalloc: device ordinal %d out of range", dev);
    // makes the device's primary context current if no context is (CUDA 12)
    err = cudaSetDevice(dev);
    if (err != cudaSuccess)
        return fail(R2S_ERR_CUDA, "noalloc: cudaSetDevice(%d) failed (%s)", dev,
                    cudaGetErrorString(err));
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    unsigned long long ctx_id = 0;
    if (int rc = current_context_id(dev, &ctx_id)) return rc;
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (slot.ptr == nullptr || slot.ctx_id != ctx_id) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess || p == nullptr)
            return fail(R2S_ERR_CUDA, "noalloc: cudaGetSymbolAddress failed on device %d (%s)", dev,
                        cudaGetErrorString(err));
        slot.ptr = static_cast<float*>(p);
        slot.ctx_id = ctx_id;
    }
    *out = slot.ptr;
    return R2S_OK;
}

}  // namespace
}  // namespace r2s

extern "C" int r2s_rasterize_to_pixels_bwd_noalloc_f32(
    int mode, const float* means2d, const float* conics, const float* opacities, const float* mus,
    const int32_t* offsets, const int32_t* flatten_ids, const float* v_image, int64_t C, int64_t N,
    int64_t n_isects, uint32_t W, uint32_t H, uint32_t T, uint32_t ntx, uint32_t nty,
    float* v_means2d_abs, float* v_means2d, float* v_conics, float* v_opacities, float* v_mus,
    r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "rasterize_to_pixels_bwd_noalloc: negative size");
    // C * N is compared by division: the product of two large sizes could
    // overflow int64 and wrap to a small value
    if (N > 0 && C > r2s::kNoAllocMaxPairs / N)
        return r2s::fail(R2S_ERR_UNSUPPORTED,
                         "rasterize_to_pixels_bwd_noalloc: %lld views x %lld Gaussians exceed the "
                         "static scratch of %lld (view, Gaussian) pairs; use "
                         "r2s_rasterize_to_pixels_bwd with caller scratch",
                         (long long)C, (long long)N, (long long)r2s::kNoAllocMaxPairs);
    float* scratch = nullptr;
    if (int rc = r2s::noalloc_scratch(&scratch)) return rc;
    float* stats = scratch;
    float* splats = scratch + (size_t)r2s::kNoAllocMaxPairs * 8;
    return r2s_rasterize_to_pixels_bwd(R2S_F32, mode, means2d, conics, opacities, mus, offsets,
                                       flatten_ids, v_image, C, N, n_isects, W, H, T, ntx, nty,
                                       splats, stats, v_means2d_abs, v_means2d, v_conics,
                                       v_opacities, v_mus, stream);
}

namespace r2s {
R2S_DBG_DEFINE_READER(debug_flags_raster)
}  // namespace r2s
