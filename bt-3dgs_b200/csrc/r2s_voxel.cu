// 3D voxelization forward and backward.
//
// Forward (reference: csrc/VoxelizeToVoxelsFwd.cu:68-221): one CTA per brick,
// one thread per voxel.  Threads are laid out x-fastest (the reference maps
// threadIdx.x to z, VoxelizeToVoxelsFwd.cu:98-108, which makes every store
// stride dim1*dim2); here a warp owns an 8x4x1 voxel row block, its stores
// are contiguous 32-byte segments, and it evaluates only the staged
// Gaussians whose cut-off box (alpha >= 1e-6) reaches its voxels.
//
// Backward (reference: csrc/VoxelizeToVoxelsBwd.cu:70-250 and 321-441): one
// CTA per brick with the brick's upstream gradient in shared memory; the
// float32 8^3 kernel gives each thread one record, narrows its culling box to
// the rows of each z-slice that the ellipsoid's slice can reach (brick_rows in
// r2s_cull.cuh), sorts the brick's records by their slice range, walks those
// rows and reduces ten moments of the contributing voxels,
//   S0 = sum v e, S_i = sum v e d_i, S_ij = sum v e d_i d_j (i <= j),
// which map linearly to the reference gradients:
//   v_means3d = w Q (Sx, Sy, Sz),   v_opacity = S0,
//   v_conics  = -w (Sxx/2, Sxy, Sxz, Syy/2, Syz, Szz/2).
//
// Z-slabs: the fused entry points take a brick-layer range and a volume
// pointer at the slab's first voxel row, so one GPU can voxelize only its
// slab of the global grid with keys and offsets of the global binning.
#include <math_constants.h>

#include <algorithm>

#include "r2s_common.cuh"
#include "r2s_cull.cuh"
#include "r2s_debug.cuh"
#include "r2s_cutoff.cuh"
#include "r2s_refexpr.cuh"

namespace r2s {

namespace {

constexpr float kLog2eV = 1.4426950408889634f;
constexpr float kAlphaMin3D = 1e-6f;

__host__ __device__ __forceinline__ size_t al16v(size_t x) { return (x + 15) & ~size_t(15); }

__device__ __forceinline__ void cull_range_v(float m, float e, float origin, int lim, int& lo,
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

// Cut-off extents of w*exp(-sigma) >= thresh from a 3D conic (symmetric
// inverse covariance, upper triangle c00 c01 c02 c11 c12 c22).
__device__ __forceinline__ void conic3_cull(const float q[6], float amp, float thresh, float e[3]) {
    bool nan = isnan(amp);
#pragma unroll
    for (int k = 0; k < 6; ++k) nan |= isnan(q[k]);
    if (nan) {
        e[0] = e[1] = e[2] = CUDART_INF_F;
        return;
    }
    const float aa = fabsf(amp);
    if (!(aa >= thresh)) {
        e[0] = e[1] = e[2] = -1.f;
        return;
    }
    // covariance = inverse(conic) by cofactors
    const float c00 = q[3] * q[5] - q[4] * q[4];
    const float c11 = q[0] * q[5] - q[2] * q[2];
    const float c22 = q[0] * q[3] - q[1] * q[1];
    const float c01 = q[2] * q[4] - q[1] * q[5];
    const float c02 = q[1] * q[4] - q[2] * q[3];
    const float det = q[0] * c00 + q[1] * c01 + q[2] * c02;
    if (!(q[0] > 0.f && q[3] > 0.f && q[5] > 0.f && det > 0.f && c00 > 0.f && c11 > 0.f &&
          c22 > 0.f)) {
        e[0] = e[1] = e[2] = CUDART_INF_F;
        return;
    }
    const float cond = (q[0] * q[3] * q[5]) / det;
    if (!isfinite(cond) || cond > 1e6f) {
        e[0] = e[1] = e[2] = CUDART_INF_F;
        return;
    }
    const float s_cut = logf(aa / thresh) * 1.0001f + 1e-4f;
    const float rel = 1.0f + 1e-4f + 4e-7f * cond;
    e[0] = sqrtf(2.0f * s_cut * (c00 / det) * rel) * 1.0001f + 1e-3f;
    e[1] = sqrtf(2.0f * s_cut * (c11 / det) * rel) * 1.0001f + 1e-3f;
    e[2] = sqrtf(2.0f * s_cut * (c22 / det) * rel) * 1.0001f + 1e-3f;
}

template <typename S>
struct VoxSrc {
    const float4* vsplats;  // fused float32 records [N][4]
    const S* means3d;       // [N][3]
    const S* conics;        // [N][6]
    const S* opac;          // [N]
};

template <typename S, bool SPLATS>
__device__ __forceinline__ void load_vgauss(const VoxSrc<S>& src, int64_t g, S m[3], S q[6], S& w,
                                            float e[3]) {
    if constexpr (SPLATS) {
        const float4 a = src.vsplats[4 * g], b = src.vsplats[4 * g + 1],
                     c = src.vsplats[4 * g + 2], d = src.vsplats[4 * g + 3];
        m[0] = a.x; m[1] = a.y; m[2] = a.z;
        q[0] = a.w; q[1] = b.x; q[2] = b.y; q[3] = b.z; q[4] = b.w; q[5] = c.x;
        w = c.y;
        e[0] = c.z; e[1] = c.w; e[2] = d.x;
    } else {
#pragma unroll
        for (int k = 0; k < 3; ++k) m[k] = src.means3d[3 * g + k];
#pragma unroll
        for (int k = 0; k < 6; ++k) q[k] = src.conics[6 * g + k];
        w = src.opac[g];
        float qf[6];
#pragma unroll
        for (int k = 0; k < 6; ++k) qf[k] = (float)q[k];
        conic3_cull(qf, (float)w, kAlphaMin3D, e);
    }
}

struct BrickGeom {
    int T;
    int nthr;  // T^3
    __device__ __forceinline__ void voxel(int tid, int& lx, int& ly, int& lz) const {
        lz = tid / (T * T);
        const int r = tid - lz * T * T;
        ly = r / T;
        lx = r - ly * T;
    }
};

// ===========================================================================
// Forward
// ===========================================================================
template <typename S, bool SPLATS>
__global__ void voxel_fwd_kernel(VoxSrc<S> src, const int32_t* __restrict__ offsets,
                                 const int32_t* __restrict__ flatten_ids, int64_t n_keys,
                                 int64_t n_isects, uint32_t dim2, uint32_t dim1, uint32_t dim0,
                                 BrickGeom geo, uint32_t nt2, uint32_t nt1, uint32_t layer_begin,
                                 S* __restrict__ vol) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nthr = geo.nthr, T = geo.T;
    const size_t arr = al16v((size_t)nthr * sizeof(S));
    S* s_p[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) s_p[k] = reinterpret_cast<S*>(smem_raw + k * arr);
    uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem_raw + 10 * arr);
    const int n_warps = (nthr + 31) >> 5;
    const size_t mask_bytes = al16v((size_t)max(nthr, n_warps * 6) * 4);
    uint2* s_box = reinterpret_cast<uint2*>(smem_raw + 10 * arr + mask_bytes);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bx = blockIdx.x, by = blockIdx.y, bz_local = blockIdx.z;
    const uint32_t bz = bz_local + layer_begin;
    const int64_t key = ((int64_t)bz_local * nt1 + by) * nt2 + bx;
    const int X0 = bx * T, Y0 = by * T, Z0 = bz * T;
    const int xmax = min(T - 1, (int)dim2 - 1 - X0);
    const int ymax = min(T - 1, (int)dim1 - 1 - Y0);
    const int zmax = min(T - 1, (int)dim0 - 1 - Z0);
    int lx, ly, lz;
    geo.voxel(tid, lx, ly, lz);
    const bool inside = lx <= xmax && ly <= ymax && lz <= zmax;
    {
        // per-warp voxel bounding box of the inside voxels, built with shared
        // atomics (exact for partial warps too); s_mask doubles as scratch
        int* bb = reinterpret_cast<int*>(s_mask);  // [n_warps][6]
        for (int i = tid; i < n_warps * 6; i += nthr) bb[i] = (i % 6) & 1 ? -1 : 255;
        __syncthreads();
        if (inside) {
            atomicMin(&bb[warp * 6 + 0], lx);
            atomicMax(&bb[warp * 6 + 1], lx);
            atomicMin(&bb[warp * 6 + 2], ly);
            atomicMax(&bb[warp * 6 + 3], ly);
            atomicMin(&bb[warp * 6 + 4], lz);
            atomicMax(&bb[warp * 6 + 5], lz);
        }
        __syncthreads();
        if (tid < n_warps) {
            const int* q = bb + tid * 6;
            uint2 b;
            if (q[1] < 0) {
                b.x = 0x00ff00ffu;  // empty: lo 255 > hi 0
                b.y = 0x000000ffu;
            } else {
                b.x = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16) |
                      ((uint32_t)q[3] << 24);
                b.y = (uint32_t)q[4] | ((uint32_t)q[5] << 8);
            }
            s_box[tid] = b;
        }
        __syncthreads();
    }
    const S px = static_cast<S>(X0 + lx) + static_cast<S>(0.5);
    const S py = static_cast<S>(Y0 + ly) + static_cast<S>(0.5);
    const S pz = static_cast<S>(Z0 + lz) + static_cast<S>(0.5);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    const unsigned wmask = (nthr - warp * 32) >= 32 ? 0xffffffffu : ((1u << (nthr - warp * 32)) - 1u);
    S acc = static_cast<S>(0);
    __syncthreads();

    for (int b0 = start; b0 < end; b0 += nthr) {
        const int n = min(nthr, end - b0);
        __syncthreads();
        if (tid < n) {
            const int64_t g = flatten_ids[b0 + tid];
            S m[3], q[6], w;
            float e[3];
            load_vgauss<S, SPLATS>(src, g, m, q, w, e);
            int xl, xh, yl, yh, zl, zh;
            cull_range_v((float)m[0], e[0], (float)X0, xmax, xl, xh);
            cull_range_v((float)m[1], e[1], (float)Y0, ymax, yl, yh);
            cull_range_v((float)m[2], e[2], (float)Z0, zmax, zl, zh);
            uint32_t msk = 0;
            if (xl <= xh && yl <= yh && zl <= zh) {
                for (int wv = 0; wv < n_warps; ++wv) {
                    const uint2 b = s_box[wv];
                    const int bx0 = b.x & 0xff, bx1 = (b.x >> 8) & 0xff;
                    const int by0 = (b.x >> 16) & 0xff, by1 = b.x >> 24;
                    const int bz0 = b.y & 0xff, bz1 = (b.y >> 8) & 0xff;
                    if (xl <= bx1 && xh >= bx0 && yl <= by1 && yh >= by0 && zl <= bz1 && zh >= bz0)
                        msk |= 1u << wv;
                }
            }
            s_p[0][tid] = m[0];
            s_p[1][tid] = m[1];
            s_p[2][tid] = m[2];
            if constexpr (std::is_same<S, float>::value) {
                s_p[3][tid] = 0.5f * kLog2eV * q[0];
                s_p[4][tid] = kLog2eV * q[1];
                s_p[5][tid] = kLog2eV * q[2];
                s_p[6][tid] = 0.5f * kLog2eV * q[3];
                s_p[7][tid] = kLog2eV * q[4];
                s_p[8][tid] = 0.5f * kLog2eV * q[5];
            } else {
#pragma unroll
                for (int k = 0; k < 6; ++k) s_p[3 + k][tid] = q[k];
            }
            s_p[9][tid] = w;
            s_mask[tid] = msk;
        }
        __syncthreads();
        for (int c0 = 0; c0 < n; c0 += 32) {
            const int j = c0 + lane;
            unsigned bits = __ballot_sync(wmask, j < n && ((s_mask[j] >> warp) & 1u));
            while (bits) {
                const int t = c0 + __ffs(bits) - 1;
                bits &= bits - 1;
                const S dx = px - s_p[0][t];
                const S dy = py - s_p[1][t];
                const S dz = pz - s_p[2][t];
                if constexpr (std::is_same<S, float>::value) {
                    const float u = fmaf(s_p[3][t], dx, fmaf(s_p[4][t], dy, s_p[5][t] * dz));
                    const float v = fmaf(s_p[6][t], dy, s_p[7][t] * dz);
                    const float s = fmaf(dx, u, fmaf(dy, v, s_p[8][t] * dz * dz));
                    const float al = s_p[9][t] * exp2f(-s);
                    acc += (s < 0.f || fabsf(al) < kAlphaMin3D) ? 0.f : al;
                } else {
                    const S sig = static_cast<S>(0.5) * (s_p[3][t] * dx * dx + s_p[6][t] * dy * dy +
                                                         s_p[8][t] * dz * dz) +
                                  s_p[4][t] * dx * dy + s_p[5][t] * dx * dz + s_p[7][t] * dy * dz;
                    const S al = s_p[9][t] * expf_neg(sig);
                    const bool skip = sig < static_cast<S>(0) ||
                                      fabsf(static_cast<float>(al)) < static_cast<S>(1e-6);
                    acc += skip ? static_cast<S>(0) : al;
                }
            }
        }
    }
    if (inside)
        vol[((int64_t)(Z0 + lz - (int)layer_begin * T) * dim1 + (Y0 + ly)) * dim2 + X0 + lx] = acc;
}

// ===========================================================================
// Backward statistics
// ===========================================================================
template <typename S>
__device__ __forceinline__ void vstats_red(S* dst, const S v[10]) {
    if constexpr (std::is_same<S, float>::value) {
        red_add_v4(dst, v[0], v[1], v[2], v[3]);
        red_add_v4(dst + 4, v[4], v[5], v[6], v[7]);
        red_add_v2(dst + 8, v[8], v[9]);
    } else {
        for (int k = 0; k < 10; ++k) atomicAdd(dst + k, v[k]);
    }
}
// float moments into the float64 per-Gaussian sums of the fused path: the
// sum over a Gaussian's bricks is then exact to ~1e-16 whatever order the
// atomics land in, so repeated or differently sharded runs agree
__device__ __forceinline__ void vstats_red(double* dst, const float v[10]) {
#pragma unroll
    for (int k = 0; k < 10; ++k) atomicAdd(dst + k, (double)v[k]);
}

// per-Gaussian statistics of the voxel backward: float64 for the fused
// path (splat records), the input type for the reference-layout wrappers
template <typename S, bool SPLATS>
using VStat = typename std::conditional<SPLATS, double, S>::type;

template <typename S, bool SPLATS, int EXPMODE>
__global__ void voxel_bwd_kernel(VoxSrc<S> src, const int32_t* __restrict__ offsets,
                                 const int32_t* __restrict__ flatten_ids, int64_t n_keys,
                                 int64_t n_isects, const S* __restrict__ v_vol, uint32_t dim2,
                                 uint32_t dim1, uint32_t dim0, int T, uint32_t nt2, uint32_t nt1,
                                 uint32_t layer_begin, VStat<S, SPLATS>* __restrict__ stats) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nthr = blockDim.x;
    const int TT = T * T, TTT = T * T * T;
    S* s_v = reinterpret_cast<S*>(smem_raw);
    const size_t arr = al16v((size_t)nthr * sizeof(S));
    unsigned char* base = smem_raw + al16v((size_t)TTT * sizeof(S));
    S* s_p[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) s_p[k] = reinterpret_cast<S*>(base + k * arr);
    int32_t* s_g = reinterpret_cast<int32_t*>(base + 10 * arr);
    uint2* s_box = reinterpret_cast<uint2*>(base + 10 * arr + al16v((size_t)nthr * 4));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_warps = nthr >> 5;
    const uint32_t bx = blockIdx.x, by = blockIdx.y, bz_local = blockIdx.z;
    const uint32_t bz = bz_local + layer_begin;
    const int64_t key = ((int64_t)bz_local * nt1 + by) * nt2 + bx;
    const int X0 = bx * T, Y0 = by * T, Z0 = bz * T;
    const int xmax = min(T - 1, (int)dim2 - 1 - X0);
    const int ymax = min(T - 1, (int)dim1 - 1 - Y0);
    const int zmax = min(T - 1, (int)dim0 - 1 - Z0);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (start >= end) return;
    const int64_t zoff = (int64_t)layer_begin * T;
    for (int p = tid; p < TTT; p += nthr) {
        const int z = p / TT, r = p - z * TT, y = r / T, x = r - y * T;
        s_v[p] = (x <= xmax && y <= ymax && z <= zmax)
                     ? v_vol[((Z0 + z - zoff) * dim1 + (Y0 + y)) * (int64_t)dim2 + X0 + x]
                     : static_cast<S>(0);
    }
    for (int b0 = start; b0 < end; b0 += nthr) {
        const int n = min(nthr, end - b0);
        __syncthreads();
        if (tid < n) {
            const int64_t g = flatten_ids[b0 + tid];
            S m[3], q[6], w;
            float e[3];
            load_vgauss<S, SPLATS>(src, g, m, q, w, e);
            int xl, xh, yl, yh, zl, zh;
            cull_range_v((float)m[0], e[0], (float)X0, xmax, xl, xh);
            cull_range_v((float)m[1], e[1], (float)Y0, ymax, yl, yh);
            cull_range_v((float)m[2], e[2], (float)Z0, zmax, zl, zh);
            if (xl > xh || yl > yh || zl > zh) xl = 1, xh = 0, yl = yh = zl = zh = 0;
#pragma unroll
            for (int k = 0; k < 3; ++k) s_p[k][tid] = m[k];
#pragma unroll
            for (int k = 0; k < 6; ++k) s_p[3 + k][tid] = q[k];
            s_p[9][tid] = w;
            s_g[tid] = (int32_t)g;
            uint2 b;
            b.x = (uint32_t)xl | ((uint32_t)xh << 8) | ((uint32_t)yl << 16) | ((uint32_t)yh << 24);
            b.y = (uint32_t)zl | ((uint32_t)zh << 8);
            s_box[tid] = b;
        }
        __syncthreads();
        for (int t = warp; t < n; t += n_warps) {
            const uint2 b = s_box[t];
            const int xl = b.x & 0xff, xh = (b.x >> 8) & 0xff;
            if (xl > xh) continue;
            const int yl = (b.x >> 16) & 0xff, yh = b.x >> 24;
            const int zl = b.y & 0xff, zh = (b.y >> 8) & 0xff;
            const int wx = xh - xl + 1, wy = yh - yl + 1;
            const int wxy = wx * wy;
            const int npx = wxy * (zh - zl + 1);
            const float inv_wxy = 1.0f / (float)wxy, inv_wx = 1.0f / (float)wx;
            const S mx = s_p[0][t], my = s_p[1][t], mz = s_p[2][t];
            const S q0 = s_p[3][t], q1 = s_p[4][t], q2 = s_p[5][t], q3 = s_p[6][t],
                    q4 = s_p[7][t], q5 = s_p[8][t], w = s_p[9][t];
            S acc[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
            for (int p = lane; p < npx; p += 32) {
                const int zz = __float2int_rz(((float)p + 0.5f) * inv_wxy);
                const int r = p - zz * wxy;
                const int yy = __float2int_rz(((float)r + 0.5f) * inv_wx);
                const int xx = r - yy * wx;
                const int lx = xl + xx, ly = yl + yy, lz = zl + zz;
                const S v = s_v[(lz * T + ly) * T + lx];
                const S dx = static_cast<S>(X0 + lx) + static_cast<S>(0.5) - mx;
                const S dy = static_cast<S>(Y0 + ly) + static_cast<S>(0.5) - my;
                const S dz = static_cast<S>(Z0 + lz) + static_cast<S>(0.5) - mz;
                S e;
                bool skip;
                if constexpr (std::is_same<S, float>::value) {
                    const float A = 0.5f * kLog2eV * q0, B = kLog2eV * q1, Cq = kLog2eV * q2;
                    const float D = 0.5f * kLog2eV * q3, E = kLog2eV * q4, F = 0.5f * kLog2eV * q5;
                    const float u = fmaf(A, dx, fmaf(B, dy, Cq * dz));
                    const float vv = fmaf(D, dy, E * dz);
                    const float s = fmaf(dx, u, fmaf(dy, vv, F * dz * dz));
                    e = exp2f(-s);
                    skip = s < 0.f || fabsf(w * e) < kAlphaMin3D;
                } else {
                    const S sig = static_cast<S>(0.5) * (q0 * dx * dx + q3 * dy * dy + q5 * dz * dz) +
                                  q1 * dx * dy + q2 * dx * dz + q4 * dy * dz;
                    if constexpr (EXPMODE == 0) {
                        e = expf_neg(sig);
                        skip = sig < static_cast<S>(0) ||
                               fabsf(static_cast<float>(w * e)) < static_cast<S>(1e-6);
                    } else {
                        e = exp(-sig);
                        skip = sig < static_cast<S>(0) || fabs(w * e) < static_cast<S>(1e-6);
                    }
                }
                const S ve = skip ? static_cast<S>(0) : v * e;
                const S vx = ve * dx, vy = ve * dy, vz = ve * dz;
                acc[0] += ve;
                acc[1] += vx;
                acc[2] += vy;
                acc[3] += vz;
                acc[4] += vx * dx;
                acc[5] += vx * dy;
                acc[6] += vx * dz;
                acc[7] += vy * dy;
                acc[8] += vy * dz;
                acc[9] += vz * dz;
            }
#pragma unroll
            for (int k = 0; k < 10; ++k) acc[k] = warp_sum(acc[k]);
            if (lane == 0) vstats_red(stats + (int64_t)s_g[t] * 12, acc);
        }
    }
}

// ===========================================================================
// float32, 8x8x8 bricks: the fast kernels
// ===========================================================================
//
// Validity test as in the 16x16 rasterizer: with s = sigma*log2(e) the
// reference's test (sigma >= 0 and |w exp(-sigma)| >= 1e-6) is
// 0 <= s <= log2(|w| 1e6), decided by one unsigned compare of the bits of s.
// In the forward, pairs within rounding of the cut-off may be decided
// differently from the reference's float test (each such pair moves a voxel
// by at most ~1e-6); the 8x8x8 backward re-decides them exactly
// (r2s_cutoff.cuh).

// The forward evaluates -s (negated coefficients, exact) and compare its bits as
// signed integers with INT_MIN + bits(s_thr); s = -0.0 (a conic that is not
// positive definite, voxel centre on the mean) counts as s < 0.
__device__ __forceinline__ bool sn_valid_v(float sn, int thr_n) {
    return __float_as_int(sn) <= thr_n;
}

__device__ __forceinline__ int thr_neg_v(float thr) {
    return (int)(__float_as_uint(thr) ^ 0x80000000u);
}

struct VRecord {
    float m[3];
    // negated pre-scaled conic: -sigma log2(e) = dx (A dx + B dy + Cq dz) + dy (D dy + E dz) + F dz^2
    float A, B, Cq, D, E, F;
    float w;
    float e[3];
    float band;  // cut-off band of the voxel backward (cutoff_band_v)
};

__device__ __forceinline__ VRecord load_vrecord(const float4* __restrict__ vsplats, int64_t g) {
    const float4 a = vsplats[4 * g], b = vsplats[4 * g + 1], c = vsplats[4 * g + 2],
                 d = vsplats[4 * g + 3];
    VRecord r;
    r.m[0] = a.x;
    r.m[1] = a.y;
    r.m[2] = a.z;
    r.A = -0.5f * kLog2eV * a.w;
    r.B = -kLog2eV * b.x;
    r.Cq = -kLog2eV * b.y;
    r.D = -0.5f * kLog2eV * b.z;
    r.E = -kLog2eV * b.w;
    r.F = -0.5f * kLog2eV * c.x;
    r.w = c.y;
    r.e[0] = c.z;
    r.e[1] = c.w;
    r.e[2] = d.x;
    r.band = d.y;
    return r;
}

// The natural conic (P00, P01, P02, P11, P12, P22) of a voxel splat record.
__device__ __forceinline__ void raw_conic(const float4* __restrict__ vsplats, int64_t g,
                                          float q[6]) {
    const float4 a = vsplats[4 * g], b = vsplats[4 * g + 1], c = vsplats[4 * g + 2];
    q[0] = a.w;
    q[1] = b.x;
    q[2] = b.y;
    q[3] = b.z;
    q[4] = b.w;
    q[5] = c.x;
}

// First and last slice with rows of a brick_rows table (ezl > ezh: none).
__device__ __forceinline__ void table_slices(uint32_t tlo, uint32_t thi, int& ezl, int& ezh) {
    ezl = 8;
    ezh = -1;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t byte = ((k < 4 ? tlo : thi) >> (8 * (k & 3))) & 0xffu;
        if ((byte & 15u) <= (byte >> 4)) {
            ezl = min(ezl, k);
            ezh = k;
        }
    }
}

// Launch order of the brick CTAs.  The per-brick kernels below map their
// linear block index through `order` (when given) to a brick key, so that
// the GPU, which starts blocks in linear order, begins with the bricks that
// hold the most records: the classic longest-first schedule, which keeps a
// long brick from starting last and idling the other SMs at the end of a
// launch whose bricks fill about one wave (a z-slab of a multi-GPU split).
__device__ __forceinline__ int64_t brick_of_block(const int32_t* __restrict__ order,
                                                  uint32_t nt2, uint32_t nt1, int& bx, int& by,
                                                  int& bzl) {
    const int64_t lin = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const int64_t key = order != nullptr ? (int64_t)order[lin] : lin;
    bx = (int)(key % nt2);
    by = (int)((key / nt2) % nt1);
    bzl = (int)(key / ((int64_t)nt2 * nt1));
    return key;
}

constexpr int kOrderThreads = 1024;

// order[] = brick keys grouped by floor(log2(records)) from the largest
// group down (an approximate longest-first order; empty bricks last).  One
// CTA: a histogram of the 33 groups, their descending prefix, a scatter.
__global__ void __launch_bounds__(kOrderThreads)
brick_order_kernel(const int32_t* __restrict__ offsets, int64_t n_keys, int64_t n_isects,
                   int32_t* __restrict__ order) {
    __shared__ int s_cnt[33];
    __shared__ int s_cur[33];
    const int tid = threadIdx.x;
    if (tid < 33) s_cnt[tid] = 0;
    __syncthreads();
    auto group = [&](int64_t k) {
        const int64_t end = k + 1 < n_keys ? (int64_t)offsets[k + 1] : n_isects;
        const int64_t c = end - (int64_t)offsets[k];
        return c > 0 ? 32 - __clz((unsigned)min(c, (int64_t)INT32_MAX)) : 0;  // 0..31
    };
    for (int64_t k = tid; k < n_keys; k += kOrderThreads) atomicAdd(&s_cnt[group(k)], 1);
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int b = 32; b >= 0; --b) {
            s_cur[b] = run;
            run += s_cnt[b];
        }
    }
    __syncthreads();
    for (int64_t k = tid; k < n_keys; k += kOrderThreads)
        order[atomicAdd(&s_cur[group(k)], 1)] = (int32_t)k;
}

// Row table of every (record, brick) pair of the brick lists: rows[i] =
// brick_rows of record i against its brick (per-slice first | last row,
// 0x0f for none).  One CTA per brick; computed once per binning and read by
// the forward and the backward, so neither pays for it in its staging.
constexpr int kVRowsThreads = 128;

__global__ void __launch_bounds__(kVRowsThreads)
voxel_rows8_kernel(const float4* __restrict__ vsplats, const int32_t* __restrict__ offsets,
                   const int32_t* __restrict__ flatten_ids, int64_t n_keys, int64_t n_isects,
                   int64_t n_splats, uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t nt2,
                   uint32_t nt1, uint32_t layer_begin, const int32_t* __restrict__ order,
                   uint2* __restrict__ rows) {
    int bxi, byi, bzl;
    const int64_t key = brick_of_block(order, nt2, nt1, bxi, byi, bzl);
    const uint32_t bz = bzl + layer_begin;
    const int X0 = bxi * 8, Y0 = byi * 8, Z0 = bz * 8;
    const int xmax = min(7, (int)dim2 - 1 - X0);
    const int ymax = min(7, (int)dim1 - 1 - Y0);
    const int zmax = min(7, (int)dim0 - 1 - Z0);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (R2S_DBG_BAD(start >= 0 && start <= end && end <= n_isects, R2S_DBG_TILE_RANGE)) return;
    for (int i = start + threadIdx.x; i < end; i += kVRowsThreads) {
        const int64_t g = flatten_ids[i];
        if (R2S_DBG_BAD(g >= 0 && g < n_splats, R2S_DBG_RECORD_ID)) continue;
        const VRecord r = load_vrecord(vsplats, g);
        int xl, xh, yl, yh, zl, zh;
        cull_range_v(r.m[0], r.e[0], (float)X0, xmax, xl, xh);
        cull_range_v(r.m[1], r.e[1], (float)Y0, ymax, yl, yh);
        cull_range_v(r.m[2], r.e[2], (float)Z0, zmax, zl, zh);
        float q[6];
        raw_conic(vsplats, g, q);
        uint32_t tlo, thi;
        int ezl, ezh;
        brick_rows(r.m[0], r.m[1], r.m[2], q, s_threshold_v(r.w), (float)X0, (float)Y0,
                   (float)Z0, xl, xh, yl, yh, zl, zh, tlo, thi, ezl, ezh);
        rows[i] = make_uint2(tlo, thi);
    }
}

// A group of 2 warps covers a brick's 512 voxels (a warp owns four z-slices,
// a thread 4x2 voxels (x, z)).  A CTA holds GROUPS groups; they take the
// staged records of each batch in turn (record t of the batch to group
// t mod GROUPS) and add their partial sums in group order at the end.  One
// group per CTA is the fastest on launches of many records (the full config-2
// grid: 20M records, 2.44 ms against 2.80 ms with four groups); launches of
// fewer records per SM (a z-slab of a multi-GPU split, a small grid) finish
// sooner with four (2-4M records: 0.43-0.54 ms against 0.63-0.69 ms), since
// with one group an SM runs a handful of heavy bricks at low occupancy once
// the light ones are done.  On centred slabs of the config-2 grid four groups
// are 14 % faster at 3.8M records and 3 % slower at 7.7M; they cross near
// 6.5M records on 148 SMs.
constexpr int kVFwd8Batch = 128;  // records staged per group and batch
constexpr int64_t kVFwd8GroupedRecordsPerSM = 44032;  // fewer per launch: four groups

template <int GROUPS>
__global__ void __launch_bounds__(64 * GROUPS)
voxel_fwd8_kernel(const float4* __restrict__ vsplats, const int32_t* __restrict__ offsets,
                  const int32_t* __restrict__ flatten_ids, const uint2* __restrict__ rows,
                  int64_t n_keys, int64_t n_isects, int64_t n_splats, uint32_t dim2,
                  uint32_t dim1, uint32_t dim0, uint32_t nt2, uint32_t nt1, uint32_t layer_begin,
                  const int32_t* __restrict__ order, float* __restrict__ vol) {
    constexpr int kThreads = 64 * GROUPS, kBatch = kVFwd8Batch * GROUPS;
    __shared__ float4 s_a[kBatch];  // mx, my, mz, A
    __shared__ float4 s_b[kBatch];  // B, Cq, D, E
    __shared__ float4 s_c[kBatch];  // F, w, s threshold, warp mask (bits)

    const int tid = threadIdx.x, grp = tid >> 6, gt = tid & 63, warp = gt >> 5;
    int bxi, byi, bzl;
    const int64_t key = brick_of_block(order, nt2, nt1, bxi, byi, bzl);
    const uint32_t bz = bzl + layer_begin;
    const int X0 = bxi * 8, Y0 = byi * 8, Z0 = bz * 8;
    const int xmax = min(7, (int)dim2 - 1 - X0);
    const int ymax = min(7, (int)dim1 - 1 - Y0);
    const int zmax = min(7, (int)dim0 - 1 - Z0);
    const int lx = (gt & 1) * 4, ly = (gt >> 1) & 7, lz = (gt >> 4) * 2;
    const float2 px01 = make_float2((float)(X0 + lx) + 0.5f, (float)(X0 + lx) + 1.5f);
    const float2 px23 = make_float2((float)(X0 + lx) + 2.5f, (float)(X0 + lx) + 3.5f);
    const float py = (float)(Y0 + ly) + 0.5f;
    const float pz0 = (float)(Z0 + lz) + 0.5f, pz1 = (float)(Z0 + lz) + 1.5f;
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (R2S_DBG_BAD(start >= 0 && start <= end && end <= n_isects, R2S_DBG_TILE_RANGE))
        return;  // uniform over the CTA
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // [z][x]

    for (int b0 = start; b0 < end; b0 += kBatch) {
        const int n = min(kBatch, end - b0);
        __syncthreads();
        for (int j = tid; j < n; j += kThreads) {
            const int64_t g = flatten_ids[b0 + j];
            if (R2S_DBG_BAD(g >= 0 && g < n_splats, R2S_DBG_RECORD_ID)) {
                s_c[j] = make_float4(0.f, 0.f, 0.f, __uint_as_float(0u));  // no warp evaluates it
                continue;
            }
            const VRecord r = load_vrecord(vsplats, g);
            int xl, xh, yl, yh, zl, zh;
            cull_range_v(r.m[0], r.e[0], (float)X0, xmax, xl, xh);
            cull_range_v(r.m[1], r.e[1], (float)Y0, ymax, yl, yh);
            cull_range_v(r.m[2], r.e[2], (float)Z0, zmax, zl, zh);
            // bit h: warp h's four slices can hold a passing voxel -- from the
            // row table when there is one, else from the culling box
            uint32_t msk = 0;
            if (rows != nullptr) {
                const uint2 tab = rows[b0 + j];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint32_t byte = ((k < 4 ? tab.x : tab.y) >> (8 * (k & 3))) & 0xffu;
                    if ((byte & 15u) <= (byte >> 4)) msk |= 1u << (k >> 2);
                }
            } else if (xl <= xh && yl <= yh && zl <= zh) {
#pragma unroll
                for (int k = 0; k < 2; ++k)
                    if (zl <= 4 * k + 3 && zh >= 4 * k) msk |= 1u << k;
            }
            s_a[j] = make_float4(r.m[0], r.m[1], r.m[2], r.A);
            s_b[j] = make_float4(r.B, r.Cq, r.D, r.E);
            s_c[j] = make_float4(r.F, r.w, __int_as_float(thr_neg_v(s_threshold_v(r.w))),
                                 __uint_as_float(msk));
        }
        __syncthreads();
        for (int t = grp; t < n; t += GROUPS) {
            const float4 c = s_c[t];
            if (!((__float_as_uint(c.w) >> warp) & 1u)) continue;  // warp-uniform
            const float4 a = s_a[t], b = s_b[t];
            const int thr_n = __float_as_int(c.z);
            const float2 nmx = make_float2(-a.x, -a.x);
            const float2 dx01 = fadd2(px01, nmx), dx23 = fadd2(px23, nmx);
            const float dy = py - a.y;
            const float bdy = b.x * dy, ddy = b.z * dy;
            const float2 A2 = make_float2(a.w, a.w);
#pragma unroll
            for (int zz = 0; zz < 2; ++zz) {
                const float dz = (zz ? pz1 : pz0) - a.z;
                const float u = fmaf(b.y, dz, bdy);
                const float q = fmaf(dy, fmaf(b.w, dz, ddy), c.x * dz * dz);
                const float2 u2 = make_float2(u, u), q2 = make_float2(q, q);
                // -s = dx (A dx + u) + q
                const float2 s01 = ffma2(dx01, ffma2(A2, dx01, u2), q2);
                const float2 s23 = ffma2(dx23, ffma2(A2, dx23, u2), q2);
                const float e0 = exp2f(s01.x), e1 = exp2f(s01.y);
                const float e2 = exp2f(s23.x), e3 = exp2f(s23.y);
                if (sn_valid_v(s01.x, thr_n)) acc[zz][0] = fmaf(c.y, e0, acc[zz][0]);
                if (sn_valid_v(s01.y, thr_n)) acc[zz][1] = fmaf(c.y, e1, acc[zz][1]);
                if (sn_valid_v(s23.x, thr_n)) acc[zz][2] = fmaf(c.y, e2, acc[zz][2]);
                if (sn_valid_v(s23.y, thr_n)) acc[zz][3] = fmaf(c.y, e3, acc[zz][3]);
            }
        }
    }
    if constexpr (GROUPS > 1) {  // the groups' sums, added in group order by group 0
        __syncthreads();  // the last batch's records are no longer read
        float* const s_part = reinterpret_cast<float*>(s_a);  // [group - 1][8][64]
        static_assert((GROUPS - 1) * 8 * 64 <= kBatch * 4, "partial sums fit in s_a");
        if (grp > 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) s_part[((grp - 1) * 8 + k) * 64 + gt] = acc[k >> 2][k & 3];
        }
        __syncthreads();
        if (grp > 0) return;
#pragma unroll
        for (int g = 1; g < GROUPS; ++g)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k >> 2][k & 3] += s_part[((g - 1) * 8 + k) * 64 + gt];
    }
    if (ly > ymax) return;
    const int64_t zoff = (int64_t)layer_begin * 8;
#pragma unroll
    for (int zz = 0; zz < 2; ++zz) {
        if (lz + zz > zmax) continue;
        if (R2S_DBG_BAD(Z0 + lz + zz - zoff <
                                min((int64_t)(layer_begin + gridDim.z) * 8, (int64_t)dim0) - zoff &&
                            Y0 + ly < (int)dim1 && X0 + lx < (int)dim2,
                        R2S_DBG_PIXEL))
            continue;
        float* row = vol + ((Z0 + lz + zz - zoff) * (int64_t)dim1 + (Y0 + ly)) * dim2 + X0 + lx;
        if (lx + 3 <= xmax && (dim2 & 3) == 0) {
            *reinterpret_cast<float4*>(row) =
                make_float4(acc[zz][0], acc[zz][1], acc[zz][2], acc[zz][3]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (lx + k <= xmax) row[k] = acc[zz][k];
        }
    }
}

constexpr int kVBwd8Threads = 256;  // one brick per CTA, one Gaussian record per thread
constexpr int kVBwd8Batch = 1024;   // records staged and sorted per batch

// Backward statistics of 8x8x8 bricks, one record per thread.  Staging
// narrows each record's culling box to the rows of every z-slice where its
// ellipsoid reaches the brick (brick_rows: per-slice row ranges and the
// slices that have rows) and counting-sorts each batch of 1024 records by
// that slice range, so that a group of 32 lanes walks similar slices.  A
// thread walks, per slice of its warp's union, the union of its lanes' rows
// in that slice, and the 8 voxels of each row in packed pairs.  Per-column
// sums Col_x = sum v e over rows give S0, Sx, Sxx; per-row sums R0 = sum_x v e
// and R1 = sum_x v e dx give the y/z moments, so every moment is a direct sum.
__global__ void __launch_bounds__(kVBwd8Threads, 3)
voxel_bwd8_kernel(const float4* __restrict__ vsplats, const int32_t* __restrict__ offsets,
                  const int32_t* __restrict__ flatten_ids, const uint2* __restrict__ rows,
                  int64_t n_keys, int64_t n_isects, int64_t n_splats,
                  const float* __restrict__ v_vol, uint32_t dim2, uint32_t dim1, uint32_t dim0,
                  uint32_t nt2, uint32_t nt1, uint32_t layer_begin,
                  const int32_t* __restrict__ order, double* __restrict__ stats) {
    __shared__ __align__(16) float s_v[512];
    __shared__ uint2 s_tab[kVBwd8Batch];     // per-slice rows (byte k: first | last << 4)
    __shared__ int32_t s_g[kVBwd8Batch];
    __shared__ uint8_t s_zr[kVBwd8Batch];    // first slice | last slice << 4; 0x0f: none
    __shared__ uint16_t s_perm[kVBwd8Batch];
    __shared__ int32_t s_cnt[65];            // bucket 64: records that reach no voxel
    __shared__ int s_next;                   // next group to take
    __shared__ uint16_t s_fix[kVBwd8Batch];  // records with a voxel in the cut-off band
    __shared__ int s_nfix;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int bxi, byi, bzl;
    const int64_t key = brick_of_block(order, nt2, nt1, bxi, byi, bzl);
    const uint32_t bz = bzl + layer_begin;
    const int X0 = bxi * 8, Y0 = byi * 8, Z0 = bz * 8;
    const int xmax = min(7, (int)dim2 - 1 - X0);
    const int ymax = min(7, (int)dim1 - 1 - Y0);
    const int zmax = min(7, (int)dim0 - 1 - Z0);
    const int start = offsets[key];
    const int end = key + 1 < n_keys ? offsets[key + 1] : (int)n_isects;
    if (start >= end) return;
    if (R2S_DBG_BAD(start >= 0 && end <= n_isects, R2S_DBG_TILE_RANGE)) return;  // CTA-uniform
    const int64_t zoff = (int64_t)layer_begin * 8;
    for (int p = tid; p < 512; p += kVBwd8Threads) {
        const int z = p >> 6, y = (p >> 3) & 7, x = p & 7;
        bool in = x <= xmax && y <= ymax && z <= zmax;
        if (in && R2S_DBG_BAD(Z0 + z - zoff < min((int64_t)(layer_begin + gridDim.z) * 8,
                                                   (int64_t)dim0) - zoff,
                              R2S_DBG_PIXEL))
            in = false;
        s_v[p] = in ? v_vol[((Z0 + z - zoff) * (int64_t)dim1 + (Y0 + y)) * dim2 + X0 + x] : 0.f;
    }
    const float X0f = (float)X0, Y0f = (float)Y0, Z0f = (float)Z0;

    for (int base = start; base < end; base += kVBwd8Batch) {
        if (tid < 65) s_cnt[tid] = 0;
        if (tid == 0) s_nfix = 0;
        __syncthreads();
        constexpr int kPer = kVBwd8Batch / kVBwd8Threads;
        int bucket[kPer], rank[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int idx = k * kVBwd8Threads + tid;
            const int i = base + idx;
            int32_t g = 0;
            uint32_t tlo = 0x0f0f0f0fu, thi = 0x0f0f0f0fu;
            int ezl = 8, ezh = -1;
            if (i < end && R2S_DBG_BAD(flatten_ids[i] >= 0 && flatten_ids[i] < n_splats,
                                        R2S_DBG_RECORD_ID)) {
                // checked build: an id outside the records stays unstaged
            } else if (i < end) {
                g = flatten_ids[i];
                if (rows != nullptr) {
                    const uint2 tab = rows[i];
                    tlo = tab.x;
                    thi = tab.y;
                    table_slices(tlo, thi, ezl, ezh);
                } else {
                    const VRecord r = load_vrecord(vsplats, g);
                    int xl, xh, yl, yh, zl, zh;
                    cull_range_v(r.m[0], r.e[0], X0f, xmax, xl, xh);
                    cull_range_v(r.m[1], r.e[1], Y0f, ymax, yl, yh);
                    cull_range_v(r.m[2], r.e[2], Z0f, zmax, zl, zh);
                    float q[6];
                    raw_conic(vsplats, g, q);
                    brick_rows(r.m[0], r.m[1], r.m[2], q, s_threshold_v(r.w), X0f, Y0f, Z0f, xl,
                               xh, yl, yh, zl, zh, tlo, thi, ezl, ezh);
                }
            }
            const bool live = ezl <= ezh;
            bucket[k] = live ? ezl * 8 + ezh : 64;
            s_g[idx] = g;
            s_tab[idx] = make_uint2(tlo, thi);
            s_zr[idx] = live ? (uint8_t)(ezl | (ezh << 4)) : (uint8_t)0x0f;
            rank[k] = atomicAdd(&s_cnt[bucket[k]], 1);
        }
        __syncthreads();
        if (warp == 0) {  // exclusive scan of the 65 bucket counts, 3 per lane
            int c[3], sum = 0;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int b = lane * 3 + j;
                c[j] = b < 65 ? s_cnt[b] : 0;
                sum += c[j];
            }
            const int excl = warp_inclusive_scan(sum) - sum;
            int run = excl;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int b = lane * 3 + j;
                if (b < 65) s_cnt[b] = run;
                run += c[j];
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            s_perm[s_cnt[bucket[k]] + rank[k]] = (uint16_t)(k * kVBwd8Threads + tid);
        if (tid == 0) s_next = kVBwd8Threads / 32;
        __syncthreads();
        const int n_groups = (min(kVBwd8Batch, end - base) + 31) >> 5;

        // groups are taken from a shared counter: sorted groups differ in cost
        auto process = [&](int grp) {
            const int idx = s_perm[grp * 32 + lane];
            const uint32_t zr = s_zr[idx];
            const int zl = zr & 15, zh = zr >> 4;
            const bool live = zl <= zh;
            const int z0 = __reduce_min_sync(0xffffffffu, live ? zl : 15);
            const int z1 = __reduce_max_sync(0xffffffffu, live ? zh : 0);
            if (z0 > z1) return;  // warp-uniform
            const int64_t g = s_g[idx];
            const uint2 tab = s_tab[idx];
            const VRecord r = load_vrecord(vsplats, g);

            // z = s_thr - s from the chain (s_thr enters through the slice
            // term): kept when z >= 0, in the cut-off band when |z| <= band;
            // the sums run over 2^z and are scaled by 2^-s_thr per record
            const float s_thr = s_threshold_v(r.w);
            float z_min = CUDART_INF_F;
            const float2 A2 = make_float2(r.A, r.A);
            float2 dx[4], col[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                dx[j] = make_float2((X0f + (2 * j + 0.5f)) - r.m[0], (X0f + (2 * j + 1.5f)) - r.m[0]);
                col[j] = make_float2(0.f, 0.f);
            }
            float Sy = 0.f, Sz = 0.f, Syy = 0.f, Syz = 0.f, Szz = 0.f, Sxy = 0.f, Sxz = 0.f;
            for (int z = z0; z <= z1; ++z) {
                const uint32_t byte = ((z < 4 ? tab.x : tab.y) >> (8 * (z & 3))) & 0xffu;
                const int ylo = live ? (int)(byte & 15u) : 15, yhi = live ? (int)(byte >> 4) : 0;
                const int y0 = __reduce_min_sync(0xffffffffu, ylo);
                const int y1 = __reduce_max_sync(0xffffffffu, yhi);
                if (y0 > y1) continue;  // warp-uniform: no row of this slice
                const float dz = (Z0f + ((float)z + 0.5f)) - r.m[2];
                const float cdz = r.Cq * dz, edz = r.E * dz, fzz = fmaf(r.F * dz, dz, s_thr);
                for (int y = y0; y <= y1; ++y) {
                    const bool rin = y >= ylo && y <= yhi;
                    const float dy = (Y0f + ((float)y + 0.5f)) - r.m[1];
                    const float by = fmaf(r.B, dy, cdz);
                    const float rest = fmaf(dy, fmaf(r.D, dy, edz), fzz);
                    const float2 by2 = make_float2(by, by), rest2 = make_float2(rest, rest);
                    const float4* vr = reinterpret_cast<const float4*>(s_v + z * 64 + y * 8);
                    const float4 va = vr[0], vb = vr[1];
                    float2 r0 = make_float2(0.f, 0.f), r1 = r0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 v2 = j == 0   ? make_float2(va.x, va.y)
                                          : j == 1 ? make_float2(va.z, va.w)
                                          : j == 2 ? make_float2(vb.x, vb.y)
                                                   : make_float2(vb.z, vb.w);
                        const float2 z2 = ffma2(dx[j], ffma2(A2, dx[j], by2), rest2);  // s_thr - s
                        float e0 = exp2f(z2.x), e1 = exp2f(z2.y);
                        z_min = fminf(z_min, fminf(fabsf(z2.x), fabsf(z2.y)));
                        e0 = (rin && z2.x >= 0.f) ? e0 : 0.f;
                        e1 = (rin && z2.y >= 0.f) ? e1 : 0.f;
                        const float2 ve = fmul2(v2, make_float2(e0, e1));
                        col[j] = fadd2(col[j], ve);
                        r0 = fadd2(r0, ve);
                        r1 = ffma2(ve, dx[j], r1);
                    }
                    const float R0 = r0.x + r0.y, R1 = r1.x + r1.y;
                    Sy = fmaf(dy, R0, Sy);
                    Sz = fmaf(dz, R0, Sz);
                    Syy = fmaf(dy * dy, R0, Syy);
                    Syz = fmaf(dy * dz, R0, Syz);
                    Szz = fmaf(dz * dz, R0, Szz);
                    Sxy = fmaf(dy, R1, Sxy);
                    Sxz = fmaf(dz, R1, Sxz);
                }
            }
            if (!live) return;
            if (!(z_min > r.band)) s_fix[atomicAdd(&s_nfix, 1)] = (uint16_t)idx;  // also NaN
            float S0 = 0.f, Sx = 0.f, Sxx = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                S0 += col[j].x + col[j].y;
                const float2 cx = fmul2(col[j], dx[j]);
                Sx += cx.x + cx.y;
                Sxx = fmaf(cx.x, dx[j].x, Sxx);
                Sxx = fmaf(cx.y, dx[j].y, Sxx);
            }
            const float k = exp2f(-s_thr);  // 2^-s_thr: the sums back to e^-sigma
            const float m[10] = {S0 * k,  Sx * k,  Sy * k,  Sz * k,  Sxx * k,
                                 Sxy * k, Sxz * k, Syy * k, Syz * k, Szz * k};
            vstats_red(stats + g * 12, m);
                };
        int grp = warp;
        while (grp < n_groups) {
            process(grp);
            __syncwarp();
            int nxt = 0;
            if (lane == 0) nxt = atomicAdd(&s_next, 1);
            grp = __shfl_sync(0xffffffffu, nxt, 0);
        }
        __syncthreads();
        // records with a voxel in the cut-off band: every voxel of the brick
        // re-decided by the reference's own test, two voxels per thread;
        // where the decisions differ (a few voxels in a million records), the
        // voxel's moments are added to or taken back from the record's
        // float64 sums
        const int n_fix = s_nfix;
        for (int f = 0; f < n_fix; ++f) {
            const int idx = s_fix[f];
            const int64_t g = s_g[idx];
            const uint2 tab = s_tab[idx];
            const float4 a = vsplats[4 * g], b = vsplats[4 * g + 1], c = vsplats[4 * g + 2];
            const float kc[6] = {a.w, b.x, b.y, b.z, b.w, c.x};  // raw conic (raw_conic)
            // the pre-scaled coefficients of load_vrecord, operation for operation
            const float A = -0.5f * kLog2eV * a.w, B = -kLog2eV * b.x, Cq = -kLog2eV * b.y;
            const float D = -0.5f * kLog2eV * b.z, E = -kLog2eV * b.w, F = -0.5f * kLog2eV * c.x;
            const float s_thr = s_threshold_v(c.y);
            const float band = vsplats[4 * g + 3].y;
#pragma unroll 1
            for (int vox = tid; vox < 512; vox += kVBwd8Threads) {
                const int z = vox >> 6, y = (vox >> 3) & 7, x = vox & 7;
                if (x > xmax || y > ymax || z > zmax) continue;
                // the main loop's fast decision, operation for operation; a
                // voxel outside the row table is dropped by both tests
                const uint32_t byte = ((z < 4 ? tab.x : tab.y) >> (8 * (z & 3))) & 0xffu;
                if (y < (int)(byte & 15u) || y > (int)(byte >> 4)) continue;
                const float dx = (X0f + ((float)x + 0.5f)) - a.x;
                const float dy = (Y0f + ((float)y + 0.5f)) - a.y;
                const float dz = (Z0f + ((float)z + 0.5f)) - a.z;
                const float cdz = Cq * dz, edz = E * dz, fzz = fmaf(F * dz, dz, s_thr);
                const float by = fmaf(B, dy, cdz);
                const float rest = fmaf(dy, fmaf(D, dy, edz), fzz);
                const float zz = fmaf(dx, fmaf(A, dx, by), rest);
                const bool fast = zz >= 0.f;
                // outside the band the sign of z is the reference's decision
                const bool exact =
                    fabsf(zz) > band ? zz >= 0.f : ref_keep3d(kc, c.y, dx, dy, dz);
                if (fast == exact) continue;
                const float ve = (exact ? 1.0f : -1.0f) * s_v[vox] * (exp2f(zz) * exp2f(-s_thr));
                const float vx = ve * dx, vy = ve * dy, vz = ve * dz;
                const float mv[10] = {ve, vx, vy, vz, vx * dx, vx * dy, vx * dz, vy * dy, vy * dz,
                                      vz * dz};
                vstats_red(stats + g * 12, mv);
            }
        }
        __syncthreads();
    }
}

template <typename S>
__global__ void voxel_unpack_kernel(const S* __restrict__ stats, const S* __restrict__ conics,
                                    const S* __restrict__ opac, int64_t N, S* __restrict__ v_m3,
                                    S* __restrict__ v_con, S* __restrict__ v_op) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    const S* st = stats + g * 12;
    const S* q = conics + g * 6;
    const S w = opac[g];
    v_m3[3 * g] = w * (q[0] * st[1] + q[1] * st[2] + q[2] * st[3]);
    v_m3[3 * g + 1] = w * (q[1] * st[1] + q[3] * st[2] + q[4] * st[3]);
    v_m3[3 * g + 2] = w * (q[2] * st[1] + q[4] * st[2] + q[5] * st[3]);
    const S h = static_cast<S>(0.5);
    v_con[6 * g] = -w * h * st[4];
    v_con[6 * g + 1] = -w * st[5];
    v_con[6 * g + 2] = -w * st[6];
    v_con[6 * g + 3] = -w * h * st[7];
    v_con[6 * g + 4] = -w * st[8];
    v_con[6 * g + 5] = -w * h * st[9];
    v_op[g] = st[0];
}

int check_bricks(uint32_t T, uint32_t nt2, uint32_t nt1, uint32_t layers) {
    R2S_REQUIRE(T > 0 && T * T * T <= 1024,
                "3D tile_size must be positive with tile_size**3 <= 1024");
    R2S_REQUIRE(nt2 > 0 && nt1 > 0 && nt2 <= 65535 && nt1 <= 65535 && layers <= 65535,
                "voxelize: brick grid out of range");
    return R2S_OK;
}

template <typename S, bool SPLATS>
int launch_voxel_fwd(const VoxSrc<S>& src, const int32_t* offsets, const int32_t* flatten_ids,
                     int64_t n_isects, uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t T,
                     uint32_t nt2, uint32_t nt1, uint32_t layer_begin, uint32_t layer_end, S* vol,
                     cudaStream_t stream) {
    BrickGeom geo;
    geo.T = (int)T;
    geo.nthr = (int)(T * T * T);
    const int n_warps = (geo.nthr + 31) / 32;
    const size_t smem = 10 * al16v((size_t)geo.nthr * sizeof(S)) +
                        al16v((size_t)std::max(geo.nthr, n_warps * 6) * 4) + n_warps * 8;
    auto kern = voxel_fwd_kernel<S, SPLATS>;
    if (int rc = set_dynamic_smem(kern, smem, "voxelize")) return rc;
    const uint32_t layers = layer_end - layer_begin;
    const dim3 grid(nt2, nt1, layers);
    kern<<<grid, geo.nthr, smem, stream>>>(src, offsets, flatten_ids,
                                           (int64_t)layers * nt1 * nt2, n_isects, dim2, dim1, dim0,
                                           geo, nt2, nt1, layer_begin, vol);
    return check_launch("voxelize_to_voxels_fwd");
}

template <typename S, bool SPLATS, int EXPMODE>
int launch_voxel_bwd(const VoxSrc<S>& src, const int32_t* offsets, const int32_t* flatten_ids,
                     const S* v_vol, int64_t N, int64_t n_isects, uint32_t dim2, uint32_t dim1,
                     uint32_t dim0, uint32_t T, uint32_t nt2, uint32_t nt1, uint32_t layer_begin,
                     uint32_t layer_end, VStat<S, SPLATS>* stats, cudaStream_t stream) {
    cudaMemsetAsync(stats, 0, (size_t)N * 12 * sizeof(VStat<S, SPLATS>), stream);
    if (n_isects == 0) return check_launch("voxelize_to_voxels_bwd");
    const int nthr = 256;
    const size_t smem = al16v((size_t)T * T * T * sizeof(S)) + 10 * al16v((size_t)nthr * sizeof(S)) +
                        al16v((size_t)nthr * 4) + (size_t)nthr * 8;
    auto kern = voxel_bwd_kernel<S, SPLATS, EXPMODE>;
    if (int rc = set_dynamic_smem(kern, smem, "voxelize")) return rc;
    const uint32_t layers = layer_end - layer_begin;
    const dim3 grid(nt2, nt1, layers);
    kern<<<grid, nthr, smem, stream>>>(src, offsets, flatten_ids, (int64_t)layers * nt1 * nt2,
                                       n_isects, v_vol, dim2, dim1, dim0, (int)T, nt2, nt1,
                                       layer_begin, stats);
    return check_launch("voxelize_to_voxels_bwd");
}

}  // namespace

}  // namespace r2s

using namespace r2s;

extern "C" int r2s_voxelize_to_voxels_fwd(int dtype, const void* means3d, const void* conics,
                                          const void* opacities, const int32_t* offsets,
                                          const int32_t* flatten_ids, int64_t N, int64_t n_isects,
                                          uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t T,
                                          uint32_t nt2, uint32_t nt1, uint32_t nt0, void* volume,
                                          r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0 && n_isects >= 0, "voxelize_to_voxels_fwd: negative size");
    const size_t es = dtype == R2S_F64 ? 8 : 4;
    const int64_t nvox = (int64_t)dim0 * dim1 * dim2;
    if (nvox == 0) return R2S_OK;
    if (N == 0 || n_isects == 0) {
        cudaMemsetAsync(volume, 0, nvox * es, stream);
        return check_launch("voxelize_to_voxels_fwd");
    }
    if (int rc = check_bricks(T, nt2, nt1, nt0)) return rc;
    R2S_REQUIRE((uint64_t)nt2 * T >= dim2 && (uint64_t)nt1 * T >= dim1 && (uint64_t)nt0 * T >= dim0,
                "voxelize: brick grid does not cover the volume");
    return R2S_DTYPE_DISPATCH(dtype, "voxelize_to_voxels_fwd", [&] {
        VoxSrc<scalar_t> src{nullptr, (const scalar_t*)means3d, (const scalar_t*)conics,
                             (const scalar_t*)opacities};
        return launch_voxel_fwd<scalar_t, false>(src, offsets, flatten_ids, n_isects, dim2, dim1,
                                                 dim0, T, nt2, nt1, 0, nt0, (scalar_t*)volume,
                                                 stream);
    });
}

extern "C" int r2s_voxelize_to_voxels_bwd(int dtype, int mode, const void* means3d,
                                          const void* conics, const void* opacities,
                                          const int32_t* offsets, const int32_t* flatten_ids,
                                          const void* v_volume, int64_t N, int64_t n_isects,
                                          uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t T,
                                          uint32_t nt2, uint32_t nt1, uint32_t nt0, void* stats,
                                          void* v_means3d, void* v_conics, void* v_opacities,
                                          r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0 && n_isects >= 0, "voxelize_to_voxels_bwd: negative size");
    R2S_REQUIRE(mode == 0 || mode == 1, "voxelize_to_voxels_bwd: mode must be 0 or 1");
    const size_t es = dtype == R2S_F64 ? 8 : 4;
    if (N == 0) return R2S_OK;
    if (n_isects == 0 || (int64_t)dim0 * dim1 * dim2 == 0) {
        cudaMemsetAsync(v_means3d, 0, N * 3 * es, stream);
        cudaMemsetAsync(v_conics, 0, N * 6 * es, stream);
        cudaMemsetAsync(v_opacities, 0, N * es, stream);
        return check_launch("voxelize_to_voxels_bwd");
    }
    if (int rc = check_bricks(T, nt2, nt1, nt0)) return rc;
    return R2S_DTYPE_DISPATCH(dtype, "voxelize_to_voxels_bwd", [&] {
        VoxSrc<scalar_t> src{nullptr, (const scalar_t*)means3d, (const scalar_t*)conics,
                             (const scalar_t*)opacities};
        int rc = mode == 0 ? launch_voxel_bwd<scalar_t, false, 0>(
                                 src, offsets, flatten_ids, (const scalar_t*)v_volume, N, n_isects,
                                 dim2, dim1, dim0, T, nt2, nt1, 0, nt0, (scalar_t*)stats, stream)
                           : launch_voxel_bwd<scalar_t, false, 1>(
                                 src, offsets, flatten_ids, (const scalar_t*)v_volume, N, n_isects,
                                 dim2, dim1, dim0, T, nt2, nt1, 0, nt0, (scalar_t*)stats, stream);
        if (rc) return rc;
        voxel_unpack_kernel<scalar_t><<<grid_for(N), kThreads, 0, stream>>>(
            (const scalar_t*)stats, (const scalar_t*)conics, (const scalar_t*)opacities, N,
            (scalar_t*)v_means3d, (scalar_t*)v_conics, (scalar_t*)v_opacities);
        return check_launch("voxelize_to_voxels_bwd");
    });
}

extern "C" int r2s_voxel_rows_f32(const float* vsplats, const int32_t* offsets,
                                  const int32_t* flatten_ids, int64_t N, int64_t n_isects,
                                  uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t T,
                                  uint32_t nt2, uint32_t nt1, uint32_t nt0, uint32_t layer_begin,
                                  uint32_t layer_end, const int32_t* brick_order, uint32_t* rows,
                                  r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0 && n_isects >= 0, "voxel_rows: negative size");
    R2S_REQUIRE(T == 8, "voxel_rows: the row table is built for 8-voxel bricks");
    R2S_REQUIRE(layer_begin <= layer_end && layer_end <= nt0, "voxel_rows: bad layer range");
    if (int rc = check_bricks(T, nt2, nt1, nt0)) return rc;
    if (N == 0 || n_isects == 0 || layer_end == layer_begin) return R2S_OK;
    R2S_REQUIRE(rows != nullptr, "voxel_rows: null output");
    const dim3 grid(nt2, nt1, layer_end - layer_begin);
    voxel_rows8_kernel<<<grid, kVRowsThreads, 0, stream>>>(
        (const float4*)vsplats, offsets, flatten_ids,
        (int64_t)(layer_end - layer_begin) * nt1 * nt2, n_isects, N, dim2, dim1, dim0, nt2, nt1,
        layer_begin, brick_order, reinterpret_cast<uint2*>(rows));
    return check_launch("voxel_rows");
}

extern "C" int r2s_voxel_splats_fwd_f32(const float* vsplats, const int32_t* offsets,
                                        const int32_t* flatten_ids, const uint32_t* rows,
                                        int64_t N, int64_t n_isects,
                                        uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t T,
                                        uint32_t nt2, uint32_t nt1, uint32_t nt0,
                                        uint32_t layer_begin, uint32_t layer_end,
                                        const int32_t* brick_order, float* volume,
                                        r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0 && n_isects >= 0, "voxel_splats_fwd: negative size");
    R2S_REQUIRE(layer_begin <= layer_end && layer_end <= nt0, "voxel_splats_fwd: bad layer range");
    if (int rc = check_bricks(T, nt2, nt1, nt0)) return rc;
    const int64_t zb = (int64_t)layer_begin * T;
    const int64_t ze = std::min<int64_t>((int64_t)layer_end * T, dim0);
    if (ze <= zb || (int64_t)dim1 * dim2 == 0) return R2S_OK;
    if (N == 0 || n_isects == 0) {
        cudaMemsetAsync(volume, 0, (size_t)(ze - zb) * dim1 * dim2 * 4, stream);
        return check_launch("voxel_splats_fwd");
    }
    if (T == 8) {
        const dim3 grid(nt2, nt1, layer_end - layer_begin);
        const int64_t n_keys = (int64_t)(layer_end - layer_begin) * nt1 * nt2;
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (n_isects < kVFwd8GroupedRecordsPerSM * std::max(sms, 1))
            voxel_fwd8_kernel<4><<<grid, 64 * 4, 0, stream>>>(
                (const float4*)vsplats, offsets, flatten_ids, reinterpret_cast<const uint2*>(rows),
                n_keys, n_isects, N, dim2, dim1, dim0, nt2, nt1, layer_begin, brick_order, volume);
        else
            voxel_fwd8_kernel<1><<<grid, 64, 0, stream>>>(
                (const float4*)vsplats, offsets, flatten_ids, reinterpret_cast<const uint2*>(rows),
                n_keys, n_isects, N, dim2, dim1, dim0, nt2, nt1, layer_begin, brick_order, volume);
        return check_launch("voxel_splats_fwd");
    }
    VoxSrc<float> src{(const float4*)vsplats, nullptr, nullptr, nullptr};
    return launch_voxel_fwd<float, true>(src, offsets, flatten_ids, n_isects, dim2, dim1, dim0, T,
                                         nt2, nt1, layer_begin, layer_end, volume, stream);
}

extern "C" int r2s_voxel_splats_bwd_f32(const float* vsplats, const int32_t* offsets,
                                        const int32_t* flatten_ids, const uint32_t* rows,
                                        const float* v_volume,
                                        int64_t N, int64_t n_isects, uint32_t dim2, uint32_t dim1,
                                        uint32_t dim0, uint32_t T, uint32_t nt2, uint32_t nt1,
                                        uint32_t nt0, uint32_t layer_begin, uint32_t layer_end,
                                        const int32_t* brick_order, double* stats,
                                        r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0 && n_isects >= 0, "voxel_splats_bwd: negative size");
    R2S_REQUIRE(layer_begin <= layer_end && layer_end <= nt0, "voxel_splats_bwd: bad layer range");
    if (int rc = check_bricks(T, nt2, nt1, nt0)) return rc;
    if (N == 0) return R2S_OK;
    if (T == 8) {
        cudaMemsetAsync(stats, 0, (size_t)N * 12 * sizeof(double), stream);
        if (n_isects > 0 && layer_end > layer_begin) {
            const dim3 grid(nt2, nt1, layer_end - layer_begin);
            voxel_bwd8_kernel<<<grid, kVBwd8Threads, 0, stream>>>(
                (const float4*)vsplats, offsets, flatten_ids, reinterpret_cast<const uint2*>(rows),
                (int64_t)(layer_end - layer_begin) * nt1 * nt2, n_isects, N, v_volume, dim2,
                dim1, dim0, nt2, nt1, layer_begin, brick_order, stats);
        }
        return check_launch("voxel_splats_bwd");
    }
    VoxSrc<float> src{(const float4*)vsplats, nullptr, nullptr, nullptr};
    return launch_voxel_bwd<float, true, 0>(src, offsets, flatten_ids, v_volume, N, n_isects, dim2,
                                            dim1, dim0, T, nt2, nt1, layer_begin, layer_end, stats,
                                            stream);
}

extern "C" int r2s_brick_order(const int32_t* offsets, int64_t n_keys, int64_t n_isects,
                               int32_t* order, r2s_stream_t stream) {
    R2S_REQUIRE(n_keys >= 0 && n_isects >= 0, "brick_order: negative size");
    if (n_keys == 0) return R2S_OK;
    R2S_REQUIRE(n_keys <= INT32_MAX, "brick_order: too many bricks");
    brick_order_kernel<<<1, kOrderThreads, 0, stream>>>(offsets, n_keys, n_isects, order);
    return check_launch("brick_order");
}

namespace r2s {
R2S_DBG_DEFINE_READER(debug_flags_voxel)
}  // namespace r2s
