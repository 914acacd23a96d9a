// Tile binning by stable counting placement.
//
// The reference (csrc/IsectTiles.cpp:30-170, csrc/IsectTilesKernel.cu:137-445)
// emits one (key, value) record per (splat, tile) with key = segment *
// n_tiles + tile and value = the splat's flattened index, then CUB-radix-sorts
// the keys stably.  Because records are emitted in ascending value order, the
// sorted result is: for every key, the values of all splats covering that
// tile, ascending.  This file produces exactly that order without a sort:
//
//   phase 1  per (segment, chunk of items): histogram of records per tile
//            (one CTA per chunk, shared-memory counters)
//   phase 2  per (segment, tile): exclusive prefix over chunks (column scan),
//            then an exclusive scan of the per-tile totals -> tile offsets
//            and n_isects (the reference's isect_offset_encode output falls
//            out of this scan directly)
//   phase 3  per (segment, chunk): one warp walks the chunk's items in order,
//            one item per step with its records spread over the lanes, and
//            writes each record to offsets[tile] + running count; an item's
//            records cover distinct tiles, so lanes never share a counter and
//            item order is kept without ranking
//
// The sorted keys (isect_ids) are a run-length expansion of the offsets and
// are written by a separate coalesced kernel only when a caller asks for them.
//
// Segments are views (2D: items s*N + i, rects [C*N]) or z-layers of bricks
// (3D, "layered": items i in [0, N) restricted to Gaussians whose brick range
// contains the layer, rects [N]).
#include "r2s_common.cuh"
#include "r2s_tiles.cuh"
#include "r2s_debug.cuh"

namespace r2s {

namespace {

constexpr int64_t kMinChunk = 2048;
constexpr int64_t kMaxChunk = 65536;
constexpr int64_t kHistBudget = int64_t(256) << 20;  // bytes of per-chunk histograms
constexpr int kSmemLimit = 200 * 1024;

struct BinPlan {
    int64_t chunk;
    int64_t n_chunks;
    int64_t hist_elems;
    int64_t totals_elems;
    int64_t bytes;
};

inline int64_t align256(int64_t b) { return (b + 255) & ~int64_t(255); }

BinPlan make_plan(int64_t S, int64_t N, int64_t T) {
    BinPlan p{};
    p.chunk = kMinChunk;
    for (;;) {
        p.n_chunks = (N + p.chunk - 1) / p.chunk;
        if (p.n_chunks < 1) p.n_chunks = 1;
        if (S * p.n_chunks * T * 4 <= kHistBudget || p.chunk >= kMaxChunk) break;
        p.chunk *= 2;
    }
    p.hist_elems = S * p.n_chunks * T;
    p.totals_elems = S * T;
    p.bytes = align256(p.hist_elems * 4) + align256(p.totals_elems * 4) + 256;
    return p;
}

struct ItemRect {
    uint32_t x0, x1, y0, y1;
    int n;
};

template <bool LAYERED>
__device__ __forceinline__ ItemRect load_rect(const void* rects, int64_t s, int64_t i, int64_t N,
                                              int64_t layer) {
    ItemRect r;
    uint32_t px, py;
    if constexpr (LAYERED) {
        const Rect3 q = reinterpret_cast<const Rect3*>(rects)[i];
        const uint32_t z0 = lo16(q.z), z1 = hi16(q.z);
        px = q.x;
        py = q.y;
        if (layer < (int64_t)z0 || layer >= (int64_t)z1) px = py = 0;
    } else {
        const Rect2 q = reinterpret_cast<const Rect2*>(rects)[s * N + i];
        px = q.x;
        py = q.y;
    }
    r.x0 = lo16(px);
    r.x1 = hi16(px);
    r.y0 = lo16(py);
    r.y1 = hi16(py);
    r.n = (r.x1 > r.x0 && r.y1 > r.y0) ? (int)((r.x1 - r.x0) * (r.y1 - r.y0)) : 0;
    return r;
}

// Phase 1: per-(segment, chunk) tile histogram.
template <bool LAYERED>
__global__ void __launch_bounds__(256) bin_count_kernel(const void* __restrict__ rects, int64_t N,
                                                        int T, uint32_t tiles_x,
                                                        int64_t seg_base, int64_t chunk,
                                                        int64_t n_chunks,
                                                        int32_t* __restrict__ hist) {
    extern __shared__ int32_t h[];
    const int64_t k = blockIdx.x;
    const int64_t s = blockIdx.y;
    for (int t = threadIdx.x; t < T; t += blockDim.x) h[t] = 0;
    __syncthreads();
    const int64_t i0 = k * chunk;
    const int64_t i1 = min(N, i0 + chunk);
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const ItemRect r = load_rect<LAYERED>(rects, s, i, N, seg_base + s);
        if (r.n == 0) continue;
        for (uint32_t y = r.y0; y < r.y1; ++y)
            for (uint32_t x = r.x0; x < r.x1; ++x) atomicAdd(&h[y * tiles_x + x], 1);
    }
    __syncthreads();
    int32_t* out = hist + (s * n_chunks + k) * (int64_t)T;
    for (int t = threadIdx.x; t < T; t += blockDim.x) out[t] = h[t];
}

// Phase 2a: exclusive prefix of every (segment, tile) column over chunks.
__global__ void bin_colscan_kernel(int32_t* __restrict__ hist, int64_t S, int64_t n_chunks, int T,
                                   int32_t* __restrict__ totals) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= S * T) return;
    const int64_t s = idx / T, t = idx - s * T;
    int32_t* col = hist + s * n_chunks * T + t;
    int32_t run = 0;
    // eight loads in flight per thread: the column walk is latency-bound
    int64_t k = 0;
    for (; k + 8 <= n_chunks; k += 8) {
        int32_t v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = col[(k + u) * T];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            col[(k + u) * T] = run;
            run += v[u];
        }
    }
    for (; k < n_chunks; ++k) {
        const int32_t v = col[k * T];
        col[k * T] = run;
        run += v;
    }
    totals[idx] = run;
}

// Phase 2b: exclusive scan of the per-tile totals (single CTA).
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) bin_scan_kernel(const int32_t* __restrict__ totals,
                                                                int64_t n,
                                                                int32_t* __restrict__ offsets,
                                                                int64_t* __restrict__ n_isects) {
    __shared__ int64_t part[kScanThreads];
    const int tid = threadIdx.x;
    const int64_t per = (n + kScanThreads - 1) / kScanThreads;
    const int64_t b = tid * per, e = min(n, b + per);
    int64_t local = 0;
    for (int64_t j = b; j < e; ++j) local += totals[j];
    part[tid] = local;
    __syncthreads();
    for (int o = 1; o < kScanThreads; o <<= 1) {
        int64_t v = tid >= o ? part[tid - o] : 0;
        __syncthreads();
        part[tid] += v;
        __syncthreads();
    }
    int64_t run = part[tid] - local;
    for (int64_t j = b; j < e; ++j) {
        offsets[j] = static_cast<int32_t>(run);
        run += totals[j];
    }
    if (tid == kScanThreads - 1) *n_isects = part[tid];
}

// Phase 3: one warp per (segment, chunk) places the chunk's records.
template <bool LAYERED>
__global__ void bin_place_kernel(const void* __restrict__ rects, int64_t S, int64_t N, int T,
                                 uint32_t tiles_x, int64_t seg_base, int64_t chunk,
                                 int64_t n_chunks, const int32_t* __restrict__ hist,
                                 const int32_t* __restrict__ offsets,
                                 int32_t* __restrict__ flatten_ids, int64_t n_isects) {
    extern __shared__ int32_t smem[];
    const int warps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int32_t* cnt = smem + (int64_t)warp * T;
    const int64_t gw = (int64_t)blockIdx.x * warps + warp;
    if (gw >= S * n_chunks) return;
    const int64_t s = gw / n_chunks;
    const int64_t k = gw - s * n_chunks;
    const int32_t* hrow = hist + (s * n_chunks + k) * (int64_t)T;
    const int32_t* orow = offsets + s * (int64_t)T;
    for (int t = lane; t < T; t += 32) cnt[t] = orow[t] + hrow[t];
    __syncwarp();

    const int64_t i0 = k * chunk;
    const int64_t i1 = min(N, i0 + chunk);
    const int64_t id_base = LAYERED ? 0 : s * N;
    for (int64_t base = i0; base < i1; base += 32) {
        const int64_t i = base + lane;
        ItemRect r{0, 0, 0, 0, 0};
        if (i < i1) r = load_rect<LAYERED>(rects, s, i, N, seg_base + s);
        unsigned todo = __ballot_sync(0xffffffffu, r.n > 0);
        const uint32_t px = pack16(r.x0, r.x1), py = pack16(r.y0, r.y1);
        // One item at a time, in item order: its records cover distinct tiles,
        // so every lane owns a different counter and no ranking is needed.
        while (todo) {
            const int j = __ffs(todo) - 1;
            todo &= todo - 1;
            const uint32_t qx = __shfl_sync(0xffffffffu, px, j);
            const uint32_t qy = __shfl_sync(0xffffffffu, py, j);
            const int x0 = (int)lo16(qx), w = (int)(hi16(qx) - lo16(qx));
            const int y0 = (int)lo16(qy), h = (int)(hi16(qy) - lo16(qy));
            const int n = w * h;
            const int32_t id = (int32_t)(id_base + base + j);
            int dy = lane / w;
            int dx = lane - dy * w;
            const int sdy = 32 / w, sdx = 32 - sdy * w;
            for (int q = lane; q < n; q += 32) {
                const int tile = (y0 + dy) * (int)tiles_x + x0 + dx;
                const int pos = cnt[tile];
                if (!R2S_DBG_BAD(pos >= 0 && pos < n_isects, R2S_DBG_SLOT)) flatten_ids[pos] = id;
                cnt[tile] = pos + 1;
                dy += sdy;
                dx += sdx;
                if (dx >= w) { dx -= w; ++dy; }
            }
            __syncwarp();
        }
    }
}

// Warp walk over items [w0, w1) in item order: for every record (item, tile)
// calls emit(tile, item - i_base) on one lane.  One item per step, its records
// spread over the lanes; an item's records cover distinct tiles, so lanes of
// one step never share a tile.
template <bool LAYERED, typename Emit>
__device__ __forceinline__ void walk_items(const void* __restrict__ rects, int64_t s, int64_t N,
                                           int64_t layer, int64_t w0, int64_t w1, int64_t i_base,
                                           uint32_t tiles_x, Emit&& emit) {
    const int lane = threadIdx.x & 31;
    for (int64_t base = w0; base < w1; base += 32) {
        const int64_t i = base + lane;
        ItemRect r{0, 0, 0, 0, 0};
        if (i < w1) r = load_rect<LAYERED>(rects, s, i, N, layer);
        // the owner lane decodes its item once: (x0 | w << 16), (y0 | n << 16), 1 / w
        const uint32_t w = r.x1 - r.x0;
        const uint32_t pa = r.x0 | (w << 16), pb = r.y0 | ((uint32_t)r.n << 16);
        const float prw = r.n > 0 ? 1.0f / (float)w : 0.f;
        unsigned todo = __ballot_sync(0xffffffffu, r.n > 0);
        const int local0 = (int)(base - i_base);
        int j = todo ? __ffs(todo) - 1 : 0;
        uint32_t qa = __shfl_sync(0xffffffffu, pa, j), qb = __shfl_sync(0xffffffffu, pb, j);
        float qr = __shfl_sync(0xffffffffu, prw, j);
        while (todo) {
            todo &= todo - 1;
            // fetch the next item while this one is placed
            const int jn = todo ? __ffs(todo) - 1 : 0;
            const uint32_t na = __shfl_sync(0xffffffffu, pa, jn);
            const uint32_t nb = __shfl_sync(0xffffffffu, pb, jn);
            const float nr = __shfl_sync(0xffffffffu, prw, jn);
            const int x0 = (int)(qa & 0xffffu), iw = (int)(qa >> 16);
            const int y0 = (int)(qb & 0xffffu), n = (int)(qb >> 16);
            // q / w for q < 2^21 records by a float reciprocal: (q + 0.5) / w
            // lies at least 0.5 / w from an integer, far above the rounding
            int dy = (int)(((float)lane + 0.5f) * qr);
            int dx = lane - dy * iw;
            const int sdy = (int)(32.5f * qr), sdx = 32 - sdy * iw;
            for (int q = lane; q < n; q += 32) {
                emit((y0 + dy) * (int)tiles_x + x0 + dx, local0 + j);
                dy += sdy;
                dx += sdx;
                if (dx >= iw) {
                    dx -= iw;
                    ++dy;
                }
            }
            __syncwarp();
            j = jn;
            qa = na;
            qb = nb;
            qr = nr;
        }
    }
}

// Per-tile record counts of items [w0, w1), one item per lane (order-free),
// into 16-bit counters packed two per 32-bit word (tile t: half t & 1 of word
// t >> 1, added with one 32-bit atomic; counts stay below 2^16).
template <bool LAYERED>
__device__ __forceinline__ void count_items(const void* __restrict__ rects, int64_t s, int64_t N,
                                            int64_t layer, int64_t w0, int64_t w1,
                                            uint32_t tiles_x, uint32_t* words) {
    for (int64_t i = w0 + (threadIdx.x & 31); i < w1; i += 32) {
        const ItemRect r = load_rect<LAYERED>(rects, s, i, N, layer);
        if (r.n == 0) continue;
        for (uint32_t y = r.y0; y < r.y1; ++y)
            for (uint32_t x = r.x0; x < r.x1; ++x) {
                const uint32_t t = y * tiles_x + x;
                atomicAdd(&words[t >> 1], (t & 1u) ? 0x10000u : 1u);
            }
    }
}

// Exclusive scan of v[0, n) into out[0, n) by one CTA; returns the total to
// every thread.  scratch holds 33 ints (one per warp, <= 32 warps, and the total).
__device__ __forceinline__ int block_exclusive_scan(const int32_t* v, int32_t* out, int n,
                                                    int32_t* scratch) {
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (n + nthr - 1) / nthr;
    const int b = min(n, tid * per), e = min(n, b + per);
    int local = 0;
    for (int j = b; j < e; ++j) local += v[j];
    const int incl = warp_inclusive_scan(local);
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = nthr >> 5;
        const int x = lane < nw ? scratch[lane] : 0;
        const int xi = warp_inclusive_scan(x);
        if (lane < nw) scratch[lane] = xi - x;
        if (lane == nw - 1) scratch[32] = xi;
    }
    __syncthreads();
    int run = scratch[warp] + incl - local;
    for (int j = b; j < e; ++j) {
        const int c = v[j];
        out[j] = run;
        run += c;
    }
    const int total = scratch[32];
    __syncthreads();
    return total;
}

constexpr int kStagedWarps = 16;

// Phase 3, staged: one CTA per (segment, chunk).  16 warps take consecutive
// sub-chunks; shared-memory atomics give per-(warp, tile) 16-bit counts (a chunk
// holds at most 2^16 items), whose prefix over
// warps and tiles places every record of the chunk in a tile-major staging
// buffer in shared memory (16-bit item offsets), in item order per tile.  The
// buffer is then written out one tile run at a time, so each tile's records
// of the chunk reach global memory as one contiguous store sequence.  A chunk
// with more records than the buffer holds writes its records directly.
template <bool LAYERED>
__global__ void __launch_bounds__(kStagedWarps * 32)
bin_place_staged_kernel(const void* __restrict__ rects, int64_t N, int T, uint32_t tiles_x,
                        int64_t seg_base, int64_t chunk, int64_t n_chunks,
                        const int32_t* __restrict__ hist, const int32_t* __restrict__ offsets,
                        int32_t* __restrict__ flatten_ids, int cap, int64_t n_isects) {
    extern __shared__ __align__(16) int32_t smem[];
    __shared__ int32_t s_scan[33];
    const int tid = threadIdx.x, nthr = blockDim.x, warp = tid >> 5, lane = tid & 31;
    const int TW = (T + 1) >> 1;  // 32-bit words per warp row of 16-bit counters
    uint32_t* wcw = reinterpret_cast<uint32_t*>(smem);  // [warps][TW]
    uint16_t* wc = reinterpret_cast<uint16_t*>(smem);   // [warps][2 TW]: counts, then positions
    int32_t* gpos = smem + kStagedWarps * TW;  // [T] first global position of the chunk's run
    int32_t* tot = gpos + T;             // [T] records of the chunk per tile
    int32_t* lofs = tot + T;             // [T] first staging slot per tile
    uint16_t* stage = reinterpret_cast<uint16_t*>(lofs + T);

    const int64_t s = blockIdx.x / n_chunks;
    const int64_t k = blockIdx.x - s * n_chunks;
    const int64_t i0 = k * chunk;
    const int64_t i1 = min(N, i0 + chunk);
    const int64_t layer = seg_base + s;
    const int64_t id0 = (LAYERED ? 0 : s * N) + i0;
    const int64_t per = (((i1 - i0) + kStagedWarps * 32 - 1) / (kStagedWarps * 32)) * 32;
    const int64_t w0 = min(i1, i0 + warp * per), w1 = min(i1, w0 + per);
    const int32_t* hrow = hist + (s * n_chunks + k) * (int64_t)T;
    const int32_t* orow = offsets + s * (int64_t)T;
    for (int t = tid; t < kStagedWarps * TW; t += nthr) wcw[t] = 0u;
    for (int t = tid; t < T; t += nthr) gpos[t] = orow[t] + hrow[t];
    __syncthreads();

    count_items<LAYERED>(rects, s, N, layer, w0, w1, tiles_x, wcw + warp * TW);
    uint16_t* mine = wc + warp * 2 * TW;
    __syncthreads();
    for (int t = tid; t < T; t += nthr) {
        int run = 0;
#pragma unroll
        for (int w = 0; w < kStagedWarps; ++w) {
            const int c = wc[w * 2 * TW + t];
            wc[w * 2 * TW + t] = (uint16_t)run;
            run += c;
        }
        tot[t] = run;
    }
    __syncthreads();
    const int total = block_exclusive_scan(tot, lofs, T, s_scan);
    if (total <= cap) {
        walk_items<LAYERED>(rects, s, N, layer, w0, w1, i0, tiles_x, [&](int tile, int local) {
            const int p = mine[tile];
            mine[tile] = (uint16_t)(p + 1);
            stage[lofs[tile] + p] = (uint16_t)local;
        });
        __syncthreads();
        for (int t = warp; t < T; t += kStagedWarps) {
            const int n = tot[t];
            const uint16_t* src = stage + lofs[t];
            int32_t* dst = flatten_ids + gpos[t];
            for (int j = lane; j < n; j += 32)
                if (!R2S_DBG_BAD(gpos[t] >= 0 && (int64_t)gpos[t] + j < n_isects, R2S_DBG_SLOT))
                    dst[j] = (int32_t)(id0 + src[j]);
        }
    } else {
        walk_items<LAYERED>(rects, s, N, layer, w0, w1, i0, tiles_x, [&](int tile, int local) {
            const int p = mine[tile];
            mine[tile] = (uint16_t)(p + 1);
            if (!R2S_DBG_BAD(gpos[tile] + p >= 0 && (int64_t)gpos[tile] + p < n_isects,
                             R2S_DBG_SLOT))
                flatten_ids[gpos[tile] + p] = (int32_t)(id0 + local);
        });
    }
}

// Run-length expansion of the offsets into sorted int64 keys: one warp per key.
__global__ void decode_keys_kernel(const int32_t* __restrict__ offsets, int64_t n_keys,
                                   int64_t n_isects, int64_t key_base,
                                   int64_t* __restrict__ isect_ids) {
    const int64_t key = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (key >= n_keys) return;
    const int64_t b = offsets[key];
    const int64_t e = key + 1 < n_keys ? (int64_t)offsets[key + 1] : n_isects;
    const int64_t v = key_base + key;
    for (int64_t j = b + lane; j < e; j += 32) isect_ids[j] = v;
}

// offsets[k] = lower_bound(isect_ids, k) for a sorted key array.
__global__ void offset_encode_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t n_keys,
                                     int32_t* __restrict__ offsets) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n_keys) return;
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (ids[mid] < k) lo = mid + 1; else hi = mid;
    }
    offsets[k] = static_cast<int32_t>(lo);
}

template <typename S>
__global__ void rects_2d_kernel(const S* __restrict__ means2d, const int32_t* __restrict__ radii,
                                int rect_radii, int64_t total, uint32_t tile, uint32_t ntx,
                                uint32_t nty, Rect2* __restrict__ rects,
                                int32_t* __restrict__ tiles_per_gauss) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const S rx = static_cast<S>(rect_radii ? radii[2 * idx] : radii[idx]);
    const S ry = static_cast<S>(rect_radii ? radii[2 * idx + 1] : radii[idx]);
    int32_t count;
    rects[idx] = tile_rect_2d<S>(means2d[2 * idx], means2d[2 * idx + 1], rx, ry, tile, ntx, nty,
                                 count);
    tiles_per_gauss[idx] = count;
}

template <typename S>
__global__ void rects_3d_kernel(const S* __restrict__ means3d, const int32_t* __restrict__ radii,
                                int64_t N, uint32_t tile, uint32_t nt2, uint32_t nt1,
                                uint32_t nt0, Rect3* __restrict__ rects,
                                int32_t* __restrict__ tiles_per_gauss) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    int32_t count;
    rects[g] = tile_rect_3d<S>(means3d[3 * g], means3d[3 * g + 1], means3d[3 * g + 2],
                               static_cast<S>(radii[3 * g]), static_cast<S>(radii[3 * g + 1]),
                               static_cast<S>(radii[3 * g + 2]), tile, nt2, nt1, nt0, count);
    tiles_per_gauss[g] = count;
}

struct WsView {
    int32_t* hist;
    int32_t* totals;
};

WsView carve(void* ws, const BinPlan& p) {
    char* b = reinterpret_cast<char*>(ws);
    WsView v;
    v.hist = reinterpret_cast<int32_t*>(b);
    v.totals = reinterpret_cast<int32_t*>(b + align256(p.hist_elems * 4));
    return v;
}

int check_shape(int64_t S, int64_t N, int64_t T, uint32_t tiles_x) {
    R2S_REQUIRE(S >= 0 && N >= 0 && T >= 0, "binning: negative size");
    R2S_REQUIRE(N < (int64_t(1) << 31), "binning: more than 2^31 items per segment");
    R2S_REQUIRE(S * N < (int64_t(1) << 31), "binning: flattened index exceeds int32");
    R2S_REQUIRE(tiles_x > 0 || T == 0, "binning: tiles_x must be positive");
    if ((int64_t)T * 4 + 96 * 4 > kSmemLimit)
        return fail(R2S_ERR_UNSUPPORTED,
                    "binning: %lld tiles per segment exceed the shared-memory counters "
                    "of this build (max %d)",
                    (long long)T, (kSmemLimit - 384) / 4);
    return R2S_OK;
}

}  // namespace

int bin_prepare_impl(const void* rects, int64_t S, int64_t N, int64_t T, uint32_t tiles_x,
                     bool layered, int64_t seg_base, void* ws, int64_t ws_bytes,
                     int32_t* offsets, int64_t* n_isects_dev, cudaStream_t stream) {
    if (int rc = check_shape(S, N, T, tiles_x)) return rc;
    const BinPlan p = make_plan(S, N, T);
    R2S_REQUIRE(ws_bytes >= p.bytes || S * T == 0,
                "binning: workspace of %lld bytes is smaller than the required %lld",
                (long long)ws_bytes, (long long)p.bytes);
    if (S * T == 0) {
        cudaMemsetAsync(n_isects_dev, 0, sizeof(int64_t), stream);
        return check_launch("bin_prepare");
    }
    const WsView w = carve(ws, p);
    if (N > 0) {
        const dim3 grid((unsigned)p.n_chunks, (unsigned)S);
        const size_t smem = (size_t)T * 4;
        if (layered) {
            if (int rc = set_dynamic_smem(bin_count_kernel<true>, smem, "binning")) return rc;
            bin_count_kernel<true><<<grid, 256, smem, stream>>>(rects, N, (int)T, tiles_x, seg_base,
                                                                p.chunk, p.n_chunks, w.hist);
        } else {
            if (int rc = set_dynamic_smem(bin_count_kernel<false>, smem, "binning")) return rc;
            bin_count_kernel<false><<<grid, 256, smem, stream>>>(rects, N, (int)T, tiles_x, seg_base,
                                                                 p.chunk, p.n_chunks, w.hist);
        }
        bin_colscan_kernel<<<grid_for(S * T), kThreads, 0, stream>>>(w.hist, S, p.n_chunks,
                                                                     (int)T, w.totals);
    } else {
        cudaMemsetAsync(w.totals, 0, S * T * 4, stream);
    }
    bin_scan_kernel<<<1, kScanThreads, 0, stream>>>(w.totals, S * T, offsets, n_isects_dev);
    return check_launch("bin_prepare");
}

int bin_place_impl(const void* rects, int64_t S, int64_t N, int64_t T, uint32_t tiles_x,
                   bool layered, int64_t seg_base, const void* ws, int64_t ws_bytes,
                   const int32_t* offsets, int64_t n_isects, int32_t* flatten_ids,
                   int64_t* isect_ids, cudaStream_t stream) {
    if (int rc = check_shape(S, N, T, tiles_x)) return rc;
    R2S_REQUIRE(n_isects >= 0, "binning: negative n_isects");
    if (n_isects > INT32_MAX)
        return fail(R2S_ERR_CAPACITY,
                    "binning: %lld intersections exceed the int32 index space of the "
                    "tile offsets; split the views into smaller batches",
                    (long long)n_isects);
    if (n_isects == 0 || S * T == 0 || N == 0) return R2S_OK;
    const BinPlan p = make_plan(S, N, T);
    R2S_REQUIRE(ws_bytes >= p.bytes, "binning: workspace too small");
    const WsView w = carve(const_cast<void*>(ws), p);
    // staged placement when the per-(warp, tile) counters leave room for a
    // staging buffer of at least 4096 records: in 112 KB, two 16-warp CTAs per
    // SM (2 x (112 + 1) KB of the SM's 228 KB; 2304 tiles per segment, a 768^2
    // detector, leave 6656 records), else in 224 KB, one CTA per SM (4096
    // bricks per layer, a 512^3 grid, leave 24576)
    constexpr int64_t kStagedSmemTwo = 112 * 1024, kStagedSmemOne = 224 * 1024;
    const int64_t fixed = (int64_t)kStagedWarps * ((T + 1) / 2) * 4 + (int64_t)3 * T * 4;
    const int64_t budget = fixed + 4096 * 2 <= kStagedSmemTwo ? kStagedSmemTwo : kStagedSmemOne;
    const int64_t cap = ((budget - fixed) / 2) & ~int64_t(7);
    if (cap >= 4096 && p.chunk <= 65536) {
        const size_t smem = (size_t)(fixed + cap * 2);
        const unsigned blocks = (unsigned)(S * p.n_chunks);
        if (layered) {
            if (int rc = set_dynamic_smem(bin_place_staged_kernel<true>, smem, "bin_place"))
                return rc;
            bin_place_staged_kernel<true><<<blocks, kStagedWarps * 32, smem, stream>>>(
                rects, N, (int)T, tiles_x, seg_base, p.chunk, p.n_chunks, w.hist, offsets,
                flatten_ids, (int)cap, n_isects);
        } else {
            if (int rc = set_dynamic_smem(bin_place_staged_kernel<false>, smem, "bin_place"))
                return rc;
            bin_place_staged_kernel<false><<<blocks, kStagedWarps * 32, smem, stream>>>(
                rects, N, (int)T, tiles_x, seg_base, p.chunk, p.n_chunks, w.hist, offsets,
                flatten_ids, (int)cap, n_isects);
        }
        if (isect_ids != nullptr) {
            const int64_t n_keys = S * T;
            decode_keys_kernel<<<(unsigned)((n_keys * 32 + 255) / 256), 256, 0, stream>>>(
                offsets, n_keys, n_isects, seg_base * T, isect_ids);
        }
        return check_launch("bin_place");
    }
    const int per_warp = (int)T * 4;
    int warps = kSmemLimit / per_warp;
    warps = warps > 8 ? 8 : (warps < 1 ? 1 : warps);
    const int64_t n_warps = S * p.n_chunks;
    const unsigned blocks = (unsigned)((n_warps + warps - 1) / warps);
    const size_t smem = (size_t)warps * per_warp;
    if (layered) {
        if (int rc = set_dynamic_smem(bin_place_kernel<true>, smem, "bin_place")) return rc;
        bin_place_kernel<true><<<blocks, warps * 32, smem, stream>>>(
            rects, S, N, (int)T, tiles_x, seg_base, p.chunk, p.n_chunks, w.hist, offsets,
            flatten_ids, n_isects);
    } else {
        if (int rc = set_dynamic_smem(bin_place_kernel<false>, smem, "bin_place")) return rc;
        bin_place_kernel<false><<<blocks, warps * 32, smem, stream>>>(
            rects, S, N, (int)T, tiles_x, seg_base, p.chunk, p.n_chunks, w.hist, offsets,
            flatten_ids, n_isects);
    }
    if (isect_ids != nullptr) {
        const int64_t n_keys = S * T;
        decode_keys_kernel<<<(unsigned)((n_keys * 32 + 255) / 256), 256, 0, stream>>>(
            offsets, n_keys, n_isects, seg_base * T, isect_ids);
    }
    return check_launch("bin_place");
}

}  // namespace r2s

using namespace r2s;

extern "C" int64_t r2s_bin_workspace_bytes(int64_t S, int64_t N, int64_t T, int layered) {
    (void)layered;
    if (S < 0 || N < 0 || T < 0) return -1;
    return make_plan(S, N, T).bytes;
}

extern "C" int r2s_bin_prepare(const void* rects, int64_t S, int64_t N, int64_t T,
                               uint32_t tiles_x, int layered, int64_t seg_base, void* ws,
                               int64_t ws_bytes, int32_t* offsets, int64_t* n_isects_dev,
                               r2s_stream_t stream) {
    return bin_prepare_impl(rects, S, N, T, tiles_x, layered != 0, seg_base, ws, ws_bytes,
                            offsets, n_isects_dev, stream);
}

extern "C" int r2s_bin_place(const void* rects, int64_t S, int64_t N, int64_t T, uint32_t tiles_x,
                             int layered, int64_t seg_base, const void* ws, int64_t ws_bytes,
                             const int32_t* offsets, int64_t n_isects, int32_t* flatten_ids,
                             int64_t* isect_ids, r2s_stream_t stream) {
    return bin_place_impl(rects, S, N, T, tiles_x, layered != 0, seg_base, ws, ws_bytes, offsets,
                          n_isects, flatten_ids, isect_ids, stream);
}

extern "C" int r2s_isect_tiles_prepare(int dtype, const void* means2d, const int32_t* radii,
                                       int radii_is_rect, int64_t C, int64_t N, uint32_t tile,
                                       uint32_t ntx, uint32_t nty, int32_t* tiles_per_gauss,
                                       void* rects, void* ws, int64_t ws_bytes,
                                       int32_t* offsets, int64_t* n_isects_dev,
                                       r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "isect_tiles: negative size");
    R2S_REQUIRE(tile > 0, "isect_tiles: tile_size must be positive");
    R2S_REQUIRE(ntx < 65536 && nty < 65536, "isect_tiles: tile grid too large");
    const int64_t total = C * N;
    if (total > 0) {
        int rc = R2S_DTYPE_DISPATCH(dtype, "isect_tiles", [&] {
            rects_2d_kernel<scalar_t><<<grid_for(total), kThreads, 0, stream>>>(
                (const scalar_t*)means2d, radii, radii_is_rect, total, tile, ntx, nty,
                (Rect2*)rects, tiles_per_gauss);
            return check_launch("isect_tiles");
        });
        if (rc) return rc;
    }
    return bin_prepare_impl(rects, C, N, (int64_t)ntx * nty, ntx, false, 0, ws, ws_bytes, offsets,
                            n_isects_dev, stream);
}

extern "C" int r2s_isect_tiles_3d_prepare(int dtype, const void* means3d, const int32_t* radii,
                                          int64_t N, uint32_t tile, uint32_t nt2, uint32_t nt1,
                                          uint32_t nt0, int32_t* tiles_per_gauss, void* rects,
                                          void* ws, int64_t ws_bytes, int32_t* offsets,
                                          int64_t* n_isects_dev, r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0, "isect_tiles_3d: negative size");
    R2S_REQUIRE(tile > 0, "isect_tiles_3d: tile_size must be positive");
    R2S_REQUIRE(nt0 < 65536 && nt1 < 65536 && nt2 < 65536, "isect_tiles_3d: brick grid too large");
    if (N > 0) {
        int rc = R2S_DTYPE_DISPATCH(dtype, "isect_tiles_3d", [&] {
            rects_3d_kernel<scalar_t><<<grid_for(N), kThreads, 0, stream>>>(
                (const scalar_t*)means3d, radii, N, tile, nt2, nt1, nt0, (Rect3*)rects,
                tiles_per_gauss);
            return check_launch("isect_tiles_3d");
        });
        if (rc) return rc;
    }
    return bin_prepare_impl(rects, nt0, N, (int64_t)nt1 * nt2, nt2, true, 0, ws, ws_bytes, offsets,
                            n_isects_dev, stream);
}

extern "C" int r2s_isect_offset_encode(const int64_t* isect_ids, int64_t n_isects, int64_t n_keys,
                                       int32_t* offsets, r2s_stream_t stream) {
    R2S_REQUIRE(n_isects >= 0 && n_keys >= 0, "isect_offset_encode: negative size");
    if (n_keys == 0) return R2S_OK;
    offset_encode_kernel<<<grid_for(n_keys), kThreads, 0, stream>>>(isect_ids, n_isects, n_keys,
                                                                    offsets);
    return check_launch("isect_offset_encode");
}

namespace r2s {
R2S_DBG_DEFINE_READER(debug_flags_binning)
}  // namespace r2s
