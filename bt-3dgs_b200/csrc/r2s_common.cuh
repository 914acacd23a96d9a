// Shared device/host helpers for the r2s sm_100a library.
//
// Everything in this library is launched on a caller-provided stream and
// writes only caller-provided buffers: no kernel allocates, no entry point
// calls cudaMalloc.  Entry points return an int status (R2S_OK on success);
// the message of the last failure on the calling thread is kept by
// r2s_last_error().
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <type_traits>

#include "../../include/r2s.h"

namespace r2s {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------
// Host-side status helpers (implemented in r2s_runtime.cpp)
// ---------------------------------------------------------------------------
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
// torch.nn.functional.softplus in float, bit for bit (r2s_precise.cu, built
// without fast math)
int launch_softplus_f32(const float* x, float* y, int64_t n, cudaStream_t stream);

// Opt a kernel in to `bytes` of dynamic shared memory; R2S_ERR_CUDA on failure.
template <typename Kernel>
inline int set_dynamic_smem(Kernel kernel, size_t bytes, const char* what) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return fail(R2S_ERR_CUDA, "%s: cannot reserve %zu bytes of shared memory: %s", what, bytes,
                    cudaGetErrorString(e));
    }
    return R2S_OK;
}

#define R2S_REQUIRE(cond, ...)                                                 \
    do {                                                                       \
        if (!(cond)) return ::r2s::fail(R2S_ERR_ARG, __VA_ARGS__);             \
    } while (0)

#define R2S_DTYPE_DISPATCH(dtype, NAME, ...)                                   \
    [&]() -> int {                                                             \
        if ((dtype) == R2S_F32) {                                              \
            using scalar_t = float;                                            \
            return __VA_ARGS__();                                              \
        } else if ((dtype) == R2S_F64) {                                       \
            using scalar_t = double;                                           \
            return __VA_ARGS__();                                              \
        }                                                                      \
        return ::r2s::fail(R2S_ERR_ARG, "%s: unsupported dtype code %d", NAME, \
                           (int)(dtype));                                      \
    }()

inline unsigned grid_for(int64_t n, int threads = kThreads) {
    return (unsigned)((n + threads - 1) / threads);
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// exp(-x) as the reference evaluates it in its forward and pixel-mode kernels:
// CUDA's __expf on the float value, for both float and double instantiations.
template <typename S>
__device__ __forceinline__ S expf_neg(S x) {
    return static_cast<S>(__expf(-static_cast<float>(x)));
}

// exp(-x) at the scalar type's own precision (the reference's per-Gaussian
// backward uses exp()).
template <typename S>
__device__ __forceinline__ S exp_neg_native(S x) {
    if constexpr (std::is_same<S, float>::value) {
        return __expf(-x);
    } else {
        return exp(-x);
    }
}

template <typename S>
__device__ __forceinline__ S warp_sum(S v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Vector reduction into global memory (sm_90+): one L2 transaction for four
// consecutive floats instead of four scalar atomics.
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}
__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

// Packed float32 pairs (sm_100 f32x2 arithmetic): one instruction updates two
// adjacent pixels; each lane of the pair is rounded exactly like the scalar
// instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Packed tile rectangle of one (segment, item): [x0, x1) x [y0, y1) in tile
// units, 16 bits per bound.  An empty rectangle has x1 <= x0 or y1 <= y0.
struct Rect2 {
    uint32_t x;  // x0 | x1 << 16
    uint32_t y;  // y0 | y1 << 16
};
// 3D brick rectangle: additionally [z0, z1) in brick units.
struct Rect3 {
    uint32_t x;
    uint32_t y;
    uint32_t z;
    uint32_t pad;
};

__host__ __device__ __forceinline__ uint32_t pack16(uint32_t lo, uint32_t hi) {
    return (lo & 0xffffu) | (hi << 16);
}
__host__ __device__ __forceinline__ uint32_t lo16(uint32_t v) { return v & 0xffffu; }
__host__ __device__ __forceinline__ uint32_t hi16(uint32_t v) { return v >> 16; }

}  // namespace r2s
