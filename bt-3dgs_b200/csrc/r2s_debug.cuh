// Bounds-checked build of the library (R2S_DEBUG).
//
// `python bt-3dgs_b200/build.py --debug` compiles every source with
// -DR2S_DEBUG into r2splat/_lib/libr2s_debug.so.  In that build the hot
// kernels test the indices they read or write through before using them:
//   R2S_DBG_TILE_RANGE  a tile's record range [start, end) lies in [0, n_isects)
//   R2S_DBG_RECORD_ID   a flatten id addresses an existing (view, Gaussian) record
//   R2S_DBG_PIXEL       a pixel or voxel index lies inside the image or volume
//   R2S_DBG_SLOT        a binning write lands inside the n_isects output slots
// A failed test sets its bit in the flag word of the kernel's translation unit
// and the access is skipped -- the checked build reports a bad index instead
// of touching memory out of bounds.  r2s_debug_flags() (include/r2s.h) ORs
// and optionally clears the flag words of all units.  In the release build
// R2S_DBG_BAD(...) is the constant false: the conditions are not compiled.
//
// This replaces the CUDA sanitizer run the reference's contributor guide asks
// for (CONTRIBUTING.md:33-35) on machines where the sanitizer is unavailable:
// the GPU test suite runs its workloads through the checked build and
// requires every flag to stay clear.
#pragma once

#include <cuda_runtime.h>

namespace r2s {
enum : unsigned {
    R2S_DBG_TILE_RANGE = 1u,
    R2S_DBG_RECORD_ID = 2u,
    R2S_DBG_PIXEL = 4u,
    R2S_DBG_SLOT = 8u,
};
}  // namespace r2s

#ifdef R2S_DEBUG
// one flag word per translation unit (the library is linked without
// relocatable device code); its reader is defined by R2S_DBG_DEFINE_READER
static __device__ unsigned int g_r2s_dbg_flags;
#define R2S_DBG_BAD(cond, bit) (!(cond) ? (atomicOr(&g_r2s_dbg_flags, (bit)), true) : false)
#define R2S_DBG_DEFINE_READER(fn)                                                     \
    int fn(unsigned* flags, int clear) {                                              \
        unsigned v = 0;                                                               \
        cudaError_t e = cudaMemcpyFromSymbol(&v, g_r2s_dbg_flags, sizeof(unsigned));  \
        if (e == cudaSuccess && clear) {                                              \
            const unsigned zero = 0;                                                  \
            e = cudaMemcpyToSymbol(g_r2s_dbg_flags, &zero, sizeof(unsigned));         \
        }                                                                             \
        *flags |= v;                                                                  \
        return e == cudaSuccess ? 0 : (int)e;                                         \
    }
#else
#define R2S_DBG_BAD(cond, bit) false
#define R2S_DBG_DEFINE_READER(fn)                 \
    int fn(unsigned* flags, int clear) {          \
        (void)flags;                              \
        (void)clear;                              \
        return 0;                                 \
    }
#endif
