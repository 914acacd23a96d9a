// Status and error-message plumbing of the C ABI.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/r2s.h"

namespace r2s {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* what) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        return fail(R2S_ERR_CUDA, "%s: CUDA error %d (%s)", what, (int)err, cudaGetErrorString(err));
    return R2S_OK;
}

}  // namespace r2s

namespace r2s {
// flag words of the checked build, one per translation unit (r2s_debug.cuh)
int debug_flags_raster(unsigned* flags, int clear);
int debug_flags_voxel(unsigned* flags, int clear);
int debug_flags_binning(unsigned* flags, int clear);
}  // namespace r2s

extern "C" const char* r2s_version(void) {
#ifdef R2S_DEBUG
    return "r2s-b200 0.1.0 (sm_100a, bounds-checked build)";
#else
    return "r2s-b200 0.1.0 (sm_100a)";
#endif
}

extern "C" int r2s_debug_build(void) {
#ifdef R2S_DEBUG
    return 1;
#else
    return 0;
#endif
}

extern "C" int r2s_debug_flags(unsigned* flags, int clear) {
    if (flags == nullptr) return r2s::fail(R2S_ERR_ARG, "debug_flags: flags is null");
    *flags = 0;
    int (*readers[])(unsigned*, int) = {r2s::debug_flags_raster, r2s::debug_flags_voxel,
                                        r2s::debug_flags_binning};
    for (auto read : readers) {
        const int e = read(flags, clear);
        if (e != 0)
            return r2s::fail(R2S_ERR_CUDA, "debug_flags: reading the flag words failed (%s)",
                             cudaGetErrorString((cudaError_t)e));
    }
    return R2S_OK;
}

extern "C" size_t r2s_last_error(char* buf, size_t len) {
    const std::string& m = r2s::g_last_error;
    if (buf && len > 0) {
        const size_t n = m.size() < len - 1 ? m.size() : len - 1;
        std::memcpy(buf, m.data(), n);
        buf[n] = '\0';
    }
    return m.size();
}
