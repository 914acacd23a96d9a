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

extern "C" const char* r2s_version(void) { return "r2s-b200 0.1.0 (sm_100a)"; }

extern "C" size_t r2s_last_error(char* buf, size_t len) {
    const std::string& m = r2s::g_last_error;
    if (buf && len > 0) {
        const size_t n = m.size() < len - 1 ? m.size() : len - 1;
        std::memcpy(buf, m.data(), n);
        buf[n] = '\0';
    }
    return m.size();
}
