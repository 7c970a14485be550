// api.cu -- library-level entry points: errors, version, device error word.
#include "common.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace fp4x {

static thread_local char t_last_error[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

int num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

}  // namespace fp4x

extern "C" const char *fp4x_last_error(void) { return fp4x::t_last_error; }

extern "C" const char *fp4x_version(void) { return "fp4x 0.1.0 (sm_100a)"; }

extern "C" int fp4x_device_error(fp4x_stream_t stream, uint32_t *bits_out) {
    uint32_t bits = 0;
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&bits, fp4x::g_device_error, sizeof(bits));
    const uint32_t zero = 0;
    if (e == cudaSuccess && bits) e = cudaMemcpyToSymbol(fp4x::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) {
        fp4x::set_error("fp4x_device_error: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    if (bits_out) *bits_out = bits;
    if (bits) {
        fp4x::set_error("device-side bounded wait expired (error bits 0x%x)", bits);
        return FP4X_ETIMEOUT;
    }
    return FP4X_OK;
}

extern "C" int fp4x_set_wait_limit(uint32_t polls) {
    const cudaError_t e = cudaMemcpyToSymbol(fp4x::g_flag_wait_limit, &polls, sizeof(polls));
    if (e != cudaSuccess) {
        fp4x::set_error("fp4x_set_wait_limit: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}
