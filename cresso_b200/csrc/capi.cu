// Library info and the error plumbing of the C ABI.

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include <stdlib.h>

#include <nvtx3/nvToolsExt.h>

#include "cresso_status.h"

namespace cresso {

bool nvtx_enabled() {
    static const bool on = [] {
        const char* v = getenv("CRESSO_B200_NVTX");
        return v != nullptr && v[0] != '\0' && !(v[0] == '0' && v[1] == '\0');
    }();
    return on;
}

void nvtx_push(const char* fmt, ...) {
    char name[160];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(name, sizeof(name), fmt, ap);
    va_end(ap);
    nvtxRangePushA(name);
}

void nvtx_pop() { nvtxRangePop(); }

constexpr int kUploadBytes = 16384;
struct UploadBlob {
    uint32_t w[kUploadBytes / 4];
};

// The blob is read in place from the parameter space (__grid_constant__).
__global__ void upload_kernel(const __grid_constant__ UploadBlob blob, unsigned char* __restrict__ dst, int n) {
    if ((reinterpret_cast<uintptr_t>(dst) & 3) == 0 && (n & 3) == 0) {
        uint32_t* d = reinterpret_cast<uint32_t*>(dst);
        for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) d[i] = blob.w[i];
    } else {
        const unsigned char* src = reinterpret_cast<const unsigned char*>(blob.w);
        for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

int upload_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
    const unsigned char* p = static_cast<const unsigned char*>(src);
    unsigned char* d = static_cast<unsigned char*>(dst);
    UploadBlob blob;
    while (bytes > 0) {
        const size_t c = bytes < (size_t)kUploadBytes ? bytes : (size_t)kUploadBytes;
        memcpy(blob.w, p, c);
        upload_kernel<<<1, 256, 0, stream>>>(blob, d, (int)c);
        const int st = check_launch("upload_kernel");
        if (st != CRESSO_OK) return st;
        p += c;
        d += c;
        bytes -= c;
    }
    return CRESSO_OK;
}

static thread_local char g_last_error[1024] = {0};
static std::atomic<int64_t> g_launches{0};

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return CRESSO_OK;
    return set_error(CRESSO_ECUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return CRESSO_OK;
    }
    return set_error(CRESSO_ECUDA, "launch of %s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Copies the device status word into a host word the device can write (pinned
// host memory under unified addressing) from a kernel: a posted write over the
// bus, so the copy never queues on a copy engine behind the caller's transfers.
__global__ void status_copy_kernel(const int32_t* __restrict__ word, volatile int32_t* host_word) {
    *host_word = *word;
}

}  // namespace cresso

extern "C" {

int cresso_status_copy(const void* status_word, void* host_word, cresso_stream_t stream) {
    CRESSO_REQUIRE(status_word != nullptr && host_word != nullptr, CRESSO_EINVAL, "status_copy: NULL word");
    cresso::status_copy_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(reinterpret_cast<const int32_t*>(status_word),
                                                                  reinterpret_cast<volatile int32_t*>(host_word));
    CRESSO_LAUNCHED("status_copy_kernel");
    return CRESSO_OK;
}

const char* cresso_version(void) { return "cresso_b200 0.1.0 (CRESSO5 step, abi 1)"; }

const char* cresso_arch(void) { return "sm_100a"; }

int cresso_last_error(char* buf, size_t n) {
    const size_t len = strlen(cresso::g_last_error);
    if (buf != nullptr && n > 0) {
        const size_t c = len < n - 1 ? len : n - 1;
        memcpy(buf, cresso::g_last_error, c);
        buf[c] = '\0';
    }
    return (int)len;
}

int64_t cresso_launch_count(void) { return cresso::g_launches.load(std::memory_order_relaxed); }

int cresso_abi_layout(int64_t* out, int n) {
    if (out == nullptr || n < 4) return cresso::set_error(CRESSO_EINVAL, "abi_layout: need an array of >= 4");
    out[0] = (int64_t)sizeof(cresso_hparams);
    out[1] = (int64_t)sizeof(cresso_tensor_desc);
    out[2] = CRESSO_MAX_NDIM;
    out[3] = CRESSO_MAX_RANK;
    return CRESSO_OK;
}

}  // extern "C"
