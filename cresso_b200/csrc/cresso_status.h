// Status / error plumbing of the C ABI: entry points return an int status and
// leave a message in a thread-local buffer that cresso_last_error() copies out.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cresso_b200.h"

namespace cresso {

int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
// Status of the last kernel launch on this thread (cudaGetLastError).
int check_launch(const char* what);

// Copies `bytes` of host memory to device memory in stream order, carried as the
// parameters of kernel launches (16 KB per launch) instead of a DMA copy: the
// per-step plan uploads then never wait behind large host-to-device copies that
// other streams have queued on the copy engine (a caller prefetching the next
// step's gradients, for instance).  The host buffer may be released on return.
int upload_async(void* dst, const void* src, size_t bytes, cudaStream_t stream);

// NVTX ranges around the library's launches, on when the environment variable
// CRESSO_B200_NVTX is set to a value other than "0" when the library first
// checks it (a profiler then shows one range per entry call and per stage).
bool nvtx_enabled();
void nvtx_push(const char* fmt, ...);
void nvtx_pop();
struct NvtxRange {
    bool on;
    template <typename... Args>
    explicit NvtxRange(const char* fmt, Args... args) : on(nvtx_enabled()) {
        if (on) nvtx_push(fmt, args...);
    }
    ~NvtxRange() {
        if (on) nvtx_pop();
    }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace cresso

#define CRESSO_REQUIRE(cond, code, ...)                    \
    do {                                                   \
        if (!(cond)) return ::cresso::set_error((code), __VA_ARGS__); \
    } while (0)

#define CRESSO_CUDA(call)                                        \
    do {                                                         \
        int _st = ::cresso::check_cuda((call), #call);           \
        if (_st != CRESSO_OK) return _st;                        \
    } while (0)

#define CRESSO_LAUNCHED(name)                                    \
    do {                                                         \
        int _st = ::cresso::check_launch(name);                  \
        if (_st != CRESSO_OK) return _st;                        \
    } while (0)
