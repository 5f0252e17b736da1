// Segment copies for the multi-GPU exchange of tensors stepped whole.
//
// Under row sharding a tensor passed whole is stepped by one owner rank; its
// parameter and floating-point state tensors (hundreds of small tensors for a
// LoRA-heavy set: eight 0-d states per tensor) then travel to every rank in one
// all-gather of a byte buffer.  Packing them into that buffer, and unpacking the
// gathered buffer into the tensors, is one launch each over a device table of
// (source, destination, bytes) rows, instead of one copy per tensor.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "cresso_common.cuh"
#include "cresso_status.h"

namespace cresso {

// Block b copies the segments b, b + gridDim.x, ...: 16-byte vectors when both
// ends are 16-byte aligned, bytes otherwise (and for the tail).
__global__ void __launch_bounds__(kThreads) copy_segments_kernel(const uint64_t* __restrict__ table, int64_t n) {
    for (int64_t s = blockIdx.x; s < n; s += gridDim.x) {
        const unsigned char* src = reinterpret_cast<const unsigned char*>(table[3 * s]);
        unsigned char* dst = reinterpret_cast<unsigned char*>(table[3 * s + 1]);
        const int64_t nb = (int64_t)table[3 * s + 2];
        int64_t head = 0;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
            const int64_t nv = nb >> 4;
            const int4* s4 = reinterpret_cast<const int4*>(src);
            int4* d4 = reinterpret_cast<int4*>(dst);
            for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) d4[i] = s4[i];
            head = nv << 4;
        }
        for (int64_t i = head + threadIdx.x; i < nb; i += blockDim.x) dst[i] = src[i];
    }
}

}  // namespace cresso

using namespace cresso;

extern "C" {

int cresso_copy_segments(const uint64_t* table, int64_t n_segments, cresso_stream_t stream) {
    CRESSO_REQUIRE(n_segments >= 0, CRESSO_EINVAL, "copy_segments: n_segments must be >= 0");
    if (n_segments == 0) return CRESSO_OK;
    CRESSO_REQUIRE(table != nullptr, CRESSO_EINVAL, "copy_segments: NULL table");
    const int grid = (int)std::min<int64_t>(n_segments, 148 * 8);
    copy_segments_kernel<<<grid, kThreads, 0, (cudaStream_t)stream>>>(table, n_segments);
    CRESSO_LAUNCHED("copy_segments_kernel");
    return CRESSO_OK;
}

}  // extern "C"
