// f3s_internal.cuh -- pieces shared by the translation units of libfused3s.so:
// the workspace header layout, the host-side error plumbing and block-level
// scan primitives.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "fused3s.h"
#include "f3s_ptx.cuh"

namespace f3s {

// Every workspace starts with this 256-byte header; kernel scratch follows.
struct WsHeader {
    int abort;    // per-launch stop flag (cleared by each entry point)
    int counter;  // work-queue ticket counter (forward) / heavy-window count (convert)
    int status;   // first error code, sticky until f3s_workspace_status()
    int aux;
    int pad[60];
};
static_assert(sizeof(WsHeader) == 256, "workspace header is 256 bytes");
constexpr size_t kWsHeaderBytes = sizeof(WsHeader);

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline ErrorSink sink_of(void* ws) {
    WsHeader* h = static_cast<WsHeader*>(ws);
    return ErrorSink{&h->abort, &h->status};
}

// Host-side: remember the CUDA error behind an F3S_ERR_CUDA return.
void note_cuda_error(cudaError_t e);

#define F3S_CUDA_TRY(call)                       \
    do {                                         \
        cudaError_t e_ = (call);                 \
        if (e_ != cudaSuccess) {                 \
            ::f3s::note_cuda_error(e_);          \
            return F3S_ERR_CUDA;                 \
        }                                        \
    } while (0)

#define F3S_LAUNCH_CHECK()                            \
    do {                                              \
        cudaError_t e_ = cudaGetLastError();          \
        if (e_ != cudaSuccess) {                      \
            ::f3s::note_cuda_error(e_);               \
            return F3S_ERR_CUDA;                      \
        }                                             \
    } while (0)

int num_sms_of_current_device();

// ------------------------------------------------------------------ scans --
__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Exclusive scan across a block of BT threads; `total` receives the block
// sum.  `scratch` must hold BT/32 + 1 ints of shared memory.  Contains
// __syncthreads(), so every thread of the block must call it.
template <int BT>
__device__ __forceinline__ int block_exclusive_scan(int v, int& total, int* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    constexpr int NW = BT / 32;
    int inc = warp_inclusive_scan(v);
    if (lane == 31) scratch[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        int s = lane < NW ? scratch[lane] : 0;
        int si = warp_inclusive_scan(s);
        if (lane < NW) scratch[lane] = si - s;
        if (lane == NW - 1) scratch[NW] = si;
    }
    __syncthreads();
    int res = scratch[wid] + inc - v;
    total = scratch[NW];
    __syncthreads();
    return res;
}

// Device-wide exclusive scan of n int32 values: out[i] = sum in[0..i), and
// out[n] = total when `write_total`.  `tile_sums` needs scan_tiles(n) ints.
// Sums must fit in int32 (callers guarantee it).
constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;
inline int64_t scan_tiles(int64_t n) { return (n + kScanTile - 1) / kScanTile; }
int device_exclusive_scan(const int* in, int* out, int64_t n, bool write_total, int* tile_sums,
                          cudaStream_t stream);

}  // namespace f3s
