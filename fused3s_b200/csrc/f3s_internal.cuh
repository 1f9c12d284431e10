// f3s_internal.cuh -- pieces shared by the translation units of libfused3s.so:
// the workspace header layout, the host-side error plumbing and block-level
// scan primitives.
#pragma once
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
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

// ------------------------------------------------------ per-context state --
// The calling thread's current CUDA context: its device and the driver's
// unique context id (cuCtxGetId).  Host-side state the library keeps per
// device -- kernel attributes, the no-alloc scratch address, library-owned
// workspaces -- belongs to one context: cudaDeviceReset destroys it and the
// next primary context of the device gets a new id, so every such cache is
// keyed on the id and rebuilt when it changes.
constexpr int kMaxDevices = 64;
struct ContextKey {
    int device;
    unsigned long long id;
};
int current_context(ContextKey* key);

// A value computed once per context of each device, under a lock (several
// host threads may call the library at once).  get() returns the cached
// value when it was made in the current context, else calls make(&value)
// and caches it on success.
template <class T>
class PerContext {
  public:
    template <class Make>
    int get(T* out, Make&& make) {
        ContextKey k{};
        int rc = current_context(&k);
        if (rc != F3S_SUCCESS) return rc;
        std::lock_guard<std::mutex> lock(mu_);
        Slot& s = slots_[k.device];
        if (!s.valid || s.id != k.id) {
            T v{};
            rc = make(&v);
            if (rc != F3S_SUCCESS) return rc;
            s.value = v;
            s.id = k.id;
            s.valid = true;
        }
        if (out) *out = s.value;
        return F3S_SUCCESS;
    }

  private:
    struct Slot {
        bool valid = false;
        unsigned long long id = 0;
        T value{};
    };
    std::mutex mu_;
    Slot slots_[kMaxDevices];
};

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
// persistent CTAs a forward launch may use on the current device
int forward_grid_limit();

// NVTX range around an entry point's host side (its enqueue), named after
// the call; free when no profiler is attached.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

// The part of a plan one forward launch runs, and the K / V rows it holds:
// pieces [begin, end) of the plan (end -1: to the last), K / V holding the
// graph's rows 16 * kv_col_base ... 16 * kv_col_base + kv_rows - 1 (kv_rows -1:
// all rows from 0), and whether the split windows are merged right after.
struct PieceRange {
    int begin = 0;
    int end = -1;
    int kv_col_base = 0;
    int kv_rows = -1;
    bool merge = true;
};

// The fused forward behind every forward entry point (f3s_forward.cu).
int forward_impl(const void* Q, const void* K, const void* V, void* O, int o_dtype, const int* offsets,
                 const int* cols, const int* order, const uint8_t* block_hints, const void* plan, int num_items,
                 int num_nodes, int heads, int head_dim, int q_window_base, int q_rows, void* ws, size_t ws_bytes,
                 cudaStream_t stream, uint64_t timeout_ns, const PieceRange& range);

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
