// f3s_api.cu -- C-ABI glue of libfused3s.so: status strings, the workspace
// status read-back, the reference-signature launch, the fp32 -> fp16 cast and
// the per-context bookkeeping the other translation units share.
#include <atomic>
#include <map>
#include <mutex>
#include <utility>
#include <cuda.h>
#include "f3s_internal.cuh"

namespace f3s {

static std::atomic<int> g_last_cuda_error{0};

void note_cuda_error(cudaError_t e) { g_last_cuda_error.store((int)e); }

int num_sms_of_current_device() {
    static std::atomic<int> cache[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    if (dev >= 0 && dev < kMaxDevices) {
        const int c = cache[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 1;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 1;
    if (dev >= 0 && dev < kMaxDevices) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

// Upper bound on the persistent CTAs of a forward launch, per device (0: one
// per SM).  Set by f3s_set_forward_sm_limit.
static std::atomic<int> g_forward_sm_limit[kMaxDevices] = {};

int forward_grid_limit() {
    const int sms = num_sms_of_current_device();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return sms;
    const int lim = g_forward_sm_limit[dev].load(std::memory_order_relaxed);
    return lim > 0 && lim < sms ? lim : sms;
}

int set_forward_sm_limit(int max_ctas) {
    int dev = 0;
    F3S_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return F3S_ERR_UNSUPPORTED;
    if (max_ctas < 0) return F3S_ERR_INVALID_VALUE;
    g_forward_sm_limit[dev].store(max_ctas, std::memory_order_relaxed);
    return F3S_SUCCESS;
}

// Driver entry points for the context identity, looked up once through the
// runtime (the library links no libcuda).
using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

int current_context(ContextKey* key) {
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(p);
    });
    int dev = 0;
    F3S_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return F3S_ERR_UNSUPPORTED;
    if (!get_current || !get_id) return F3S_ERR_CUDA;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
        // no context current on this thread yet: cudaSetDevice makes the
        // device's primary context current (creating it if needed)
        F3S_CUDA_TRY(cudaSetDevice(dev));
        if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return F3S_ERR_CUDA;
    }
    unsigned long long id = 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return F3S_ERR_CUDA;
    key->device = dev;
    key->id = id;
    return F3S_SUCCESS;
}


// Library-owned forward workspaces for the reference-signature launch, one
// per (context, stream): the launch's ticket counter and status word live
// there, so launches on different streams never share them.  Allocated on
// first use of a stream and kept until the process exits (256 bytes each);
// entries of a destroyed context are never matched again.
static void* legacy_workspace(cudaStream_t stream, int* rc) {
    static std::map<std::pair<unsigned long long, uintptr_t>, void*> ws;
    static std::mutex mu;
    ContextKey k{};
    *rc = current_context(&k);
    if (*rc != F3S_SUCCESS) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(k.id, reinterpret_cast<uintptr_t>(stream));
    auto it = ws.find(key);
    if (it != ws.end()) return it->second;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, kWsHeaderBytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, kWsHeaderBytes);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        *rc = F3S_ERR_CUDA;
        return nullptr;
    }
    ws[key] = p;
    return p;
}

__global__ void k_half_from_float(const float* __restrict__ in, __half* __restrict__ out, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __float2half_rn(in[i]);
}

}  // namespace f3s

extern "C" {

const char* f3s_status_string(int status) {
    switch (status) {
        case F3S_SUCCESS: return "F3S_SUCCESS";
        case F3S_ERR_INVALID_VALUE: return "F3S_ERR_INVALID_VALUE: invalid argument";
        case F3S_ERR_UNSUPPORTED: return "F3S_ERR_UNSUPPORTED: head_dim must be 64 or 128";
        case F3S_ERR_BAD_CSR: return "F3S_ERR_BAD_CSR: column index outside [0, N) or row_ptr not monotone";
        case F3S_ERR_WORKSPACE: return "F3S_ERR_WORKSPACE: workspace too small";
        case F3S_ERR_CUDA: return "F3S_ERR_CUDA: CUDA runtime error";
        case F3S_ERR_TIMEOUT: return "F3S_ERR_TIMEOUT: a bounded device wait expired";
        case F3S_ERR_BAD_FORMAT: return "F3S_ERR_BAD_FORMAT: window id or block column out of range";
        case F3S_ERR_TOO_LARGE: return "F3S_ERR_TOO_LARGE: exceeds int32 limits of the format";
        default: return "F3S_ERR_UNKNOWN";
    }
}

int f3s_version(void) { return 1 * 10000 + 1 * 100 + 0; }

int f3s_set_forward_sm_limit(int32_t max_ctas) { return f3s::set_forward_sm_limit(max_ctas); }

int f3s_last_cuda_error(void) { return f3s::g_last_cuda_error.load(); }

int f3s_workspace_status(void* d_workspace, f3s_stream_t stream) {
    if (!d_workspace) return F3S_ERR_INVALID_VALUE;
    f3s::WsHeader* h = static_cast<f3s::WsHeader*>(d_workspace);
    cudaStream_t s = (cudaStream_t)stream;
    int st = 0;
    F3S_CUDA_TRY(cudaStreamSynchronize(s));
    F3S_CUDA_TRY(cudaMemcpyAsync(&st, &h->status, sizeof(int), cudaMemcpyDeviceToHost, s));
    F3S_CUDA_TRY(cudaStreamSynchronize(s));
    if (st != 0) {
        F3S_CUDA_TRY(cudaMemsetAsync(&h->status, 0, sizeof(int), s));
        F3S_CUDA_TRY(cudaStreamSynchronize(s));
    }
    return st;
}

int f3s_1tb1rw_launch(const void* Q, const void* K, const void* V, float* O_out, const int32_t* window_offsets,
                      const int32_t* block_col_indices, const int32_t* window_order, int32_t num_row_windows,
                      int32_t feat_dim, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_1tb1rw_launch");
    if (num_row_windows < 0 || (int64_t)num_row_windows * 16 > INT32_MAX) return F3S_ERR_INVALID_VALUE;
    int rc = 0;
    void* ws = f3s::legacy_workspace((cudaStream_t)stream, &rc);
    if (!ws) return rc;
    const int rows = num_row_windows * 16;
    return f3s::forward_impl(Q, K, V, O_out, F3S_OUT_F32, window_offsets, block_col_indices, window_order, nullptr,
                             nullptr, num_row_windows, rows, 1, feat_dim, 0, rows, ws, f3s::kWsHeaderBytes,
                             (cudaStream_t)stream, 10ull * 1000 * 1000 * 1000, f3s::PieceRange{});
}

int f3s_half_from_float(const float* d_in, void* d_out, int64_t n, f3s_stream_t stream) {
    if (n < 0 || (n > 0 && (!d_in || !d_out))) return F3S_ERR_INVALID_VALUE;
    if (n == 0) return F3S_SUCCESS;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)f3s::num_sms_of_current_device() * 16);
    f3s::k_half_from_float<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(d_in, static_cast<__half*>(d_out), n);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

}  // extern "C"
