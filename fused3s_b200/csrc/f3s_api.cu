// f3s_api.cu -- C-ABI glue of libfused3s.so: status strings, the workspace
// status read-back, the reference-signature launch and the fp32 -> fp16 cast.
#include <atomic>
#include <mutex>
#include "f3s_internal.cuh"

namespace f3s {

static std::atomic<int> g_last_cuda_error{0};

void note_cuda_error(cudaError_t e) { g_last_cuda_error.store((int)e); }

int num_sms_of_current_device() {
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    if (dev < 64 && cache[dev] > 0) return cache[dev];
    int n = 1;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 1;
    if (dev < 64) cache[dev] = n;
    return n;
}

int forward_impl(const void* Q, const void* K, const void* V, void* O, int o_dtype, const int* offsets,
                 const int* cols, const int* order, const uint8_t* block_hints, const void* plan, int num_items,
                 int num_nodes, int heads, int head_dim, int q_window_base, int q_rows, void* ws, size_t ws_bytes,
                 cudaStream_t stream, uint64_t timeout_ns);

// Library-owned forward workspace for the reference-signature launch, one
// per device, allocated on first use and kept until process exit.
static void* legacy_workspace(int* rc) {
    static void* ws[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev >= 64) {
        note_cuda_error(e);
        *rc = F3S_ERR_CUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!ws[dev]) {
        e = cudaMalloc(&ws[dev], kWsHeaderBytes);
        if (e != cudaSuccess) {
            note_cuda_error(e);
            *rc = F3S_ERR_CUDA;
            return nullptr;
        }
        e = cudaMemset(ws[dev], 0, kWsHeaderBytes);
        if (e != cudaSuccess) {
            note_cuda_error(e);
            *rc = F3S_ERR_CUDA;
            return nullptr;
        }
    }
    *rc = F3S_SUCCESS;
    return ws[dev];
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

int f3s_version(void) { return 1 * 10000 + 0 * 100 + 0; }

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
    if (num_row_windows < 0 || (int64_t)num_row_windows * 16 > INT32_MAX) return F3S_ERR_INVALID_VALUE;
    int rc = 0;
    void* ws = f3s::legacy_workspace(&rc);
    if (!ws) return rc;
    const int rows = num_row_windows * 16;
    return f3s::forward_impl(Q, K, V, O_out, F3S_OUT_F32, window_offsets, block_col_indices, window_order, nullptr,
                             nullptr, num_row_windows, rows, 1, feat_dim, 0, rows, ws, f3s::kWsHeaderBytes,
                             (cudaStream_t)stream, 10ull * 1000 * 1000 * 1000);
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
