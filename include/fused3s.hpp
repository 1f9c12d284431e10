// fused3s.hpp -- the reference's C++ host API for the fused3s_v2 path,
// rebuilt on the C ABI of libfused3s.so (fused3s.h).  Header-only.
//
// A caller of the reference (tests/test_fused_3s_v2.cu) keeps its code and
// swaps the include / link line:
//
//   reference                                   here
//   GraphData, load_csr_graph   utils.cuh:19-40  same names, same fields
//   blockSparseFormat           utils.cuh:42-46  same names, same fields
//   convert_csr_to_block_sparse converter.cu:13  same signature, runs on the GPU
//   generate_balanced_window_order utils.cuh:48  same signature, runs on the GPU
//   f3s_1tb1rw_kernel<<<nrw, dim3(32,4)>>>(...)  f3s_1tb1rw_launch(same args, stream)
//   float2half_kernel<<<...>>>(in, out, n)       f3s_half_from_float(in, out, n, stream)
//
// Differences, each deliberate:
//   * failures throw fused3s::Error (with the f3s_status) instead of exit();
//   * load_csr_graph reads col_idx.txt, the file the reference's exporter
//     writes (the reference opens col_ind.txt, utils.cuh:36, and reads zeros);
//   * generate_balanced_window_order breaks ties by ascending window id.  The
//     block-count sequence along the order is the reference's; define
//     F3S_REFERENCE_TIE_ORDER before including this header to get the
//     reference's exact permutation (std::sort on the host, as the reference
//     does) instead.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <fstream>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "fused3s.h"

namespace fused3s {

class Error : public std::runtime_error {
   public:
    Error(int status, const std::string& where)
        : std::runtime_error(where + ": " + f3s_status_string(status)), status_(status) {}
    int status() const { return status_; }

   private:
    int status_;
};

inline void check(int status, const char* where) {
    if (status != F3S_SUCCESS) throw Error(status, where);
}

inline void check_cuda(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw Error(F3S_ERR_CUDA, std::string(where) + " (" + cudaGetErrorString(e) + ")");
}

// RAII device buffer.
template <typename T>
struct DeviceBuffer {
    T* ptr = nullptr;
    size_t count = 0;
    explicit DeviceBuffer(size_t n) : count(n) {
        if (n) check_cuda(cudaMalloc(reinterpret_cast<void**>(&ptr), n * sizeof(T)), "cudaMalloc");
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() {
        if (ptr) cudaFree(ptr);
    }
};

}  // namespace fused3s

// ---------------------------------------------------------------- types --

struct GraphData {  // include/utils.cuh:19-24
    int num_nodes;
    int num_edges;
    std::vector<int> row_ptr;
    std::vector<int> col_ind;
};

struct blockSparseFormat {  // include/utils.cuh:42-46
    int num_row_windows;
    std::vector<int> window_offsets;
    std::vector<int> block_col_indices;
};

// ------------------------------------------------------------- loaders --

// include/utils.cuh:26-40, reading the column file the exporter writes.
inline GraphData load_csr_graph(const std::string& dataset_dir) {
    GraphData graph;
    std::ifstream meta(dataset_dir + "/meta.txt");
    if (!(meta >> graph.num_nodes >> graph.num_edges))
        throw fused3s::Error(F3S_ERR_INVALID_VALUE, "load_csr_graph: " + dataset_dir + "/meta.txt");
    graph.row_ptr.resize(graph.num_nodes + 1);
    std::ifstream row_file(dataset_dir + "/row_ptr.txt");
    for (int i = 0; i <= graph.num_nodes; ++i)
        if (!(row_file >> graph.row_ptr[i]))
            throw fused3s::Error(F3S_ERR_INVALID_VALUE, "load_csr_graph: row_ptr.txt too short");
    std::ifstream col_file(dataset_dir + "/col_idx.txt");
    if (!col_file) col_file.open(dataset_dir + "/col_ind.txt");
    graph.col_ind.resize(graph.num_edges);
    for (int i = 0; i < graph.num_edges; ++i)
        if (!(col_file >> graph.col_ind[i]))
            throw fused3s::Error(F3S_ERR_INVALID_VALUE, "load_csr_graph: column file too short");
    return graph;
}

// ---------------------------------------------------------- converter --

// src/converter.cu:13-44 on the GPU; bit-exact output.
inline blockSparseFormat convert_csr_to_block_sparse(int num_nodes, const std::vector<int>& row_ptr,
                                                     const std::vector<int>& col_ind) {
    using fused3s::DeviceBuffer;
    if (num_nodes < 0 || row_ptr.size() != (size_t)num_nodes + 1)
        throw fused3s::Error(F3S_ERR_INVALID_VALUE, "convert_csr_to_block_sparse: row_ptr size");
    const int64_t nnz = (int64_t)col_ind.size();
    blockSparseFormat f;
    f.num_row_windows = (num_nodes + 15) / 16;
    DeviceBuffer<int32_t> d_rp(row_ptr.size()), d_col(std::max<int64_t>(nnz, 1));
    DeviceBuffer<int32_t> d_off(f.num_row_windows + 1), d_cols(std::max<int64_t>(nnz, 1));
    const size_t wsz = f3s_convert_workspace_size(num_nodes, nnz);
    DeviceBuffer<unsigned char> d_ws(wsz);
    fused3s::check_cuda(cudaMemset(d_ws.ptr, 0, wsz), "cudaMemset");
    fused3s::check_cuda(cudaMemcpy(d_rp.ptr, row_ptr.data(), row_ptr.size() * 4, cudaMemcpyHostToDevice), "H2D");
    if (nnz)
        fused3s::check_cuda(cudaMemcpy(d_col.ptr, col_ind.data(), nnz * 4, cudaMemcpyHostToDevice), "H2D");
    int64_t B = 0;
    fused3s::check(f3s_convert(d_rp.ptr, d_col.ptr, num_nodes, nnz, d_off.ptr, d_cols.ptr, d_ws.ptr, wsz, &B,
                               nullptr),
                   "f3s_convert");
    f.window_offsets.resize(f.num_row_windows + 1);
    f.block_col_indices.resize(B);
    fused3s::check_cuda(cudaMemcpy(f.window_offsets.data(), d_off.ptr, f.window_offsets.size() * 4,
                                   cudaMemcpyDeviceToHost),
                        "D2H");
    if (B)
        fused3s::check_cuda(cudaMemcpy(f.block_col_indices.data(), d_cols.ptr, B * 4, cudaMemcpyDeviceToHost),
                            "D2H");
    return f;
}

// ------------------------------------------------------------ order --

// include/utils.cuh:48-59.
inline std::vector<int> generate_balanced_window_order(const blockSparseFormat& format) {
    std::vector<int> window_order(format.num_row_windows);
#ifdef F3S_REFERENCE_TIE_ORDER
    std::iota(window_order.begin(), window_order.end(), 0);
    std::sort(window_order.begin(), window_order.end(), [&format](int a, int b) {
        return format.window_offsets[a + 1] - format.window_offsets[a] >
               format.window_offsets[b + 1] - format.window_offsets[b];
    });
#else
    using fused3s::DeviceBuffer;
    const int nrw = format.num_row_windows;
    if (nrw == 0) return window_order;
    DeviceBuffer<int32_t> d_off(nrw + 1), d_order(nrw);
    const size_t wsz = f3s_window_order_workspace_size(nrw);
    DeviceBuffer<unsigned char> d_ws(wsz);
    fused3s::check_cuda(cudaMemcpy(d_off.ptr, format.window_offsets.data(), (nrw + 1) * 4, cudaMemcpyHostToDevice),
                        "H2D");
    fused3s::check(f3s_window_order(d_off.ptr, nrw, d_order.ptr, d_ws.ptr, wsz, nullptr), "f3s_window_order");
    fused3s::check_cuda(cudaMemcpy(window_order.data(), d_order.ptr, nrw * 4, cudaMemcpyDeviceToHost), "D2H");
#endif
    return window_order;
}

// ------------------------------------------------------------ kernel --

namespace fused3s {

// The reference kernel's argument list (src/fused3s_v2.cu:81-90) plus a
// stream; launch geometry is the library's.  Buffers hold
// num_row_windows*16 rows.  Throws fused3s::Error.  (The C entry point of the
// same name returns an f3s_status instead.)
inline void f3s_1tb1rw_launch(const void* Q, const void* K, const void* V, float* O_out, const int* window_offsets,
                              const int* block_col_indices, const int* window_order, int num_row_windows,
                              int feat_dim, cudaStream_t stream = 0) {
    check(::f3s_1tb1rw_launch(Q, K, V, O_out, window_offsets, block_col_indices, window_order, num_row_windows,
                              feat_dim, reinterpret_cast<f3s_stream_t>(stream)),
          "f3s_1tb1rw_launch");
}

// fp32 -> fp16 cast (tests/test_fused_3s_v2.cu:61-64).
inline void float2half(const float* in, void* out, int64_t n, cudaStream_t stream = 0) {
    check(f3s_half_from_float(in, out, n, reinterpret_cast<f3s_stream_t>(stream)), "f3s_half_from_float");
}

// Extended forward: true num_nodes (columns >= N masked), H heads of
// head_dim in {64, 128}, node-major [N, H, d] buffers without padding.
inline void forward(const void* Q, const void* K, const void* V, float* O, const int* window_offsets,
                    const int* block_cols, const int* order, int num_items, int num_nodes, int heads, int head_dim,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream = 0) {
    check(f3s_forward(Q, K, V, O, window_offsets, block_cols, order, nullptr, nullptr, num_items, num_nodes, heads,
                      head_dim, 0,
                      num_nodes, workspace, workspace_bytes, reinterpret_cast<f3s_stream_t>(stream)),
          "f3s_forward");
}

// Work plan (f3s_make_plan) owned by the caller: windows above
// max_blocks_per_piece blocks run as several pieces, merged in piece order.
// Build once per graph, window set and (heads, head_dim).
struct Plan {
    DeviceBuffer<unsigned char> buf;
    Plan(const int* window_offsets, const int* order, int num_items, int64_t num_blocks, int max_blocks_per_piece,
         int heads, int head_dim, cudaStream_t stream = 0)
        : buf(f3s_plan_size(num_items, num_blocks, max_blocks_per_piece, heads, head_dim)) {
        if (buf.count == 0) throw Error(F3S_ERR_INVALID_VALUE, "f3s_plan_size");
        check(f3s_make_plan(window_offsets, order, num_items, num_blocks, max_blocks_per_piece, heads, head_dim,
                            buf.ptr, buf.count, reinterpret_cast<f3s_stream_t>(stream)),
              "f3s_make_plan");
    }
    const void* get() const { return buf.ptr; }
};

// Per-block L2 eviction hints (f3s_block_hints) for the windows in `order`,
// with half of `l2_bytes` as the keep budget; d_hints holds num_blocks bytes.
inline void block_hints(const int* window_offsets, const int* block_cols, const int* order, int num_items,
                        int num_row_windows, int heads, int head_dim, int64_t l2_bytes, unsigned char* d_hints,
                        cudaStream_t stream = 0) {
    DeviceBuffer<unsigned char> ws(f3s_block_hints_workspace_size(num_row_windows));
    check(f3s_block_hints(window_offsets, block_cols, order, num_items, num_row_windows,
                          16LL * heads * head_dim * 2 * 2, l2_bytes / 2, d_hints, ws.ptr, ws.count,
                          reinterpret_cast<f3s_stream_t>(stream)),
          "f3s_block_hints");
    check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");  // ws is freed on return
}

// The extended forward with an optional plan and hints and O in
// F3S_OUT_F32 / F3S_OUT_F16 / F3S_OUT_BF16 (the fp32 result rounded to
// nearest); d_O is [num_nodes, heads, head_dim] of that type.
inline void forward_ex(const void* Q, const void* K, const void* V, void* O, int o_dtype, const int* window_offsets,
                       const int* block_cols, const int* order, const unsigned char* block_hints, const Plan* plan,
                       int num_items, int num_nodes, int heads, int head_dim, void* workspace,
                       size_t workspace_bytes, cudaStream_t stream = 0) {
    check(f3s_forward_ex(Q, K, V, O, o_dtype, window_offsets, block_cols, order, block_hints,
                         plan ? plan->get() : nullptr, num_items, num_nodes, heads, head_dim, 0, num_nodes, workspace,
                         workspace_bytes, reinterpret_cast<f3s_stream_t>(stream)),
          "f3s_forward_ex");
}

}  // namespace fused3s
