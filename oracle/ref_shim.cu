// ref_shim.cu -- extern "C" doors into the reference's own functions.
//
// TEST INFRASTRUCTURE ONLY (see f3s_oracle.c).  This file holds no
// algorithm: it converts plain pointers into the reference's std::vector
// structs and calls the reference functions, which oracle/Makefile compiles
// unchanged from the reference source tree into oracle/_ref/libf3s_ref.so:
//
//   convert_csr_to_block_sparse     src/converter.cu:13
//   generate_balanced_window_order  include/utils.cuh:48
//   cpu_block_sparse_attention      tests/test_fused_3s_v2.cu:17
//   cpu_sparse_attention_csr        baselines/cpu_baseline.cpp:16
//   f3s_1tb1rw_kernel               src/fused3s_v2.cu:81
//
// The reference's test file is compiled with -Dmain=ref_v2_main so that its
// CPU ground-truth function can be linked here without its main().
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <thread>
#include <vector>
#include <cuda_fp16.h>
#include "utils.cuh"

blockSparseFormat convert_csr_to_block_sparse(int num_nodes, const std::vector<int>& row_ptr,
                                              const std::vector<int>& col_ind);
void cpu_block_sparse_attention(int num_nodes, int feat_dim, const float* Q, const float* K,
                                const float* V, float* O, const blockSparseFormat& format);
void cpu_sparse_attention_csr(int num_nodes, int feat_dim, const float* Q, const float* K,
                              const float* V, const int* row_ptr, const int* col_idx,
                              float* out_mat);
__global__ void f3s_1tb1rw_kernel(const half* __restrict__ Q, const half* __restrict__ K,
                                  const half* __restrict__ V, float* __restrict__ O_out,
                                  const int* __restrict__ window_offsets,
                                  const int* __restrict__ block_col_indices,
                                  const int* __restrict__ window_order, int num_row_windows,
                                  int feat_dim);

namespace {
// The reference converter prints two statistics lines; keep them off stdout.
struct QuietCout {
    std::streambuf* old;
    QuietCout() : old(std::cout.rdbuf(nullptr)) {}
    ~QuietCout() {
        std::cout.rdbuf(old);
        std::cout.clear();
    }
};

blockSparseFormat make_format(int nrw, const int* offsets, const int* cols) {
    blockSparseFormat f;
    f.num_row_windows = nrw;
    f.window_offsets.assign(offsets, offsets + nrw + 1);
    f.block_col_indices.assign(cols, cols + offsets[nrw]);
    return f;
}

// A copy of the format in which only `mine` keep their block lists; the
// reference function skips windows whose list is empty.
blockSparseFormat restrict_format(int nrw, const int* offsets, const int* cols,
                                  const std::vector<int>& mine) {
    std::vector<char> keep(nrw, 0);
    for (int w : mine) keep[w] = 1;
    blockSparseFormat f;
    f.num_row_windows = nrw;
    f.window_offsets.resize(nrw + 1);
    f.window_offsets[0] = 0;
    for (int w = 0; w < nrw; ++w) {
        if (keep[w])
            for (int b = offsets[w]; b < offsets[w + 1]; ++b) f.block_col_indices.push_back(cols[b]);
        f.window_offsets[w + 1] = (int)f.block_col_indices.size();
    }
    return f;
}
}  // namespace

extern "C" {

// Returns B; offsets_out has nrw+1 entries, cols_out room for nnz entries.
long long ref_convert(int num_nodes, const int* row_ptr, long long nnz, const int* col_ind,
                      int* offsets_out, int* cols_out) {
    std::vector<int> rp(row_ptr, row_ptr + num_nodes + 1);
    std::vector<int> ci(col_ind, col_ind + nnz);
    blockSparseFormat f;
    {
        QuietCout q;
        f = convert_csr_to_block_sparse(num_nodes, rp, ci);
    }
    std::memcpy(offsets_out, f.window_offsets.data(), f.window_offsets.size() * sizeof(int));
    if (!f.block_col_indices.empty())
        std::memcpy(cols_out, f.block_col_indices.data(), f.block_col_indices.size() * sizeof(int));
    return (long long)f.block_col_indices.size();
}

void ref_window_order(int nrw, const int* offsets, int* order_out) {
    blockSparseFormat f;
    f.num_row_windows = nrw;
    f.window_offsets.assign(offsets, offsets + nrw + 1);
    std::vector<int> o = generate_balanced_window_order(f);
    if (!o.empty()) std::memcpy(order_out, o.data(), o.size() * sizeof(int));
}

// Single-head block attention, [num_nodes, d] row-major.  windows == NULL
// runs every window; otherwise only the listed ones.  The listed windows are
// dealt to nthreads threads; each thread runs the unchanged reference
// function on its own restricted format copy (rows are disjoint).
void ref_block_attention(int num_nodes, int d, const float* Q, const float* K, const float* V,
                         float* O, int nrw, const int* offsets, const int* cols,
                         const int* windows, int nwin, int nthreads) {
    if (windows == nullptr && nthreads <= 1) {
        blockSparseFormat f = make_format(nrw, offsets, cols);
        cpu_block_sparse_attention(num_nodes, d, Q, K, V, O, f);
        return;
    }
    if (nthreads < 1) nthreads = 1;
    std::vector<int> all;
    if (windows == nullptr) {
        all.resize(nrw);
        for (int w = 0; w < nrw; ++w) all[w] = w;
    } else {
        all.assign(windows, windows + nwin);
    }
    std::vector<std::vector<int>> parts(nthreads);
    for (size_t i = 0; i < all.size(); ++i) parts[i % nthreads].push_back(all[i]);
    std::vector<blockSparseFormat> fmts(nthreads);
    for (int t = 0; t < nthreads; ++t) fmts[t] = restrict_format(nrw, offsets, cols, parts[t]);
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t)
        th.emplace_back([&, t] { cpu_block_sparse_attention(num_nodes, d, Q, K, V, O, fmts[t]); });
    for (auto& x : th) x.join();
}

void ref_edge_attention(int num_nodes, int d, const float* Q, const float* K, const float* V,
                        const int* row_ptr, const int* col_idx, float* out) {
    cpu_sparse_attention_csr(num_nodes, d, Q, K, V, row_ptr, col_idx, out);
}

// Launch the reference's own v2 kernel exactly as its test does
// (tests/test_fused_3s_v2.cu:123-131) on the given stream.  Q/K/V/O are
// device pointers with nrw*16 rows of feat_dim (== 64) columns.
int ref_v2_launch(const void* Q, const void* K, const void* V, float* O, const int* offsets,
                  const int* cols, const int* order, int nrw, int feat_dim, void* stream) {
    dim3 block_dim(32, 4);
    dim3 grid_dim(nrw);
    f3s_1tb1rw_kernel<<<grid_dim, block_dim, 0, (cudaStream_t)stream>>>(
        (const half*)Q, (const half*)K, (const half*)V, O, offsets, cols, order, nrw, feat_dim);
    return (int)cudaGetLastError();
}

}  // extern "C"
