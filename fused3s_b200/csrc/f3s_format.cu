// f3s_format.cu -- the graph-format half of the hot path on the GPU:
//   * CSR -> 16x16 block-sparse row windows, bit-exact to the reference
//     converter (src/converter.cu:13-44);
//   * the descending-workload window order (include/utils.cuh:48-59) as a
//     stable LSD radix sort;
//   * the device-wide exclusive scan both of them use.
//
// All of this is integer work bound by HBM / L2 latency, not by tensor
// cores; kernels are sized in CTAs of 256 threads, coalesced loads, and the
// per-window work of the converter stays in shared memory.
#include <algorithm>
#include <climits>
#include <mutex>
#include "f3s_internal.cuh"

namespace f3s {

// =========================================================================
// Device-wide exclusive scan (three launches: tile sums, scan of the tile
// sums in one CTA, tile scan + add).
// =========================================================================

__global__ void __launch_bounds__(kScanThreads) k_scan_tile_sums(const int* __restrict__ in, int64_t n,
                                                               int* __restrict__ tile_sums) {
    __shared__ int scratch[kScanThreads / 32 + 1];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    int s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int64_t i = base + (int64_t)k * kScanThreads + threadIdx.x;
        if (i < n) s += in[i];
    }
    int total;
    block_exclusive_scan<kScanThreads>(s, total, scratch);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// One CTA of 1024 threads scans the tile sums in place (exclusive), in
// chunks of 4096 with a running carry.
__global__ void __launch_bounds__(1024) k_scan_carry(int* __restrict__ tile_sums, int64_t ntiles) {
    __shared__ int scratch[1024 / 32 + 1];
    int carry = 0;
    for (int64_t base = 0; base < ntiles; base += 4096) {
        int v[4];
        int s = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            int64_t i = base + threadIdx.x * 4 + k;
            v[k] = i < ntiles ? tile_sums[i] : 0;
            s += v[k];
        }
        int total;
        int ex = block_exclusive_scan<1024>(s, total, scratch) + carry;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            int64_t i = base + threadIdx.x * 4 + k;
            if (i < ntiles) tile_sums[i] = ex;
            ex += v[k];
        }
        carry += total;
    }
}

__global__ void __launch_bounds__(kScanThreads) k_scan_tiles(const int* __restrict__ in,
                                                           int* __restrict__ out, int64_t n,
                                                           const int* __restrict__ tile_sums,
                                                           int write_total) {
    __shared__ int buf[kScanTile];
    __shared__ int scratch[kScanThreads / 32 + 1];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int j = k * kScanThreads + threadIdx.x;
        int64_t i = base + j;
        buf[j] = i < n ? in[i] : 0;
    }
    __syncthreads();
    int v[kScanItems];
    int s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = buf[threadIdx.x * kScanItems + k];
        s += v[k];
    }
    int total;
    int ex = block_exclusive_scan<kScanThreads>(s, total, scratch) + tile_sums[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        buf[threadIdx.x * kScanItems + k] = ex;
        ex += v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int j = k * kScanThreads + threadIdx.x;
        int64_t i = base + j;
        if (i < n) out[i] = buf[j];
    }
    if (write_total && blockIdx.x == gridDim.x - 1 && threadIdx.x == kScanThreads - 1)
        out[n] = ex;  // last thread of the last tile holds the grand total
}

int device_exclusive_scan(const int* in, int* out, int64_t n, bool write_total, int* tile_sums,
                          cudaStream_t stream) {
    if (n <= 0) {
        if (write_total) F3S_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(int), stream));
        return F3S_SUCCESS;
    }
    const int64_t nt = scan_tiles(n);
    k_scan_tile_sums<<<(unsigned)nt, kScanThreads, 0, stream>>>(in, n, tile_sums);
    F3S_LAUNCH_CHECK();
    k_scan_carry<<<1, 1024, 0, stream>>>(tile_sums, nt);
    F3S_LAUNCH_CHECK();
    k_scan_tiles<<<(unsigned)nt, kScanThreads, 0, stream>>>(in, out, n, tile_sums, write_total ? 1 : 0);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

// =========================================================================
// CSR -> block-sparse converter
//
// Window w owns the contiguous edge range [row_ptr[16w], row_ptr[min(16w+16,
// N)]).  Its active block columns are the sorted unique keys v >> 4.
//   1. k_convert_light: one CTA per window; validates the CSR rows; windows
//      with at most kConvCap edges are bitonic-sorted in shared memory and
//      de-duplicated; their unique keys go to scratch at the window's own
//      edge offset.  Longer windows are queued as heavy.
//   2. k_convert_heavy: persistent CTAs take heavy windows; a bitmap over the
//      block-column range (up to 2^20 columns per pass, 128 KB of shared
//      memory) gives the sorted unique keys directly.
//   3. exclusive scan of the per-window counts -> window_offsets.
//   4. k_convert_compact: one warp per window copies its keys to
//      block_cols[window_offsets[w] ...].
// =========================================================================

constexpr int kConvThreads = 256;
constexpr int kConvCap = 4096;            // keys sorted in shared memory per window
constexpr int kHeavyThreads = 1024;
constexpr int kHeavyBitmapBits = 1 << 20;  // 128 KB of shared memory per pass

__global__ void __launch_bounds__(kConvThreads)
    k_convert_light(const int* __restrict__ row_ptr, const int* __restrict__ col, int N, int64_t nnz,
                    int* __restrict__ tmp, int* __restrict__ counts, int* __restrict__ heavy_list,
                    WsHeader* hdr) {
    __shared__ int keys[kConvCap];
    __shared__ int rp[17];
    __shared__ int scratch[kConvThreads / 32 + 1];
    const ErrorSink err{&hdr->abort, &hdr->status};
    const int w = blockIdx.x;
    const int t = threadIdx.x;
    const int r0 = w * 16;
    const int nrows = min(16, N - r0);
    if (t <= nrows) rp[t] = row_ptr[r0 + t];
    __syncthreads();
    bool bad = false;
    if (t < nrows && rp[t + 1] < rp[t]) bad = true;
    if (t == 0 && (rp[0] < 0 || (int64_t)rp[nrows] > nnz)) bad = true;
    if (__syncthreads_or(bad)) {
        if (t == 0) {
            raise_error(err, F3S_ERR_BAD_CSR);
            counts[w] = 0;
        }
        return;
    }
    const int lo = rp[0];
    const int L = rp[nrows] - lo;
    if (L == 0) {
        if (t == 0) counts[w] = 0;
        return;
    }
    if (L > kConvCap) {
        if (t == 0) heavy_list[atomicAdd(&hdr->counter, 1)] = w;
        return;
    }
    int P = 1;
    while (P < L) P <<= 1;
    bad = false;
    for (int i = t; i < P; i += kConvThreads) {
        int k = INT_MAX;
        if (i < L) {
            int v = col[lo + i];
            if (v < 0 || v >= N) bad = true;
            k = v >> 4;
        }
        keys[i] = k;
    }
    if (__syncthreads_or(bad)) {
        if (t == 0) {
            raise_error(err, F3S_ERR_BAD_CSR);
            counts[w] = 0;
        }
        return;
    }
    // bitonic sort of keys[0, P) ascending
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = t; i < (P >> 1); i += kConvThreads) {
                int a = 2 * j * (i / j) + (i % j);
                int b = a + j;
                int x = keys[a], y = keys[b];
                bool up = (a & k) == 0;
                if ((x > y) == up) {
                    keys[a] = y;
                    keys[b] = x;
                }
            }
            __syncthreads();
        }
    }
    // unique: thread t owns keys [t*ipt, (t+1)*ipt)
    const int ipt = P > kConvThreads ? P / kConvThreads : 1;
    const int i0 = t * ipt;
    int cnt = 0;
    for (int i = i0; i < i0 + ipt && i < L; ++i)
        if (i == 0 || keys[i] != keys[i - 1]) ++cnt;
    int total;
    int pos = block_exclusive_scan<kConvThreads>(cnt, total, scratch);
    for (int i = i0; i < i0 + ipt && i < L; ++i)
        if (i == 0 || keys[i] != keys[i - 1]) tmp[lo + pos++] = keys[i];
    if (t == 0) counts[w] = total;
}

__global__ void __launch_bounds__(kHeavyThreads)
    k_convert_heavy(const int* __restrict__ row_ptr, const int* __restrict__ col, int N, int nrw,
                    int* __restrict__ tmp, int* __restrict__ counts,
                    const int* __restrict__ heavy_list, WsHeader* hdr, int bitmap_bits) {
    extern __shared__ uint32_t bitmap[];
    __shared__ int scratch[kHeavyThreads / 32 + 1];
    const ErrorSink err{&hdr->abort, &hdr->status};
    const int t = threadIdx.x;
    const int nheavy = load_volatile(&hdr->counter);
    for (int hi = blockIdx.x; hi < nheavy; hi += gridDim.x) {
        const int w = heavy_list[hi];
        const int lo = row_ptr[w * 16];
        const int L = row_ptr[min(w * 16 + 16, N)] - lo;
        int written = 0;
        bool bad = false;
        for (int kbase = 0; kbase < nrw; kbase += bitmap_bits) {
            const int kend = min(nrw, kbase + bitmap_bits);
            const int words = (kend - kbase + 31) >> 5;
            for (int i = t; i < words; i += kHeavyThreads) bitmap[i] = 0u;
            __syncthreads();
            for (int i = t; i < L; i += kHeavyThreads) {
                int v = col[lo + i];
                if (v < 0 || v >= N) {
                    bad = true;
                    continue;
                }
                int k = (v >> 4) - kbase;
                if (k >= 0 && k < kend - kbase) atomicOr(&bitmap[k >> 5], 1u << (k & 31));
            }
            __syncthreads();
            const int wpt = (words + kHeavyThreads - 1) / kHeavyThreads;
            const int w0 = t * wpt;
            int cnt = 0;
            for (int i = w0; i < w0 + wpt && i < words; ++i) cnt += __popc(bitmap[i]);
            int total;
            int pos = written + block_exclusive_scan<kHeavyThreads>(cnt, total, scratch);
            for (int i = w0; i < w0 + wpt && i < words; ++i) {
                uint32_t m = bitmap[i];
                while (m) {
                    int b = __ffs(m) - 1;
                    m &= m - 1;
                    tmp[lo + pos++] = kbase + i * 32 + b;
                }
            }
            written += total;
            __syncthreads();
        }
        if (__syncthreads_or(bad)) {
            if (t == 0) raise_error(err, F3S_ERR_BAD_CSR);
        }
        if (t == 0) counts[w] = written;
    }
}

__global__ void __launch_bounds__(256) k_convert_compact(const int* __restrict__ row_ptr, int nrw,
                                                         const int* __restrict__ tmp,
                                                         const int* __restrict__ offsets,
                                                         int* __restrict__ cols) {
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= nrw) return;
    const int lo = row_ptr[w * 16];
    const int off = offsets[w];
    const int cnt = offsets[w + 1] - off;
    for (int i = lane; i < cnt; i += 32) cols[off + i] = tmp[lo + i];
}

struct ConvertLayout {
    size_t tmp, counts, heavy, tiles, total;
};

static ConvertLayout convert_layout(int32_t num_nodes, int64_t nnz) {
    const int64_t nrw = ((int64_t)num_nodes + 15) / 16;
    ConvertLayout L;
    size_t off = kWsHeaderBytes;
    L.tmp = off;
    off = align_up(off + (size_t)std::max<int64_t>(nnz, 1) * 4, 256);
    L.counts = off;
    off = align_up(off + (size_t)std::max<int64_t>(nrw, 1) * 4, 256);
    L.heavy = off;
    off = align_up(off + (size_t)std::max<int64_t>(nrw, 1) * 4, 256);
    L.tiles = off;
    off = align_up(off + (size_t)std::max<int64_t>(scan_tiles(nrw), 1) * 4, 256);
    L.total = off;
    return L;
}

static int convert_impl(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes,
                        int64_t nnz, int32_t* d_window_offsets, int32_t* d_block_cols,
                        void* d_workspace, size_t workspace_bytes, int64_t* h_num_blocks,
                        cudaStream_t stream) {
    if (num_nodes < 0 || nnz < 0 || nnz > INT_MAX) return num_nodes < 0 || nnz < 0 ? F3S_ERR_INVALID_VALUE : F3S_ERR_TOO_LARGE;
    if (!d_row_ptr || !d_window_offsets || !d_workspace || (nnz > 0 && (!d_col_ind || !d_block_cols)))
        return F3S_ERR_INVALID_VALUE;
    const ConvertLayout L = convert_layout(num_nodes, nnz);
    if (workspace_bytes < L.total) return F3S_ERR_WORKSPACE;
    const int nrw = (int)(((int64_t)num_nodes + 15) / 16);
    char* ws = static_cast<char*>(d_workspace);
    WsHeader* hdr = reinterpret_cast<WsHeader*>(ws);
    int* tmp = reinterpret_cast<int*>(ws + L.tmp);
    int* counts = reinterpret_cast<int*>(ws + L.counts);
    int* heavy = reinterpret_cast<int*>(ws + L.heavy);
    int* tiles = reinterpret_cast<int*>(ws + L.tiles);

    // clear abort flag and heavy counter (adjacent words), keep the sticky status
    F3S_CUDA_TRY(cudaMemsetAsync(hdr, 0, 2 * sizeof(int), stream));
    if (nrw == 0) {
        F3S_CUDA_TRY(cudaMemsetAsync(d_window_offsets, 0, sizeof(int), stream));
    } else {
        k_convert_light<<<nrw, kConvThreads, 0, stream>>>(d_row_ptr, d_col_ind, num_nodes, nnz, tmp,
                                                          counts, heavy, hdr);
        F3S_LAUNCH_CHECK();
        const int bits = std::min(nrw, kHeavyBitmapBits);
        const size_t smem = (size_t)((bits + 31) / 32) * 4;
        // the bitmap kernel's shared-memory attribute, once per CUDA context
        static PerContext<int> attr_once;
        int rc = attr_once.get(nullptr, [](int*) -> int {
            F3S_CUDA_TRY(cudaFuncSetAttribute(k_convert_heavy, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (kHeavyBitmapBits / 32) * 4));
            return F3S_SUCCESS;
        });
        if (rc != F3S_SUCCESS) return rc;
        const int grid = std::max(1, std::min(nrw, num_sms_of_current_device()));
        k_convert_heavy<<<grid, kHeavyThreads, smem, stream>>>(d_row_ptr, d_col_ind, num_nodes, nrw, tmp,
                                                               counts, heavy, hdr, bits);
        F3S_LAUNCH_CHECK();
        rc = device_exclusive_scan(counts, d_window_offsets, nrw, true, tiles, stream);
        if (rc != F3S_SUCCESS) return rc;
        k_convert_compact<<<(nrw + 7) / 8, 256, 0, stream>>>(d_row_ptr, nrw, tmp, d_window_offsets,
                                                             d_block_cols);
        F3S_LAUNCH_CHECK();
    }
    if (h_num_blocks) {
        int st = f3s_workspace_status(d_workspace, (f3s_stream_t)stream);
        if (st != F3S_SUCCESS) return st;
        int32_t b = 0;
        F3S_CUDA_TRY(cudaMemcpyAsync(&b, d_window_offsets + nrw, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     stream));
        F3S_CUDA_TRY(cudaStreamSynchronize(stream));
        *h_num_blocks = b;
    }
    return F3S_SUCCESS;
}

// =========================================================================
// Window order: stable LSD radix sort of key = nrw - blocks(w) (so ascending
// keys = descending block counts), values = window ids starting as iota.
// 8-bit digits; ceil(bits(nrw) / 8) passes.
//   k_order_init       keys / values
//   k_radix_hist       per-tile digit histogram, digit-major [256][ntiles]
//   scan               exclusive scan of the histogram -> global bases
//   k_radix_scatter    stable in-tile ranks via warp match + per-warp counts
// =========================================================================

constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsRounds = 8;  // items per lane
constexpr int kRsTile = kRsThreads * kRsRounds;

__global__ void __launch_bounds__(256) k_order_init(const int* __restrict__ offsets, int nrw,
                                                    uint32_t* __restrict__ keys, int* __restrict__ vals) {
    int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w < nrw) {
        keys[w] = (uint32_t)(nrw - (offsets[w + 1] - offsets[w]));
        vals[w] = w;
    }
}

__global__ void __launch_bounds__(kRsThreads) k_radix_hist(const uint32_t* __restrict__ keys, int n,
                                                          int shift, int ntiles, int* __restrict__ hist) {
    __shared__ int h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int base = blockIdx.x * kRsTile;
    for (int k = 0; k < kRsRounds; ++k) {
        int i = base + k * kRsThreads + threadIdx.x;
        if (i < n) atomicAdd(&h[(keys[i] >> shift) & 255u], 1);
    }
    __syncthreads();
    hist[threadIdx.x * ntiles + blockIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(kRsThreads)
    k_radix_scatter(const uint32_t* __restrict__ keys_in, const int* __restrict__ vals_in, int n, int shift,
                    int ntiles, const int* __restrict__ hist_scanned, uint32_t* __restrict__ keys_out,
                    int* __restrict__ vals_out) {
    __shared__ int wcount[kRsWarps][256];
    __shared__ int tile_base[256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int base = blockIdx.x * kRsTile + warp * (kRsRounds * 32);
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int d = lane; d < 256; d += 32) wcount[warp][d] = 0;
    __syncwarp();
    // pass 1: per-warp digit counts
    for (int r = 0; r < kRsRounds; ++r) {
        int i = base + r * 32 + lane;
        int d = i < n ? (int)((keys_in[i] >> shift) & 255u) : -1;
        unsigned peers = __match_any_sync(0xffffffffu, d);
        if (d >= 0 && (peers & lt_mask) == 0) wcount[warp][d] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    {
        const int d = threadIdx.x;  // 256 threads == 256 digits
        int run = 0;
        for (int ww = 0; ww < kRsWarps; ++ww) {
            int c = wcount[ww][d];
            wcount[ww][d] = run;
            run += c;
        }
        tile_base[d] = hist_scanned[d * ntiles + blockIdx.x];
    }
    __syncthreads();
    // pass 2: stable ranks
    for (int r = 0; r < kRsRounds; ++r) {
        int i = base + r * 32 + lane;
        uint32_t k = 0;
        int v = 0, d = -1;
        if (i < n) {
            k = keys_in[i];
            v = vals_in[i];
            d = (int)((k >> shift) & 255u);
        }
        unsigned peers = __match_any_sync(0xffffffffu, d);
        int prior = d >= 0 ? wcount[warp][d] : 0;
        __syncwarp();
        if (d >= 0) {
            int pos = tile_base[d] + prior + __popc(peers & lt_mask);
            if (keys_out) keys_out[pos] = k;
            vals_out[pos] = v;
            if ((peers & lt_mask) == 0) wcount[warp][d] = prior + __popc(peers);
        }
        __syncwarp();
    }
}

struct OrderLayout {
    size_t keys0, keys1, vals0, vals1, hist, tiles, total;
    int ntiles;
};

static OrderLayout order_layout(int32_t nrw) {
    OrderLayout L;
    const size_t n = (size_t)std::max(nrw, 1);
    L.ntiles = (int)((n + kRsTile - 1) / kRsTile);
    size_t off = kWsHeaderBytes;
    L.keys0 = off;
    off = align_up(off + n * 4, 256);
    L.keys1 = off;
    off = align_up(off + n * 4, 256);
    L.vals0 = off;
    off = align_up(off + n * 4, 256);
    L.vals1 = off;
    off = align_up(off + n * 4, 256);
    L.hist = off;
    const size_t hn = (size_t)256 * L.ntiles;
    off = align_up(off + (hn + 1) * 4, 256);
    L.tiles = off;
    off = align_up(off + (size_t)std::max<int64_t>(scan_tiles(hn), 1) * 4, 256);
    L.total = off;
    return L;
}

static int window_order_impl(const int32_t* d_offsets, int32_t nrw, int32_t* d_order, void* d_workspace,
                             size_t workspace_bytes, cudaStream_t stream) {
    if (nrw < 0) return F3S_ERR_INVALID_VALUE;
    if (nrw == 0) return F3S_SUCCESS;
    if (!d_offsets || !d_order || !d_workspace) return F3S_ERR_INVALID_VALUE;
    const OrderLayout L = order_layout(nrw);
    if (workspace_bytes < L.total) return F3S_ERR_WORKSPACE;
    char* ws = static_cast<char*>(d_workspace);
    uint32_t* keys[2] = {reinterpret_cast<uint32_t*>(ws + L.keys0), reinterpret_cast<uint32_t*>(ws + L.keys1)};
    int* vals[2] = {reinterpret_cast<int*>(ws + L.vals0), reinterpret_cast<int*>(ws + L.vals1)};
    int* hist = reinterpret_cast<int*>(ws + L.hist);
    int* tiles = reinterpret_cast<int*>(ws + L.tiles);
    k_order_init<<<(nrw + 255) / 256, 256, 0, stream>>>(d_offsets, nrw, keys[0], vals[0]);
    F3S_LAUNCH_CHECK();
    int bits = 32 - __builtin_clz((unsigned)nrw);  // keys lie in [0, nrw]
    const int passes = (bits + 7) / 8;
    const int64_t hn = (int64_t)256 * L.ntiles;
    for (int p = 0; p < passes; ++p) {
        const int src = p & 1, dst = src ^ 1;
        const bool last = p == passes - 1;
        k_radix_hist<<<L.ntiles, kRsThreads, 0, stream>>>(keys[src], nrw, 8 * p, L.ntiles, hist);
        F3S_LAUNCH_CHECK();
        int rc = device_exclusive_scan(hist, hist, hn, false, tiles, stream);
        if (rc != F3S_SUCCESS) return rc;
        k_radix_scatter<<<L.ntiles, kRsThreads, 0, stream>>>(keys[src], vals[src], nrw, 8 * p, L.ntiles, hist,
                                                             last ? nullptr : keys[dst],
                                                             last ? d_order : vals[dst]);
        F3S_LAUNCH_CHECK();
    }
    return F3S_SUCCESS;
}

// =========================================================================
// L2 eviction hints per block.
//
// A block column's K/V tile is read once per window that lists it.  Columns
// listed by many windows are worth keeping in L2; columns listed by a single
// window are never reused.  popularity[c] = number of listed windows that
// reference c; the most popular columns, up to an L2 byte budget, get hint 1
// (evict-last), single-use columns hint 2 (evict-first), the rest hint 0.
// The hint is stored per block (hint of the block's column), so the fused
// kernel loads it alongside the block's column index instead of after it.
//   k_hint_popularity  one warp per listed window, atomics per block
//   k_hint_histogram   histogram of min(popularity, 4095)
//   k_hint_threshold   one CTA: the smallest popularity whose columns (with
//                      all more popular ones) still fit the budget
//   k_hint_mark        writes the per-block hints
// =========================================================================

constexpr int kHintBins = 4096;

__global__ void __launch_bounds__(256) k_hint_popularity(const int* __restrict__ offsets,
                                                         const int* __restrict__ cols, const int* __restrict__ order,
                                                         int num_items, int* __restrict__ pop) {
    const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (i >= num_items) return;
    const int w = order[i];
    const int b1 = offsets[w + 1];
    for (int b = offsets[w] + lane; b < b1; b += 32) atomicAdd(&pop[cols[b]], 1);
}

__global__ void __launch_bounds__(256) k_hint_histogram(const int* __restrict__ pop, int nrw,
                                                        int* __restrict__ hist) {
    __shared__ int h[kHintBins];
    for (int i = threadIdx.x; i < kHintBins; i += 256) h[i] = 0;
    __syncthreads();
    for (int c = blockIdx.x * 256 + threadIdx.x; c < nrw; c += gridDim.x * 256)
        atomicAdd(&h[min(pop[c], kHintBins - 1)], 1);
    __syncthreads();
    for (int i = threadIdx.x; i < kHintBins; i += 256)
        if (h[i]) atomicAdd(&hist[i], h[i]);
}

// T = the smallest bin b >= 2 with sum(hist[b..]) <= budget (kHintBins if
// none): those columns, the most popular, fit the budget together.
__global__ void __launch_bounds__(1024) k_hint_threshold(const int* __restrict__ hist, int64_t budget_cols,
                                                         int* __restrict__ thr) {
    __shared__ int scratch[1024 / 32 + 1];
    __shared__ int best;
    constexpr int kPer = kHintBins / 1024;
    // thread t owns bins [kHintBins - kPer (t + 1), kHintBins - kPer t), walked downwards
    const int top = kHintBins - kPer * threadIdx.x;
    int v[kPer];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        v[i] = hist[top - 1 - i];
        sum += v[i];
    }
    if (threadIdx.x == 0) best = kHintBins;
    int total;
    int above = block_exclusive_scan<1024>(sum, total, scratch);  // columns in higher bins
    int local = kHintBins;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        above += v[i];
        const int b = top - 1 - i;
        if (b >= 2 && (int64_t)above <= budget_cols) local = b;
    }
    atomicMin(&best, local);
    __syncthreads();
    if (threadIdx.x == 0) *thr = best;
}

__global__ void __launch_bounds__(256) k_hint_mark(const int* __restrict__ pop, const int* __restrict__ cols,
                                                   const int* __restrict__ offsets, int nrw,
                                                   const int* __restrict__ thr, uint8_t* __restrict__ hints) {
    const int t = *thr;
    const int nb = offsets[nrw];
    for (int b = blockIdx.x * 256 + threadIdx.x; b < nb; b += gridDim.x * 256) {
        const int q = pop[cols[b]];
        hints[b] = (uint8_t)(q >= t ? 1 : (q == 1 ? 2 : 0));
    }
}

struct HintLayout {
    size_t pop, hist, thr, total;
};

static HintLayout hint_layout(int32_t nrw) {
    HintLayout L;
    size_t off = kWsHeaderBytes;
    L.pop = off;
    off = align_up(off + (size_t)std::max(nrw, 1) * 4, 256);
    L.hist = off;
    off = align_up(off + (size_t)kHintBins * 4, 256);
    L.thr = off;
    L.total = align_up(off + 4, 256);
    return L;
}

static int block_hints_impl(const int32_t* d_offsets, const int32_t* d_cols, const int32_t* d_order,
                            int32_t num_items, int32_t nrw, int64_t bytes_per_column, int64_t l2_budget_bytes,
                            uint8_t* d_hints, void* d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (nrw < 0 || num_items < 0 || bytes_per_column <= 0 || l2_budget_bytes < 0) return F3S_ERR_INVALID_VALUE;
    if (nrw == 0) return F3S_SUCCESS;
    if (!d_offsets || !d_cols || !d_hints || !d_workspace || (num_items > 0 && !d_order))
        return F3S_ERR_INVALID_VALUE;
    const HintLayout L = hint_layout(nrw);
    if (workspace_bytes < L.total) return F3S_ERR_WORKSPACE;
    char* ws = static_cast<char*>(d_workspace);
    int* pop = reinterpret_cast<int*>(ws + L.pop);
    int* hist = reinterpret_cast<int*>(ws + L.hist);
    int* thr = reinterpret_cast<int*>(ws + L.thr);
    F3S_CUDA_TRY(cudaMemsetAsync(pop, 0, (size_t)nrw * 4, stream));
    F3S_CUDA_TRY(cudaMemsetAsync(hist, 0, (size_t)kHintBins * 4, stream));
    if (num_items > 0) {
        k_hint_popularity<<<(num_items + 7) / 8, 256, 0, stream>>>(d_offsets, d_cols, d_order, num_items, pop);
        F3S_LAUNCH_CHECK();
    }
    const int sms = num_sms_of_current_device();
    k_hint_histogram<<<std::max(1, std::min((nrw + 255) / 256, sms * 4)), 256, 0, stream>>>(pop, nrw, hist);
    F3S_LAUNCH_CHECK();
    k_hint_threshold<<<1, 1024, 0, stream>>>(hist, l2_budget_bytes / bytes_per_column, thr);
    F3S_LAUNCH_CHECK();
    k_hint_mark<<<sms * 8, 256, 0, stream>>>(pop, d_cols, d_offsets, nrw, thr, d_hints);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

// =========================================================================
// Converter for callers that cannot allocate device memory.
//
// Its scratch lives in the library itself: a fixed 32 MiB array in device
// global memory that every GPU loading this library holds until the process
// exits.  Host code only ever sees a host-side stand-in for the array's name,
// so the real device address is looked up once per device, with that device
// current, through cudaGetSymbolAddress.  Every call shares the array;
// calls whose work overlaps on the GPU (other streams, other host threads)
// race on it.
// =========================================================================

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address in the current context, looked up with the
// device current the first time a context uses it (and again after a device
// reset, whose new context places the array anew).
static int noalloc_scratch_address(void** out) {
    static PerContext<void*> addr;
    return addr.get(out, [](void** p) -> int {
        *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(p, g_noalloc_scratch);
        if (e != cudaSuccess || *p == nullptr) {
            note_cuda_error(e);
            return F3S_ERR_CUDA;
        }
        return F3S_SUCCESS;
    });
}

static int convert_noalloc_impl(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes,
                                int64_t nnz, int32_t* d_window_offsets, int32_t* d_block_cols,
                                int64_t* h_num_blocks, cudaStream_t stream) {
    if (num_nodes < 0 || nnz < 0 || h_num_blocks == nullptr) return F3S_ERR_INVALID_VALUE;
    if (nnz > INT_MAX) return F3S_ERR_TOO_LARGE;
    if (convert_layout(num_nodes, nnz).total > kNoAllocScratchBytes) return F3S_ERR_WORKSPACE;
    void* ws = nullptr;
    int rc = noalloc_scratch_address(&ws);
    if (rc != F3S_SUCCESS) return rc;
    // the array keeps the previous call's contents: the header (abort flag,
    // heavy-window counter, status word) must start at zero; everything
    // after it is written before it is read within one call
    F3S_CUDA_TRY(cudaMemsetAsync(ws, 0, kWsHeaderBytes, stream));
    return convert_impl(d_row_ptr, d_col_ind, num_nodes, nnz, d_window_offsets, d_block_cols, ws,
                        kNoAllocScratchBytes, h_num_blocks, stream);
}

}  // namespace f3s

extern "C" {

int f3s_convert_noalloc(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes, int64_t nnz,
                        int32_t* d_window_offsets, int32_t* d_block_cols, int64_t* h_num_blocks,
                        f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_convert_noalloc");
    return f3s::convert_noalloc_impl(d_row_ptr, d_col_ind, num_nodes, nnz, d_window_offsets, d_block_cols,
                                     h_num_blocks, (cudaStream_t)stream);
}

size_t f3s_convert_workspace_size(int32_t num_nodes, int64_t nnz) {
    if (num_nodes < 0 || nnz < 0) return 0;
    return f3s::convert_layout(num_nodes, nnz).total;
}

int f3s_convert(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes, int64_t nnz,
                int32_t* d_window_offsets, int32_t* d_block_cols, void* d_workspace, size_t workspace_bytes,
                int64_t* h_num_blocks, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_convert");
    return f3s::convert_impl(d_row_ptr, d_col_ind, num_nodes, nnz, d_window_offsets, d_block_cols,
                             d_workspace, workspace_bytes, h_num_blocks, (cudaStream_t)stream);
}

size_t f3s_block_hints_workspace_size(int32_t num_row_windows) {
    if (num_row_windows < 0) return 0;
    return f3s::hint_layout(num_row_windows).total;
}

int f3s_block_hints(const int32_t* d_window_offsets, const int32_t* d_block_cols, const int32_t* d_order,
                    int32_t num_items, int32_t num_row_windows, int64_t bytes_per_column, int64_t l2_budget_bytes,
                    uint8_t* d_block_hints, void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_block_hints");
    return f3s::block_hints_impl(d_window_offsets, d_block_cols, d_order, num_items, num_row_windows,
                                 bytes_per_column, l2_budget_bytes, d_block_hints, d_workspace, workspace_bytes,
                                 (cudaStream_t)stream);
}

size_t f3s_window_order_workspace_size(int32_t num_row_windows) {
    if (num_row_windows < 0) return 0;
    return f3s::order_layout(num_row_windows).total;
}

int f3s_window_order(const int32_t* d_window_offsets, int32_t num_row_windows, int32_t* d_order,
                     void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_window_order");
    return f3s::window_order_impl(d_window_offsets, num_row_windows, d_order, d_workspace, workspace_bytes,
                                  (cudaStream_t)stream);
}

}  // extern "C"
