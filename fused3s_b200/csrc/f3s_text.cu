// f3s_text.cu -- whitespace-separated decimal integers (the reference's
// meta.txt / row_ptr.txt / col_idx.txt, read with `>>` at
// include/utils.cuh:26-40) parsed on the GPU, so a CSR read from disk goes
// to the device as raw bytes and is decoded there.
//
// Two passes over tiles of kTextTile bytes (a thread per 16 consecutive
// bytes): count the starts of numbers per tile, scan the tile counts, then
// recount with a block scan to give every number its rank and let the thread
// that holds its first byte decode it.  A number is a maximal run of
// [0-9+-]; separators are space, tab, CR and LF.  Any other byte, a sign not
// followed by digits only, or a value outside int32 records an error in the
// workspace.  Byte-bound: each byte is read twice (plus at most 11 bytes
// past a tile end for the numbers that straddle it).
#include "f3s_internal.cuh"

namespace f3s {

constexpr int kTextThreads = 256;
constexpr int kTextBytesPerThread = 16;
constexpr int kTextTile = kTextThreads * kTextBytesPerThread;
// a text holds at most (n_bytes + 1) / 2 numbers: the counts stay in int32
constexpr int64_t kMaxTextBytes = (int64_t)INT32_MAX - 1;

__device__ __forceinline__ bool text_num_char(unsigned char c) { return (c >= '0' && c <= '9') || c == '-' || c == '+'; }
__device__ __forceinline__ bool text_space(unsigned char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

// number starts among this thread's bytes [i0, i0 + 16); flags bad bytes
__device__ __forceinline__ int text_starts(const unsigned char* __restrict__ t, int64_t n, int64_t i0, uint32_t& mask,
                                           bool& bad) {
    unsigned char prev = i0 > 0 ? t[i0 - 1] : ' ';
    int cnt = 0;
    mask = 0;
#pragma unroll
    for (int k = 0; k < kTextBytesPerThread; ++k) {
        const int64_t i = i0 + k;
        if (i >= n) break;
        const unsigned char c = t[i];
        const bool num = text_num_char(c);
        if (!num && !text_space(c)) bad = true;
        if (num && !text_num_char(prev)) {
            mask |= 1u << k;
            ++cnt;
        }
        prev = c;
    }
    return cnt;
}

__global__ void __launch_bounds__(kTextThreads) k_text_count(const unsigned char* __restrict__ t, int64_t n,
                                                             int* __restrict__ tile_counts, WsHeader* hdr) {
    __shared__ int scratch[kTextThreads / 32 + 1];
    const int64_t i0 = (int64_t)blockIdx.x * kTextTile + (int64_t)threadIdx.x * kTextBytesPerThread;
    uint32_t mask;
    bool bad = false;
    const int c = text_starts(t, n, i0, mask, bad);
    if (bad) raise_error(ErrorSink{&hdr->abort, &hdr->status}, F3S_ERR_INVALID_VALUE);
    int total;
    block_exclusive_scan<kTextThreads>(c, total, scratch);
    if (threadIdx.x == 0) tile_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kTextThreads) k_text_parse(const unsigned char* __restrict__ t, int64_t n,
                                                             const int* __restrict__ tile_offsets,
                                                             int32_t* __restrict__ out, int64_t max_count,
                                                             WsHeader* hdr) {
    __shared__ int scratch[kTextThreads / 32 + 1];
    const int64_t i0 = (int64_t)blockIdx.x * kTextTile + (int64_t)threadIdx.x * kTextBytesPerThread;
    uint32_t mask;
    bool bad = false;
    const int c = text_starts(t, n, i0, mask, bad);
    int total;
    const int before = block_exclusive_scan<kTextThreads>(c, total, scratch);
    int64_t rank = (int64_t)tile_offsets[blockIdx.x] + before;
    while (mask) {
        const int k = __ffs(mask) - 1;
        mask &= mask - 1;
        int64_t i = i0 + k;
        bool neg = false;
        if (t[i] == '-' || t[i] == '+') {
            neg = t[i] == '-';
            ++i;
        }
        int64_t v = 0;
        int digits = 0;
        bool ok = true;
        for (; i < n && text_num_char(t[i]); ++i) {
            const unsigned char ch = t[i];
            if (ch < '0' || ch > '9' || digits >= 11) {  // sign inside a number, or too long for int32
                ok = false;
                break;
            }
            v = v * 10 + (ch - '0');
            ++digits;
        }
        if (neg) v = -v;
        if (!ok || digits == 0) {
            raise_error(ErrorSink{&hdr->abort, &hdr->status}, digits >= 11 ? F3S_ERR_TOO_LARGE : F3S_ERR_INVALID_VALUE);
        } else if (v > INT32_MAX || v < INT32_MIN) {
            raise_error(ErrorSink{&hdr->abort, &hdr->status}, F3S_ERR_TOO_LARGE);
        } else if (rank >= max_count) {
            raise_error(ErrorSink{&hdr->abort, &hdr->status}, F3S_ERR_WORKSPACE);
        } else {
            out[rank] = (int32_t)v;
        }
        ++rank;
    }
}

struct TextLayout {
    size_t counts, tiles, total;
};

static TextLayout text_layout(int64_t n_bytes) {
    TextLayout L{};
    const int64_t nt = (n_bytes + kTextTile - 1) / kTextTile;
    size_t off = kWsHeaderBytes;
    L.counts = off;
    off = align_up(off + (size_t)(nt + 1) * 4, 256);
    L.tiles = off;
    off = align_up(off + (size_t)std::max<int64_t>(scan_tiles(nt), 1) * 4, 256);
    L.total = off;
    return L;
}

static int parse_int32_impl(const char* d_text, int64_t n_bytes, int32_t* d_out, int64_t max_count,
                            int64_t* h_count, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (n_bytes < 0 || max_count < 0 || !h_count || !ws) return F3S_ERR_INVALID_VALUE;
    if (n_bytes > kMaxTextBytes) return F3S_ERR_TOO_LARGE;
    *h_count = 0;
    if (n_bytes == 0) return F3S_SUCCESS;
    if (!d_text || (max_count > 0 && !d_out)) return F3S_ERR_INVALID_VALUE;
    const TextLayout L = text_layout(n_bytes);
    if (ws_bytes < L.total) return F3S_ERR_WORKSPACE;
    char* w = static_cast<char*>(ws);
    WsHeader* hdr = reinterpret_cast<WsHeader*>(w);
    int* counts = reinterpret_cast<int*>(w + L.counts);
    int* tiles = reinterpret_cast<int*>(w + L.tiles);
    const int64_t nt = (n_bytes + kTextTile - 1) / kTextTile;
    const unsigned char* t = reinterpret_cast<const unsigned char*>(d_text);
    F3S_CUDA_TRY(cudaMemsetAsync(hdr, 0, kWsHeaderBytes, stream));
    k_text_count<<<(unsigned)nt, kTextThreads, 0, stream>>>(t, n_bytes, counts, hdr);
    F3S_LAUNCH_CHECK();
    int rc = device_exclusive_scan(counts, counts, nt, true, tiles, stream);
    if (rc != F3S_SUCCESS) return rc;
    k_text_parse<<<(unsigned)nt, kTextThreads, 0, stream>>>(t, n_bytes, counts, d_out, max_count, hdr);
    F3S_LAUNCH_CHECK();
    int found = 0, status = 0;
    F3S_CUDA_TRY(cudaMemcpyAsync(&found, counts + nt, sizeof(int), cudaMemcpyDeviceToHost, stream));
    F3S_CUDA_TRY(cudaMemcpyAsync(&status, &hdr->status, sizeof(int), cudaMemcpyDeviceToHost, stream));
    F3S_CUDA_TRY(cudaStreamSynchronize(stream));
    if (status != 0) return status;
    *h_count = found;
    return F3S_SUCCESS;
}

}  // namespace f3s

extern "C" {

size_t f3s_parse_int32_workspace_size(int64_t n_bytes) {
    if (n_bytes < 0) return 0;
    return f3s::text_layout(n_bytes).total;
}

int f3s_parse_int32(const char* d_text, int64_t n_bytes, int32_t* d_out, int64_t max_count, int64_t* h_count,
                    void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    return f3s::parse_int32_impl(d_text, n_bytes, d_out, max_count, h_count, d_workspace, workspace_bytes,
                                 (cudaStream_t)stream);
}

}  // extern "C"
