/* The C-ABI call sequence a C caller of fused3S would write (convert, order,
 * plan, hints, forward, status), compiled with a C compiler to keep the header
 * plain C.  Not executed: it only has to compile against include/fused3s.h. */
#include <stdint.h>
#include <stdlib.h>
#include "fused3s.h"

int run(const int32_t* d_row_ptr, const int32_t* d_col, int32_t N, int64_t nnz, int32_t* d_offsets,
        int32_t* d_cols, int32_t* d_order, const void* d_Q, const void* d_K, const void* d_V, float* d_O,
        void* d_O16, uint8_t* d_hints, void* d_ws, size_t ws_bytes, void* d_plan, size_t plan_bytes,
        const char* d_text, int64_t text_bytes, f3s_stream_t stream) {
    const int32_t H = 8, d = 64, nrw = (N + 15) / 16;
    int64_t B = 0, count = 0;
    int st = f3s_convert(d_row_ptr, d_col, N, nnz, d_offsets, d_cols, d_ws, ws_bytes, &B, stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_convert_noalloc(d_row_ptr, d_col, N, nnz, d_offsets, d_cols, &B, stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_window_order(d_offsets, nrw, d_order, d_ws, f3s_window_order_workspace_size(nrw), stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_block_hints(d_offsets, d_cols, d_order, nrw, nrw, 16LL * H * d * 4, 63LL << 20, d_hints, d_ws,
                         f3s_block_hints_workspace_size(nrw), stream);
    if (st != F3S_SUCCESS) return st;
    if (plan_bytes < f3s_plan_size(nrw, B, 64, H, d)) return F3S_ERR_WORKSPACE;
    st = f3s_make_plan(d_offsets, d_order, nrw, B, 64, H, d, d_plan, plan_bytes, stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_forward(d_Q, d_K, d_V, d_O, d_offsets, d_cols, d_order, d_hints, d_plan, nrw, N, H, d, 0, N, d_ws,
                     f3s_forward_workspace_size(), stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_forward_ex(d_Q, d_K, d_V, d_O16, F3S_OUT_F16, d_offsets, d_cols, d_order, NULL, NULL, nrw, N, H, d,
                        0, N, d_ws, f3s_forward_workspace_size(), stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_workspace_status(d_ws, stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_1tb1rw_launch(d_Q, d_K, d_V, d_O, d_offsets, d_cols, d_order, nrw, d, stream);
    if (st != F3S_SUCCESS) return st;
    st = f3s_parse_int32(d_text, text_bytes, (int32_t*)d_cols, nnz, &count, d_ws,
                         f3s_parse_int32_workspace_size(text_bytes), stream);
    if (st != F3S_SUCCESS) return st;
    {
        int32_t piece[4] = {0, 0, 0, -1};
        int32_t off_h[2] = {0, 0};
        st = f3s_load_plan(piece, 1, NULL, 0, 0, off_h, 1, H, d, d_plan, f3s_plan_size_for(1, 0, 0, H, d), stream);
        if (st != F3S_SUCCESS) return st;
    }
    {
        void* buf = NULL;
        char handle[F3S_IPC_HANDLE_BYTES];
        st = f3s_peer_alloc(1 << 20, &buf, handle);
        if (st != F3S_SUCCESS) return st;
        st = f3s_peer_copy(buf, d_O, 1 << 20, stream);
        f3s_peer_free(buf);
    }
    return st == F3S_SUCCESS ? f3s_half_from_float(d_O, d_O16, 16, stream) : st;
}
