/*
 * fused3s.h -- C ABI of libfused3s.so, the B200 (sm_100a) fused 3S engine:
 * CSR -> 16x16 block-sparse row windows -> descending-workload window order
 * -> fused SDDMM + online softmax + SpMM -> fp32 O.
 *
 * Plain pointers and sizes only.  Every device pointer is caller-owned
 * memory on the current device.  Every call is asynchronous on `stream`
 * unless it says it synchronises.  Calls never exit the process: they return
 * an f3s_status.  Errors found by a kernel (bad CSR, bad window id, an
 * expired bounded wait) are recorded in the caller's workspace and read back
 * with f3s_workspace_status().
 *
 * Reference interfaces replaced (paths relative to the fatalhawk/fused3S
 * project root):
 *   f3s_convert        <- blockSparseFormat convert_csr_to_block_sparse(
 *                           int, const std::vector<int>&, const std::vector<int>&)
 *                           src/converter.cu:13 (declared by callers at
 *                           tests/test_fused_3s_v2.cu:10)
 *   f3s_window_order   <- std::vector<int> generate_balanced_window_order(
 *                           const blockSparseFormat&)   include/utils.cuh:48
 *   f3s_forward        <- __global__ f3s_1tb1rw_kernel(...) src/fused3s_v2.cu:81-90,
 *                           launched <<<nrw, dim3(32,4)>>> at
 *                           tests/test_fused_3s_v2.cu:123-131
 *   f3s_1tb1rw_launch  <- the same kernel with its exact argument list
 *   f3s_half_from_float<- __global__ float2half_kernel tests/test_fused_3s_v2.cu:61-64
 * The C++ header fused3s.hpp rebuilds the reference's own host API
 * (GraphData, blockSparseFormat, load_csr_graph, ...) on top of these.
 */
#ifndef FUSED3S_H_
#define FUSED3S_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* f3s_stream_t;

typedef enum f3s_status {
    F3S_SUCCESS = 0,
    F3S_ERR_INVALID_VALUE = 1, /* bad argument: null pointer, negative size ...   */
    F3S_ERR_UNSUPPORTED = 2,   /* head_dim / heads combination not built          */
    F3S_ERR_BAD_CSR = 3,       /* column outside [0, N) or row_ptr decreasing     */
    F3S_ERR_WORKSPACE = 4,     /* workspace smaller than the *_workspace_size()   */
    F3S_ERR_CUDA = 5,          /* a CUDA runtime call failed                      */
    F3S_ERR_TIMEOUT = 6,       /* a bounded device-side wait expired              */
    F3S_ERR_BAD_FORMAT = 7,    /* window id / block column outside its range      */
    F3S_ERR_TOO_LARGE = 8      /* exceeds the int32 limits of the format          */
} f3s_status;

/* Human-readable name of a status code (static storage). */
const char* f3s_status_string(int status);

/* Library ABI version: major * 10000 + minor * 100 + patch. */
int f3s_version(void);

/* Last CUDA error seen by a call that returned F3S_ERR_CUDA (cudaError_t). */
int f3s_last_cuda_error(void);

/* At most max_ctas persistent CTAs per forward launch on the current device
 * from now on (0: one per SM, the default).  The fused kernel holds one CTA
 * per SM for its whole run; a caller that overlaps it with another kernel
 * -- an NCCL collective on a second stream, say -- leaves that kernel SMs
 * this way.  No reference counterpart. */
int f3s_set_forward_sm_limit(int32_t max_ctas);

/* ------------------------------------------------------------------------
 * Workspace status.  Synchronises `stream`, returns the first error code a
 * kernel recorded in `d_workspace` (any of the workspaces below) and clears
 * it.  F3S_SUCCESS when none.
 * ---------------------------------------------------------------------- */
int f3s_workspace_status(void* d_workspace, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * CSR -> block-sparse row windows (src/converter.cu:13-44 semantics).
 *
 * Window w covers rows [16w, min(16w+16, N)); its active block columns are
 * the sorted unique {v / 16} over the window's edges.  Output is bit-exact
 * to the reference converter.
 *
 *   d_row_ptr        int32[num_nodes + 1]   CSR row pointers
 *   d_col_ind        int32[nnz]             CSR column indices (any order)
 *   d_window_offsets int32[nrw + 1] out     nrw = ceil(num_nodes / 16)
 *   d_block_cols     int32[nnz]      out    capacity nnz (B <= nnz always);
 *                                           first B entries are written
 *   h_num_blocks     optional host int64 out: if non-NULL the call
 *                    synchronises `stream`, checks the CSR status and stores
 *                    B = window_offsets[nrw].
 * The CSR is validated on the device (columns in [0, N), row_ptr
 * non-decreasing and within [0, nnz]); a violation is reported as
 * F3S_ERR_BAD_CSR (immediately when h_num_blocks != NULL, else through
 * f3s_workspace_status).
 * ---------------------------------------------------------------------- */
size_t f3s_convert_workspace_size(int32_t num_nodes, int64_t nnz);
int f3s_convert(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes, int64_t nnz,
                int32_t* d_window_offsets, int32_t* d_block_cols, void* d_workspace,
                size_t workspace_bytes, int64_t* h_num_blocks, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * CSR -> block-sparse row windows without any device allocation.
 * No counterpart in the reference (its converter runs on the host).
 *
 * Same output and CSR checks as f3s_convert, for callers that cannot
 * allocate device memory for the converter's scratch: a plugin inside a
 * framework whose caching allocator has already reserved the GPU's memory
 * (a cudaMalloc of its own may fail there, or take memory the framework
 * thinks it owns), or a latency-critical service that allocates everything
 * at start-up and never calls cudaMalloc / cudaFree afterwards (both can
 * stall or synchronise the device).  The caller still passes the inputs and
 * the outputs (d_window_offsets: nrw + 1 entries, d_block_cols: nnz).
 *
 * The scratch is a fixed 32 MiB array inside the library, in device memory,
 * held by every GPU that loads the library until the process exits.  A
 * graph whose f3s_convert_workspace_size(num_nodes, nnz) exceeds 32 MiB
 * (about nnz + 2 * num_nodes / 16 > 8.3 million) is rejected with
 * F3S_ERR_WORKSPACE before anything runs.  This call itself allocates
 * nothing (no cudaMalloc, cudaFree or allocating library routine).
 *
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  h_num_blocks is required: the call
 * synchronises `stream`, reads the kernels' status from the shared array and
 * returns it (F3S_ERR_BAD_CSR etc.), and stores B.  All calls share the one
 * array, so calls whose work overlaps on the GPU (from several streams or
 * host threads) race; serialise them.
 * ---------------------------------------------------------------------- */
int f3s_convert_noalloc(const int32_t* d_row_ptr, const int32_t* d_col_ind, int32_t num_nodes, int64_t nnz,
                        int32_t* d_window_offsets, int32_t* d_block_cols, int64_t* h_num_blocks,
                        f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Balanced window order (include/utils.cuh:48-59 semantics).
 *
 * d_order[i] = window ids sorted by block count, descending; ties by
 * ascending window id (a stable sort).  The block-count sequence along the
 * order equals the reference's for every input.
 * ---------------------------------------------------------------------- */
size_t f3s_window_order_workspace_size(int32_t num_row_windows);
int f3s_window_order(const int32_t* d_window_offsets, int32_t num_row_windows, int32_t* d_order,
                     void* d_workspace, size_t workspace_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused SDDMM + online softmax + SpMM (src/fused3s_v2.cu:81-246 semantics,
 * with columns >= num_nodes masked like the reference's CPU ground truth,
 * tests/test_fused_3s_v2.cu:32-37).
 *
 * For every window w listed in d_order[0 .. num_items) and every head h:
 *   O[r, h, :] = sum_c softmax_c(Q[r, h, :] . K[c, h, :]) V[c, h, :]
 * over the 16 columns of every active block of w, rows r of w with r < N.
 *
 *   d_Q     fp16 [q_rows, heads, head_dim]  rows 16*q_window_base ... of Q
 *   d_K,d_V fp16 [num_nodes, heads, head_dim]
 *   d_O     fp32 [q_rows, heads, head_dim]  same rows as d_Q; rows of listed
 *           windows are fully written (zeros for a window with no block)
 *   d_window_offsets / d_block_cols: the converter's output for all windows
 *   d_order  int32[num_items] window ids to compute (any subset, any order;
 *            each must lie in [q_window_base, q_window_base + ceil(q_rows/16)))
 *   d_block_hints optional uint8[num_blocks] L2 eviction hint of every
 *            active block from f3s_block_hints (NULL: no hint); affects
 *            speed only.
 *   d_plan   optional plan from f3s_make_plan (NULL: one work item per entry
 *            of d_order).  With a plan, d_order / num_items are not used: the
 *            plan lists the windows, heavy ones cut into pieces.
 *   q_window_base / q_rows: 0 / num_nodes on one GPU; a rank's slab when the
 *            windows are sharded across GPUs.
 * head_dim in {64, 128}; heads >= 1.  No padding of any tensor is needed:
 * rows >= num_nodes are never read or written.  All base pointers must be
 * 16-byte aligned.
 * ---------------------------------------------------------------------- */
size_t f3s_forward_workspace_size(void);
int f3s_forward(const void* d_Q, const void* d_K, const void* d_V, float* d_O,
                const int32_t* d_window_offsets, const int32_t* d_block_cols, const int32_t* d_order,
                const uint8_t* d_block_hints, const void* d_plan, int32_t num_items, int32_t num_nodes,
                int32_t heads, int32_t head_dim, int32_t q_window_base, int32_t q_rows, void* d_workspace,
                size_t workspace_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * f3s_forward with the element type of O chosen by the caller (no reference
 * counterpart: the reference writes fp32 O only).  Identical arguments and
 * semantics, except d_O is [q_rows, heads, head_dim] of o_dtype: the fp32
 * result rounded to nearest-even (F3S_OUT_F16 / F3S_OUT_BF16), which halves
 * the O write and any later all-gather of O.  F3S_OUT_F32 is f3s_forward.
 * ---------------------------------------------------------------------- */
typedef enum f3s_out_dtype {
    F3S_OUT_F32 = 0,
    F3S_OUT_F16 = 1,
    F3S_OUT_BF16 = 2
} f3s_out_dtype;

int f3s_forward_ex(const void* d_Q, const void* d_K, const void* d_V, void* d_O, int32_t o_dtype,
                   const int32_t* d_window_offsets, const int32_t* d_block_cols, const int32_t* d_order,
                   const uint8_t* d_block_hints, const void* d_plan, int32_t num_items, int32_t num_nodes,
                   int32_t heads, int32_t head_dim, int32_t q_window_base, int32_t q_rows, void* d_workspace,
                   size_t workspace_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Work plan for f3s_forward (no reference counterpart: the reference gives
 * each window one CTA, so one heavy window bounds the kernel's run time).
 *
 * For the windows in d_order[0 .. num_items) (kept in that order), a window
 * with more than max_blocks_per_piece active blocks becomes
 * ceil(blocks / max_blocks_per_piece) pieces of consecutive blocks, each its
 * own work item; the pieces' partial softmax states are merged (in piece
 * order: the result is deterministic) after the fused kernel.  num_blocks is
 * an upper bound on the active blocks of the listed windows (sizes the
 * plan).  The plan is built on the device; compute it once per graph and
 * window set, for one (heads, head_dim).  d_plan must be 256-byte aligned;
 * a plan is used by one forward at a time.
 * ---------------------------------------------------------------------- */
size_t f3s_plan_size(int32_t num_items, int64_t num_blocks, int32_t max_blocks_per_piece, int32_t heads,
                     int32_t head_dim);
int f3s_make_plan(const int32_t* d_window_offsets, const int32_t* d_order, int32_t num_items,
                  int64_t num_blocks, int32_t max_blocks_per_piece, int32_t heads, int32_t head_dim,
                  void* d_plan, size_t plan_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * A work plan whose pieces the caller built on the host (no reference
 * counterpart), for schedules f3s_make_plan does not make -- e.g. windows
 * cut at block-column chunk boundaries with the pieces ordered chunk by
 * chunk, so that all SMs read one L2-sized range of K/V at a time.
 *
 * h_pieces: int32[4 * num_pieces], per piece in processing order
 *   (window, first block, end block, partial slot), the block range inside
 *   the window's [window_offsets[w], window_offsets[w + 1]); slot -1 for a
 *   window that is one piece, else the slot of its partial state.
 * h_splits: int32[4 * num_split], per window of several pieces
 *   (window, first slot, pieces, 0): its pieces own slots first ...
 *   first + pieces - 1 and are merged in slot order (deterministic).
 * h_window_offsets: the format's offsets on the host (validation only).
 * Copies synchronously.  The plan is validated on the host and rejected
 * with F3S_ERR_BAD_FORMAT unless: every index lies in range; the pieces of
 * each listed window cover its blocks exactly once (no gap, no overlap),
 * each holding at least one block except the single piece of a window
 * without blocks; a window of one piece has slot -1 and no split record; a
 * window of several pieces has exactly one split record whose count equals
 * its pieces, and its pieces use that record's slots, each exactly once; no
 * two split records share a slot.
 * The plan then serves f3s_forward / f3s_forward_ex like one from
 * f3s_make_plan (d_order / num_items unused), and f3s_forward_pieces.
 * ---------------------------------------------------------------------- */
size_t f3s_plan_size_for(int32_t num_pieces, int32_t num_split, int32_t num_split_pieces, int32_t heads,
                         int32_t head_dim);
int f3s_load_plan(const int32_t* h_pieces, int32_t num_pieces, const int32_t* h_splits, int32_t num_split,
                  int32_t num_split_pieces, const int32_t* h_window_offsets, int32_t num_row_windows, int32_t heads,
                  int32_t head_dim, void* d_plan, size_t plan_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Sweep plan (no reference counterpart): a caller-built schedule in which
 * a window may run as several pieces that are processed one after another
 * inside one forward launch, carrying the window's running softmax state
 * (row max, row sum, unnormalised O) from piece to piece in the plan.  Its
 * purpose is locality: windows cut at block-column chunk boundaries and the
 * pieces listed chunk by chunk make every SM read one L2-sized range of K / V
 * at a time, while no partial state per piece is kept.
 *
 * h_pieces: int32[4 * num_pieces] in processing order, (window, first block,
 *   end block, unused).  The pieces of a window must appear in ascending
 *   block order and cover its blocks [window_offsets[w], window_offsets[w+1])
 *   exactly once; a piece holds at least one block unless its window has
 *   none.  Windows must lie in [q_window_base, q_window_base + q_windows).
 * Validated on the host (F3S_ERR_BAD_FORMAT); copies synchronously.
 * A piece waits (bounded) until the previous piece of its window has stored
 * the state: run a sweep plan with f3s_forward / f3s_forward_ex (one launch
 * runs every piece), with a workspace of f3s_sweep_workspace_size(q_rows,
 * heads) bytes (per-window counters, cleared by each launch).  The result
 * equals the unsplit forward within the same tolerance.
 * ---------------------------------------------------------------------- */
size_t f3s_sweep_plan_size(int32_t num_pieces, int32_t q_windows, int32_t heads, int32_t head_dim);
size_t f3s_sweep_workspace_size(int32_t q_rows, int32_t heads);
int f3s_load_sweep_plan(const int32_t* h_pieces, int32_t num_pieces, const int32_t* h_window_offsets,
                        int32_t num_row_windows, int32_t q_window_base, int32_t q_windows, int32_t heads,
                        int32_t head_dim, void* d_plan, size_t plan_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Part of a plan's work, with K / V holding only some block columns (no
 * reference counterpart: the reference reads all of K / V on one device).
 *
 * Runs pieces [piece_begin, piece_end) of d_plan (piece_end -1: to the
 * plan's last piece) and does not merge.  d_K / d_V hold the graph's rows
 * 16 * kv_col_base ... 16 * kv_col_base + kv_rows - 1 (kv_rows ends on a
 * block-column boundary unless it reaches num_nodes); every block of the
 * launched pieces must have its column inside that range
 * (F3S_ERR_BAD_FORMAT otherwise, through f3s_workspace_status).  A piece of
 * a window of one piece (slot -1) writes the window's O rows; a piece of a
 * split window writes its partial softmax state into the plan.  Once every
 * piece of the split windows has run -- over one or several calls, e.g. one
 * per K / V slice passed around a ring of GPUs -- f3s_plan_merge writes
 * their O rows.  f3s_forward_ex with a plan equals f3s_forward_pieces over
 * all pieces with the whole K / V, then f3s_plan_merge.  (Not for sweep
 * plans, whose pieces must all run in one launch.)
 * Other arguments as f3s_forward_ex (d_order is not needed).
 * ---------------------------------------------------------------------- */
int f3s_forward_pieces(const void* d_Q, const void* d_K, const void* d_V, void* d_O, int32_t o_dtype,
                       const int32_t* d_window_offsets, const int32_t* d_block_cols, const uint8_t* d_block_hints,
                       const void* d_plan, int32_t piece_begin, int32_t piece_end, int32_t kv_col_base,
                       int32_t kv_rows, int32_t num_nodes, int32_t heads, int32_t head_dim, int32_t q_window_base,
                       int32_t q_rows, void* d_workspace, size_t workspace_bytes, f3s_stream_t stream);

/* Combines the partial states of every split window of d_plan (in slot
 * order: deterministic) and writes their O rows ([q_rows, heads, head_dim]
 * of o_dtype, rows 16 * q_window_base ...). */
int f3s_plan_merge(const void* d_plan, void* d_O, int32_t o_dtype, int32_t num_nodes, int32_t heads,
                   int32_t head_dim, int32_t q_window_base, int32_t q_rows, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * L2 eviction hints for f3s_forward, one per active block (no reference
 * counterpart: a speed hint computed once per graph and window set).
 *
 * Counts, for the windows listed in d_order[0 .. num_items), how many of
 * them reference each block column; the most popular columns whose K/V
 * bytes (bytes_per_column = 16 * heads * head_dim * 2 * 2) fit in
 * l2_budget_bytes get hint 1 (keep: evict-last), columns referenced by one
 * listed window get hint 2 (stream: evict-first), the rest 0.  Every block
 * gets its column's hint, so the forward reads it next to the block's
 * column index.  d_block_hints: uint8[d_window_offsets[num_row_windows]]
 * (entries of unlisted windows' blocks are written but not meaningful).
 * ---------------------------------------------------------------------- */
size_t f3s_block_hints_workspace_size(int32_t num_row_windows);
int f3s_block_hints(const int32_t* d_window_offsets, const int32_t* d_block_cols, const int32_t* d_order,
                    int32_t num_items, int32_t num_row_windows, int64_t bytes_per_column,
                    int64_t l2_budget_bytes, uint8_t* d_block_hints, void* d_workspace,
                    size_t workspace_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Drop-in launch with the reference kernel's exact argument list
 * (src/fused3s_v2.cu:81-90): Q/K/V/O have num_row_windows*16 rows of
 * feat_dim columns, one head, and every one of those rows is treated as a
 * real node (the reference v2 kernel cannot know N, so padded columns are
 * not masked -- call f3s_forward with the true num_nodes for masking).
 * Uses a library-owned workspace (the launch's work counter and status
 * word) per CUDA context and stream, allocated (256 bytes) on the first
 * launch on that stream and kept until the process exits: launches on
 * different streams may run concurrently; launches on one stream run in
 * stream order.
 * ---------------------------------------------------------------------- */
int f3s_1tb1rw_launch(const void* Q, const void* K, const void* V, float* O_out,
                      const int32_t* window_offsets, const int32_t* block_col_indices,
                      const int32_t* window_order, int32_t num_row_windows, int32_t feat_dim,
                      f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * fp32 -> fp16 (round to nearest even), n elements
 * (tests/test_fused_3s_v2.cu:61-64).
 * ---------------------------------------------------------------------- */
int f3s_half_from_float(const float* d_in, void* d_out, int64_t n, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Throughput of mma.sync.m16n8k16 (f16 x f16 -> f32), the tensor-core
 * instruction of the fused kernel, on the current device: one CTA of
 * warps_per_sm warps per SM, each warp running 8 independent accumulator
 * chains for iters iterations; writes TFLOP/s to *h_tflops (synchronises
 * `stream`).  The tensor-side roofline denominator of the fused kernel (no
 * reference counterpart).
 * ---------------------------------------------------------------------- */
int f3s_probe_mma_sync(int32_t warps_per_sm, int32_t iters, double* h_tflops, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Self-test of the failure path: launches a kernel that waits on an
 * mbarrier nobody arrives on, with the given bound.  The wait gives up,
 * records F3S_ERR_TIMEOUT in the workspace and the kernel returns normally;
 * read it with f3s_workspace_status().  No fault, trap or hang.
 * ---------------------------------------------------------------------- */
int f3s_selftest_wait_timeout(uint64_t timeout_ns, void* d_workspace, size_t workspace_bytes,
                              f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Decimal text -> int32 on the GPU (the reference reads row_ptr.txt and
 * col_idx.txt with std::ifstream >>, include/utils.cuh:26-40; here the file
 * bytes are copied to the device as they are and decoded there).
 *
 * d_text: n_bytes of whitespace-separated integers (space, tab, CR, LF;
 * optional sign).  Writes the numbers in order to d_out[0 .. *h_count) and
 * synchronises the stream.  Errors: F3S_ERR_INVALID_VALUE for any other
 * byte or a malformed number, F3S_ERR_TOO_LARGE for a value outside int32 or
 * n_bytes >= 2^31 - 1 (split larger files at a separator), F3S_ERR_WORKSPACE
 * when the text holds more than max_count numbers.
 * ---------------------------------------------------------------------- */
size_t f3s_parse_int32_workspace_size(int64_t n_bytes);
int f3s_parse_int32(const char* d_text, int64_t n_bytes, int32_t* d_out, int64_t max_count, int64_t* h_count,
                    void* d_workspace, size_t workspace_bytes, f3s_stream_t stream);

/* ------------------------------------------------------------------------
 * Peer buffers for exchanging O between the ranks of a sharded forward (no
 * reference counterpart: the reference runs on one GPU).
 *
 * f3s_peer_alloc allocates `bytes` of device memory on the current device
 * and writes its CUDA IPC handle (F3S_IPC_HANDLE_BYTES bytes) to
 * ipc_handle; another process on the box passes the handle to
 * f3s_peer_open to map the buffer (peer access enabled over NVLink), and
 * unmaps it with f3s_peer_close before the owner calls f3s_peer_free.
 * f3s_peer_copy is a stream-ordered copy between any two device pointers
 * (local or mapped): it runs on a copy engine, so it overlaps kernels that
 * hold every SM.  Copies into another rank's buffer are complete when the
 * copying stream passes them; a stream-ordered collective after them tells
 * the owner.
 * ---------------------------------------------------------------------- */
#define F3S_IPC_HANDLE_BYTES 64
int f3s_peer_alloc(size_t bytes, void** d_ptr, void* ipc_handle);
int f3s_peer_open(const void* ipc_handle, void** d_ptr);
int f3s_peer_close(void* d_ptr);
int f3s_peer_free(void* d_ptr);
int f3s_peer_copy(void* d_dst, const void* d_src, size_t bytes, f3s_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FUSED3S_H_ */
