// f3s_forward.cu -- fused SDDMM + online softmax + SpMM over 16x16 block-sparse
// row windows, for sm_100a.
//
// Semantics: tests/test_fused_3s_v2.cu:17-59 (block semantics: every column
// of every active block of the row's window is scored; columns >= N are
// masked), computed the way src/fused3s_v2.cu:81-246 does (fp16 Q/K/V, fp32
// scores, online softmax with fp32 running max / sum, P rounded to fp16 for
// P.V, fp32 accumulation, fp32 O).
//
// Design (B200-first, not a translation of the v2 kernel):
//   * Persistent CTAs, one per SM, pull work items (window, head-group) from a
//     device-wide ticket counter in the caller's workspace, in the order given
//     by `order` (descending workload), so heavy windows start first and the
//     tail balances itself.
//   * Memory layout is node-major [N, H, d] fp16.  A CTA takes HG heads of a
//     window at once, so one active block's K (or V) tile is 16 * HG * d * 2
//     contiguous bytes in HBM.  It is fetched with at most two TMA boxes of
//     a 3-D tensor map {64 elems, head-chunk, node} (strides grow with the
//     dimension, as the driver documents; 128-byte swizzle): one of HA
//     head-chunks, HA odd, and one of the remaining chunk.  In shared memory
//     the tile is node-major with a node stride of HA * 128 B, an odd
//     multiple of the swizzle row, so ldmatrix reads are conflict-free
//     (chunk_row()).  Up to 32 blocks are issued per round, one per lane of
//     the producer warp; each lane issues its block's K and V boxes.
//   * L2 eviction priority per load: Q tiles (read once) evict-first; K/V
//     tiles by the caller's per-block hint, the hint of the block's column
//     (popular columns evict-last, columns used by one window evict-first).
//   * Warp specialisation: warp 8 is the producer (ticket fetch, window
//     metadata, block-column list read 32 at a time, TMA issue into a ring of
//     STAGES K/V stages guarded by full/empty mbarriers); warps 0-7 consume.
//     Consumer warp (hh, sp) owns head hh of the group and the blocks whose
//     global issue index is sp mod SPLITS (SPLITS = 8 / HG), each split with
//     its own sub-ring of stages; partial (m, l, O) of the splits are merged
//     through shared memory at the end of the window.
//   * Per block and head: S = Q K^T with mma.sync m16n8k16 (Q fragments stay
//     in registers for the whole window), row max / sum with quad shuffles,
//     exp2 on the MUFU, P packed to fp16 straight from the accumulator
//     fragments into the A operand of O += P V (V via ldmatrix.trans).
//     16-wide contractions are too narrow for tcgen05's M >= 64 tiles without
//     packing unrelated windows; at 16 flop/byte the kernel is HBM-bound and
//     the warp-level tensor path is not the limiter.
//   * Every mbarrier wait is bounded (global timer) and aborts the CTA with a
//     status word in the workspace instead of hanging.
#include <algorithm>
#include <mutex>
#include <type_traits>
#include <vector>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include "f3s_internal.cuh"

namespace f3s {

// Consumer warps per CTA (plus one producer warp): 8 -- one per head of an
// 8-head group, or SPLITS = 8 / HG per head.  F3S_WIDE_CONSUMERS builds the
// d = 64, 8-head variant with 16 consumer warps (two per head, alternate
// blocks) for comparison.
constexpr int kConsumerWarps = 8;
template <int D, int HG>
constexpr int consumer_warps() {
#ifdef F3S_WIDE_CONSUMERS
    return D == 64 && HG == 8 ? 16 : kConsumerWarps;
#else
    return kConsumerWarps;
#endif
}
constexpr int kSmemBudget = 227 * 1024;
constexpr uint64_t kWaitTimeoutNs = 10ull * 1000 * 1000 * 1000;  // 10 s: far above any legal wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyLog2 = 8.0f;  // running-max slack before an O rescale (p <= 256)

template <int D, int HG>
struct FwdCfg {
    static constexpr int CW = consumer_warps<D, HG>();  // consumer warps
    static constexpr int THREADS = (CW + 1) * 32;
    static constexpr int SPLITS = CW / HG;
    static constexpr int HC = HG * D / 64;           // 128-byte head-chunks per node in one tile
    // A tile arrives as two TMA boxes of HA and HB head-chunks (HA odd,
    // HB = 0 or 1), node-major in shared memory: see chunk_row().
    static constexpr int HA = (HC % 2 == 0) ? HC - 1 : HC;
    static constexpr int HB = HC - HA;
    static constexpr int NBOX = HB ? 2 : 1;
    static constexpr int TILE = 16 * HG * D * 2;     // bytes of one Q, K or V tile
    static constexpr int SLOT_F = 16 * D + 64;       // floats per merge slot (O partial + m/l)
    static constexpr int MERGE = (SPLITS - 1) * HG * SLOT_F * 4;
    // Q double buffer + merge area + barriers/metadata (<= 1 KB for <= 32
    // stages) + 1 KB slack for aligning the dynamic shared memory base
    static constexpr int FIXED = 2 * TILE + MERGE + 1024 + 1024;
    static constexpr int STAGES_FIT = (kSmemBudget - FIXED) / (2 * TILE);
    // Each split owns a sub-ring of S_SUB stages: block j of a window goes to
    // split j % SPLITS, and a split's l-th block (counted over its windows)
    // to slot l % S_SUB of its sub-ring.  Every stage is then consumed by one
    // split, strictly in order, so a waiter is never two phases ahead of a
    // stage (the mbarrier parity would alias).
    static constexpr int S_SUB = (STAGES_FIT > 32 ? 32 : STAGES_FIT) / SPLITS;
    static constexpr int STAGES = S_SUB * SPLITS;
    static_assert(S_SUB >= 2, "need at least two stages per split");
    // Blocks a consumer warp takes per step (one max update and one vote per
    // step; their QK^T / exp / P.V chains interleave).  A step holds NB
    // stages of the split's sub-ring until its end, so NB leaves stages for
    // the producer to keep loading.  Measured on B200 (C1 / C3 / c4s / C4):
    // 2 is fastest; 3 ties; 4 is slower; issuing the next step's QK^T before
    // this step's softmax (two steps in flight) was slower too.
#ifndef F3S_BLOCKS_PER_STEP
#define F3S_BLOCKS_PER_STEP 2
#endif
    static constexpr int NB_WANT = D == 64 ? F3S_BLOCKS_PER_STEP : 2;
    static constexpr int NB_ROOM = S_SUB - 2 > 1 ? S_SUB - 2 : 1;  // keep two stages loading if possible
    static constexpr int NB = NB_WANT < NB_ROOM ? NB_WANT : NB_ROOM;
    static_assert(NB >= 1 && NB < S_SUB, "a step must leave the producer a stage");
    // blocks the producer issues per round (one per lane); a multiple of
    // SPLITS that divides 32, and at most STAGES
    static constexpr int ISSUE_W = STAGES >= 32 ? 32 : (STAGES >= 16 ? 16 : (STAGES >= 8 ? 8 : (STAGES >= 4 ? 4 : 2)));
    static_assert(ISSUE_W % SPLITS == 0 && ISSUE_W <= STAGES, "issue width");
    static constexpr int Q_OFF = 0;
    static constexpr int KV_OFF = 2 * TILE;
    static constexpr int MERGE_OFF = KV_OFF + STAGES * 2 * TILE;
    static constexpr int BAR_OFF = MERGE_OFF + MERGE;
    static constexpr int NBARS = 2 * STAGES + 6;
    static constexpr int META_OFF = BAR_OFF + NBARS * 8;
    static constexpr int WINFO_OFF = (META_OFF + STAGES * 4 + 15) / 16 * 16;
    static constexpr int SINK_OFF = WINFO_OFF + 4 * 16;  // one word per consumer warp, written, never read
    static constexpr int SMEM = SINK_OFF + CW * 4 + 1024;  // + slack to align the base to 1 KB
    static_assert(STAGES >= 2, "need at least two K/V stages");
    static_assert(SMEM <= kSmemBudget, "shared memory budget");
    static_assert(D % 64 == 0, "head_dim must be a multiple of 64");
};

// ---------------------------------------------------------------- plans --
// A plan cuts every window with more than T active blocks into pieces of at
// most T consecutive blocks so that one heavy window spreads over many SMs.
// Each piece is a work item; a piece of a split window writes its partial
// (running max m, sum l, unnormalised O) for its 16 rows and HG heads into
// the plan's scratch, and k_merge_pieces combines the pieces of each window
// in piece order (deterministic) and writes O.
struct PlanHeader {
    int num_pieces;        // work items (pieces) in the plan
    int num_split;         // windows that were split
    int num_split_pieces;  // pieces of split windows (partial slots used)
    int max_pieces, max_split, max_split_pieces;
    int max_blocks;        // T
    int heads, head_dim, groups, hg;
    int status;            // 0, or an f3s_status if the plan overflowed
    long long splits_off;  // byte offsets of the sections; pieces follow the header
    long long partials_off;
    long long states_off;  // sweep plans: one running (m, l, O) state per window and head
    int mode;              // kPlanPieces, or kPlanSweep
    int pad[45];
};
static_assert(sizeof(PlanHeader) == 256, "plan header is 256 bytes");

// Plan modes.  0 (make_plan / load_plan): a split window's pieces write
// partial states into their own slots, merged after the kernel
// (k_merge_pieces).  kPlanSweep: a window's pieces run one after another
// (each waits for the previous one), carrying one running state per window
// and head: a piece loads it, folds in its own blocks and stores it back; the
// last writes O.
constexpr int kPlanSweep = 1;
// piece info of a sweep plan: index of the piece within its window, and a
// flag for the window's last piece
constexpr int kSweepLast = 1 << 30;
constexpr int kSweepIndexMask = kSweepLast - 1;

struct FwdParams {
    void* O;            // [q_rows, H, D] of o_dtype
    const int* offsets;
    const int* cols;
    const int* order;
    PlanHeader* plan;          // plan (device), or null: one work item per entry of `order`
    WsHeader* hdr;
    uint64_t timeout_ns;
    int num_items;      // entries of `order`
    int groups;         // head groups per window (heads / HG)
    int num_nodes;      // N (rows of K and V)
    int nrw_total;      // ceil(N / 16)
    int heads;          // H
    int q_window_base;  // first window of the Q / O slab
    int q_windows;      // windows in the slab
    int q_rows;         // rows of the Q / O slab
    int tail;           // N % 16 (0: no masked column)
    const uint8_t* hints;  // per block L2 hint (1 keep, 2 stream, else normal) or null
    int o_dtype;           // f3s_out_dtype of O
    int piece_begin;       // with a plan: first piece of this launch
    int piece_end;         // with a plan: end of the launch's pieces, or -1 for all
    int kv_col_base;       // first block column held in K / V (row 16 * kv_col_base of the graph)
    int kv_cols;           // block columns held in K / V
    int* seq;              // sweep plans: per window and head, pieces of the window done this launch
    long long seq_cap;     // entries of seq
};

// O stores: fp32 as computed, or rounded to nearest into fp16 / bf16.
// Streaming stores (O is written once).  idx is an element index; pairs
// start at even, quads at multiples of 4 (aligned for every type).
__device__ __forceinline__ void store_o2(void* O, int64_t idx, float a, float b, int dt) {
    if (dt == F3S_OUT_F16) {
        const __half2 v = __floats2half2_rn(a, b);
        __stcs(reinterpret_cast<unsigned int*>(static_cast<__half*>(O) + idx), *reinterpret_cast<const unsigned int*>(&v));
    } else if (dt == F3S_OUT_BF16) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        __stcs(reinterpret_cast<unsigned int*>(static_cast<__nv_bfloat16*>(O) + idx),
               *reinterpret_cast<const unsigned int*>(&v));
    } else {
        __stcs(reinterpret_cast<float2*>(static_cast<float*>(O) + idx), make_float2(a, b));
    }
}

__device__ __forceinline__ void store_o4(void* O, int64_t idx, float4 v, int dt) {
    if (dt == F3S_OUT_F32) {
        __stcs(reinterpret_cast<float4*>(static_cast<float*>(O) + idx), v);
        return;
    }
    uint2 w;
    if (dt == F3S_OUT_F16) {
        const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        w = make_uint2(*reinterpret_cast<const unsigned int*>(&a), *reinterpret_cast<const unsigned int*>(&b));
        __stcs(reinterpret_cast<uint2*>(static_cast<__half*>(O) + idx), w);
    } else {
        const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        w = make_uint2(*reinterpret_cast<const unsigned int*>(&a), *reinterpret_cast<const unsigned int*>(&b));
        __stcs(reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(O) + idx), w);
    }
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, const ErrorSink& e, uint64_t tmo) {
    bool ok = mbar_wait_bounded(bar, parity, e, tmo);
    return __all_sync(0xffffffffu, ok);
}

// Inline fast path: one try_wait per lane and a vote; the bounded slow path
// only when the phase is not complete yet.
__device__ __forceinline__ bool wait_fast(uint32_t bar, uint32_t parity, const ErrorSink& e, uint64_t tmo) {
    const bool ready = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ready)) return true;
    return wait_warp(bar, parity, e, tmo);
}

// Tensor maps of Q, K and V: 3-D {64 elems, head-chunk, node} views with a
// box of HA head-chunks (a) and one of a single head-chunk (b).
struct FwdMaps {
    CUtensorMap qa, qb, ka, kb, va, vb;
};

// Shared-memory row (128-byte unit) of head-chunk hc of node n in a tile.
// Box a holds head-chunks [0, HA) node-major (row n*HA + hc), box b the last
// one (row 16*HA + n).  HA is odd, so the 8 nodes an ldmatrix phase reads
// from one head-chunk fall on 8 different 128-byte swizzle rows
// ((n*HA + hc) mod 8 are distinct): conflict-free.
template <int HA>
__device__ __forceinline__ uint32_t chunk_row(int hc, int n) {
    return hc < HA ? (uint32_t)(n * HA + hc) : (uint32_t)(16 * HA + n);
}

template <int D, int HG>
__global__ void __launch_bounds__(FwdCfg<D, HG>::THREADS, 1)
    k_fused3s(const __grid_constant__ FwdMaps maps, const FwdParams p) {
    using C = FwdCfg<D, HG>;
    constexpr int S = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* sp8 = smem_raw + (sbase - raw);
    const uint32_t q_s = sbase + C::Q_OFF;
    const uint32_t kv_s = sbase + C::KV_OFF;
    float* merge = reinterpret_cast<float*>(sp8 + C::MERGE_OFF);
    const uint32_t bar0 = sbase + C::BAR_OFF;
    int* stage_col = reinterpret_cast<int*>(sp8 + C::META_OFF);
    int4* winfo = reinterpret_cast<int4*>(sp8 + C::WINFO_OFF);
    const uint32_t sink_s = sbase + C::SINK_OFF;
    auto full = [&](uint32_t s) { return bar0 + 8u * s; };
    auto empty = [&](uint32_t s) { return bar0 + 8u * (S + s); };
    auto qfull = [&](uint32_t q) { return bar0 + 8u * (2 * S + q); };
    auto qempty = [&](uint32_t q) { return bar0 + 8u * (2 * S + 2 + q); };
    const uint32_t mfull = bar0 + 8u * (2 * S + 4);
    const uint32_t mempty = bar0 + 8u * (2 * S + 5);
    // Block j of a window belongs to split j % SPLITS; a split's l-th block
    // (counted over all its windows) uses slot l % S_SUB of its sub-ring, in
    // phase l / S_SUB.
    auto slot_of = [](uint32_t sp, uint32_t l) -> uint32_t { return sp * C::S_SUB + l % C::S_SUB; };
    auto par_of = [](uint32_t l) -> uint32_t { return (l / C::S_SUB) & 1u; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const ErrorSink err{&p.hdr->abort, &p.hdr->status};

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), HG);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(qfull(q), 1);
            mbar_init(qempty(q), C::CW);
        }
        mbar_init(mfull, C::SPLITS > 1 ? (C::SPLITS - 1) * HG : 1);
        mbar_init(mempty, HG);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == C::CW) {
        // ------------------------------------------------------ producer --
        // The whole warp runs this loop.  A block's K and V tiles are NBOX
        // boxes each, issued by the lane that claimed the block (rounds of
        // up to ISSUE_W blocks below); lanes [0, NBOX) issue a window's Q
        // boxes.
        if (lane == 0) {
            tma_prefetch_desc(&maps.qa);
            tma_prefetch_desc(&maps.qb);
            tma_prefetch_desc(&maps.ka);
            tma_prefetch_desc(&maps.kb);
            tma_prefetch_desc(&maps.va);
            tma_prefetch_desc(&maps.vb);
        }
        const uint64_t pol_first = l2_policy_evict_first();
        const uint64_t pol_normal = l2_policy_evict_normal();
        const uint64_t pol_last = l2_policy_evict_last();
        const int b_total = __ldg(p.offsets + p.nrw_total);
        int n_units = p.num_items;
        const int4* pieces = nullptr;  // plan pieces (w, b0, b1, partial slot or -1)
        if (p.plan != nullptr) {
            // this launch's range of the plan's pieces
            const int np_all = p.plan->num_pieces;
            const int pe = p.piece_end < 0 ? np_all : p.piece_end;
            pieces = reinterpret_cast<const int4*>(p.plan + 1) + p.piece_begin;
            n_units = pe - p.piece_begin;
            if (p.plan->status != 0 || p.plan->heads != p.heads || p.plan->head_dim != D || pe > np_all ||
                n_units < 0) {
                if (lane == 0) raise_error(err, F3S_ERR_BAD_FORMAT);
                n_units = 0;
            }
        }
        const int total = n_units * p.groups;
        const int bi = lane % C::NBOX;  // box of this lane: 0 = a (HA chunks), 1 = b (last chunk)
        const CUtensorMap* tq = bi ? &maps.qb : &maps.qa;
        const uint32_t box_off = bi ? (uint32_t)(C::HA * 2048) : 0u;  // 16 nodes x HA x 128 B
        const int box_hc = bi ? C::HA : 0;
        uint32_t cnt[C::SPLITS];  // blocks issued per split
#pragma unroll
        for (int t = 0; t < C::SPLITS; ++t) cnt[t] = 0;
        int k = 0;        // windows published
        bool aborted = false;
        // Work tickets and window descriptors run one item ahead, and the
        // next item's first 32 block columns (with their block hints) load
        // while this item issues: an item's first TMA never waits on a chain
        // of global loads.  (Tickets two items ahead read 4-5 % more DRAM at
        // C4 with no gain at C1.)
        auto fetch = [&](int t) -> int4 {  // (window, b0, b1, partial slot); window -1 past the end
            if (t >= total) return make_int4(-1, 0, 0, -1);
            const int unit = t / p.groups;
            if (pieces != nullptr) return __ldg(pieces + unit);
            const int wd = __ldg(p.order + unit);
            if (wd < 0 || wd >= p.nrw_total) return make_int4(wd, 0, 0, -1);
            return make_int4(wd, __ldg(p.offsets + wd), __ldg(p.offsets + wd + 1), -1);
        };
        auto first_chunk = [&](const int4& dd, int& c, int& h) {
            const bool ok = dd.x >= 0 && dd.y >= 0 && dd.z <= b_total && dd.y + lane < dd.z;
            c = ok ? __ldg(p.cols + dd.y + lane) : 0;
            h = (ok && p.hints != nullptr) ? (int)__ldg(p.hints + dd.y + lane) : 0;
        };
        int t0 = 0, t1 = 0;
        if (lane == 0) {
            t0 = atomicAdd(&p.hdr->counter, 1);
            t1 = atomicAdd(&p.hdr->counter, 1);
        }
        t0 = __shfl_sync(0xffffffffu, t0, 0);
        t1 = __shfl_sync(0xffffffffu, t1, 0);
        int4 d0 = fetch(t0), d1 = fetch(t1);
        int c0 = 0, h0 = 0;
        first_chunk(d0, c0, h0);
        for (;;) {
            const bool end = t0 >= total;
            int w = -1, g = 0, b0 = 0, b1 = 0, pslot = -1;
            int t2 = total;
            int c1 = 0, h1 = 0;
            if (!end) {
                if (lane == 0 && t1 < total) t2 = atomicAdd(&p.hdr->counter, 1);
                first_chunk(d1, c1, h1);
                g = t0 - (t0 / p.groups) * p.groups;
                w = d0.x;
                b0 = d0.y;
                b1 = d0.z;
                pslot = d0.w;
                if (w < p.q_window_base || w >= p.q_window_base + p.q_windows || b0 < 0 || b1 < b0 ||
                    b1 > b_total) {
                    if (lane == 0) raise_error(err, F3S_ERR_BAD_FORMAT);
                    aborted = true;
                    break;
                }
            }
            const int q = k & 1;
            if (!wait_fast(qempty(q), ((k >> 1) & 1) ^ 1, err, p.timeout_ns)) {
                aborted = true;
                break;
            }
            const int z0 = g * C::HC;
            if (lane == 0) {
                if (end) {
                    winfo[2 * q] = make_int4(-1, 0, 0, 0);
                    mbar_arrive(qfull(q));
                } else {
                    winfo[2 * q] = make_int4(w, g, b0, b1);
                    winfo[2 * q + 1] = make_int4(pslot, 0, 0, 0);
                    if (b1 > b0)
                        mbar_arrive_expect_tx(qfull(q), C::TILE);
                    else
                        mbar_arrive(qfull(q));
                }
            }
            if (end) break;
            __syncwarp();
            if (b1 > b0 && lane < C::NBOX)
                tma_load_3d_hint(q_s + q * C::TILE + box_off, tq, qfull(q), 0, z0 + box_hc,
                                 16 * (w - p.q_window_base), pol_first);
            ++k;
            int myc = c0, myh = h0;
            for (int base = b0; base < b1; base += 32) {
                const int n = min(32, b1 - base);
                // next chunk of the block list, in flight while this one issues
                const int nbase = base + 32;
                const bool more = nbase + lane < b1;
                const int nc = more ? __ldg(p.cols + nbase + lane) : 0;
                const int nh = (more && p.hints != nullptr) ? (int)__ldg(p.hints + nbase + lane) : 0;
                // every block column must lie in the K / V rows this launch holds
                if (__any_sync(0xffffffffu, lane < n && (myc < p.kv_col_base || myc - p.kv_col_base >= p.kv_cols))) {
                    if (lane == 0) raise_error(err, F3S_ERR_BAD_FORMAT);
                    aborted = true;
                    break;
                }
                // Up to W blocks per round, one per lane: each lane claims its
                // block's stage (split lane % SPLITS, that split's next slots
                // in lane order) and issues the block's K and V boxes as soon
                // as its own stage is free, so the ring stays as full as with
                // one block at a time while the issues overlap.  W <= STAGES:
                // no lane waits on a stage filled in the same round.
                for (int sub = 0; sub < n; sub += C::ISSUE_W) {
                    const int m = min(C::ISSUE_W, n - sub);
                    const bool act = lane < m;
                    const int c = __shfl_sync(0xffffffffu, myc, (sub + lane) & 31);
                    const int h = __shfl_sync(0xffffffffu, myh, (sub + lane) & 31);
                    const int bsp = lane % C::SPLITS;  // base - b0 and sub are multiples of SPLITS
                    uint32_t l = 0;
#pragma unroll
                    for (int t = 0; t < C::SPLITS; ++t)
                        if (t == bsp) l = cnt[t];
                    l += (uint32_t)(lane / C::SPLITS);
                    const uint32_t s = slot_of(bsp, l);
                    const uint32_t par = par_of(l) ^ 1u;
                    const uint64_t pol = h == 1 ? pol_last : (h == 2 ? pol_first : pol_normal);
                    const int kr = 16 * (c - p.kv_col_base);  // first row of the block in K / V
                    auto issue = [&]() {
                        stage_col[s] = c;
                        mbar_arrive_expect_tx(full(s), 2 * C::TILE);
                        const uint32_t dst = kv_s + s * 2 * C::TILE;
                        tma_load_3d_hint(dst, &maps.ka, full(s), 0, z0, kr, pol);
                        tma_load_3d_hint(dst + C::TILE, &maps.va, full(s), 0, z0, kr, pol);
                        if constexpr (C::NBOX == 2) {
                            tma_load_3d_hint(dst + C::HA * 2048, &maps.kb, full(s), 0, z0 + C::HA, kr, pol);
                            tma_load_3d_hint(dst + C::TILE + C::HA * 2048, &maps.vb, full(s), 0, z0 + C::HA, kr,
                                             pol);
                        }
                    };
                    bool issued = !act;
                    if (act && mbar_try_wait(empty(s), par)) {
                        issue();
                        issued = true;
                    }
                    if (!__all_sync(0xffffffffu, issued)) {
                        // bounded retry loop, uniform over the warp
                        const uint64_t t_start = global_timer_ns();
                        for (int spin = 1;; ++spin) {
                            if (!issued && mbar_try_wait(empty(s), par)) {
                                issue();
                                issued = true;
                            }
                            if (__all_sync(0xffffffffu, issued)) break;
                            if ((spin & 15) == 0) {
                                bool stop = __any_sync(0xffffffffu, load_volatile(err.abort) != 0);
                                if (!stop && global_timer_ns() - t_start > p.timeout_ns) {
                                    if (lane == 0) raise_error(err, F3S_ERR_TIMEOUT);
                                    stop = true;
                                }
                                if (__any_sync(0xffffffffu, stop)) {
                                    aborted = true;
                                    break;
                                }
                            }
                        }
                    }
                    // a split's stages free in slot order, so its issued lanes
                    // are a prefix: the counts stay exact even on abort
                    const uint32_t done = __ballot_sync(0xffffffffu, issued && act);
#pragma unroll
                    for (int t = 0; t < C::SPLITS; ++t) {
                        uint32_t mask_t = 0;
#pragma unroll
                        for (int j = t; j < 32; j += C::SPLITS) mask_t |= 1u << j;
                        cnt[t] += (uint32_t)__popc(done & mask_t);
                    }
                    if (aborted) break;
                }
                if (aborted) break;
                myc = nc;
                myh = nh;
            }
            if (aborted) break;
            t0 = t1;
            t1 = __shfl_sync(0xffffffffu, t2, 0);
            d0 = d1;
            d1 = fetch(t1);
            c0 = c1;
            h0 = h1;
        }
        if (aborted && lane == 0) {
            // let this CTA's own bulk copies land before it exits
#pragma unroll
            for (int t = 0; t < C::SPLITS; ++t) {
                const uint32_t n = cnt[t] < (uint32_t)C::S_SUB ? cnt[t] : (uint32_t)C::S_SUB;
                for (uint32_t l = cnt[t] - n; l < cnt[t]; ++l) mbar_drain(full(slot_of(t, l)), par_of(l), 100000000ull);
            }
            for (int kk = k > 2 ? k - 2 : 0; kk < k; ++kk) mbar_drain(qfull(kk & 1), (kk >> 1) & 1, 100000000ull);
        }
        return;
    }

    // ---------------------------------------------------------- consumers --
    const int hh = warp % HG;
    const int sp = warp / HG;
    const int g4 = lane >> 2, t4 = lane & 3;
    const int a_row = (lane & 7) + (((lane >> 3) & 1) << 3);  // ldmatrix rows for Q (A) and V (B, trans)
    const int a_chk = lane >> 4;
    const int b_row = (lane & 7) + ((lane >> 4) << 3);  // ldmatrix rows for K (B)
    const int b_chk = (lane >> 3) & 1;
    constexpr int KS = D / 16;  // k-steps of QK^T, and 16-column pairs of PV
    constexpr int NT = D / 8;   // n-tiles of the O accumulator
    // Per-lane shared-memory offsets of this warp's head inside a tile, per
    // 16-wide k-step: ldmatrix rows of K (B operand of Q K^T) and of V (B
    // operand of P V, transposed), computed once.
    // (The wide variant, with fewer registers per thread, recomputes them.)
    constexpr bool HOIST = C::CW == kConsumerWarps;
    uint32_t offk[HOIST ? KS : 1], offv[HOIST ? KS : 1];
    auto koff = [&](int ks) -> uint32_t {
        return swz128(chunk_row<C::HA>(hh * (D / 64) + ks / 4, b_row), (ks & 3) * 2 + b_chk);
    };
    auto voff = [&](int ks) -> uint32_t {
        return swz128(chunk_row<C::HA>(hh * (D / 64) + ks / 4, a_row), (ks & 3) * 2 + a_chk);
    };
    if constexpr (HOIST) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            offk[ks] = koff(ks);
            offv[ks] = voff(ks);
        }
    }
    // position of this split's next block in its sub-ring (slot l % S_SUB
    // and phase parity (l / S_SUB) & 1 of its l-th block over all windows)
    uint32_t ring_pos = 0, ring_par = 0;
    const bool sweep = p.plan != nullptr && p.plan->mode == kPlanSweep;
    constexpr int SE = NT * 4 + 4;  // floats of one lane's running state (O fragments, m0, l0, m1, l1)
    for (int k = 0;; ++k) {
        const int q = k & 1;
        if (!wait_warp(qfull(q), (k >> 1) & 1, err, p.timeout_ns)) return;
        const int4 wi = winfo[2 * q];
        const int pslot = winfo[2 * q + 1].x;
        if (wi.x < 0) return;
        const int w = wi.x, g = wi.y, nb = wi.w - wi.z;
        uint32_t qa[KS][4];
        uint32_t qdep = 0;
        if (nb > 0) {
            const uint32_t qt = q_s + q * C::TILE;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const uint32_t row = chunk_row<C::HA>(hh * (D / 64) + ks / 4, a_row);
                ldsm_x4(qt + swz128(row, (ks & 3) * 2 + a_chk), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) qdep ^= qa[ks][0] ^ qa[ks][1] ^ qa[ks][2] ^ qa[ks][3];
        }
        // Free the Q slot only once the fragments are in registers: the
        // arrive follows a store of a value computed from them.  An arrive issued right
        // after the ldmatrix instructions let the producer's next Q copy into
        // this slot race with them (rows of a warp's Q were seen to change in
        // sweep plans, where a warp that waited on its flag is the last to
        // arrive and the producer is already waiting).
        __syncwarp();
        if (lane == 0) mbar_arrive_after(qempty(q), sink_s + 4u * (uint32_t)warp, qdep);

        float o[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        // Running row max m (log2 units) and sum l.  The max moves lazily:
        // only when a row's block max exceeds it by more than kLazyLog2, so
        // most blocks skip the O rescale; p = 2^(s*log2e - m) <= 2^kLazyLog2
        // stays well inside fp16, and O / l is unchanged because both use
        // the same m.
        float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
        bool ok = true;
        auto qk_tile = [&](uint32_t kt, float (&sc)[2][4]) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t k0, k1, k2, k3;
                uint32_t ko;
                if constexpr (HOIST) ko = offk[ks]; else ko = koff(ks);
                ldsm_x4(kt + ko, k0, k1, k2, k3);
                if (ks == 0) {
                    mma_16816_zero(sc[0], qa[ks], k0, k1);
                    mma_16816_zero(sc[1], qa[ks], k2, k3);
                } else {
                    mma_16816(sc[0], qa[ks], k0, k1);
                    mma_16816(sc[1], qa[ks], k2, k3);
                }
            }
        };
        auto mask_tail = [&](float (&sc)[2][4], int col) {
            if (col == p.nrw_total - 1) {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (nt * 8 + 2 * t4 + (i & 1) >= p.tail) sc[nt][i] = -INFINITY;
            }
        };
        auto pv_tile = [&](uint32_t vt, const uint32_t (&pa)[4]) {
#pragma unroll
            for (int jj = 0; jj < KS; ++jj) {
                uint32_t v0, v1, v2, v3;
                uint32_t vo;
                if constexpr (HOIST) vo = offv[jj]; else vo = voff(jj);
                ldsm_x4_t(vt + vo, v0, v1, v2, v3);
                mma_16816(o[2 * jj], pa, v0, v1);
                mma_16816(o[2 * jj + 1], pa, v2, v3);
            }
        };
        // NB blocks per step (this split's next NB blocks of the window, j,
        // j + SPLITS, ...; the blocks j = sp, sp + SPLITS, ... are its next
        // blocks in the sub-ring, in order): their QK^T, exp and P.V chains
        // interleave, and one max update / rescale covers 16 * NB columns.
        constexpr int NB = C::NB;
        struct Step {
            float sc[NB][2][4];
            uint32_t st[NB];
            int n;  // blocks in the step (0: past the window's end)
        };
        // Waits for the step's stages and issues its QK^T: all NB blocks when
        // `whole` is std::true_type (the common case, without per-block
        // tests), else the split's remaining blocks of the window (< NB).
        auto fetch = [&](Step& S, int j, auto whole) -> bool {
            constexpr bool FULL = decltype(whole)::value;
            if constexpr (FULL) {
                S.n = NB;
            } else {
                S.n = (nb - 1 - j) / C::SPLITS + 1;  // this split's blocks from j on, warp-uniform
            }
            uint32_t ph[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                S.st[b] = sp * C::S_SUB + ring_pos;
                ph[b] = ring_par;
                if ((FULL || b < S.n) && ++ring_pos == (uint32_t)C::S_SUB) {
                    ring_pos = 0;
                    ring_par ^= 1u;
                }
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (FULL || b < S.n) {
                    if (!wait_fast(full(S.st[b]), ph[b], err, p.timeout_ns)) return false;
                    qk_tile(kv_s + S.st[b] * 2 * C::TILE, S.sc[b]);
                    if (p.tail != 0) mask_tail(S.sc[b], stage_col[S.st[b]]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) S.sc[b][0][i] = S.sc[b][1][i] = -INFINITY;
                }
            }
            return true;
        };
        // Softmax update and P.V of a fetched step; frees its stages.
        auto process = [&](Step& S, auto whole) {
            constexpr bool FULL = decltype(whole)::value;
            float mx0 = fmaxf(fmaxf(S.sc[0][0][0], S.sc[0][0][1]), fmaxf(S.sc[0][1][0], S.sc[0][1][1]));
            float mx1 = fmaxf(fmaxf(S.sc[0][0][2], S.sc[0][0][3]), fmaxf(S.sc[0][1][2], S.sc[0][1][3]));
#pragma unroll
            for (int b = 1; b < NB; ++b) {
                mx0 = fmaxf(mx0, fmaxf(fmaxf(S.sc[b][0][0], S.sc[b][0][1]), fmaxf(S.sc[b][1][0], S.sc[b][1][1])));
                mx1 = fmaxf(mx1, fmaxf(fmaxf(S.sc[b][0][2], S.sc[b][0][3]), fmaxf(S.sc[b][1][2], S.sc[b][1][3])));
            }
            // A row's max exceeds its running max by more than kLazyLog2 iff
            // one of the row's four lanes holds such a value (scaling by
            // log2e is monotonic), so the vote needs no row reduction: the
            // shuffles run only on the rare update, which then applies the
            // row-max rule exactly as before.
            const bool up_lane = mx0 * kLog2e > m0 + kLazyLog2 || mx1 * kLog2e > m1 + kLazyLog2;
            if (__any_sync(0xffffffffu, up_lane)) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2)) * kLog2e;
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2)) * kLog2e;
                const bool up0 = mx0 > m0 + kLazyLog2, up1 = mx1 > m1 + kLazyLog2;
                const float mn0 = up0 ? mx0 : m0, mn1 = up1 ? mx1 : m1;
                const float c0 = fast_exp2(m0 - mn0), c1 = fast_exp2(m1 - mn1);
                l0 *= c0;
                l1 *= c1;
#pragma unroll
                for (int jn = 0; jn < NT; ++jn) {
                    o[jn][0] *= c0;
                    o[jn][1] *= c0;
                    o[jn][2] *= c1;
                    o[jn][3] *= c1;
                }
                m0 = mn0;
                m1 = mn1;
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (FULL || b < S.n) {
                    float pr[2][4];
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        pr[nt][0] = fast_exp2(fmaf(S.sc[b][nt][0], kLog2e, -m0));
                        pr[nt][1] = fast_exp2(fmaf(S.sc[b][nt][1], kLog2e, -m0));
                        pr[nt][2] = fast_exp2(fmaf(S.sc[b][nt][2], kLog2e, -m1));
                        pr[nt][3] = fast_exp2(fmaf(S.sc[b][nt][3], kLog2e, -m1));
                    }
                    l0 += (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
                    l1 += (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
                    uint32_t pa[4];
                    pa[0] = pack_half2(pr[0][0], pr[0][1]);
                    pa[1] = pack_half2(pr[0][2], pr[0][3]);
                    pa[2] = pack_half2(pr[1][0], pr[1][1]);
                    pa[3] = pack_half2(pr[1][2], pr[1][3]);
                    pv_tile(kv_s + S.st[b] * 2 * C::TILE + C::TILE, pa);
                }
            }
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    if (FULL || b < S.n) mbar_arrive(empty(S.st[b]));
            }
        };
        Step A;
        for (int j = sp; j < nb; j += NB * C::SPLITS) {
            if ((nb - 1 - j) / C::SPLITS + 1 >= NB) {
                if (!(ok = fetch(A, j, std::true_type{}))) break;
                process(A, std::true_type{});
            } else {
                if (!(ok = fetch(A, j, std::false_type{}))) break;
                process(A, std::false_type{});
            }
        }
        if (!ok) return;
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

        if constexpr (C::SPLITS > 1) {
            if (sp > 0) {
                if (!wait_warp(mempty, (k & 1) ^ 1, err, p.timeout_ns)) return;
                float* slot = merge + ((sp - 1) * HG + hh) * C::SLOT_F;
#pragma unroll
                for (int r = 0; r < NT * 4; ++r) slot[r * 32 + lane] = o[r >> 2][r & 3];
                if (t4 == 0) {
                    float4 ml = make_float4(m0, l0, m1, l1);
                    *reinterpret_cast<float4*>(slot + 16 * D + g4 * 4) = ml;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(mfull);
                continue;
            }
            if (!wait_warp(mfull, k & 1, err, p.timeout_ns)) return;
#pragma unroll 1
            for (int s2 = 1; s2 < C::SPLITS; ++s2) {
                const float* slot = merge + ((s2 - 1) * HG + hh) * C::SLOT_F;
                const float4 ml = *reinterpret_cast<const float4*>(slot + 16 * D + g4 * 4);
                const float M0 = fmaxf(m0, ml.x), M1 = fmaxf(m1, ml.z);
                const float a0 = fast_exp2(m0 - M0), b0s = fast_exp2(ml.x - M0);
                const float a1 = fast_exp2(m1 - M1), b1s = fast_exp2(ml.z - M1);
                l0 = l0 * a0 + ml.y * b0s;
                l1 = l1 * a1 + ml.w * b1s;
                m0 = M0;
                m1 = M1;
#pragma unroll
                for (int r = 0; r < NT * 4; ++r) {
                    const float other = slot[r * 32 + lane];
                    const bool lo_row = (r & 3) < 2;
                    o[r >> 2][r & 3] = o[r >> 2][r & 3] * (lo_row ? a0 : a1) + other * (lo_row ? b0s : b1s);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(mempty);
        }

        if (sweep) {
            // Sweep plan: the window's running state (this warp's head) is
            // carried from piece to piece.  Piece k > 0 waits for piece k - 1
            // (an earlier ticket, so it is running or done), folds the stored
            // state in with the same max / scale rule as the split merge, and
            // either stores the state back and releases piece k + 1, or, as
            // the last piece, normalises and writes O below.
            const int kpiece = pslot & kSweepIndexMask;
            const bool last = (pslot & kSweepLast) != 0;
            const long long fidx = ((long long)(w - p.q_window_base) * p.groups + g) * HG + hh;
            if (fidx >= p.seq_cap) {
                if (lane == 0) raise_error(err, F3S_ERR_BAD_FORMAT);
                return;
            }
            int* flag = p.seq + fidx;
            float4* st4 = reinterpret_cast<float4*>(reinterpret_cast<char*>(p.plan) + p.plan->states_off) +
                          fidx * (SE / 4) * 32;
            if (kpiece > 0) {
                // Every lane waits on the flag with its own acquire load (one
                // transaction per poll for the warp) and reads the stored
                // state with strong GPU-scope loads, so each lane's reads are
                // ordered after its own acquire, whatever the cache holds.
                if (!__all_sync(0xffffffffu, flag_wait_bounded(flag, kpiece, err, p.timeout_ns))) return;
                const float4 ml = ld_relaxed_gpu_f4(st4 + NT * 32 + lane);  // (m0, l0, m1, l1) of the pieces before
                const float M0 = fmaxf(m0, ml.x), M1 = fmaxf(m1, ml.z);
                const float a0 = fast_exp2(ml.x - M0), b0s = fast_exp2(m0 - M0);
                const float a1 = fast_exp2(ml.z - M1), b1s = fast_exp2(m1 - M1);
                l0 = ml.y * a0 + l0 * b0s;
                l1 = ml.w * a1 + l1 * b1s;
                m0 = M0;
                m1 = M1;
#pragma unroll
                for (int jn = 0; jn < NT; ++jn) {
                    const float4 v = ld_relaxed_gpu_f4(st4 + jn * 32 + lane);
                    o[jn][0] = v.x * a0 + o[jn][0] * b0s;
                    o[jn][1] = v.y * a0 + o[jn][1] * b0s;
                    o[jn][2] = v.z * a1 + o[jn][2] * b1s;
                    o[jn][3] = v.w * a1 + o[jn][3] * b1s;
                }
            }
            if (!last) {
#pragma unroll
                for (int jn = 0; jn < NT; ++jn)
                    __stcs(st4 + jn * 32 + lane, make_float4(o[jn][0], o[jn][1], o[jn][2], o[jn][3]));
                __stcs(st4 + NT * 32 + lane, make_float4(m0, l0, m1, l1));
                __threadfence();  // every lane: its state stores before the release below
                __syncwarp();
                if (lane == 0) st_release_gpu(flag, kpiece + 1);
                continue;
            }
        } else if (pslot >= 0) {
            // piece of a split window: partial (m, l, unnormalised O) of the
            // 16 rows and this warp's head -> plan scratch, merged later
            float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(p.plan) + p.plan->partials_off);
            float* slot = partials + ((size_t)pslot * p.groups + g) * (size_t)(HG * 16 * (D + 2));
            float* op = slot + (size_t)hh * 16 * D + 2 * t4;
#pragma unroll
            for (int jn = 0; jn < NT; ++jn) {
                *reinterpret_cast<float2*>(op + g4 * D + jn * 8) = make_float2(o[jn][0], o[jn][1]);
                *reinterpret_cast<float2*>(op + (g4 + 8) * D + jn * 8) = make_float2(o[jn][2], o[jn][3]);
            }
            if (t4 == 0) {
                float* ml = slot + (size_t)HG * 16 * D + (size_t)hh * 32;
                *reinterpret_cast<float2*>(ml + 2 * g4) = make_float2(m0, l0);
                *reinterpret_cast<float2*>(ml + 2 * (g4 + 8)) = make_float2(m1, l1);
            }
            continue;
        }
        // ------------------------------------------------ normalise, store --
        const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
        const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
        const int h = g * HG + hh;
        const int ra = 16 * w + g4, rb = ra + 8;
        const int64_t sa = (int64_t)(ra - 16 * p.q_window_base), sb = sa + 8;
        if (ra < p.num_nodes && sa < p.q_rows) {
            const int64_t dst = (sa * p.heads + h) * D + 2 * t4;
#pragma unroll
            for (int jn = 0; jn < NT; ++jn) store_o2(p.O, dst + jn * 8, o[jn][0] * inv0, o[jn][1] * inv0, p.o_dtype);
        }
        if (rb < p.num_nodes && sb < p.q_rows) {
            const int64_t dst = (sb * p.heads + h) * D + 2 * t4;
#pragma unroll
            for (int jn = 0; jn < NT; ++jn) store_o2(p.O, dst + jn * 8, o[jn][2] * inv1, o[jn][3] * inv1, p.o_dtype);
        }
    }
}

// ------------------------------------------------------------ plan kernels --

// Per listed window: number of pieces, pieces of split windows, split flag.
__global__ void __launch_bounds__(256) k_plan_count(const int* __restrict__ offsets, const int* __restrict__ order,
                                                    int n, int T, int* __restrict__ npieces, int* __restrict__ nsplitp,
                                                    int* __restrict__ nsplitw) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= n) return;
    const int w = order[i];
    const int nb = offsets[w + 1] - offsets[w];
    const bool split = nb > T;
    const int cnt = split ? (nb + T - 1) / T : 1;
    npieces[i] = cnt;
    nsplitp[i] = split ? cnt : 0;
    nsplitw[i] = split ? 1 : 0;
}

// After the three exclusive scans (totals at index n): write the pieces and
// the split-window records, within the plan's capacities.
__global__ void __launch_bounds__(256) k_plan_fill(const int* __restrict__ offsets, const int* __restrict__ order,
                                                   int n, int T, const int* __restrict__ poff,
                                                   const int* __restrict__ soff, const int* __restrict__ woff,
                                                   PlanHeader* ph) {
    int4* pieces = reinterpret_cast<int4*>(ph + 1);
    int4* splits = reinterpret_cast<int4*>(reinterpret_cast<char*>(ph) + ph->splits_off);
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i == 0) {
        ph->num_pieces = poff[n];
        ph->num_split = woff[n];
        ph->num_split_pieces = soff[n];
        if (poff[n] > ph->max_pieces || woff[n] > ph->max_split || soff[n] > ph->max_split_pieces)
            ph->status = F3S_ERR_WORKSPACE;
    }
    if (i >= n) return;
    if (poff[n] > ph->max_pieces || woff[n] > ph->max_split || soff[n] > ph->max_split_pieces) return;
    const int w = order[i];
    const int b0 = offsets[w], b1 = offsets[w + 1];
    const int cnt = poff[i + 1] - poff[i];
    const bool split = woff[i + 1] > woff[i];
    for (int k = 0; k < cnt; ++k) {
        const int lo = split ? b0 + k * T : b0;
        const int hi = split ? min(b1, lo + T) : b1;
        pieces[poff[i] + k] = make_int4(w, lo, hi, split ? soff[i] + k : -1);
    }
    if (split) splits[woff[i]] = make_int4(w, soff[i], cnt, 0);
}

// One CTA per (split window, head group): O = sum_k c_k O_k with
// c_k = 2^(m_k - M) / sum_j 2^(m_j - M) l_j over the window's pieces, summed
// in piece order (deterministic).  Per unit: a warp per row finds M and the
// sum (lanes over pieces); the coefficients of up to 32 pieces are staged in
// shared memory; each thread then accumulates float4s of O with the loads of
// consecutive pieces in flight together.
template <int D>
__global__ void __launch_bounds__(256) k_merge_pieces(const PlanHeader* __restrict__ ph, void* __restrict__ O,
                                                      int heads, int num_nodes, int q_window_base, int q_rows,
                                                      int o_dtype) {
    constexpr int kMaxRows = 8 * 16;            // hg * 16 <= 128 rows of (head, node)
    constexpr int kChunk = 32;                  // pieces per coefficient chunk
    constexpr int kEpt = kMaxRows * D / 4 / 256 > 8 ? 8 : kMaxRows * D / 4 / 256;  // float4s per thread
    __shared__ float s_max[kMaxRows], s_inv[kMaxRows];
    __shared__ float s_coef[kChunk][kMaxRows];
    if (ph->status != 0 || ph->heads != heads || ph->head_dim != D) return;
    const int4* splits = reinterpret_cast<const int4*>(reinterpret_cast<const char*>(ph) + ph->splits_off);
    const float* partials = reinterpret_cast<const float*>(reinterpret_cast<const char*>(ph) + ph->partials_off);
    const int groups = ph->groups, hg = ph->hg;
    const int rows = hg * 16;
    if (rows > kMaxRows || rows * D / 4 > kEpt * 256) return;  // plans are built with hg * d <= 512
    const size_t slot_f = (size_t)rows * (D + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int unit = blockIdx.x; unit < ph->num_split * groups; unit += gridDim.x) {
        const int sidx = unit / groups, g = unit - sidx * groups;
        const int4 sw = splits[sidx];  // (window, first slot, pieces, -)
        const float* base = partials + ((size_t)sw.y * groups + g) * slot_f;
        const size_t pstride = (size_t)groups * slot_f;  // floats between consecutive pieces
        const float* ml_base = base + (size_t)rows * D;  // (m, l) pairs per row
        for (int row = warp; row < rows; row += 8) {
            float mx = -INFINITY;
            for (int k = lane; k < sw.z; k += 32) mx = fmaxf(mx, __ldcs(ml_base + k * pstride + 2 * row));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float sum = 0.f;
            for (int k = lane; k < sw.z; k += 32) {
                const float2 v = __ldcs(reinterpret_cast<const float2*>(ml_base + k * pstride + 2 * row));
                sum = fmaf(fast_exp2(v.x - mx), v.y, sum);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                s_max[row] = mx;
                s_inv[row] = sum > 0.f ? 1.f / sum : 0.f;
            }
        }
        float4 acc[kEpt];
#pragma unroll
        for (int e = 0; e < kEpt; ++e) acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int kc = 0; kc < sw.z; kc += kChunk) {
            const int nk = min(kChunk, sw.z - kc);
            __syncthreads();  // s_max / s_inv written; previous chunk's coefficients consumed
            for (int i = threadIdx.x; i < nk * rows; i += 256) {
                const int kk = i / rows, row = i - kk * rows;
                const float m = __ldcs(ml_base + (kc + kk) * pstride + 2 * row);
                s_coef[kk][row] = fast_exp2(m - s_max[row]) * s_inv[row];
            }
            __syncthreads();
#pragma unroll
            for (int e = 0; e < kEpt; ++e) {
                const int idx = threadIdx.x + e * 256;
                if (idx < rows * D / 4) {
                    const int row = idx / (D / 4);
                    const float4* src = reinterpret_cast<const float4*>(base + (size_t)kc * pstride) + idx;
                    const size_t step4 = pstride / 4;
                    float4 a = acc[e];
#pragma unroll 4
                    for (int kk = 0; kk < nk; ++kk) {
                        const float4 v = __ldcs(src + kk * step4);
                        const float c = s_coef[kk][row];
                        a.x = fmaf(c, v.x, a.x);
                        a.y = fmaf(c, v.y, a.y);
                        a.z = fmaf(c, v.z, a.z);
                        a.w = fmaf(c, v.w, a.w);
                    }
                    acc[e] = a;
                }
            }
        }
#pragma unroll
        for (int e = 0; e < kEpt; ++e) {
            const int idx = threadIdx.x + e * 256;
            if (idx < rows * D / 4) {
                const int row = idx / (D / 4), c4 = idx - row * (D / 4);
                const int hh = row >> 4, r = row & 15;
                const int node = 16 * sw.x + r;
                const int64_t srow = (int64_t)node - 16 * (int64_t)q_window_base;
                if (node < num_nodes && srow >= 0 && srow < q_rows)  // windows outside the slab: never written
                    store_o4(O, (srow * heads + (int64_t)g * hg + hh) * D + 4 * c4, acc[e], o_dtype);
            }
        }
        __syncthreads();  // s_max / s_inv reused by the next unit
    }
}

__global__ void k_plan_init(PlanHeader* ph, const PlanHeader h) {
    if (threadIdx.x == 0) *ph = h;
}

struct PlanLayout {
    size_t pieces, splits, npieces, nsplitp, nsplitw, tiles, partials, total;
    int max_pieces, max_split, max_split_pieces, groups, hg;
};

static int pick_head_group(int heads, int head_dim);

static PlanLayout plan_layout(int num_items, int64_t num_blocks, int T, int heads, int head_dim) {
    PlanLayout L{};
    L.hg = pick_head_group(heads, head_dim);
    L.groups = heads / L.hg;
    const int64_t per_t = T > 0 ? num_blocks / T : 0;
    L.max_pieces = (int)std::min<int64_t>(INT32_MAX / 2, (int64_t)num_items + 2 * per_t + 1);
    L.max_split = (int)std::min<int64_t>(num_items, per_t + 1);
    L.max_split_pieces = (int)std::min<int64_t>(INT32_MAX / 2, 2 * per_t + 1);
    size_t off = sizeof(PlanHeader);
    L.pieces = off;
    off = align_up(off + (size_t)L.max_pieces * 16, 256);
    L.splits = off;
    off = align_up(off + (size_t)std::max(L.max_split, 1) * 16, 256);
    const size_t nn = (size_t)num_items + 1;
    L.npieces = off;
    off = align_up(off + nn * 4, 256);
    L.nsplitp = off;
    off = align_up(off + nn * 4, 256);
    L.nsplitw = off;
    off = align_up(off + nn * 4, 256);
    L.tiles = off;
    off = align_up(off + (size_t)std::max<int64_t>(scan_tiles(num_items), 1) * 4, 256);
    L.partials = off;
    off = align_up(off + (size_t)L.max_split_pieces * L.groups * L.hg * 16 * (head_dim + 2) * 4, 256);
    L.total = off;
    return L;
}

// ------------------------------------------------------------------ host --

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// Tensor map over fp16 [rows, heads, head_dim] viewed as the 3-D tensor
// {64 elems, heads*head_dim/64 head-chunks, rows}: strides 128 B and
// heads*head_dim*2 B, each the previous dimension's full extent, as the
// driver documents.  The box is {64, box_chunks, 16}: box_chunks head-chunks
// of 16 consecutive nodes.  (A map whose head-chunk stride lies below the
// node stride is accepted by the encoder but is outside the documented
// contract -- and faulted here on a 17 GB tensor -- so it is never built.)
static bool encode_map(CUtensorMap* m, const void* base, int rows, int heads, int head_dim, int box_chunks) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {64, (cuuint64_t)heads * head_dim / 64, (cuuint64_t)rows};
    cuuint64_t strides[2] = {128, (cuuint64_t)heads * head_dim * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)box_chunks, 16};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Per-variant "max dynamic shared memory" attribute, set once per CUDA
// context of each device (a device reset makes a new context that needs it
// again); thread-safe.
template <int D, int HG>
static int ensure_smem_attr() {
    static PerContext<int> once;
    return once.get(nullptr, [](int*) -> int {
        F3S_CUDA_TRY(cudaFuncSetAttribute(k_fused3s<D, HG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          FwdCfg<D, HG>::SMEM));
        return F3S_SUCCESS;
    });
}

template <int D, int HG>
static int launch_variant(const void* Q, const void* K, const void* V, FwdParams prm, int q_rows, int kv_rows,
                          bool merge, cudaStream_t stream) {
    using C = FwdCfg<D, HG>;
    int rc = ensure_smem_attr<D, HG>();
    if (rc != F3S_SUCCESS) return rc;
    FwdMaps maps;
    const int hb = C::HB ? C::HB : 1;  // box b is unused when HB == 0; encode a valid map anyway
    if (!encode_map(&maps.qa, Q, q_rows, prm.heads, D, C::HA) || !encode_map(&maps.qb, Q, q_rows, prm.heads, D, hb) ||
        !encode_map(&maps.ka, K, kv_rows, prm.heads, D, C::HA) || !encode_map(&maps.kb, K, kv_rows, prm.heads, D, hb) ||
        !encode_map(&maps.va, V, kv_rows, prm.heads, D, C::HA) || !encode_map(&maps.vb, V, kv_rows, prm.heads, D, hb))
        return F3S_ERR_INVALID_VALUE;
    const int sms = num_sms_of_current_device();
    const int ctas = forward_grid_limit();
    const int items = prm.num_items * prm.groups;
    const int grid = prm.plan ? ctas : std::max(1, std::min(items, ctas));
    k_fused3s<D, HG><<<grid, C::THREADS, C::SMEM, stream>>>(maps, prm);
    F3S_LAUNCH_CHECK();
    if (prm.plan && merge) {
        k_merge_pieces<D><<<2 * sms, 256, 0, stream>>>(prm.plan, prm.O, prm.heads, prm.num_nodes, prm.q_window_base,
                                                       prm.q_rows, prm.o_dtype);
        F3S_LAUNCH_CHECK();
    }
    return F3S_SUCCESS;
}

// Heads per CTA: the largest power of two <= min(8, 512 / head_dim) that
// divides `heads` (so one tile is at most 16 KB and STAGES >= 4).
static int pick_head_group(int heads, int head_dim) {
    int cap = std::min(8, 512 / head_dim);
    int hg = 1;
    while (hg * 2 <= cap && heads % (hg * 2) == 0) hg *= 2;
    return hg;
}

// A plan whose pieces the caller built (host arrays), e.g. cut at block-column
// chunk boundaries and ordered chunk by chunk.  Layout: header, pieces,
// split records, partial states -- the sections the kernels read.
struct LoadedPlanLayout {
    size_t pieces, splits, partials, total;
    int groups, hg;
};

static LoadedPlanLayout loaded_plan_layout(int num_pieces, int num_split, int num_split_pieces, int heads,
                                           int head_dim) {
    LoadedPlanLayout L{};
    L.hg = pick_head_group(heads, head_dim);
    L.groups = heads / L.hg;
    size_t off = sizeof(PlanHeader);
    L.pieces = off;
    off = align_up(off + (size_t)std::max(num_pieces, 1) * 16, 256);
    L.splits = off;
    off = align_up(off + (size_t)std::max(num_split, 1) * 16, 256);
    L.partials = off;
    off = align_up(off + (size_t)std::max(num_split_pieces, 1) * L.groups * L.hg * 16 * (head_dim + 2) * 4, 256);
    L.total = off;
    return L;
}

// Host-side validation of a caller-built plan.  Every index the kernels
// derive from it stays inside its buffers (piece ranges inside their
// window's blocks, slots below num_split_pieces, split records inside the
// slot range), and the plan is consistent, so the result is the same as the
// unsplit forward:
//   * the pieces of a window cover its blocks [offsets[w], offsets[w+1])
//     exactly once; a piece holds at least one block, except the single
//     piece of a window that has none;
//   * a window of one piece has slot -1 and no split record;
//   * a window of several pieces has one split record (w, first, count)
//     with count equal to its pieces, and its pieces use the slots first ...
//     first + count - 1, each exactly once;
//   * no two split records share a slot.
static int validate_plan(const int32_t* pieces, int num_pieces, const int32_t* splits, int num_split,
                         int num_split_pieces, const int32_t* offsets, int nrw) {
    for (int i = 0; i < num_pieces; ++i) {
        const int32_t* pc = pieces + 4 * (size_t)i;
        if (pc[0] < 0 || pc[0] >= nrw || pc[1] < offsets[pc[0]] || pc[2] < pc[1] || pc[2] > offsets[pc[0] + 1] ||
            pc[3] < -1 || pc[3] >= num_split_pieces)
            return F3S_ERR_BAD_FORMAT;
    }
    // split records: at most one per window, slot ranges disjoint
    std::vector<int> split_of(nrw, -1);
    std::vector<int> slot_owner(num_split_pieces, -1);
    for (int i = 0; i < num_split; ++i) {
        const int32_t* sw = splits + 4 * (size_t)i;
        if (sw[0] < 0 || sw[0] >= nrw || sw[1] < 0 || sw[2] < 1 || (int64_t)sw[1] + sw[2] > num_split_pieces)
            return F3S_ERR_BAD_FORMAT;
        if (split_of[sw[0]] >= 0) return F3S_ERR_BAD_FORMAT;
        split_of[sw[0]] = i;
        for (int k = sw[1]; k < sw[1] + sw[2]; ++k) {
            if (slot_owner[k] >= 0) return F3S_ERR_BAD_FORMAT;
            slot_owner[k] = sw[0];
        }
    }
    // pieces grouped by window: coverage and slot use
    std::vector<int> idx(num_pieces);
    for (int i = 0; i < num_pieces; ++i) idx[i] = i;
    std::sort(idx.begin(), idx.end(), [&](int a, int b) {
        const int32_t* pa = pieces + 4 * (size_t)a;
        const int32_t* pb = pieces + 4 * (size_t)b;
        return pa[0] != pb[0] ? pa[0] < pb[0] : pa[1] < pb[1];
    });
    std::vector<char> slot_used(num_split_pieces, 0);
    for (int i = 0; i < num_pieces;) {
        const int w = pieces[4 * (size_t)idx[i]];
        int j = i;
        while (j < num_pieces && pieces[4 * (size_t)idx[j]] == w) ++j;
        const int n = j - i;
        const int b0 = offsets[w], b1 = offsets[w + 1];
        int at = b0;
        for (int k = i; k < j; ++k) {
            const int32_t* pc = pieces + 4 * (size_t)idx[k];
            if (pc[1] != at) return F3S_ERR_BAD_FORMAT;  // gap or overlap
            if (pc[2] == pc[1] && !(b1 == b0 && n == 1)) return F3S_ERR_BAD_FORMAT;
            at = pc[2];
            if (n == 1) {
                if (pc[3] != -1 || split_of[w] >= 0) return F3S_ERR_BAD_FORMAT;
            } else {
                if (pc[3] < 0 || slot_owner[pc[3]] != w || slot_used[pc[3]]) return F3S_ERR_BAD_FORMAT;
                slot_used[pc[3]] = 1;
            }
        }
        if (at != b1) return F3S_ERR_BAD_FORMAT;
        if (n > 1 && (split_of[w] < 0 || splits[4 * (size_t)split_of[w] + 2] != n)) return F3S_ERR_BAD_FORMAT;
        i = j;
    }
    // every split record's window has its pieces
    for (int i = 0; i < num_split; ++i)
        for (int k = splits[4 * (size_t)i + 1]; k < splits[4 * (size_t)i + 1] + splits[4 * (size_t)i + 2]; ++k)
            if (!slot_used[k]) return F3S_ERR_BAD_FORMAT;
    return F3S_SUCCESS;
}

int load_plan_impl(const int32_t* pieces, int num_pieces, const int32_t* splits, int num_split,
                   int num_split_pieces, const int32_t* offsets, int nrw, int heads, int head_dim, void* plan,
                   size_t plan_bytes, cudaStream_t stream) {
    if (num_pieces < 0 || num_split < 0 || num_split_pieces < 0 || nrw < 0 || heads <= 0) return F3S_ERR_INVALID_VALUE;
    if (head_dim != 64 && head_dim != 128) return F3S_ERR_UNSUPPORTED;
    if (!plan || (num_pieces > 0 && (!pieces || !offsets)) || (num_split > 0 && !splits)) return F3S_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(plan) & 255) != 0) return F3S_ERR_INVALID_VALUE;
    const LoadedPlanLayout L = loaded_plan_layout(num_pieces, num_split, num_split_pieces, heads, head_dim);
    if (plan_bytes < L.total) return F3S_ERR_WORKSPACE;
    if ((int64_t)num_pieces * L.groups > INT32_MAX) return F3S_ERR_TOO_LARGE;
    if (num_split > 0 && !offsets) return F3S_ERR_INVALID_VALUE;
    const int rc = validate_plan(pieces, num_pieces, splits, num_split, num_split_pieces, offsets, nrw);
    if (rc != F3S_SUCCESS) return rc;
    PlanHeader h{};
    h.num_pieces = h.max_pieces = num_pieces;
    h.num_split = h.max_split = num_split;
    h.num_split_pieces = h.max_split_pieces = num_split_pieces;
    h.max_blocks = 0;
    h.heads = heads;
    h.head_dim = head_dim;
    h.groups = L.groups;
    h.hg = L.hg;
    h.splits_off = (long long)L.splits;
    h.partials_off = (long long)L.partials;
    char* base = static_cast<char*>(plan);
    F3S_CUDA_TRY(cudaMemcpyAsync(base, &h, sizeof(h), cudaMemcpyHostToDevice, stream));
    if (num_pieces > 0)
        F3S_CUDA_TRY(cudaMemcpyAsync(base + L.pieces, pieces, (size_t)num_pieces * 16, cudaMemcpyHostToDevice, stream));
    if (num_split > 0)
        F3S_CUDA_TRY(cudaMemcpyAsync(base + L.splits, splits, (size_t)num_split * 16, cudaMemcpyHostToDevice, stream));
    F3S_CUDA_TRY(cudaStreamSynchronize(stream));  // the caller's host arrays may go away on return
    return F3S_SUCCESS;
}

// Sweep plans: header, pieces (window, first block, end block, info), and
// the running states (per window of the slab, head group and head: 32 lanes
// x (head_dim / 2 + 4) floats, the consumer warp's O fragments and m / l).
struct SweepPlanLayout {
    size_t pieces, states, total;
    int groups, hg;
};

static SweepPlanLayout sweep_plan_layout(int num_pieces, int q_windows, int heads, int head_dim) {
    SweepPlanLayout L{};
    L.hg = pick_head_group(heads, head_dim);
    L.groups = heads / L.hg;
    size_t off = sizeof(PlanHeader);
    L.pieces = off;
    off = align_up(off + (size_t)std::max(num_pieces, 1) * 16, 256);
    L.states = off;
    const size_t lane_floats = (size_t)head_dim / 2 + 4;  // NT * 4 + 4 with NT = head_dim / 8
    off = align_up(off + (size_t)std::max(q_windows, 1) * heads * 32 * lane_floats * 4, 256);
    L.total = off;
    return L;
}

// A window's pieces must appear in the plan in ascending column order and
// cover its blocks exactly once; each gets its index within the window and
// the last one a flag.  Windows outside the slab are rejected.
int load_sweep_plan_impl(const int32_t* pieces, int num_pieces, const int32_t* offsets, int nrw, int q_window_base,
                         int q_windows, int heads, int head_dim, void* plan, size_t plan_bytes, cudaStream_t stream) {
    if (num_pieces < 0 || nrw < 0 || heads <= 0 || q_window_base < 0 || q_windows < 0) return F3S_ERR_INVALID_VALUE;
    if (head_dim != 64 && head_dim != 128) return F3S_ERR_UNSUPPORTED;
    if (!plan || (num_pieces > 0 && (!pieces || !offsets))) return F3S_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(plan) & 255) != 0) return F3S_ERR_INVALID_VALUE;
    const SweepPlanLayout L = sweep_plan_layout(num_pieces, q_windows, heads, head_dim);
    if (plan_bytes < L.total) return F3S_ERR_WORKSPACE;
    if ((int64_t)num_pieces * L.groups > INT32_MAX) return F3S_ERR_TOO_LARGE;
    std::vector<int32_t> out((size_t)num_pieces * 4);
    std::vector<int> seen(q_windows, 0), next_block(q_windows, -1), count(q_windows, 0);
    for (int i = 0; i < num_pieces; ++i) {
        const int32_t* pc = pieces + 4 * (size_t)i;
        const int w = pc[0];
        if (w < q_window_base || w >= q_window_base + q_windows || w >= nrw) return F3S_ERR_BAD_FORMAT;
        const int s = w - q_window_base;
        if (count[s] == 0) next_block[s] = offsets[w];
        if (pc[1] != next_block[s] || pc[2] < pc[1] || pc[2] > offsets[w + 1]) return F3S_ERR_BAD_FORMAT;
        if (pc[2] == pc[1] && offsets[w + 1] != offsets[w]) return F3S_ERR_BAD_FORMAT;  // empty piece of a window with blocks
        if (count[s] >= kSweepIndexMask) return F3S_ERR_TOO_LARGE;
        next_block[s] = pc[2];
        out[4 * (size_t)i + 0] = w;
        out[4 * (size_t)i + 1] = pc[1];
        out[4 * (size_t)i + 2] = pc[2];
        out[4 * (size_t)i + 3] = count[s]++;
    }
    for (int s = 0; s < q_windows; ++s)
        if (count[s] > 0 && next_block[s] != offsets[q_window_base + s + 1]) return F3S_ERR_BAD_FORMAT;  // not covered
    for (int i = num_pieces - 1; i >= 0; --i) {  // the last piece of every window
        const int s = out[4 * (size_t)i] - q_window_base;
        if (!seen[s]) {
            seen[s] = 1;
            out[4 * (size_t)i + 3] |= kSweepLast;
        }
    }
    PlanHeader h{};
    h.num_pieces = h.max_pieces = num_pieces;
    h.heads = heads;
    h.head_dim = head_dim;
    h.groups = L.groups;
    h.hg = L.hg;
    h.splits_off = (long long)L.states;  // no split records
    h.partials_off = (long long)L.states;
    h.states_off = (long long)L.states;
    h.mode = kPlanSweep;
    char* base = static_cast<char*>(plan);
    F3S_CUDA_TRY(cudaMemcpyAsync(base, &h, sizeof(h), cudaMemcpyHostToDevice, stream));
    if (num_pieces > 0)
        F3S_CUDA_TRY(cudaMemcpyAsync(base + L.pieces, out.data(), out.size() * 4, cudaMemcpyHostToDevice, stream));
    F3S_CUDA_TRY(cudaStreamSynchronize(stream));  // `out` goes away on return
    return F3S_SUCCESS;
}

int make_plan_impl(const int* offsets, const int* order, int num_items, int64_t num_blocks, int T, int heads,
                   int head_dim, void* plan, size_t plan_bytes, cudaStream_t stream) {
    if (num_items < 0 || num_blocks < 0 || T < 1 || heads <= 0) return F3S_ERR_INVALID_VALUE;
    if (head_dim != 64 && head_dim != 128) return F3S_ERR_UNSUPPORTED;
    if (!plan || (num_items > 0 && (!offsets || !order))) return F3S_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(plan) & 255) != 0) return F3S_ERR_INVALID_VALUE;
    const PlanLayout L = plan_layout(num_items, num_blocks, T, heads, head_dim);
    if (plan_bytes < L.total) return F3S_ERR_WORKSPACE;
    PlanHeader h{};
    h.max_pieces = L.max_pieces;
    h.max_split = L.max_split;
    h.max_split_pieces = L.max_split_pieces;
    h.max_blocks = T;
    h.heads = heads;
    h.head_dim = head_dim;
    h.groups = L.groups;
    h.hg = L.hg;
    h.splits_off = (long long)L.splits;
    h.partials_off = (long long)L.partials;
    PlanHeader* ph = static_cast<PlanHeader*>(plan);
    k_plan_init<<<1, 32, 0, stream>>>(ph, h);
    F3S_LAUNCH_CHECK();
    if (num_items == 0) return F3S_SUCCESS;
    char* base = static_cast<char*>(plan);
    int* np = reinterpret_cast<int*>(base + L.npieces);
    int* sp = reinterpret_cast<int*>(base + L.nsplitp);
    int* sw = reinterpret_cast<int*>(base + L.nsplitw);
    int* tiles = reinterpret_cast<int*>(base + L.tiles);
    const int grid = (num_items + 255) / 256;
    k_plan_count<<<grid, 256, 0, stream>>>(offsets, order, num_items, T, np, sp, sw);
    F3S_LAUNCH_CHECK();
    int rc;
    if ((rc = device_exclusive_scan(np, np, num_items, true, tiles, stream)) != F3S_SUCCESS) return rc;
    if ((rc = device_exclusive_scan(sp, sp, num_items, true, tiles, stream)) != F3S_SUCCESS) return rc;
    if ((rc = device_exclusive_scan(sw, sw, num_items, true, tiles, stream)) != F3S_SUCCESS) return rc;
    k_plan_fill<<<grid, 256, 0, stream>>>(offsets, order, num_items, T, np, sp, sw, ph);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

int forward_impl(const void* Q, const void* K, const void* V, void* O, int o_dtype, const int* offsets,
                 const int* cols, const int* order, const uint8_t* block_hints, const void* plan, int num_items,
                 int num_nodes, int heads, int head_dim, int q_window_base, int q_rows, void* ws, size_t ws_bytes,
                 cudaStream_t stream, uint64_t timeout_ns, const PieceRange& range) {
    if (o_dtype != F3S_OUT_F32 && o_dtype != F3S_OUT_F16 && o_dtype != F3S_OUT_BF16) return F3S_ERR_INVALID_VALUE;
    if (num_items < 0 || num_nodes < 0 || heads <= 0 || q_window_base < 0 || q_rows < 0)
        return F3S_ERR_INVALID_VALUE;
    if (head_dim != 64 && head_dim != 128) return F3S_ERR_UNSUPPORTED;
    if (!ws) return F3S_ERR_INVALID_VALUE;
    if (ws_bytes < kWsHeaderBytes) return F3S_ERR_WORKSPACE;
    if ((int64_t)heads * head_dim * 2 * 16 > (int64_t)1 << 40) return F3S_ERR_TOO_LARGE;
    // the piece range and the K / V slice
    if (!plan && (range.begin != 0 || range.end != -1)) return F3S_ERR_INVALID_VALUE;
    if (range.begin < 0 || (range.end != -1 && range.end < range.begin)) return F3S_ERR_INVALID_VALUE;
    const int kv_rows = range.kv_rows < 0 ? num_nodes : range.kv_rows;
    if (range.kv_col_base < 0 || (int64_t)range.kv_col_base * 16 + kv_rows > (int64_t)num_nodes)
        return F3S_ERR_INVALID_VALUE;
    // a slice that stops inside the graph must end on a block-column boundary
    if (kv_rows % 16 != 0 && (int64_t)range.kv_col_base * 16 + kv_rows != (int64_t)num_nodes)
        return F3S_ERR_INVALID_VALUE;
    if (plan) num_items = 0;  // the plan lists the work
    if ((!plan && num_items == 0) || num_nodes == 0 || q_rows == 0 || (plan && range.end == range.begin))
        return F3S_SUCCESS;
    if (kv_rows == 0) return F3S_ERR_INVALID_VALUE;
    if (!Q || !K || !V || !O || !offsets || !cols || (!plan && !order)) return F3S_ERR_INVALID_VALUE;
    auto misaligned = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) != 0; };
    if (misaligned(Q) || misaligned(K) || misaligned(V) || misaligned(O)) return F3S_ERR_INVALID_VALUE;
    const int hg = pick_head_group(heads, head_dim);
    FwdParams prm{};
    prm.O = O;
    prm.o_dtype = o_dtype;
    prm.offsets = offsets;
    prm.cols = cols;
    prm.order = order;
    prm.plan = static_cast<PlanHeader*>(const_cast<void*>(plan));
    prm.hints = block_hints;
    prm.hdr = static_cast<WsHeader*>(ws);
    prm.timeout_ns = timeout_ns;
    prm.num_items = num_items;
    prm.groups = heads / hg;
    prm.num_nodes = num_nodes;
    prm.nrw_total = (int)(((int64_t)num_nodes + 15) / 16);
    prm.heads = heads;
    prm.q_window_base = q_window_base;
    prm.q_windows = (int)(((int64_t)q_rows + 15) / 16);
    prm.q_rows = q_rows;
    prm.tail = num_nodes & 15;
    prm.piece_begin = range.begin;
    prm.piece_end = range.end;
    prm.kv_col_base = range.kv_col_base;
    prm.kv_cols = (int)(((int64_t)kv_rows + 15) / 16);
    if ((int64_t)num_items * prm.groups > INT32_MAX) return F3S_ERR_TOO_LARGE;
    // sweep plans: the per-window, per-head piece counters follow the
    // workspace header (f3s_sweep_workspace_size)
    prm.seq = reinterpret_cast<int*>(static_cast<char*>(ws) + kWsHeaderBytes);
    prm.seq_cap = (long long)((ws_bytes - kWsHeaderBytes) / sizeof(int));
    // zero the abort flag and the ticket counter (adjacent words) and the
    // sweep counters this launch can use; the status word stays sticky
    F3S_CUDA_TRY(cudaMemsetAsync(ws, 0, 2 * sizeof(int), stream));
    if (plan && prm.seq_cap > 0) {
        const long long need = (long long)prm.q_windows * heads;
        const long long n = need < prm.seq_cap ? need : prm.seq_cap;
        F3S_CUDA_TRY(cudaMemsetAsync(prm.seq, 0, (size_t)n * sizeof(int), stream));
    }
    const bool m = range.merge;
    if (head_dim == 64) {
        switch (hg) {
            case 1: return launch_variant<64, 1>(Q, K, V, prm, q_rows, kv_rows, m, stream);
            case 2: return launch_variant<64, 2>(Q, K, V, prm, q_rows, kv_rows, m, stream);
            case 4: return launch_variant<64, 4>(Q, K, V, prm, q_rows, kv_rows, m, stream);
            default: return launch_variant<64, 8>(Q, K, V, prm, q_rows, kv_rows, m, stream);
        }
    }
    switch (hg) {
        case 1: return launch_variant<128, 1>(Q, K, V, prm, q_rows, kv_rows, m, stream);
        case 2: return launch_variant<128, 2>(Q, K, V, prm, q_rows, kv_rows, m, stream);
        default: return launch_variant<128, 4>(Q, K, V, prm, q_rows, kv_rows, m, stream);
    }
}

// The merge of a plan's split windows on its own (after f3s_forward_pieces
// ran every piece of those windows).
int plan_merge_impl(const void* plan, void* O, int o_dtype, int num_nodes, int heads, int head_dim,
                    int q_window_base, int q_rows, cudaStream_t stream) {
    if (o_dtype != F3S_OUT_F32 && o_dtype != F3S_OUT_F16 && o_dtype != F3S_OUT_BF16) return F3S_ERR_INVALID_VALUE;
    if (num_nodes < 0 || heads <= 0 || q_window_base < 0 || q_rows < 0) return F3S_ERR_INVALID_VALUE;
    if (head_dim != 64 && head_dim != 128) return F3S_ERR_UNSUPPORTED;
    if (!plan || (reinterpret_cast<uintptr_t>(plan) & 255) != 0) return F3S_ERR_INVALID_VALUE;
    if (num_nodes == 0 || q_rows == 0) return F3S_SUCCESS;
    if (!O || (reinterpret_cast<uintptr_t>(O) & 15) != 0) return F3S_ERR_INVALID_VALUE;
    const int sms = num_sms_of_current_device();
    const PlanHeader* ph = static_cast<const PlanHeader*>(plan);
    if (head_dim == 64)
        k_merge_pieces<64><<<2 * sms, 256, 0, stream>>>(ph, O, heads, num_nodes, q_window_base, q_rows, o_dtype);
    else
        k_merge_pieces<128><<<2 * sms, 256, 0, stream>>>(ph, O, heads, num_nodes, q_window_base, q_rows, o_dtype);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

// -------------------------------------------------- failure-path self-test --
__global__ void k_wait_selftest(WsHeader* hdr, uint64_t timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = smem_addr(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const ErrorSink err{&hdr->abort, &hdr->status};
        // nobody arrives: the bounded wait gives up and records the timeout
        mbar_wait_bounded(b, 0, err, timeout_ns);
    }
}

int selftest_wait_timeout(uint64_t timeout_ns, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (!ws) return F3S_ERR_INVALID_VALUE;
    if (ws_bytes < kWsHeaderBytes) return F3S_ERR_WORKSPACE;
    if (timeout_ns > 5ull * 1000 * 1000 * 1000) return F3S_ERR_INVALID_VALUE;
    F3S_CUDA_TRY(cudaMemsetAsync(ws, 0, 2 * sizeof(int), stream));
    k_wait_selftest<<<1, 32, 0, stream>>>(static_cast<WsHeader*>(ws), timeout_ns);
    F3S_LAUNCH_CHECK();
    return F3S_SUCCESS;
}

}  // namespace f3s

extern "C" {

size_t f3s_forward_workspace_size(void) { return f3s::kWsHeaderBytes; }

size_t f3s_plan_size(int32_t num_items, int64_t num_blocks, int32_t max_blocks_per_piece, int32_t heads,
                     int32_t head_dim) {
    if (num_items < 0 || num_blocks < 0 || max_blocks_per_piece < 1 || heads <= 0) return 0;
    if (head_dim != 64 && head_dim != 128) return 0;
    return f3s::plan_layout(num_items, num_blocks, max_blocks_per_piece, heads, head_dim).total;
}

int f3s_make_plan(const int32_t* d_window_offsets, const int32_t* d_order, int32_t num_items, int64_t num_blocks,
                  int32_t max_blocks_per_piece, int32_t heads, int32_t head_dim, void* d_plan, size_t plan_bytes,
                  f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_make_plan");
    return f3s::make_plan_impl(d_window_offsets, d_order, num_items, num_blocks, max_blocks_per_piece, heads,
                               head_dim, d_plan, plan_bytes, (cudaStream_t)stream);
}

size_t f3s_plan_size_for(int32_t num_pieces, int32_t num_split, int32_t num_split_pieces, int32_t heads,
                         int32_t head_dim) {
    if (num_pieces < 0 || num_split < 0 || num_split_pieces < 0 || heads <= 0) return 0;
    if (head_dim != 64 && head_dim != 128) return 0;
    return f3s::loaded_plan_layout(num_pieces, num_split, num_split_pieces, heads, head_dim).total;
}

int f3s_load_plan(const int32_t* h_pieces, int32_t num_pieces, const int32_t* h_splits, int32_t num_split,
                  int32_t num_split_pieces, const int32_t* h_window_offsets, int32_t num_row_windows, int32_t heads,
                  int32_t head_dim, void* d_plan, size_t plan_bytes, f3s_stream_t stream) {
    return f3s::load_plan_impl(h_pieces, num_pieces, h_splits, num_split, num_split_pieces, h_window_offsets,
                               num_row_windows, heads, head_dim, d_plan, plan_bytes, (cudaStream_t)stream);
}

size_t f3s_sweep_plan_size(int32_t num_pieces, int32_t q_windows, int32_t heads, int32_t head_dim) {
    if (num_pieces < 0 || q_windows < 0 || heads <= 0) return 0;
    if (head_dim != 64 && head_dim != 128) return 0;
    return f3s::sweep_plan_layout(num_pieces, q_windows, heads, head_dim).total;
}

size_t f3s_sweep_workspace_size(int32_t q_rows, int32_t heads) {
    if (q_rows < 0 || heads <= 0) return 0;
    const size_t q_windows = ((size_t)q_rows + 15) / 16;
    return f3s::kWsHeaderBytes + f3s::align_up(q_windows * heads * sizeof(int), 256);
}

int f3s_load_sweep_plan(const int32_t* h_pieces, int32_t num_pieces, const int32_t* h_window_offsets,
                        int32_t num_row_windows, int32_t q_window_base, int32_t q_windows, int32_t heads,
                        int32_t head_dim, void* d_plan, size_t plan_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_load_sweep_plan");
    return f3s::load_sweep_plan_impl(h_pieces, num_pieces, h_window_offsets, num_row_windows, q_window_base,
                                     q_windows, heads, head_dim, d_plan, plan_bytes, (cudaStream_t)stream);
}

int f3s_forward(const void* d_Q, const void* d_K, const void* d_V, float* d_O, const int32_t* d_window_offsets,
                const int32_t* d_block_cols, const int32_t* d_order, const uint8_t* d_block_hints, const void* d_plan,
                int32_t num_items, int32_t num_nodes, int32_t heads, int32_t head_dim, int32_t q_window_base,
                int32_t q_rows, void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_forward");
    return f3s::forward_impl(d_Q, d_K, d_V, d_O, F3S_OUT_F32, d_window_offsets, d_block_cols, d_order,
                             d_block_hints, d_plan, num_items, num_nodes, heads, head_dim, q_window_base, q_rows,
                             d_workspace, workspace_bytes, (cudaStream_t)stream, f3s::kWaitTimeoutNs, f3s::PieceRange{});
}

int f3s_forward_pieces(const void* d_Q, const void* d_K, const void* d_V, void* d_O, int32_t o_dtype,
                       const int32_t* d_window_offsets, const int32_t* d_block_cols, const uint8_t* d_block_hints,
                       const void* d_plan, int32_t piece_begin, int32_t piece_end, int32_t kv_col_base,
                       int32_t kv_rows, int32_t num_nodes, int32_t heads, int32_t head_dim, int32_t q_window_base,
                       int32_t q_rows, void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_forward_pieces");
    if (!d_plan || kv_rows < 0) return F3S_ERR_INVALID_VALUE;
    f3s::PieceRange r;
    r.begin = piece_begin;
    r.end = piece_end;
    r.kv_col_base = kv_col_base;
    r.kv_rows = kv_rows;
    r.merge = false;
    return f3s::forward_impl(d_Q, d_K, d_V, d_O, o_dtype, d_window_offsets, d_block_cols, nullptr, d_block_hints,
                             d_plan, 0, num_nodes, heads, head_dim, q_window_base, q_rows, d_workspace,
                             workspace_bytes, (cudaStream_t)stream, f3s::kWaitTimeoutNs, r);
}

int f3s_plan_merge(const void* d_plan, void* d_O, int32_t o_dtype, int32_t num_nodes, int32_t heads,
                   int32_t head_dim, int32_t q_window_base, int32_t q_rows, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_plan_merge");
    return f3s::plan_merge_impl(d_plan, d_O, o_dtype, num_nodes, heads, head_dim, q_window_base, q_rows,
                                (cudaStream_t)stream);
}

int f3s_forward_ex(const void* d_Q, const void* d_K, const void* d_V, void* d_O, int32_t o_dtype,
                   const int32_t* d_window_offsets, const int32_t* d_block_cols, const int32_t* d_order,
                   const uint8_t* d_block_hints, const void* d_plan, int32_t num_items, int32_t num_nodes,
                   int32_t heads, int32_t head_dim, int32_t q_window_base, int32_t q_rows, void* d_workspace,
                   size_t workspace_bytes, f3s_stream_t stream) {
    f3s::NvtxRange nvtx_("f3s_forward");
    return f3s::forward_impl(d_Q, d_K, d_V, d_O, o_dtype, d_window_offsets, d_block_cols, d_order, d_block_hints,
                             d_plan, num_items, num_nodes, heads, head_dim, q_window_base, q_rows, d_workspace,
                             workspace_bytes, (cudaStream_t)stream, f3s::kWaitTimeoutNs, f3s::PieceRange{});
}

int f3s_selftest_wait_timeout(uint64_t timeout_ns, void* d_workspace, size_t workspace_bytes, f3s_stream_t stream) {
    return f3s::selftest_wait_timeout(timeout_ns, d_workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
