/*
 * f3s_oracle.c -- CPU restatement of the reference fused-3S hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in fused3s_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product path never calls it
 * and has no CPU fallback.
 *
 * Every function restates one reference function (paths are relative to the
 * fatalhawk/fused3S project root):
 *
 *   orc_convert            src/converter.cu:13-44
 *   orc_convert_mt         the same, windows split over threads
 *   orc_window_order       include/utils.cuh:48-59 (stable tie order, see below)
 *   orc_block_attention    tests/test_fused_3s_v2.cu:17-59
 *   orc_edge_attention     baselines/cpu_baseline.cpp:16-91
 *
 * Parity pin: tests/test_oracle.py checks every function here against the
 * reference's own functions compiled from its sources (oracle/Makefile ->
 * oracle/_ref/libf3s_ref.so) and against the committed fixtures in
 * tests/golden/ that were produced by those compiled reference functions.
 *
 * The floating-point statements of orc_block_attention follow the reference
 * loop statement by statement (same accumulation order, same -1e9 mask and
 * max seed, std::exp == expf, division-then-PV), so with the same compiler
 * flags the result is bit-identical to the compiled reference.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <pthread.h>

/* ------------------------------------------------------------------------ */
/* CSR -> 16x16 block-sparse row windows (src/converter.cu:13-44)           */
/* ------------------------------------------------------------------------ */

static int cmp_i32(const void* a, const void* b) {
    int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

/*
 * For each row window w (rows [16w, min(16w+16, N))) collect {v / 16} over
 * the window's edges, sorted ascending and de-duplicated: the iteration
 * order of the reference's std::set<int> (converter.cu:20,29,34).  C integer
 * division truncates toward zero exactly like the reference's `v / 16`.
 *
 * offsets_out: int32[nrw + 1]; cols_out: int32 with room for nnz entries
 * (the number of unique block columns never exceeds the number of edges).
 * Returns the total number of active blocks B = offsets_out[nrw].
 */
int64_t orc_convert(int32_t num_nodes, const int32_t* row_ptr,
                    const int32_t* col_ind, int32_t* offsets_out,
                    int32_t* cols_out) {
    int32_t nrw = (num_nodes + 15) / 16;
    int64_t total = 0;
    int64_t cap = 0;
    int32_t* buf = NULL;
    offsets_out[0] = 0;
    for (int32_t w = 0; w < nrw; ++w) {
        int32_t start = w * 16;
        int32_t end = start + 16 < num_nodes ? start + 16 : num_nodes;
        int64_t len = 0;
        for (int32_t u = start; u < end; ++u)
            if (row_ptr[u + 1] > row_ptr[u]) len += row_ptr[u + 1] - row_ptr[u];
        if (len > cap) {
            cap = len * 2;
            buf = (int32_t*)realloc(buf, (size_t)cap * sizeof(int32_t));
        }
        int64_t n = 0;
        for (int32_t u = start; u < end; ++u)
            for (int32_t j = row_ptr[u]; j < row_ptr[u + 1]; ++j)
                buf[n++] = col_ind[j] / 16;
        if (n > 1) qsort(buf, (size_t)n, sizeof(int32_t), cmp_i32);
        for (int64_t i = 0; i < n; ++i)
            if (i == 0 || buf[i] != buf[i - 1]) cols_out[total++] = buf[i];
        offsets_out[w + 1] = (int32_t)total;
    }
    free(buf);
    return total;
}

/* ------------------------------------------------------------------------ */
/* Threaded driver for orc_convert (large graphs)                           */
/* ------------------------------------------------------------------------ */

/*
 * Same output as orc_convert.  Windows are cut into nthreads contiguous
 * ranges; each worker runs orc_convert's per-window loop (the same
 * statements, on the rows of its range) into its own buffer, and the
 * buffers are concatenated in window order after the offsets are summed.
 */
typedef struct {
    int32_t num_nodes;
    const int32_t *row_ptr, *col_ind;
    int32_t w0, w1;
    int32_t* counts; /* [w1 - w0] unique block columns per window */
    int32_t* cols;   /* the range's block columns, window after window */
    int64_t ncols;
} orc_conv_part;

static void* orc_conv_worker(void* arg) {
    orc_conv_part* p = (orc_conv_part*)arg;
    int64_t cap = 0, total = 0, room = 0;
    int32_t* buf = NULL;
    for (int32_t w = p->w0; w < p->w1; ++w) {
        int32_t start = w * 16;
        int32_t end = start + 16 < p->num_nodes ? start + 16 : p->num_nodes;
        int64_t len = 0;
        for (int32_t u = start; u < end; ++u)
            if (p->row_ptr[u + 1] > p->row_ptr[u]) len += p->row_ptr[u + 1] - p->row_ptr[u];
        if (len > cap) {
            cap = len * 2;
            buf = (int32_t*)realloc(buf, (size_t)cap * sizeof(int32_t));
        }
        if (total + len > room) {
            room = (total + len) * 2 + 1024;
            p->cols = (int32_t*)realloc(p->cols, (size_t)room * sizeof(int32_t));
        }
        int64_t n = 0;
        for (int32_t u = start; u < end; ++u)
            for (int32_t j = p->row_ptr[u]; j < p->row_ptr[u + 1]; ++j)
                buf[n++] = p->col_ind[j] / 16;
        if (n > 1) qsort(buf, (size_t)n, sizeof(int32_t), cmp_i32);
        int64_t before = total;
        for (int64_t i = 0; i < n; ++i)
            if (i == 0 || buf[i] != buf[i - 1]) p->cols[total++] = buf[i];
        p->counts[w - p->w0] = (int32_t)(total - before);
    }
    free(buf);
    p->ncols = total;
    return NULL;
}

int64_t orc_convert_mt(int32_t num_nodes, const int32_t* row_ptr,
                       const int32_t* col_ind, int32_t* offsets_out,
                       int32_t* cols_out, int32_t nthreads) {
    int32_t nrw = (num_nodes + 15) / 16;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > nrw) nthreads = nrw > 0 ? nrw : 1;
    orc_conv_part* parts = (orc_conv_part*)calloc((size_t)nthreads, sizeof(orc_conv_part));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int32_t t = 0; t < nthreads; ++t) {
        orc_conv_part* p = &parts[t];
        p->num_nodes = num_nodes;
        p->row_ptr = row_ptr;
        p->col_ind = col_ind;
        p->w0 = (int32_t)((int64_t)nrw * t / nthreads);
        p->w1 = (int32_t)((int64_t)nrw * (t + 1) / nthreads);
        p->counts = (int32_t*)malloc(((size_t)(p->w1 - p->w0) + 1) * sizeof(int32_t));
        pthread_create(&th[t], NULL, orc_conv_worker, p);
    }
    int64_t total = 0;
    offsets_out[0] = 0;
    for (int32_t t = 0; t < nthreads; ++t) {
        orc_conv_part* p = &parts[t];
        pthread_join(th[t], NULL);
        for (int32_t w = p->w0; w < p->w1; ++w) {
            total += p->counts[w - p->w0];
            offsets_out[w + 1] = (int32_t)total;
        }
        if (p->ncols) memcpy(cols_out + (total - p->ncols), p->cols, (size_t)p->ncols * sizeof(int32_t));
        free(p->counts);
        free(p->cols);
    }
    free(parts);
    free(th);
    return total;
}

/* ------------------------------------------------------------------------ */
/* Descending-workload window order (include/utils.cuh:48-59)               */
/* ------------------------------------------------------------------------ */

/*
 * The reference sorts iota(nrw) with std::sort and the comparator
 * blocks(a) > blocks(b).  std::sort is not stable, so its tie order is an
 * artefact of libstdc++'s introsort.  This restatement fixes ties by
 * ascending window id (what std::stable_sort gives with the same
 * comparator).  The sequence of block counts along the order is identical
 * to the reference's for every input; the permutation itself is identical
 * whenever the reference's std::sort leaves equal keys in index order.
 *
 * Implementation: a counting sort on the block count (stable by
 * construction), descending.
 */
void orc_window_order(int32_t nrw, const int32_t* offsets, int32_t* order_out) {
    int32_t maxc = 0;
    for (int32_t w = 0; w < nrw; ++w) {
        int32_t c = offsets[w + 1] - offsets[w];
        if (c > maxc) maxc = c;
    }
    int64_t* start = (int64_t*)calloc((size_t)maxc + 2, sizeof(int64_t));
    for (int32_t w = 0; w < nrw; ++w) start[offsets[w + 1] - offsets[w]]++;
    /* descending: windows with count k start after all windows with count > k */
    int64_t run = 0;
    for (int64_t k = maxc; k >= 0; --k) {
        int64_t c = start[k];
        start[k] = run;
        run += c;
    }
    for (int32_t w = 0; w < nrw; ++w)
        order_out[start[offsets[w + 1] - offsets[w]]++] = w;
    free(start);
}

/* ------------------------------------------------------------------------ */
/* Block-semantics attention (tests/test_fused_3s_v2.cu:17-59)              */
/* ------------------------------------------------------------------------ */

/*
 * For every real row r of window w: score every column of every active
 * block of w (dense within the block), with columns >= num_nodes scored
 * -1e9; softmax over all of them (max seeded with -1e9, exp, divide by the
 * sum); then O[r] = sum over real columns of P * V.  Rows of windows with no
 * active block are left untouched (the reference's `if (S.empty())
 * continue;`).
 *
 * Generalised to H heads in node-major layout [rows, H, d]: head h of node n
 * lives at (n * H + h) * d.  With H == 1 the indexing is the reference's
 * `row * feat_dim + f`.
 *
 * windows / nwin: optional subset of window ids (NULL = all windows).
 * heads / nheads: optional subset of heads (NULL = all heads).
 */
void orc_block_attention(int32_t num_nodes, int32_t H, int32_t d,
                         const float* Q, const float* K, const float* V,
                         float* O, int32_t nrw, const int32_t* offsets,
                         const int32_t* cols, const int32_t* windows,
                         int32_t nwin, const int32_t* heads, int32_t nheads) {
    int32_t maxb = 0;
    for (int32_t w = 0; w < nrw; ++w) {
        int32_t c = offsets[w + 1] - offsets[w];
        if (c > maxb) maxb = c;
    }
    size_t cap = (size_t)maxb * 16 + 1;
    float* S = (float*)malloc(cap * sizeof(float));
    float* P = (float*)malloc(cap * sizeof(float));
    int32_t* gcol = (int32_t*)malloc(cap * sizeof(int32_t));
    int32_t nw = windows ? nwin : nrw;
    int32_t nh = heads ? nheads : H;
    for (int32_t iw = 0; iw < nw; ++iw) {
        int32_t w = windows ? windows[iw] : iw;
        int32_t b0 = offsets[w], b1 = offsets[w + 1];
        for (int32_t ih = 0; ih < nh; ++ih) {
            int32_t h = heads ? heads[ih] : ih;
            for (int32_t r = 0; r < 16; ++r) {
                int32_t row = w * 16 + r;
                if (row >= num_nodes) continue;
                const float* q = Q + ((int64_t)row * H + h) * d;
                size_t n = 0;
                for (int32_t b = b0; b < b1; ++b) {
                    int32_t bc = cols[b];
                    for (int32_t c = 0; c < 16; ++c) {
                        int32_t col = bc * 16 + c;
                        float sum = 0.0f;
                        if (col < num_nodes) {
                            const float* k = K + ((int64_t)col * H + h) * d;
                            for (int32_t f = 0; f < d; ++f) sum += q[f] * k[f];
                        } else {
                            sum = -1e9f;
                        }
                        S[n] = sum;
                        gcol[n] = col;
                        ++n;
                    }
                }
                if (n == 0) continue;
                float max_val = -1e9f;
                for (size_t i = 0; i < n; ++i)
                    if (S[i] > max_val) max_val = S[i];
                float exp_sum = 0.0f;
                for (size_t i = 0; i < n; ++i) {
                    P[i] = expf(S[i] - max_val);
                    exp_sum += P[i];
                }
                for (size_t i = 0; i < n; ++i) P[i] /= exp_sum;
                float* o = O + ((int64_t)row * H + h) * d;
                for (int32_t f = 0; f < d; ++f) {
                    float out_val = 0.0f;
                    for (size_t i = 0; i < n; ++i) {
                        int32_t gc = gcol[i];
                        if (gc < num_nodes)
                            out_val += P[i] * V[((int64_t)gc * H + h) * d + f];
                    }
                    o[f] = out_val;
                }
            }
        }
    }
    free(S);
    free(P);
    free(gcol);
}

/* ------------------------------------------------------------------------ */
/* Edge-semantics attention (baselines/cpu_baseline.cpp:16-91)              */
/* ------------------------------------------------------------------------ */

/*
 * True CSR attention: the softmax of row i runs only over its listed
 * neighbours.  Single head, [num_nodes, d] row-major.  Kept as the
 * secondary (naive) CPU reference; it is not the parity oracle because the
 * hot path has block semantics.
 */
void orc_edge_attention(int32_t num_nodes, int32_t d, const float* Q,
                        const float* K, const float* V, const int32_t* row_ptr,
                        const int32_t* col_idx, float* out) {
    size_t cap = 16;
    float* a = (float*)malloc(cap * sizeof(float));
    for (int32_t i = 0; i < num_nodes; ++i) {
        int32_t s = row_ptr[i], e = row_ptr[i + 1];
        int32_t n = e - s;
        float* o = out + (int64_t)i * d;
        if (n <= 0) {
            for (int32_t f = 0; f < d; ++f) o[f] = 0.0f;
            continue;
        }
        if ((size_t)n > cap) {
            cap = (size_t)n * 2;
            a = (float*)realloc(a, cap * sizeof(float));
        }
        for (int32_t j = 0; j < n; ++j) {
            int32_t c = col_idx[s + j];
            float dot = 0.0f;
            for (int32_t f = 0; f < d; ++f)
                dot += Q[(int64_t)i * d + f] * K[(int64_t)c * d + f];
            a[j] = dot;
        }
        float m = -1e9f;
        for (int32_t j = 0; j < n; ++j)
            if (a[j] > m) m = a[j];
        float z = 0.0f;
        for (int32_t j = 0; j < n; ++j) {
            a[j] = expf(a[j] - m);
            z += a[j];
        }
        for (int32_t j = 0; j < n; ++j) a[j] /= z;
        for (int32_t f = 0; f < d; ++f) o[f] = 0.0f;
        for (int32_t j = 0; j < n; ++j) {
            int32_t c = col_idx[s + j];
            float wgt = a[j];
            for (int32_t f = 0; f < d; ++f) o[f] += wgt * V[(int64_t)c * d + f];
        }
    }
    free(a);
}

/* ------------------------------------------------------------------------ */
/* Threaded driver for orc_block_attention                                  */
/* ------------------------------------------------------------------------ */

typedef struct {
    int32_t num_nodes, H, d;
    const float *Q, *K, *V;
    float* O;
    int32_t nrw;
    const int32_t *offsets, *cols, *windows;
    int32_t nwin;
    const int32_t* heads;
    int32_t nheads;
} orc_job;

typedef struct {
    const orc_job* job;
    int32_t* mine;
    int32_t nmine;
} orc_part;

static void* orc_worker(void* arg) {
    orc_part* p = (orc_part*)arg;
    const orc_job* j = p->job;
    orc_block_attention(j->num_nodes, j->H, j->d, j->Q, j->K, j->V, j->O,
                        j->nrw, j->offsets, j->cols, p->mine, p->nmine,
                        j->heads, j->nheads);
    return NULL;
}

/*
 * Same result as orc_block_attention; windows are dealt round-robin to
 * nthreads workers (windows write disjoint output rows).
 */
void orc_block_attention_mt(int32_t num_nodes, int32_t H, int32_t d,
                            const float* Q, const float* K, const float* V,
                            float* O, int32_t nrw, const int32_t* offsets,
                            const int32_t* cols, const int32_t* windows,
                            int32_t nwin, const int32_t* heads, int32_t nheads,
                            int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    int32_t nw = windows ? nwin : nrw;
    orc_job job = {num_nodes, H, d, Q, K, V, O, nrw, offsets, cols,
                   windows, nwin, heads, nheads};
    orc_part* parts = (orc_part*)calloc((size_t)nthreads, sizeof(orc_part));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int32_t t = 0; t < nthreads; ++t) {
        parts[t].job = &job;
        parts[t].mine = (int32_t*)malloc(((size_t)nw / nthreads + 1) * sizeof(int32_t));
    }
    for (int32_t i = 0; i < nw; ++i) {
        orc_part* p = &parts[i % nthreads];
        p->mine[p->nmine++] = windows ? windows[i] : i;
    }
    for (int32_t t = 0; t < nthreads; ++t)
        pthread_create(&th[t], NULL, orc_worker, &parts[t]);
    for (int32_t t = 0; t < nthreads; ++t) {
        pthread_join(th[t], NULL);
        free(parts[t].mine);
    }
    free(parts);
    free(th);
}
