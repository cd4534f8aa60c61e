/*
 * CPU oracle for APPNP personalised PageRank with per-iteration top-k pruning.
 * TEST INFRASTRUCTURE ONLY: built by oracle/Makefile, loaded by oracle/ppr.py.
 *
 * Restates `personal_pagerank_appnp` (NeutronGT/core/ppr_backends/appnp_backend.py:203-310)
 * one seed at a time.  Seeds are independent in the reference (row r of the SpGEMM only
 * reads row r of the state, `_aggregate_sparse_entries` keys on (row, col), top-k is per
 * row), so the seed batching of :259-262 does not change any value.
 *
 * Per seed s (state starts as {s: 1.0}, :264-266), for each of the T iterations (:272):
 *   contrib_j = state_j * (1 / max(outdeg_j, 1))                 transition values :158-162, :32
 *   acc[c]    = sum over state entries j in ASCENDING column order,
 *               for c in adj(j) in CSR order, of contrib_j           SpGEMM state x P   :167-174
 *   merged[c] = acc[c] * (1 - alpha)                                                   :175
 *   merged[s] = merged[s] + alpha   (entry created if absent)     teleport merge :180-189
 *   state     = top iter_topk of merged by (value desc, col asc)  `_segment_topk` :102-140
 *               (no pruning when iter_topk <= 0, :247-248)
 * Output: top final_keep of the last state (:291-300), emitted in (value desc, col asc)
 * order; final_keep <= 0 keeps every entry (:108-109).
 *
 * Canonical order.  The reference sums in fp32 in whatever order cuSPARSE and the CUDA
 * scatter_add_ atomics give (:74) and breaks top-k ties in torch.topk's unspecified order.
 * This restatement fixes an order instead: fp64, contributions to one column added in
 * ascending source column, ties by ascending column.  Every multiply and add is a separate
 * IEEE round-to-nearest operation (built with -ffp-contract=off), so the CUDA kernels can
 * reproduce each value bit for bit.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

typedef struct {
    double v;
    int64_t c;
} entry_t;

static inline int before(const entry_t *a, const entry_t *b) {
    /* strict "a ranks before b": larger value first, then smaller column */
    return a->v > b->v || (a->v == b->v && a->c < b->c);
}

static int cmp_rank(const void *pa, const void *pb) {
    const entry_t *a = (const entry_t *)pa, *b = (const entry_t *)pb;
    if (before(a, b)) return -1;
    if (before(b, a)) return 1;
    return 0;
}

static int cmp_col(const void *pa, const void *pb) {
    const entry_t *a = (const entry_t *)pa, *b = (const entry_t *)pb;
    return (a->c > b->c) - (a->c < b->c);
}

/* Move the k best entries (by rank) to arr[0..k), sorted by rank.  Quickselect + sort. */
static void select_topk(entry_t *arr, int64_t m, int64_t k) {
    if (k >= m) {
        qsort(arr, (size_t)m, sizeof(entry_t), cmp_rank);
        return;
    }
    int64_t lo = 0, hi = m - 1;
    while (lo < hi) {
        entry_t pivot = arr[lo + (hi - lo) / 2];
        int64_t i = lo, j = hi;
        while (i <= j) {
            while (before(&arr[i], &pivot)) i++;
            while (before(&pivot, &arr[j])) j--;
            if (i <= j) {
                entry_t t = arr[i];
                arr[i] = arr[j];
                arr[j] = t;
                i++;
                j--;
            }
        }
        if (k - 1 <= j) hi = j;
        else if (k - 1 >= i) lo = i;
        else break;
    }
    qsort(arr, (size_t)k, sizeof(entry_t), cmp_rank);
}

typedef struct {
    int64_t n;
    const int64_t *rowptr, *col;
    double alpha;
    int64_t num_iterations, iter_topk, final_keep, source_start, source_end, keep_stride;
    int64_t *out_col;
    double *out_val;
    int32_t *out_cnt;
    uint8_t *out_tie;  /* nullable: 1 where a pruning boundary was a near tie */
    double tie_rtol;
    int64_t next_seed; /* shared work counter */
} job_t;

typedef struct {
    job_t *job;
    int64_t touch, state;
    int bad;
} worker_t;

/* After select_topk(arr, m, k) with k < m: is the k-th kept value within rtol of the best
 * value left out?  Such a boundary is where the reference's unordered topk ties may pick
 * differently. */
static int boundary_near_tie(const entry_t *arr, int64_t m, int64_t k, double rtol) {
    if (k <= 0 || k >= m) return 0;
    double kept = arr[k - 1].v, best_out = arr[k].v;
    for (int64_t i = k + 1; i < m; i++)
        if (arr[i].v > best_out) best_out = arr[i].v;
    return kept - best_out <= rtol * kept;
}

static void run_seed(const job_t *jb, int64_t s, double *acc, int64_t *stamp, int64_t *sid,
                     int64_t *touched, entry_t *merged, entry_t *state, int64_t *touch_out,
                     int64_t *state_out) {
    const double oma = 1.0 - jb->alpha;
    int tie = 0;
    int64_t st_n = 1;
    state[0].c = s;
    state[0].v = 1.0;
    for (int64_t it = 0; it < jb->num_iterations; it++) {
        (*sid)++;
        int64_t nt = 0;
        for (int64_t i = 0; i < st_n; i++) {
            int64_t j = state[i].c;
            int64_t b = jb->rowptr[j], e = jb->rowptr[j + 1];
            int64_t deg = e - b;
            double inv = 1.0 / (double)(deg > 0 ? deg : 1);
            double contrib = state[i].v * inv;
            *touch_out += deg;
            for (int64_t p = b; p < e; p++) {
                int64_t c = jb->col[p];
                if (stamp[c] != *sid) {
                    stamp[c] = *sid;
                    acc[c] = 0.0;
                    touched[nt++] = c;
                }
                acc[c] = acc[c] + contrib;
            }
        }
        *state_out += st_n;
        int64_t m = 0;
        int seen_seed = 0;
        for (int64_t t = 0; t < nt; t++) {
            int64_t c = touched[t];
            double v = acc[c] * oma;
            if (c == s) {
                v = v + jb->alpha;
                seen_seed = 1;
            }
            merged[m].c = c;
            merged[m].v = v;
            m++;
        }
        if (!seen_seed) {
            merged[m].c = s;
            merged[m].v = jb->alpha;
            m++;
        }
        int64_t keep = m;
        if (jb->iter_topk > 0 && jb->iter_topk < m) {
            keep = jb->iter_topk;
            select_topk(merged, m, keep);
            tie |= boundary_near_tie(merged, m, keep, jb->tie_rtol);
        }
        memcpy(state, merged, sizeof(entry_t) * (size_t)keep);
        st_n = keep;
        qsort(state, (size_t)st_n, sizeof(entry_t), cmp_col);
    }
    int64_t keep = (jb->final_keep > 0 && jb->final_keep < st_n) ? jb->final_keep : st_n;
    select_topk(state, st_n, keep);
    tie |= boundary_near_tie(state, st_n, keep, jb->tie_rtol);
    if (jb->out_tie) jb->out_tie[s - jb->source_start] = (uint8_t)tie;
    if (keep > jb->keep_stride) keep = jb->keep_stride;
    int64_t base = (s - jb->source_start) * jb->keep_stride;
    for (int64_t i = 0; i < keep; i++) {
        jb->out_col[base + i] = state[i].c;
        jb->out_val[base + i] = state[i].v;
    }
    jb->out_cnt[s - jb->source_start] = (int32_t)keep;
}

static void *worker_main(void *arg) {
    worker_t *w = (worker_t *)arg;
    job_t *jb = w->job;
    int64_t n = jb->n;
    double *acc = (double *)malloc(sizeof(double) * (size_t)n);
    int64_t *stamp = (int64_t *)malloc(sizeof(int64_t) * (size_t)n);
    int64_t *touched = (int64_t *)malloc(sizeof(int64_t) * (size_t)n);
    entry_t *merged = (entry_t *)malloc(sizeof(entry_t) * (size_t)(n + 1));
    entry_t *state = (entry_t *)malloc(sizeof(entry_t) * (size_t)(n + 1));
    if (!acc || !stamp || !touched || !merged || !state) {
        w->bad = 1;
    } else {
        for (int64_t i = 0; i < n; i++) stamp[i] = -1;
        int64_t sid = 0;
        for (;;) {
            int64_t s = __atomic_fetch_add(&jb->next_seed, 1, __ATOMIC_RELAXED);
            if (s >= jb->source_end) break;
            run_seed(jb, s, acc, stamp, &sid, touched, merged, state, &w->touch, &w->state);
        }
    }
    free(acc);
    free(stamp);
    free(touched);
    free(merged);
    free(state);
    return NULL;
}

/* Returns 0 on success, -1 on allocation failure.  stats[0] = adjacency entries read
 * (sum of deg(j) over expanded state entries), stats[1] = state entries expanded. */
int64_t ngt_oracle_appnp(int64_t n, const int64_t *rowptr, const int64_t *col, double alpha,
                         int64_t num_iterations, int64_t iter_topk, int64_t final_keep,
                         int64_t source_start, int64_t source_end, int64_t keep_stride,
                         int64_t *out_col, double *out_val, int32_t *out_cnt, uint8_t *out_tie,
                         double tie_rtol, int nthreads, int64_t *stats) {
    if (stats) {
        stats[0] = 0;
        stats[1] = 0;
    }
    if (n <= 0 || source_end <= source_start) return 0;
    job_t jb = {n, rowptr, col, alpha, num_iterations, iter_topk, final_keep, source_start,
                source_end, keep_stride, out_col, out_val, out_cnt, out_tie, tie_rtol,
                source_start};
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    worker_t workers[256];
    pthread_t tids[256];
    for (int t = 0; t < nthreads; t++) {
        workers[t].job = &jb;
        workers[t].touch = 0;
        workers[t].state = 0;
        workers[t].bad = 0;
    }
    for (int t = 1; t < nthreads; t++) pthread_create(&tids[t], NULL, worker_main, &workers[t]);
    worker_main(&workers[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(tids[t], NULL);
    int bad = 0;
    for (int t = 0; t < nthreads; t++) {
        bad |= workers[t].bad;
        if (stats) {
            stats[0] += workers[t].touch;
            stats[1] += workers[t].state;
        }
    }
    return bad ? -1 : 0;
}
