/*
 * CPU oracle for push-based approximate personalised PageRank (the `torch_geometric` backend).
 * TEST INFRASTRUCTURE ONLY: built by oracle/Makefile, loaded by oracle/ppr.py.
 *
 * The reference's default backend, `personal_pagerank_torch_geometric`
 * (NeutronGT/core/ppr_backends/torch_geometric_backend.py:5-30), calls PyG 2.4.0's
 * `torch_geometric.utils.ppr.get_ppr(edge_index, alpha, eps)`, which is not vendored in the
 * reference.  This file restates the published method that function implements: the push
 * procedure of Andersen, Chung & Lang (2006), in the variant of Bojchevski et al. (PPRGo, 2020),
 * with a LIFO work list, per seed s over the row-stochastic walk P = D^-1 A of the CSR graph:
 *
 *   p = {s: 0}, r = {s: alpha}, stack = [s]
 *   while stack:  u = pop()
 *       res = r[u];  p[u] += res (entry created at u's first pop);  r[u] = 0
 *       for v in adj(u) in CSR order:
 *           r[v] += ((1 - alpha) * res) / deg(u)
 *           if r[v] >= (alpha * eps) * deg(v) and v is not on the stack:  push(v)
 *
 * Output per seed: the entries of p in insertion order (the seed first, then first-pop order).
 * The dispatcher then keeps the top `topk` by value when there are more
 * (torch_geometric_backend.py:19-28); the reference breaks ties in torch.topk's unspecified
 * order, this restatement by ascending node id, and emits the kept entries by (value desc,
 * node asc), as torch.topk(sorted=True) orders them.  Rows with at most topk entries stay in
 * insertion order, as the reference leaves them.
 *
 * fp64 throughout, every multiply, divide and add a separate IEEE round-to-nearest operation
 * (-ffp-contract=off), so the CUDA kernel reproduces every value bit for bit.  For an undirected
 * graph the result satisfies 0 <= pi_s(v) - p(v) < eps * deg(v) for the exact PPR pi_s of
 * teleport probability alpha (the push invariant with every residual below alpha eps deg).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int64_t n;
    const int64_t *rowptr;
    const int32_t *col;
    double alpha, eps;
    int64_t s0, s1, topk;
    int64_t *cnt;      /* [s1 - s0] kept entries per seed */
    int64_t *idx;      /* [s1 - s0][topk] */
    double *val;       /* [s1 - s0][topk] */
    int64_t next;      /* shared work counter */
    pthread_mutex_t mu;
    int64_t pushes, touched_edges, failed;
} job_t;

static int64_t take(job_t *j) {
    pthread_mutex_lock(&j->mu);
    const int64_t s = j->next++;
    pthread_mutex_unlock(&j->mu);
    return s;
}

static void *worker(void *arg) {
    job_t *j = (job_t *)arg;
    const int64_t n = j->n;
    double *r = calloc((size_t)n, sizeof(double)), *pv = calloc((size_t)n, sizeof(double));
    uint8_t *fl = calloc((size_t)n, 1);   /* bit 0: touched (in r), bit 1: in p, bit 2: on the stack */
    int64_t *stack = malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    int64_t *plist = malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    int64_t *touched = malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    int64_t pushes = 0, tedges = 0;
    if (!r || !pv || !fl || !stack || !plist || !touched) {
        pthread_mutex_lock(&j->mu);
        j->failed = 1;
        pthread_mutex_unlock(&j->mu);
        goto done;
    }
    const double alpha_eps = j->alpha * j->eps, keep = 1.0 - j->alpha;
    for (;;) {
        const int64_t s = take(j);
        if (s >= j->s1) break;
        int64_t sp = 0, np = 0, nt = 0;
        r[s] = j->alpha;
        fl[s] = 1 | 2 | 4;
        touched[nt++] = s;
        plist[np++] = s;
        pv[s] = 0.0;
        stack[sp++] = s;
        while (sp > 0) {
            const int64_t u = stack[--sp];
            fl[u] &= (uint8_t)~4u;
            const double res = r[u];
            if (fl[u] & 2) {
                pv[u] = pv[u] + res;
            } else {
                pv[u] = res;
                fl[u] |= 2;
                plist[np++] = u;
            }
            r[u] = 0.0;
            pushes++;
            const int64_t b = j->rowptr[u], e = j->rowptr[u + 1];
            if (e == b) continue;
            const double val = (keep * res) / (double)(e - b);
            tedges += e - b;
            for (int64_t q = b; q < e; q++) {
                const int64_t v = j->col[q];
                if (fl[v] & 1) {
                    r[v] = r[v] + val;
                } else {
                    r[v] = val;
                    fl[v] |= 1;
                    touched[nt++] = v;
                }
                const double thr = alpha_eps * (double)(j->rowptr[v + 1] - j->rowptr[v]);
                if (r[v] >= thr && !(fl[v] & 4)) {
                    fl[v] |= 4;
                    stack[sp++] = v;
                }
            }
        }
        /* selection */
        const int64_t o = s - j->s0, k = j->topk;
        int64_t *oi = j->idx + o * k;
        double *ov = j->val + o * k;
        if (np <= k) {
            for (int64_t i = 0; i < np; i++) {
                oi[i] = plist[i];
                ov[i] = pv[plist[i]];
            }
            j->cnt[o] = np;
        } else {
            for (int64_t t = 0; t < k; t++) {   /* k rounds of arg-best by (value desc, node asc) */
                int64_t best = -1;
                for (int64_t i = 0; i < np; i++) {
                    const int64_t c = plist[i];
                    if (c < 0) continue;
                    if (best < 0 || pv[c] > pv[plist[best]] || (pv[c] == pv[plist[best]] && c < plist[best])) best = i;
                }
                oi[t] = plist[best];
                ov[t] = pv[plist[best]];
                plist[best] = -1 - plist[best];   /* taken */
            }
            for (int64_t i = 0; i < np; i++)
                if (plist[i] < 0) plist[i] = -1 - plist[i];
            j->cnt[o] = k;
        }
        for (int64_t i = 0; i < nt; i++) {
            const int64_t v = touched[i];
            r[v] = 0.0;
            pv[v] = 0.0;
            fl[v] = 0;
        }
    }
done:
    pthread_mutex_lock(&j->mu);
    j->pushes += pushes;
    j->touched_edges += tedges;
    pthread_mutex_unlock(&j->mu);
    free(r);
    free(pv);
    free(fl);
    free(stack);
    free(plist);
    free(touched);
    return NULL;
}

/* Returns 0 on success; stats (nullable) receives {pushes, adjacency entries read}. */
int ngt_oracle_ppr_push(int64_t n, const int64_t *rowptr, const int32_t *col, double alpha, double eps,
                        int64_t seed_start, int64_t seed_end, int64_t topk, int64_t *cnt, int64_t *idx, double *val,
                        int nthreads, int64_t *stats) {
    if (n < 0 || seed_start < 0 || seed_end > n || seed_start > seed_end || topk <= 0) return 1;
    job_t j;
    memset(&j, 0, sizeof(j));
    j.n = n;
    j.rowptr = rowptr;
    j.col = col;
    j.alpha = alpha;
    j.eps = eps;
    j.s0 = seed_start;
    j.s1 = seed_end;
    j.topk = topk;
    j.cnt = cnt;
    j.idx = idx;
    j.val = val;
    j.next = seed_start;
    pthread_mutex_init(&j.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int t = 0; t < nthreads; t++) pthread_create(&th[t], NULL, worker, &j);
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&j.mu);
    if (stats) {
        stats[0] = j.pushes;
        stats[1] = j.touched_edges;
    }
    return j.failed ? 2 : 0;
}
