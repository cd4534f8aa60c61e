// APPNP personalised PageRank with per-iteration top-k (sm_100a).
//
// Replaces the propagation loop of `personal_pagerank_appnp`
// (NeutronGT/core/ppr_backends/appnp_backend.py:259-305).  The reference runs, per
// iteration and per batch of seeds, a cuSPARSE SpGEMM with a fresh handle and three
// temporary buffers (csrc/cusparse_spgemm.cu:65-267), a torch.unique + scatter_add_ merge
// (:68-77), and a Python loop calling torch.topk per row (:102-140).  Seeds are
// independent, so here one CTA owns one seed's row for all iterations and the row never
// leaves the chip between steps:
//
//   pruned mode (iter_topk > 0, the scripts' setting): the row's state has <= k entries and
//   its expansion sum_j contrib_j * e_adj(j) is a k-way merge of the state's adjacency lists
//   (CSR rows with ascending columns, as the reference's CSR writer produces them): the lists
//   are staged in shared memory (read in place from global memory when they do not fit),
//   every thread owns a column range (split at quantiles of the longest list) and merges its
//   part of every list, adding each column's contributions in list order; the teleport is
//   added and the top-k is selected from per-thread register lists, merged per warp with
//   shuffles and then across warps by one warp.
//
//   dense mode (iter_topk <= 0): the state is a dense vector of n doubles per CTA in the
//   workspace and each step pulls over the in-adjacency (transpose CSR).
//
// Canonical arithmetic (identical to oracle/appnp_oracle.c, bit for bit): fp64;
// contrib_j = state_j * (1 / max(deg_j, 1)); contributions to a column are added in
// ascending source column (pruned: the merge visits the state's lists in column order and a
// repeated edge adds its contribution once per copy; dense: the pull walks in-neighbours in
// ascending order); value = acc * (1 - alpha) [+ alpha at the seed]; ranking by
// (value desc, column asc).  All products/sums use explicit round-to-nearest intrinsics so
// no FMA contraction can change a bit.
#include <climits>

#include "common.cuh"

namespace ngt {
namespace {

constexpr int kPprThreads = 256;
constexpr int kPprWarps = kPprThreads / 32;
constexpr int kMaxCtas = 148 * 4;
constexpr int kStageCap = 12288;  // staged adjacency entries (48 KiB)

struct Cand {
    double v;
    int c;
};

__device__ __forceinline__ bool ranks_before(double va, int ca, double vb, int cb) {
    return va > vb || (va == vb && ca < cb);
}


// Per-thread sorted list of its best KMAX candidates (registers, static indexing only).
template <int KMAX>
struct TopList {
    double v[KMAX];
    int c[KMAX];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < KMAX; i++) {
            v[i] = -1.0;
            c[i] = 0x7fffffff;
        }
    }
    __device__ __forceinline__ void offer(double x, int col) {
        if (!ranks_before(x, col, v[KMAX - 1], c[KMAX - 1])) return;
        v[KMAX - 1] = x;
        c[KMAX - 1] = col;
#pragma unroll
        for (int i = KMAX - 1; i > 0; i--) {
            if (ranks_before(v[i], c[i], v[i - 1], c[i - 1])) {
                const double tv = v[i];
                v[i] = v[i - 1];
                v[i - 1] = tv;
                const int tc = c[i];
                c[i] = c[i - 1];
                c[i - 1] = tc;
            }
        }
    }
    __device__ __forceinline__ void pop() {
#pragma unroll
        for (int i = 0; i < KMAX - 1; i++) {
            v[i] = v[i + 1];
            c[i] = c[i + 1];
        }
        v[KMAX - 1] = -1.0;
        c[KMAX - 1] = 0x7fffffff;
    }
};

struct MergeSmem {
    double wv[kPprWarps];
    int wc[kPprWarps];
    int wt[kPprWarps];
    int winner;
};

// Block-wide merge of the per-thread lists: writes up to k entries in rank order to
// (out_c, out_v) in shared memory and returns the count (same value in every thread).
template <int KMAX>
__device__ int block_merge_topk(TopList<KMAX> &L, int k, MergeSmem &ms, int *out_c, double *out_v) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int count = 0;
    for (int r = 0; r < k; r++) {
        double bv = L.v[0];
        int bc = L.c[0];
        int bt = tid;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oc = __shfl_xor_sync(0xffffffffu, bc, off);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, off);
            if (ranks_before(ov, oc, bv, bc)) {
                bv = ov;
                bc = oc;
                bt = ot;
            }
        }
        if (lane == 0) {
            ms.wv[warp] = bv;
            ms.wc[warp] = bc;
            ms.wt[warp] = bt;
        }
        __syncthreads();
        if (tid == 0) {
            double gv = ms.wv[0];
            int gc = ms.wc[0], gt = ms.wt[0];
            for (int w = 1; w < kPprWarps; w++)
                if (ranks_before(ms.wv[w], ms.wc[w], gv, gc)) {
                    gv = ms.wv[w];
                    gc = ms.wc[w];
                    gt = ms.wt[w];
                }
            if (gv < 0.0) {
                ms.winner = -1;
            } else {
                ms.winner = gt;
                out_c[r] = gc;
                out_v[r] = gv;
            }
        }
        __syncthreads();
        const int win = ms.winner;
        if (win < 0) break;
        if (tid == win) L.pop();
        count = r + 1;
        __syncthreads();
    }
    return count;
}

// Exact top-k of the block's per-thread lists without block-wide barriers per round: every
// warp extracts its k best with shuffles (k rounds of a warp arg-max), warp 0 merges the
// warps' lists the same way.  Writes up to k entries in rank order to (out_c, out_v) and
// returns the count (valid in every thread after the trailing barrier).
template <int KMAX>
__device__ int block_topk(TopList<KMAX> &L, int k, double *wv, int *wc, int *count_out, int *out_c, double *out_v) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int r = 0; r < k; r++) {   // warp level
        double bv = L.v[0];
        int bc = L.c[0], bt = lane;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oc = __shfl_xor_sync(0xffffffffu, bc, off);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, off);
            if (ranks_before(ov, oc, bv, bc)) {
                bv = ov;
                bc = oc;
                bt = ot;
            }
        }
        if (lane == bt) L.pop();
        if (lane == 0) {
            wv[warp * KMAX + r] = bv;
            wc[warp * KMAX + r] = bc;
        }
    }
    __syncthreads();
    if (warp == 0) {   // lane takes candidates lane, lane + 32, ... of the warps' lists laid end to end
        constexpr int PER = (kPprWarps * KMAX + 31) / 32;
        TopList<PER> M;
        M.init();
        for (int f = lane; f < kPprWarps * k; f += 32) M.offer(wv[(f / k) * KMAX + f % k], wc[(f / k) * KMAX + f % k]);
        int cnt = 0;
        for (int r = 0; r < k; r++) {
            double bv = M.v[0];
            int bc = M.c[0], bt = lane;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const double ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oc = __shfl_xor_sync(0xffffffffu, bc, off);
                const int ot = __shfl_xor_sync(0xffffffffu, bt, off);
                if (ranks_before(ov, oc, bv, bc)) {
                    bv = ov;
                    bc = oc;
                    bt = ot;
                }
            }
            if (bv < 0.0) break;   // fewer than k candidates
            if (lane == bt) M.pop();
            if (lane == 0) {
                out_c[r] = bc;
                out_v[r] = bv;
            }
            cnt = r + 1;
        }
        if (lane == 0) *count_out = cnt;
    }
    __syncthreads();
    return *count_out;
}

struct PrunedSmem {
    int stage[kStageCap];   // the state's adjacency lists, concatenated, when they fit
    int st_col[32];         // state sorted by column (list order = canonical add order)
    double st_val[32];
    int sel_col[32];        // last selection in rank order
    double sel_val[32];
    double contrib[32];     // state value / max(degree, 1) per list
    int64_t lbeg[32];       // list start in col[]
    int llen[32];
    int wbeg[32];           // this column window's part of each list: [wbeg, wbeg + wlen)
    int wlen[32];
    int loff[33];           // window part start in stage[]
    int bounds[kPprThreads + 1];
    double wv[kPprWarps * 32];
    int wc[kPprWarps * 32];
    int st_n, staged, longest, total, cnt, seed;
};

// First index of a sorted list whose column is >= x.
template <typename Rd>
__device__ __forceinline__ int lower_bound(const Rd &rd, int len, int x) {
    int lo = 0, hi = len;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (rd(mid) < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Merge this thread's column range [lo, hi) of the state's lists into L.  `rd(i, p)` reads
// entry p of list i.  Each column's contributions are added in list order, starting at 0.0.
template <int KMAX, typename Rd>
__device__ __forceinline__ void merge_range(const PrunedSmem &S, const Rd &rd, int st_n, int lo, int hi, int seed,
                                            double alpha, double oma, TopList<KMAX> &L) {
    int p[KMAX], e[KMAX], head[KMAX];
#pragma unroll
    for (int i = 0; i < KMAX; i++) {
        p[i] = e[i] = 0;
        head[i] = INT_MAX;
        if (i < st_n) {
            const int len = S.wlen[i];
            // lists whose span misses [lo, hi) need no search
            if (len > 0 && rd(i, len - 1) >= lo && rd(i, 0) < hi) {
                p[i] = lower_bound([&](int q) { return rd(i, q); }, len, lo);
                e[i] = hi == INT_MAX ? len : lower_bound([&](int q) { return rd(i, q); }, len, hi);
                if (p[i] < e[i]) head[i] = rd(i, p[i]);
            }
        }
    }
    bool seed_seen = false;
    for (;;) {
        int v = INT_MAX;
#pragma unroll
        for (int i = 0; i < KMAX; i++) v = min(v, head[i]);
        if (v == INT_MAX) break;
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < KMAX; i++) {
            while (head[i] == v) {   // a repeated edge adds once per copy
                acc = __dadd_rn(acc, S.contrib[i]);
                p[i]++;
                head[i] = p[i] < e[i] ? rd(i, p[i]) : INT_MAX;
            }
        }
        double val = __dmul_rn(acc, oma);
        if (v == seed) {
            val = __dadd_rn(val, alpha);
            seed_seen = true;
        }
        L.offer(val, v);
    }
    // the teleport target always exists in the merged row
    if (!seed_seen && seed >= lo && seed < hi) L.offer(__dadd_rn(__dmul_rn(0.0, oma), alpha), seed);
}

// ------------------------------------------------------------------------------------
// pruned mode
// ------------------------------------------------------------------------------------
template <int KMAX>
__global__ void __launch_bounds__(kPprThreads)
    ppr_pruned_kernel(int n, const int64_t *__restrict__ rowptr, const int *__restrict__ col,
                      double alpha, double oma, int iters, int iter_topk, int final_keep,
                      int source_start, int source_end, int keep_stride, int64_t *__restrict__ out_col,
                      float *__restrict__ out_val, double *__restrict__ out_val64,
                      int *__restrict__ out_cnt, int *__restrict__ seed_counter) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrunedSmem &S = *reinterpret_cast<PrunedSmem *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (;;) {
        if (tid == 0) S.seed = atomicAdd(seed_counter, 1) + source_start;
        __syncthreads();
        const int seed = S.seed;
        if (seed >= source_end) break;
        if (tid == 0) {
            S.st_n = 1;
            S.st_col[0] = seed;
            S.st_val[0] = 1.0;
            S.sel_col[0] = seed;
            S.sel_val[0] = 1.0;
        }
        __syncthreads();
        for (int it = 0; it < iters; it++) {
            const int st_n = S.st_n;
            if (warp == 0) {   // list bounds, contributions, the longest list, total length
                int len = 0;
                if (lane < st_n) {
                    const int j = S.st_col[lane];
                    const int64_t b = rowptr[j], e = rowptr[j + 1];
                    len = (int)(e - b);
                    S.lbeg[lane] = b;
                    S.llen[lane] = len;
                    S.contrib[lane] = __dmul_rn(S.st_val[lane], __ddiv_rn(1.0, (double)(len > 0 ? len : 1)));
                }
                int tot = len, best = len, bi = lane;   // longest list (first on ties)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    tot += __shfl_xor_sync(0xffffffffu, tot, o);
                    const int ob = __shfl_xor_sync(0xffffffffu, best, o), oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ob > best || (ob == best && oi < bi)) {
                        best = ob;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    S.total = tot;
                    S.longest = bi;
                }
            }
            __syncthreads();
            TopList<KMAX> L;
            L.init();
            // Column windows: one when the lists fit the stage; otherwise the longest list is cut
            // into equal parts and every list contributes its entries inside each part's column
            // range, so a window holds about stage * 3 / 4 entries.
            const int li = S.longest, llen = S.llen[li];
            const int nwin = S.total <= kStageCap ? 1 : (S.total + (kStageCap * 3 / 4) - 1) / (kStageCap * 3 / 4);
            for (int w = 0; w < nwin; w++) {
                const int c_lo = w == 0 ? INT_MIN : __ldg(col + S.lbeg[li] + (int)(((int64_t)w * llen) / nwin));
                const int c_hi = w + 1 == nwin ? INT_MAX : __ldg(col + S.lbeg[li] + (int)(((int64_t)(w + 1) * llen) / nwin));
                if (warp == 0) {   // this window's part of every list and its place in the stage
                    int wb = 0, wl = 0;
                    if (lane < st_n) {
                        const int *lst = col + S.lbeg[lane];
                        const int len = S.llen[lane];
                        if (nwin == 1) {
                            wl = len;
                        } else {
                            wb = c_lo == INT_MIN ? 0 : lower_bound([&](int q) { return __ldg(lst + q); }, len, c_lo);
                            const int we = c_hi == INT_MAX ? len : lower_bound([&](int q) { return __ldg(lst + q); }, len, c_hi);
                            wl = we - wb;
                        }
                        S.wbeg[lane] = wb;
                        S.wlen[lane] = wl;
                    }
                    int incl = wl;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int t = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += t;
                    }
                    const int total = __shfl_sync(0xffffffffu, incl, 31);
                    if (lane < st_n) S.loff[lane] = incl - wl;
                    if (lane == 0) {
                        S.loff[st_n] = total;
                        S.staged = total <= kStageCap;
                    }
                }
                __syncthreads();
                const bool staged = S.staged;
                if (staged) {
                    for (int i = 0; i < st_n; i++) {
                        const int len = S.wlen[i], o = S.loff[i];
                        const int *src = col + S.lbeg[i] + S.wbeg[i];
                        for (int q = tid; q < len; q += kPprThreads) S.stage[o + q] = __ldg(src + q);
                    }
                }
                __syncthreads();
                {   // thread column ranges inside the window: quantiles of the longest list's part
                    const int len = S.wlen[li];
                    if (tid == 0) {
                        S.bounds[0] = c_lo;
                        S.bounds[kPprThreads] = c_hi;
                    } else {
                        const int q = (int)(((int64_t)tid * len) / kPprThreads);
                        S.bounds[tid] = q >= len ? c_hi
                                                 : (staged ? S.stage[S.loff[li] + q] : __ldg(col + S.lbeg[li] + S.wbeg[li] + q));
                    }
                }
                __syncthreads();
                const int lo = S.bounds[tid], hi = S.bounds[tid + 1];
                if (lo < hi) {
                    if (staged) {
                        int base[KMAX];
#pragma unroll
                        for (int i = 0; i < KMAX; i++) base[i] = i < st_n ? S.loff[i] : 0;
                        merge_range<KMAX>(S, [&](int i, int q) { return S.stage[base[i] + q]; }, st_n, lo, hi, seed, alpha,
                                          oma, L);
                    } else {   // a window still too large for the stage: read the lists in place
                        merge_range<KMAX>(S, [&](int i, int q) { return __ldg(col + S.lbeg[i] + S.wbeg[i] + q); }, st_n,
                                          lo, hi, seed, alpha, oma, L);
                    }
                }
                __syncthreads();   // the stage is refilled by the next window
            }
            const int cnt = block_topk<KMAX>(L, iter_topk, S.wv, S.wc, &S.cnt, S.sel_col, S.sel_val);
            if (warp == 0) {   // next state: the selection sorted by column (distinct columns)
                int c = INT_MAX;
                double v = 0.0;
                if (lane < cnt) {
                    c = S.sel_col[lane];
                    v = S.sel_val[lane];
                }
                int rank = 0;
                for (int o = 0; o < cnt; o++) rank += __shfl_sync(0xffffffffu, c, o) < c;
                if (lane < cnt) {
                    S.st_col[rank] = c;
                    S.st_val[rank] = v;
                }
                if (lane == 0) S.st_n = cnt;
            }
            __syncthreads();
        }
        if (tid == 0) {
            const int slot = seed - source_start;
            int keep = S.st_n;
            if (final_keep > 0 && final_keep < keep) keep = final_keep;
            if (keep > keep_stride) keep = keep_stride;
            for (int i = 0; i < keep; i++) {
                out_col[(size_t)slot * keep_stride + i] = S.sel_col[i];
                out_val[(size_t)slot * keep_stride + i] = (float)S.sel_val[i];
                if (out_val64) out_val64[(size_t)slot * keep_stride + i] = S.sel_val[i];
            }
            out_cnt[slot] = keep;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------
// dense mode (no pruning)
// ------------------------------------------------------------------------------------
struct DenseSmem {
    int sel_col[32];
    double sel_val[32];
    int seed;
    MergeSmem ms;
};

template <int KMAX>
__global__ void __launch_bounds__(kPprThreads)
    ppr_dense_kernel(int n, const int64_t *__restrict__ rowptr, const int64_t *__restrict__ in_rowptr,
                     const int *__restrict__ in_col, double alpha, double oma, int iters,
                     int final_keep, int source_start, int source_end, int keep_stride,
                     int64_t *__restrict__ out_col, float *__restrict__ out_val,
                     double *__restrict__ out_val64, int *__restrict__ out_cnt,
                     int *__restrict__ seed_counter, double *__restrict__ gx,
                     unsigned char *__restrict__ gp) {
    __shared__ DenseSmem S;
    const int tid = threadIdx.x;
    double *xa = gx + (size_t)blockIdx.x * 2 * n;
    double *xb = xa + n;
    unsigned char *pa = gp + (size_t)blockIdx.x * 2 * n;
    unsigned char *pb = pa + n;
    for (;;) {
        if (tid == 0) S.seed = atomicAdd(seed_counter, 1) + source_start;
        __syncthreads();
        const int seed = S.seed;
        if (seed >= source_end) break;
        for (int c = tid; c < n; c += kPprThreads) {
            xa[c] = c == seed ? 1.0 : 0.0;
            pa[c] = c == seed;
        }
        __syncthreads();
        double *x = xa, *y = xb;
        unsigned char *px = pa, *py = pb;
        for (int it = 0; it < iters; it++) {
            for (int c = tid; c < n; c += kPprThreads) {
                double acc = 0.0;
                bool pres = false;
                for (int64_t p = in_rowptr[c]; p < in_rowptr[c + 1]; p++) {
                    const int j = in_col[p];
                    if (!px[j]) continue;
                    const int64_t deg = rowptr[j + 1] - rowptr[j];
                    const double inv = __ddiv_rn(1.0, (double)(deg > 0 ? deg : 1));
                    acc = __dadd_rn(acc, __dmul_rn(x[j], inv));
                    pres = true;
                }
                double v = __dmul_rn(acc, oma);
                if (c == seed) {
                    v = __dadd_rn(v, alpha);
                    pres = true;
                }
                y[c] = v;
                py[c] = pres;
            }
            __syncthreads();
            double *t = x; x = y; y = t;
            unsigned char *tp = px; px = py; py = tp;
        }
        TopList<KMAX> L;
        L.init();
        for (int c = tid; c < n; c += kPprThreads)
            if (px[c]) L.offer(x[c], c);
        const int cnt = block_merge_topk<KMAX>(L, final_keep, S.ms, S.sel_col, S.sel_val);
        if (tid == 0) {
            const int slot = seed - source_start;
            const int keep = cnt < keep_stride ? cnt : keep_stride;
            for (int i = 0; i < keep; i++) {
                out_col[(size_t)slot * keep_stride + i] = S.sel_col[i];
                out_val[(size_t)slot * keep_stride + i] = (float)S.sel_val[i];
                if (out_val64) out_val64[(size_t)slot * keep_stride + i] = S.sel_val[i];
            }
            out_cnt[slot] = keep;
        }
        __syncthreads();
    }
}

struct PprWs {
    int *counter;
    double *gx;
    unsigned char *gp;
    size_t used;
};

PprWs carve_ppr(void *base, int64_t n, int64_t max_degree, int64_t iter_topk, int64_t num_seeds) {
    PprWs w{};
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        off = (off + 255) & ~size_t(255);
        char *r = p ? p + off : nullptr;
        off += bytes;
        return r;
    };
    const int64_t ctas = num_seeds < kMaxCtas ? (num_seeds > 0 ? num_seeds : 1) : kMaxCtas;
    w.counter = reinterpret_cast<int *>(take(sizeof(int)));
    (void)max_degree;   // the pruned mode needs no per-CTA tables
    if (iter_topk <= 0) {
        w.gx = reinterpret_cast<double *>(take(sizeof(double) * (size_t)(ctas * 2 * n)));
        w.gp = reinterpret_cast<unsigned char *>(take((size_t)(ctas * 2 * n)));
    }
    w.used = off;
    return w;
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_ppr_workspace_size(int64_t n, int64_t max_degree, int64_t iter_topk,
                                      int64_t num_seeds, size_t *bytes) {
    if (n < 0 || max_degree < 0 || num_seeds < 0 || !bytes) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    *bytes = carve_ppr(nullptr, n, max_degree, iter_topk, num_seeds).used;
    return NGT_OK;
}

extern "C" int ngt_ppr_appnp_topk(int64_t n, const int64_t *rowptr, const int32_t *col,
                                  const int64_t *in_rowptr, const int32_t *in_col, double alpha,
                                  int64_t num_iterations, int64_t iter_topk, int64_t final_keep,
                                  int64_t source_start, int64_t source_end, int64_t max_degree,
                                  int64_t keep_stride, int64_t *out_col, float *out_val,
                                  double *out_val64, int32_t *out_cnt, int32_t *info,
                                  void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || num_iterations < 1 || source_start < 0 || source_end < source_start ||
        source_end > n || keep_stride < 1 || !rowptr || !out_col || !out_val || !out_cnt || !info)
        return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || num_iterations >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    const int64_t num_seeds = source_end - source_start;
    const bool dense = iter_topk <= 0;
    const int64_t k = dense ? final_keep : iter_topk;
    if (k <= 0 || k > 32) return NGT_ERR_UNSUPPORTED;  // register top-k holds at most 32
    if (dense && (!in_rowptr || (n > 0 && !in_col))) return NGT_ERR_INVALID_ARGUMENT;
    PprWs w = carve_ppr(workspace, n, max_degree, iter_topk, num_seeds);
    if (workspace == nullptr || workspace_bytes < w.used) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(info, 0, sizeof(int32_t), st);
    cudaMemsetAsync(w.counter, 0, sizeof(int), st);
    if (num_seeds == 0) return NGT_OK;
    const int ctas = (int)(num_seeds < kMaxCtas ? num_seeds : kMaxCtas);
    const double oma = 1.0 - alpha;
    const int fk = (int)(final_keep > 0 ? final_keep : 0);
#define NGT_PPR_LAUNCH(KM)                                                                         \
    if (dense) {                                                                                   \
        ppr_dense_kernel<KM><<<ctas, kPprThreads, 0, st>>>(                                        \
            (int)n, rowptr, in_rowptr, in_col, alpha, oma, (int)num_iterations, (int)k,            \
            (int)source_start, (int)source_end, (int)keep_stride, out_col, out_val, out_val64,     \
            out_cnt, w.counter, w.gx, w.gp);                                                       \
    } else {                                                                                       \
        const size_t sm = sizeof(PrunedSmem);                                                      \
        cudaFuncSetAttribute(ppr_pruned_kernel<KM>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                             (int)sm);                                                             \
        ppr_pruned_kernel<KM><<<ctas, kPprThreads, sm, st>>>(                                      \
            (int)n, rowptr, col, alpha, oma, (int)num_iterations, (int)k, fk, (int)source_start,   \
            (int)source_end, (int)keep_stride, out_col, out_val, out_val64, out_cnt, w.counter);   \
    }                                                                                              \
    NGT_CHECK_LAUNCH();                                                                            \
    return NGT_OK;
    if (k <= 8) {
        NGT_PPR_LAUNCH(8)
    } else if (k <= 16) {
        NGT_PPR_LAUNCH(16)
    } else {
        NGT_PPR_LAUNCH(32)
    }
#undef NGT_PPR_LAUNCH
}
