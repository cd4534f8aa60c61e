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
//   pruned mode (iter_topk > 0, the scripts' setting): the row's state has <= k entries;
//   its expansion sum_j contrib_j * e_adj(j) is accumulated in an open-addressing hash
//   table (shared memory, or a per-CTA region of the workspace when the expansion of a
//   hub-heavy state does not fit), the teleport is added, and the top-k is selected with
//   per-thread register lists merged by a block tournament.
//
//   dense mode (iter_topk <= 0): the state is a dense vector of n doubles per CTA in the
//   workspace and each step pulls over the in-adjacency (transpose CSR).
//
// Canonical arithmetic (identical to oracle/appnp_oracle.c, bit for bit): fp64;
// contrib_j = state_j * (1 / max(deg_j, 1)); contributions to a column are added in
// ascending source column (pruned: the state entries are expanded one at a time with a
// barrier between them, and within one entry every column is distinct — or, for repeated
// edges, receives the same value twice, which commutes; dense: the pull walks in-neighbours
// in ascending order); value = acc * (1 - alpha) [+ alpha at the seed]; ranking by
// (value desc, column asc).  All products/sums use explicit round-to-nearest intrinsics so
// no FMA contraction can change a bit.
#include "common.cuh"

namespace ngt {
namespace {

constexpr int kPprThreads = 256;
constexpr int kPprWarps = kPprThreads / 32;
constexpr int kMaxCtas = 148 * 4;
constexpr int kSmemSlots = 4096;  // 48 KiB of keys + values
constexpr int kEmpty = -1;

struct Cand {
    double v;
    int c;
};

__device__ __forceinline__ bool ranks_before(double va, int ca, double vb, int cb) {
    return va > vb || (va == vb && ca < cb);
}

__device__ __forceinline__ uint32_t hash_slot(int c, uint32_t mask) {
    return ((uint32_t)c * 2654435761u) & mask;
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

struct PrunedSmem {
    int keys[kSmemSlots];
    double vals[kSmemSlots];
    int touched[kSmemSlots / 2];  // slots claimed this iteration (clear + scan list)
    int ntouched;
    int st_col[32];      // state sorted by column (expansion order)
    double st_val[32];
    int sel_col[32];     // last selection in rank order
    double sel_val[32];
    int st_n;
    int64_t lsum;
    int seed;
    MergeSmem ms;
};

// ------------------------------------------------------------------------------------
// pruned mode
// ------------------------------------------------------------------------------------
template <int KMAX>
__global__ void __launch_bounds__(kPprThreads)
    ppr_pruned_kernel(int n, const int64_t *__restrict__ rowptr, const int *__restrict__ col,
                      double alpha, double oma, int iters, int iter_topk, int final_keep,
                      int source_start, int source_end, int keep_stride, int64_t *__restrict__ out_col,
                      float *__restrict__ out_val, double *__restrict__ out_val64,
                      int *__restrict__ out_cnt, int *__restrict__ info, int *__restrict__ seed_counter,
                      int *__restrict__ gkeys, double *__restrict__ gvals, int *__restrict__ gtouched,
                      int64_t gcap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrunedSmem &S = *reinterpret_cast<PrunedSmem *>(smem_raw);
    const int tid = threadIdx.x;
    int *my_gkeys = gkeys ? gkeys + (size_t)blockIdx.x * gcap : nullptr;
    double *my_gvals = gvals ? gvals + (size_t)blockIdx.x * gcap : nullptr;
    int *my_gtouched = gtouched ? gtouched + (size_t)blockIdx.x * (gcap / 2) : nullptr;
    // tables start empty (the host clears the workspace regions); after every iteration
    // only the claimed slots are reset, so clearing and scanning cost O(unique columns)
    for (int s = tid; s < kSmemSlots; s += kPprThreads) {
        S.keys[s] = kEmpty;
        S.vals[s] = 0.0;
    }
    if (tid == 0) S.ntouched = 0;
    __syncthreads();

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
        bool overflow = false;
        for (int it = 0; it < iters && !overflow; it++) {
            // expansion size of this step
            if (tid == 0) {
                int64_t l = 0;
                for (int i = 0; i < S.st_n; i++) l += rowptr[S.st_col[i] + 1] - rowptr[S.st_col[i]];
                S.lsum = l;
            }
            __syncthreads();
            const int64_t need = 2 * (S.lsum + 1);
            int *keys, *touched;
            double *vals;
            uint32_t cap = 64;
            while ((int64_t)cap < need) cap <<= 1;
            if ((int64_t)cap <= kSmemSlots) {
                keys = S.keys;
                vals = S.vals;
                touched = S.touched;
            } else if (my_gkeys != nullptr && (int64_t)cap <= gcap) {
                keys = my_gkeys;
                vals = my_gvals;
                touched = my_gtouched;
            } else {
                overflow = true;
                break;
            }
            const uint32_t mask = cap - 1;
            const int st_n = S.st_n;
            for (int i = 0; i < st_n; i++) {
                const int j = S.st_col[i];
                const int64_t b = rowptr[j], e = rowptr[j + 1];
                const int64_t deg = e - b;
                const double inv = __ddiv_rn(1.0, (double)(deg > 0 ? deg : 1));
                const double contrib = __dmul_rn(S.st_val[i], inv);
                for (int64_t p = b + tid; p < e; p += kPprThreads) {
                    const int c = __ldg(col + p);
                    uint32_t slot = hash_slot(c, mask);
                    for (uint32_t probe = 0; probe <= mask; probe++) {
                        const int prev = atomicCAS(keys + slot, kEmpty, c);
                        if (prev == kEmpty) touched[atomicAdd(&S.ntouched, 1)] = (int)slot;
                        if (prev == kEmpty || prev == c) break;
                        slot = (slot + 1) & mask;
                    }
                    atomicAdd(vals + slot, contrib);
                }
                __syncthreads();  // contributions of entry i land before entry i+1's
            }
            if (tid == 0) {  // the teleport target always exists in the merged row
                uint32_t slot = hash_slot(seed, mask);
                for (uint32_t probe = 0; probe <= mask; probe++) {
                    const int prev = atomicCAS(keys + slot, kEmpty, seed);
                    if (prev == kEmpty) touched[S.ntouched++] = (int)slot;
                    if (prev == kEmpty || prev == seed) break;
                    slot = (slot + 1) & mask;
                }
            }
            __syncthreads();
            const int nt = S.ntouched;
            TopList<KMAX> L;
            L.init();
            for (int i = tid; i < nt; i += kPprThreads) {
                const int s = touched[i];
                const int c = keys[s];
                double v = __dmul_rn(vals[s], oma);
                if (c == seed) v = __dadd_rn(v, alpha);
                L.offer(v, c);
            }
            const int cnt = block_merge_topk<KMAX>(L, iter_topk, S.ms, S.sel_col, S.sel_val);
            for (int i = tid; i < nt; i += kPprThreads) {  // leave the table empty again
                const int s = touched[i];
                keys[s] = kEmpty;
                vals[s] = 0.0;
            }
            __syncthreads();
            if (tid == 0) S.ntouched = 0;
            if (tid == 0) {
                // next state: the selection sorted by column (insertion sort, <= 32 entries)
                for (int i = 0; i < cnt; i++) {
                    const int c = S.sel_col[i];
                    const double v = S.sel_val[i];
                    int p = i;
                    while (p > 0 && S.st_col[p - 1] > c) {
                        S.st_col[p] = S.st_col[p - 1];
                        S.st_val[p] = S.st_val[p - 1];
                        p--;
                    }
                    S.st_col[p] = c;
                    S.st_val[p] = v;
                }
                S.st_n = cnt;
            }
            __syncthreads();
        }
        if (tid == 0) {
            const int slot = seed - source_start;
            if (overflow) {
                atomicAdd(info, 1);
                out_cnt[slot] = 0;
            } else {
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

int64_t pruned_gcap(int64_t max_degree, int64_t iter_topk) {
    const int64_t need = 2 * (iter_topk * (max_degree > 0 ? max_degree : 1) + 1);
    int64_t cap = 64;
    while (cap < need) cap <<= 1;
    return cap;
}

struct PprWs {
    int *counter;
    int *gkeys;
    double *gvals;
    int *gtouched;
    double *gx;
    unsigned char *gp;
    int64_t gcap;
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
    if (iter_topk > 0) {
        w.gcap = pruned_gcap(max_degree, iter_topk);
        if (w.gcap > kSmemSlots) {
            w.gkeys = reinterpret_cast<int *>(take(sizeof(int) * (size_t)(ctas * w.gcap)));
            w.gvals = reinterpret_cast<double *>(take(sizeof(double) * (size_t)(ctas * w.gcap)));
            w.gtouched = reinterpret_cast<int *>(take(sizeof(int) * (size_t)(ctas * (w.gcap / 2))));
        } else {
            w.gcap = 0;
        }
    } else {
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
    if (!dense && w.gkeys != nullptr) {
        const int64_t c = num_seeds < kMaxCtas ? num_seeds : kMaxCtas;
        cudaMemsetAsync(w.gkeys, 0xff, sizeof(int) * (size_t)(c * w.gcap), st);   // kEmpty
        cudaMemsetAsync(w.gvals, 0, sizeof(double) * (size_t)(c * w.gcap), st);
    }
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
            (int)source_end, (int)keep_stride, out_col, out_val, out_val64, out_cnt, info,         \
            w.counter, w.gkeys, w.gvals, w.gtouched, w.gcap);                                      \
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
