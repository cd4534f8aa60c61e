// Push-based approximate personalised PageRank with per-seed top-k (sm_100a).
//
// Replaces the reference's default PPR backend, `personal_pagerank_torch_geometric`
// (NeutronGT/core/ppr_backends/torch_geometric_backend.py:5-30): PyG's `get_ppr(edge_index,
// alpha, eps)` followed by a per-source top-k loop in Python.  PyG's function implements the
// published push method (Andersen, Chung & Lang 2006; the variant of Bojchevski et al., PPRGo
// 2020), run per seed s over the row-stochastic walk of the CSR graph:
//
//   p = {s: 0}, r = {s: alpha}, stack = [s]
//   while stack:  u = pop()
//       res = r[u];  p[u] += res (an entry is created at u's first pop);  r[u] = 0
//       for v in adj(u) in CSR order:
//           r[v] += ((1 - alpha) * res) / deg(u)
//           if r[v] >= (alpha * eps) * deg(v) and v is not on the stack:  push(v)
//
// then keeps, for a seed with more than topk entries, the topk largest (ties: smaller node
// first), emitted by (value desc, node asc); a seed with at most topk entries keeps p in
// insertion order (seed first, then first-pop order).
//
// One warp per seed, persistent warps taking seeds from a counter.  Each warp owns a slot of
// dense per-node arrays in the workspace (r, p values, flags) plus its stack, p list and the list
// of touched nodes, through which the seed clears the flags it set (a value is only read when its
// flag says it was written, so only the flags need clearing).  A push spreads one adjacency row
// over the lanes, kPushU chunks of 32 neighbours per step with all their loads issued before any
// update: the neighbours of a row are distinct (columns ascend, so a repeated edge shows as equal
// neighbouring entries; a step holding one runs on lane 0 alone), so their updates commute, and
// the stack appends are placed with a ballot per chunk in lane (= CSR) order.  A hub seed's push
// is one warp's walk over its row, so several chunks per step cut the tail its load latency sets.
// Every operation is a separate IEEE fp64 rounding (__dmul_rn / __ddiv_rn / __dadd_rn) in the
// method's own order, so the result is bit-identical to the sequential method (the CPU
// restatement in oracle/push_oracle.c).
#include "common.cuh"

namespace ngt {
namespace {

constexpr int kPushThreads = 256;
constexpr int kPushWarps = kPushThreads / 32;
#ifndef NGT_PUSH_U
#define NGT_PUSH_U 8
#endif
constexpr int kPushU = NGT_PUSH_U;   // 32-neighbour chunks per step of a push (loads in flight together)

struct PushWs {
    double *r, *pv;
    uint8_t *fl;
    int32_t *stack, *plist, *touched;
    unsigned long long *counter;   // [0] next seed, [1] pushes, [2] adjacency entries read
    size_t used;
};

// Slot-major layout: slot k's arrays at k * n.  256-byte aligned pieces.
PushWs carve_push(void *base, int64_t n, int64_t slots) {
    PushWs w;
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        off = (off + 255) & ~size_t(255);
        char *q = p ? p + off : nullptr;
        off += bytes;
        return q;
    };
    const size_t ns = (size_t)n * (size_t)slots;
    w.counter = reinterpret_cast<unsigned long long *>(take(4 * sizeof(unsigned long long)));
    w.r = reinterpret_cast<double *>(take(ns * sizeof(double)));
    w.pv = reinterpret_cast<double *>(take(ns * sizeof(double)));
    w.stack = reinterpret_cast<int32_t *>(take(ns * sizeof(int32_t)));
    w.plist = reinterpret_cast<int32_t *>(take(ns * sizeof(int32_t)));
    w.touched = reinterpret_cast<int32_t *>(take(ns * sizeof(int32_t)));
    w.fl = reinterpret_cast<uint8_t *>(take(ns));
    w.used = off;
    return w;
}

constexpr uint8_t kTouched = 1, kInP = 2, kOnStack = 4;

// One neighbour update of the method in its sequential form (lane 0, for a step that holds a
// repeated neighbour).
__device__ __forceinline__ void relax_one(int32_t v, double val, double alpha_eps, const int64_t *__restrict__ rowptr,
                                          double *r, uint8_t *fl, int32_t *stack, int32_t *touched, int &sp, int &nt) {
    const uint8_t f = fl[v];
    const double rv = (f & kTouched) ? __dadd_rn(r[v], val) : val;
    r[v] = rv;
    uint8_t g = f | kTouched;
    if (!(f & kTouched)) touched[nt++] = v;
    const double thr = __dmul_rn(alpha_eps, (double)(rowptr[v + 1] - rowptr[v]));
    if (rv >= thr && !(f & kOnStack)) {
        g |= kOnStack;
        stack[sp++] = v;
    }
    fl[v] = g;
}

__global__ void __launch_bounds__(kPushThreads)
    ppr_push_kernel(int n, const int64_t *__restrict__ rowptr, const int32_t *__restrict__ col, double alpha,
                    double eps, int s0, int s1, int topk, int slots, int64_t *__restrict__ out_idx,
                    float *__restrict__ out_val, double *__restrict__ out_val64, int32_t *__restrict__ out_cnt,
                    int32_t *__restrict__ info, PushWs w, long long max_pushes) {
    const int lane = threadIdx.x & 31;
    const int slot = blockIdx.x * kPushWarps + (threadIdx.x >> 5);
    if (slot >= slots) return;
    const size_t base = (size_t)slot * (size_t)n;
    double *r = w.r + base, *pv = w.pv + base;
    uint8_t *fl = w.fl + base;
    int32_t *stack = w.stack + base, *plist = w.plist + base, *touched = w.touched + base;
    const double keep = 1.0 - alpha;
    const double alpha_eps = __dmul_rn(alpha, eps);
    const unsigned full = 0xffffffffu;
    const unsigned lt = (1u << lane) - 1u;
    unsigned long long pushes = 0, read = 0;

    for (;;) {
        int s = 0;
        if (lane == 0) s = (int)atomicAdd(w.counter, 1ull) + s0;
        s = __shfl_sync(full, s, 0);
        if (s >= s1) break;
        int sp = 1, np = 1, nt = 1;
        if (lane == 0) {
            r[s] = alpha;
            pv[s] = 0.0;
            fl[s] = kTouched | kInP | kOnStack;
            touched[0] = s;
            plist[0] = s;
            stack[0] = s;
        }
        __syncwarp();
        long long count = 0;
        bool capped = false;
        while (sp > 0) {
            if (++count > max_pushes) {
                capped = true;
                break;
            }
            const int u = stack[--sp];
            double res = 0.0;
            int added = 0;
            if (lane == 0) {
                const uint8_t f = fl[u];
                res = r[u];
                if (f & kInP) {
                    pv[u] = __dadd_rn(pv[u], res);
                } else {
                    pv[u] = res;
                    plist[np] = u;
                    added = 1;
                }
                fl[u] = (uint8_t)((f | kInP) & ~kOnStack);
                r[u] = 0.0;
            }
            res = __shfl_sync(full, res, 0);
            np += __shfl_sync(full, added, 0);
            __syncwarp();
            pushes++;
            const int64_t b = rowptr[u], e = rowptr[u + 1];
            if (e == b) continue;
            read += (unsigned long long)(e - b);
            const double val = __ddiv_rn(__dmul_rn(keep, res), (double)(e - b));
            for (int64_t q0 = b; q0 < e; q0 += 32 * kPushU) {
                // kPushU chunks of 32 neighbours per step: lane l takes q0 + 32 j + l.  The loads of
                // all chunks are issued before any update (the neighbours are distinct, so no chunk
                // reads what another writes), then the appends run chunk by chunk in CSR order.
                int32_t v[kPushU];
                bool act[kPushU];
                bool d = false;
#pragma unroll
                for (int j = 0; j < kPushU; j++) {
                    const int64_t q = q0 + 32 * j + lane;
                    act[j] = q < e;
                    v[j] = act[j] ? col[q] : -1;
                }
#pragma unroll
                for (int j = 0; j < kPushU; j++) {   // repeated neighbours: equal CSR neighbours
                    const int32_t prev = __shfl_up_sync(full, v[j], 1);
                    if (act[j] && lane > 0 && v[j] == prev) d = true;
                    if (j > 0) {
                        const int32_t last = __shfl_sync(full, v[j - 1], 31);
                        if (act[j] && lane == 0 && v[j] == last) d = true;
                    }
                }
                if (!__any_sync(full, d)) {
                    uint8_t f[kPushU];
                    double thr[kPushU];
#pragma unroll
                    for (int j = 0; j < kPushU; j++) {
                        f[j] = act[j] ? fl[v[j]] : (uint8_t)0;
                        thr[j] = act[j] ? __dmul_rn(alpha_eps, (double)(rowptr[v[j] + 1] - rowptr[v[j]])) : 0.0;
                    }
                    bool fresh[kPushU], push[kPushU];
#pragma unroll
                    for (int j = 0; j < kPushU; j++) {
                        fresh[j] = false;
                        push[j] = false;
                        if (act[j]) {
                            const double rv = (f[j] & kTouched) ? __dadd_rn(r[v[j]], val) : val;
                            r[v[j]] = rv;
                            fresh[j] = !(f[j] & kTouched);
                            push[j] = rv >= thr[j] && !(f[j] & kOnStack);
                            fl[v[j]] = (uint8_t)(f[j] | kTouched | (push[j] ? kOnStack : 0));
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kPushU; j++) {
                        const unsigned bf = __ballot_sync(full, fresh[j]), bp = __ballot_sync(full, push[j]);
                        if (fresh[j]) touched[nt + __popc(bf & lt)] = v[j];
                        if (push[j]) stack[sp + __popc(bp & lt)] = v[j];
                        nt += __popc(bf);
                        sp += __popc(bp);
                    }
                } else {
                    __syncwarp();
                    int sp2 = sp, nt2 = nt;
                    if (lane == 0)
                        for (int64_t qq = q0; qq < e && qq < q0 + 32 * kPushU; qq++)
                            relax_one(col[qq], val, alpha_eps, rowptr, r, fl, stack, touched, sp2, nt2);
                    sp = __shfl_sync(full, sp2, 0);
                    nt = __shfl_sync(full, nt2, 0);
                }
                __syncwarp();
            }
        }
        if (capped && lane == 0) atomicAdd(info, 1);
        // ---- selection ----
        const int o = s - s0;
        if (np <= topk) {
            for (int i = lane; i < np; i += 32) {
                const int c = plist[i];
                const double x = pv[c];
                out_idx[(int64_t)o * topk + i] = c;
                out_val[(int64_t)o * topk + i] = __double2float_rn(x);
                if (out_val64) out_val64[(int64_t)o * topk + i] = x;
            }
            if (lane == 0) out_cnt[o] = np;
        } else {
            for (int t = 0; t < topk; t++) {
                double bv = -1.0;
                int bc = -1, bi = -1;
                for (int i = lane; i < np; i += 32) {
                    const int c = plist[i];
                    if (c < 0) continue;
                    const double x = pv[c];
                    if (bi < 0 || x > bv || (x == bv && c < bc)) {
                        bv = x;
                        bc = c;
                        bi = i;
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const double ov = __shfl_xor_sync(full, bv, off);
                    const int oc = __shfl_xor_sync(full, bc, off), oi = __shfl_xor_sync(full, bi, off);
                    const bool take = oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oc < bc));
                    if (take) {
                        bv = ov;
                        bc = oc;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    out_idx[(int64_t)o * topk + t] = bc;
                    out_val[(int64_t)o * topk + t] = __double2float_rn(bv);
                    if (out_val64) out_val64[(int64_t)o * topk + t] = bv;
                    plist[bi] = -1;
                }
                __syncwarp();
            }
            if (lane == 0) out_cnt[o] = topk;
        }
        // ---- clear the flags this seed set (residuals and p values are dead once their flags are) ----
        for (int i = lane; i < nt; i += 32) fl[touched[i]] = 0;
        __syncwarp();
    }
    if (lane == 0) {
        atomicAdd(w.counter + 1, pushes);
        atomicAdd(w.counter + 2, read);
    }
}

// CSR column check and narrowing for the PPR kernels, one pass: each warp takes chunks of
// kCheckChunk entries, lane l entries c0 + 32 i + l (coalesced).  Lane 0 finds the chunk's first row
// by binary search over rowptr; each lane then advances its row while rowptr[row + 1] <= q.  Sets
// bit 0 of *flags for a column outside [0, n), bit 1 for a column below its predecessor in the same row.
constexpr int kCheckChunk = 1024;

__global__ void __launch_bounds__(256)
    csr_col32_kernel(int64_t n, int64_t nnz, const int64_t *__restrict__ rowptr, const int64_t *__restrict__ col,
                     int32_t *__restrict__ col32, int32_t *__restrict__ flags) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    int bad = 0;
    for (int64_t c0 = warp * kCheckChunk; c0 < nnz; c0 += nwarps * kCheckChunk) {
        int64_t row = 0;
        if (lane == 0) {   // last row r with rowptr[r] <= c0 (rowptr[n] = nnz > c0, so r < n)
            int64_t lo = 0, hi = n - 1;
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (rowptr[mid] <= c0) lo = mid;
                else hi = mid - 1;
            }
            row = lo;
        }
        row = __shfl_sync(full, row, 0);
        int64_t last = c0 > 0 ? col[c0 - 1] : 0;
        for (int i = 0; i < kCheckChunk / 32; i++) {
            const int64_t q = c0 + 32 * i + lane;
            const bool act = q < nnz;
            const int64_t c = act ? col[q] : 0;
            int64_t r = row;
            if (act)   // bounded by the last row, so a malformed rowptr cannot walk past its end
                while (r < n - 1 && rowptr[r + 1] <= q) r++;
            const int64_t up = __shfl_up_sync(full, c, 1);
            const int64_t prev = lane == 0 ? last : up;
            if (act) {
                if (c < 0 || c >= n) bad |= 1;
                if (q != rowptr[r] && c < prev) bad |= 2;
                col32[q] = (int32_t)c;
            }
            last = __shfl_sync(full, c, 31);
            row = __shfl_sync(full, r, 31);
            if (!__any_sync(full, q + 32 < nnz)) break;
        }
    }
    if (bad) atomicOr(flags, bad);
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_ppr_push_workspace_size(int64_t n, int64_t slots, size_t *bytes) {
    if (n < 0 || slots <= 0 || !bytes) return NGT_ERR_INVALID_ARGUMENT;
    *bytes = carve_push(nullptr, n, slots).used;
    return NGT_OK;
}

extern "C" int ngt_ppr_push_topk(int64_t n, const int64_t *rowptr, const int32_t *col, double alpha, double eps,
                                 int64_t seed_start, int64_t seed_end, int64_t topk, int64_t slots,
                                 int64_t *out_idx, float *out_val, double *out_val64, int32_t *out_cnt,
                                 int32_t *info, void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || seed_start < 0 || seed_end > n || seed_start > seed_end || topk <= 0 || slots <= 0 || !info)
        return NGT_ERR_INVALID_ARGUMENT;
    if (!(alpha > 0.0 && alpha <= 1.0) || !(eps > 0.0)) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || topk >= (int64_t)INT32_MAX || slots >= (int64_t)INT32_MAX)
        return NGT_ERR_TOO_LARGE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(info, 0, sizeof(int32_t), st) != cudaSuccess) return NGT_ERR_CUDA;
    if (seed_start == seed_end) return NGT_OK;
    if (!rowptr || !col || !out_idx || !out_val || !out_cnt) return NGT_ERR_INVALID_ARGUMENT;
    PushWs w = carve_push(workspace, n, slots);
    if (!workspace || workspace_bytes < w.used) return NGT_ERR_WORKSPACE;
    // Only the flags must start at zero (a residual or p value is read only when its flag says it was
    // written, and the lists are written before they are read): the counters and flags are cleared
    // here, and every seed clears the flags it set.
    if (cudaMemsetAsync(w.counter, 0, 4 * sizeof(unsigned long long), st) != cudaSuccess ||
        cudaMemsetAsync(w.fl, 0, (size_t)n * (size_t)slots, st) != cudaSuccess)
        return NGT_ERR_CUDA;
    // Termination guard only: a pop of a node with neighbours removes alpha * res >= alpha^2 eps of the
    // residual mass (alpha to start), so there are at most 1 + 1 / (alpha eps) of those; a node without
    // neighbours enters the stack only through an edge relaxation.  Past this bound a seed stops and
    // counts in *info.
    const double bound = 1.0 / (alpha * alpha * eps) + 4294967296.0;
    const long long max_pushes = bound > 9.0e18 ? (long long)9.0e18 : (long long)bound;
    const int blocks = (int)((slots + kPushWarps - 1) / kPushWarps);
    ppr_push_kernel<<<blocks, kPushThreads, 0, st>>>((int)n, rowptr, col, alpha, eps, (int)seed_start, (int)seed_end,
                                                    (int)topk, (int)slots, out_idx, out_val, out_val64, out_cnt,
                                                    info, w, max_pushes);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_ppr_push_stats(const void *workspace, int64_t n, int64_t slots, int64_t *pushes_and_reads,
                                  ngt_stream_t stream) {
    if (!workspace || !pushes_and_reads || n < 0 || slots <= 0) return NGT_ERR_INVALID_ARGUMENT;
    unsigned long long c[3];
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(c, workspace, sizeof(c), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return NGT_ERR_CUDA;
    pushes_and_reads[0] = (int64_t)c[1];
    pushes_and_reads[1] = (int64_t)c[2];
    return NGT_OK;
}

extern "C" int ngt_csr_col32_checked(int64_t n, int64_t nnz, const int64_t *rowptr, const int64_t *col, int32_t *col32,
                                     int32_t *flags, ngt_stream_t stream) {
    if (n < 0 || nnz < 0 || !flags || !rowptr || (nnz > 0 && (n == 0 || !col || !col32)))
        return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || nnz >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(flags, 0, sizeof(int32_t), st) != cudaSuccess) return NGT_ERR_CUDA;
    if (nnz == 0) return NGT_OK;
    const int64_t chunks = (nnz + kCheckChunk - 1) / kCheckChunk;
    const int64_t blocks = (chunks + 7) / 8 < 148 * 16 ? (chunks + 7) / 8 : 148 * 16;
    csr_col32_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, nnz, rowptr, col, col32, flags);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}
