// Sparse x sparse matrix product C = A B of CSR matrices (sm_100a).
//
// Replaces `csr_spgemm` (NeutronGT/core/ppr_backends/cusparse_ops.py:97-114) and its cuSPARSE
// kernel `csr_spgemm_cuda` (csrc/cusparse_spgemm.cu:65-267): fp32 values, A [m x n], B [n x n],
// C [m x n] with the structural entries of the product (an entry whose products cancel to zero
// stays, as cuSPARSE keeps it), columns ascending within each row.
//
// Row-wise (Gustavson) product, one warp per output row, persistent warps over rows.  Each warp
// owns a slot of dense per-column arrays in the workspace (fp32 accumulator, touched flag) and a
// list of the columns it touched.  Row i walks A's entries (j, a) in CSR order and, 32 columns at a
// time, B's row j: acc[c] = acc[c] + a * b[j][c] (one fp32 multiply, then one fp32 add, the first
// touch adding to zero), so every output value is the sum of its products in A's entry order —
// the order of the row-wise product SciPy's csr_matmat uses, bit for bit.  A step whose 32 columns
// hold a repeated column runs on lane 0 alone, in order.
// Two launches: a symbolic pass counts each row's columns (scanned into C's row pointer), then a
// numeric pass accumulates, orders the row's touched columns and writes them with their values.
// Ordering: a warp bitonic sort in shared memory up to 4,096 columns; a longer row is, when B's
// rows ascend and A's row has <= 32 entries, one ascending run per A entry, merged in pairwise
// merge-path rounds (O(nt log runs)); otherwise a bitonic sort in the slot's global scratch.  The
// slot arrays are reset through the touched list, so a call costs O(products), not O(rows x n).
#include <mutex>

#include "scan_sort.cuh"

namespace ngt {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSmemCols = 4096;   // per warp, for rows sorted in shared memory (dynamic: 128 KiB per CTA)
constexpr int kMaxRuns = 32;      // A entries per row whose ascending runs the merge path takes (one lane each)
constexpr size_t kNumericSmem = sizeof(int32_t) * (size_t)kWarps * (kSmemCols + kMaxRuns + 1);

struct SpgemmWs {
    float *acc;
    uint8_t *flag;
    int32_t *touched;          // [slots][tcap]
    int32_t *merged;           // [slots][tcap]: the other buffer of the run merges
    int64_t tcap;              // power of two >= n
    int64_t *counts;           // [m + 1]
    int64_t *partials;
    unsigned long long *next;  // [2] row counters of the two passes
    size_t used;
};

int64_t pow2_at_least(int64_t x) {
    int64_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

SpgemmWs carve_spgemm(void *base, int64_t m, int64_t n, int64_t slots) {
    SpgemmWs w;
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        off = (off + 255) & ~size_t(255);
        char *q = p ? p + off : nullptr;
        off += bytes;
        return q;
    };
    w.tcap = pow2_at_least(n > 0 ? n : 1);
    w.next = reinterpret_cast<unsigned long long *>(take(2 * sizeof(unsigned long long)));
    w.counts = reinterpret_cast<int64_t *>(take(sizeof(int64_t) * (size_t)(m + 1)));
    w.partials = reinterpret_cast<int64_t *>(take(sizeof(int64_t) * (size_t)(scan_partials_count(m + 1) + 1)));
    w.acc = reinterpret_cast<float *>(take(sizeof(float) * (size_t)n * (size_t)slots));
    w.flag = reinterpret_cast<uint8_t *>(take((size_t)n * (size_t)slots));
    w.touched = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * (size_t)w.tcap * (size_t)slots));
    w.merged = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * (size_t)w.tcap * (size_t)slots));
    w.used = off;
    return w;
}

// Ascending bitonic sort of arr[0, P) (P a power of two) by one warp.
__device__ __forceinline__ void warp_bitonic(int32_t *arr, int P, int lane) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < P; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const int32_t a = arr[i], b = arr[ixj];
                    const bool asc = (i & k) == 0;
                    if ((a > b) == asc) {
                        arr[i] = b;
                        arr[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// out[0, la + lb) = merge of the ascending, mutually distinct a[0, la) and b[0, lb) by one warp:
// lane l writes outputs [l L / 32, (l + 1) L / 32), its start found by a merge-path binary search.
__device__ __forceinline__ void warp_merge(const int32_t *a, int la, const int32_t *b, int lb, int32_t *out, int lane) {
    const int L = la + lb;
    const int d0 = (int)((int64_t)L * lane / 32), d1 = (int)((int64_t)L * (lane + 1) / 32);
    int lo = d0 - lb > 0 ? d0 - lb : 0, hi = d0 < la ? d0 : la;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < b[d0 - 1 - mid]) lo = mid + 1;
        else hi = mid;
    }
    int i = lo, j = d0 - lo;
    for (int d = d0; d < d1; d++) {
        const bool ta = j >= lb || (i < la && a[i] < b[j]);
        out[d] = ta ? a[i++] : b[j++];
    }
}

// The touched list of a row is the concatenation of one ascending run per A entry (the fresh
// columns of B's row j, in B's order) when B's rows ascend: pairwise merge rounds over the runs
// (starts in rs[0, k), rs[k] = nt) between `src` and `dst`; returns the buffer holding the result.
__device__ int32_t *merge_runs(int32_t *src, int32_t *dst, int32_t *rs, int k, int lane) {
    while (k > 1) {
        for (int r = 0; r < k; r += 2) {
            const int a0 = rs[r], a1 = rs[r + 1];
            if (r + 1 == k) {
                for (int t = a0 + lane; t < a1; t += 32) dst[t] = src[t];
            } else {
                const int a2 = rs[r + 2];
                warp_merge(src + a0, a1 - a0, src + a1, a2 - a1, dst + a0, lane);
            }
        }
        __syncwarp();
        const int nk = (k + 1) >> 1;
        int v = 0;
        if (lane <= nk) v = rs[lane < nk ? 2 * lane : k];   // new starts: every other run, then the end
        __syncwarp();
        if (lane <= nk) rs[lane] = v;
        __syncwarp();
        k = nk;
        int32_t *t = src;
        src = dst;
        dst = t;
    }
    return src;
}

template <bool NUMERIC>
__global__ void __launch_bounds__(kThreads)
    spgemm_rows(int m, int n, const int64_t *__restrict__ rowptr_a, const int32_t *__restrict__ col_a,
                const float *__restrict__ val_a, const int64_t *__restrict__ rowptr_b, const int32_t *__restrict__ col_b,
                const float *__restrict__ val_b, int slots, const int64_t *__restrict__ rowptr_c,
                int64_t *__restrict__ col_c, float *__restrict__ val_c, SpgemmWs w) {
    extern __shared__ int32_t spgemm_smem[];   // numeric pass: [kWarps][kSmemCols] sort buffers, [kWarps][kMaxRuns + 1] run starts
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int slot = blockIdx.x * kWarps + wib;
    if (slot >= slots) return;
    float *acc = w.acc + (size_t)slot * n;
    uint8_t *flag = w.flag + (size_t)slot * n;
    int32_t *touched = w.touched + (size_t)slot * w.tcap;
    const unsigned full = 0xffffffffu, lt = (1u << lane) - 1u;
    for (;;) {
        int i = 0;
        if (lane == 0) i = (int)atomicAdd(w.next + (NUMERIC ? 1 : 0), 1ull);
        i = __shfl_sync(full, i, 0);
        if (i >= m) break;
        int nt = 0;
        const int64_t arow0 = rowptr_a[i], arow1 = rowptr_a[i + 1];
        int32_t *rs = NUMERIC ? spgemm_smem + kWarps * kSmemCols + wib * (kMaxRuns + 1) : nullptr;
        const bool track = NUMERIC && arow1 - arow0 <= kMaxRuns;   // record the runs of this row
        bool ascending = true;                                      // every B row read so far ascends
        for (int64_t jj = arow0; jj < arow1; jj++) {
            const int j = col_a[jj];
            const float a = NUMERIC ? val_a[jj] : 0.f;
            const int64_t b0 = rowptr_b[j], b1 = rowptr_b[j + 1];
            if (track && lane == 0) rs[jj - arow0] = nt;
            int lastc = -1;
            for (int64_t q0 = b0; q0 < b1; q0 += 32) {
                const int64_t q = q0 + lane;
                const bool act = q < b1;
                const int c = act ? col_b[q] : -1 - lane;
                if (track) {   // B's row ascending (equal neighbours allowed)?
                    const int prev = __shfl_up_sync(full, c, 1);
                    const bool bad = act && (lane > 0 ? c < prev : c < lastc);
                    if (__any_sync(full, bad)) ascending = false;
                    const int nact = (int)(b1 - q0 < 32 ? b1 - q0 : 32);
                    lastc = __shfl_sync(full, c, nact - 1);
                }
                const bool dup = __any_sync(full, __popc(__match_any_sync(full, c)) > 1);
                if (!dup) {
                    bool fresh = false;
                    if (act) {
                        fresh = flag[c] == 0;
                        if (fresh) flag[c] = 1;
                        if (NUMERIC) {
                            const float prod = __fmul_rn(a, val_b[q]);
                            acc[c] = __fadd_rn(fresh ? 0.f : acc[c], prod);
                        }
                    }
                    const unsigned bf = __ballot_sync(full, fresh);
                    if (fresh) touched[nt + __popc(bf & lt)] = c;
                    nt += __popc(bf);
                } else {
                    __syncwarp();
                    int nt2 = nt;
                    if (lane == 0) {
                        for (int64_t qq = q0; qq < b1 && qq < q0 + 32; qq++) {
                            const int cc = col_b[qq];
                            const bool fr = flag[cc] == 0;
                            if (fr) {
                                flag[cc] = 1;
                                touched[nt2++] = cc;
                            }
                            if (NUMERIC) acc[cc] = __fadd_rn(fr ? 0.f : acc[cc], __fmul_rn(a, val_b[qq]));
                        }
                    }
                    nt = __shfl_sync(full, nt2, 0);
                }
                __syncwarp();
            }
        }
        if (!NUMERIC) {
            if (lane == 0) w.counts[i] = nt;
            for (int t = lane; t < nt; t += 32) flag[touched[t]] = 0;
        } else {
            int32_t *arr = touched;
            int P = 1;
            while (P < nt) P <<= 1;
            if (P <= kSmemCols) {
                arr = spgemm_smem + wib * kSmemCols;
                for (int t = lane; t < P; t += 32) arr[t] = t < nt ? touched[t] : INT32_MAX;
                __syncwarp();
                if (nt > 1) warp_bitonic(arr, P, lane);
            } else if (track && ascending) {   // long row: merge its ascending runs (O(nt log runs))
                if (lane == 0) rs[arow1 - arow0] = nt;
                __syncwarp();
                arr = merge_runs(touched, w.merged + (size_t)slot * w.tcap, rs, (int)(arow1 - arow0), lane);
            } else {
                for (int t = nt + lane; t < P; t += 32) arr[t] = INT32_MAX;
                __syncwarp();
                warp_bitonic(arr, P, lane);
            }
            __syncwarp();
            const int64_t o = rowptr_c[i];
            for (int t = lane; t < nt; t += 32) {
                const int c = arr[t];
                col_c[o + t] = c;
                val_c[o + t] = acc[c];
                flag[c] = 0;
            }
        }
        __syncwarp();
    }
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_csr_spgemm_workspace_size(int64_t m, int64_t n, int64_t slots, size_t *bytes) {
    if (m < 0 || n < 0 || slots <= 0 || !bytes) return NGT_ERR_INVALID_ARGUMENT;
    *bytes = carve_spgemm(nullptr, m, n, slots).used;
    return NGT_OK;
}

extern "C" int ngt_csr_spgemm_symbolic(int64_t m, int64_t n, const int64_t *rowptr_a, const int32_t *col_a,
                                       const int64_t *rowptr_b, const int32_t *col_b, int64_t slots,
                                       int64_t *rowptr_c, void *workspace, size_t workspace_bytes,
                                       ngt_stream_t stream) {
    if (m < 0 || n < 0 || slots <= 0 || !rowptr_c || !rowptr_a || !rowptr_b) return NGT_ERR_INVALID_ARGUMENT;
    if (m >= (int64_t)INT32_MAX || n >= (int64_t)INT32_MAX || slots >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    SpgemmWs w = carve_spgemm(workspace, m, n, slots);
    if (!workspace || workspace_bytes < w.used) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // the slot arrays start (and stay) zero; both row counters restart
    if (cudaMemsetAsync(workspace, 0, w.used, st) != cudaSuccess) return NGT_ERR_CUDA;
    if (m > 0) {
        spgemm_rows<false><<<(unsigned)((slots + kWarps - 1) / kWarps), kThreads, 0, st>>>(
            (int)m, (int)n, rowptr_a, col_a, nullptr, rowptr_b, col_b, nullptr, (int)slots, nullptr, nullptr, nullptr,
            w);
        NGT_CHECK_LAUNCH();
    }
    return exclusive_scan<int64_t>(w.counts, rowptr_c, m + 1, w.partials, st);
}

extern "C" int ngt_csr_spgemm_numeric(int64_t m, int64_t n, const int64_t *rowptr_a, const int32_t *col_a,
                                      const float *val_a, const int64_t *rowptr_b, const int32_t *col_b,
                                      const float *val_b, int64_t slots, const int64_t *rowptr_c, int64_t *col_c,
                                      float *val_c, void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (m < 0 || n < 0 || slots <= 0 || !rowptr_c || !rowptr_a || !rowptr_b) return NGT_ERR_INVALID_ARGUMENT;
    if (m >= (int64_t)INT32_MAX || n >= (int64_t)INT32_MAX || slots >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    SpgemmWs w = carve_spgemm(workspace, m, n, slots);
    if (!workspace || workspace_bytes < w.used) return NGT_ERR_WORKSPACE;
    if (m == 0) return NGT_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    {   // the numeric pass's sort buffers exceed the 48 KiB default: raise the limit once per device
        static std::mutex mu;
        static bool set[64] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return NGT_ERR_CUDA;
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 0 || dev >= 64 || !set[dev]) {
            if (cudaFuncSetAttribute(spgemm_rows<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kNumericSmem) != cudaSuccess)
                return NGT_ERR_CUDA;
            if (dev >= 0 && dev < 64) set[dev] = true;
        }
    }
    spgemm_rows<true><<<(unsigned)((slots + kWarps - 1) / kWarps), kThreads, kNumericSmem, st>>>(
        (int)m, (int)n, rowptr_a, col_a, val_a, rowptr_b, col_b, val_b, (int)slots, rowptr_c, col_c, val_c, w);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}
