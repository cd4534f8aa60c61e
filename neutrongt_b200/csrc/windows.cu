// Window construction between PPR and the training windows (sm_100a):
//   ngt_ppr_adjacency      the weighted, symmetric PPR adjacency the partitioner consumes
//                          (NeutronGT/core/ppr_preprocess.py:30-71, build_adj_fromat)
//   ngt_halo_merge         a window grown by its heaviest external neighbours
//                          (NeutronGT/core/metisPartition.py:397-425, _merge_related_nodes)
//   ngt_duplicate_rerange  windows reordered duplicate-nodes-first for the K/V cache
//                          (NeutronGT/core/metisPartition.py:333-363 and
//                          core/node_level_pipeline/window_state.py:52-73)
//   ngt_isolated_connections_*  random links from nodes that appear in neither the PPR list nor
//                          the graph to the nodes that do (NeutronGT/core/ppr_preprocess.py:94-132,
//                          add_isolated_connections), without the dense [isolated x others] draw
//
// The reference does these in host Python (dict / set loops, torch.unique on the CPU).  Here
// each is a handful of device passes: stable LSD radix sorts (scan_sort.cuh) stand in for the
// dictionaries and sorted() calls, segmented sums for scatter_add_, and exclusive scans for the
// list building.  Orders the reference defines (stable sort, first-encounter order of a dict,
// original order within a partition) are reproduced exactly; the one it leaves undefined (the
// order of neighbours inside a CSR row after a non-stable argsort) is pinned to the stable one.
#include "common.cuh"
#include "scan_sort.cuh"

namespace ngt {
namespace {

constexpr int kT = 256;
inline unsigned grid_for(int64_t n) { return (unsigned)((n + kT - 1) / kT); }

// ---------------------------------------------------------------------------------------------
// PPR adjacency
// ---------------------------------------------------------------------------------------------
// Undirected key (min, max) of PPR entry i; out-of-range endpoints are counted and mapped to 0.
__global__ void adj_keys_kernel(int64_t m, int64_t n, const int64_t *__restrict__ ei, uint32_t *__restrict__ ku,
                                uint32_t *__restrict__ kv, uint32_t *__restrict__ idx, int32_t *__restrict__ bad) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i >= m) return;
    int64_t s = ei[i], d = ei[m + i];
    if (s < 0 || s >= n || d < 0 || d >= n) {
        atomicAdd(bad, 1);
        s = d = 0;
    }
    ku[i] = (uint32_t)(s < d ? s : d);
    kv[i] = (uint32_t)(s < d ? d : s);
    idx[i] = (uint32_t)i;
}

__global__ void gather_u32_kernel(int64_t m, const uint32_t *__restrict__ perm, const uint32_t *__restrict__ src,
                                  uint32_t *__restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i < m) dst[i] = src[perm[i]];
}

// head[j] = 1 where sorted entry j starts a new (u, v) key
__global__ void adj_heads_kernel(int64_t m, const uint32_t *__restrict__ perm, const uint32_t *__restrict__ ku,
                                 const uint32_t *__restrict__ kv, uint32_t *__restrict__ head) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j > m) return;
    if (j == m) {
        head[j] = 0;
        return;
    }
    const uint32_t p = perm[j];
    head[j] = (j == 0 || ku[p] != ku[perm[j - 1]] || kv[p] != kv[perm[j - 1]]) ? 1u : 0u;
}

// One thread per key: the sum of its PPR values in original entry order (the order of the
// reference's CPU scatter_add_), then weight = int32(max(sum * 1000, 1)) truncated like .to(int32).
__global__ void adj_segments_kernel(int64_t m, const uint32_t *__restrict__ perm, const uint32_t *__restrict__ ku,
                                    const uint32_t *__restrict__ kv, const float *__restrict__ val,
                                    const uint32_t *__restrict__ head, const uint32_t *__restrict__ seg,
                                    uint32_t *__restrict__ uu, uint32_t *__restrict__ vv, int32_t *__restrict__ ww,
                                    int32_t *__restrict__ count) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j >= m) return;
    if (j == m - 1) *count = (int32_t)(seg[m - 1] + head[m - 1]);
    if (!head[j]) return;
    float sum = 0.f;
    for (int64_t t = j; t < m && (t == j || !head[t]); t++) sum = __fadd_rn(sum, val[perm[t]]);
    const float scaled = fmaxf(__fmul_rn(sum, 1000.f), 1.f);
    const uint32_t s = seg[j];
    uu[s] = ku[perm[j]];
    vv[s] = kv[perm[j]];
    ww[s] = __float2int_rz(scaled);
}

// Entry e < U is (u_e, v_e), entry U + e is (v_e, u_e); entries past 2U sort last (key n).
__global__ void adj_sym_kernel(int64_t m, uint32_t n, const int32_t *__restrict__ count,
                               const uint32_t *__restrict__ uu, const uint32_t *__restrict__ vv,
                               uint32_t *__restrict__ key, uint32_t *__restrict__ idx, int32_t *__restrict__ deg) {
    const int64_t e = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (e >= 2 * m) return;
    const int64_t U = *count;
    idx[e] = (uint32_t)e;
    if (e >= 2 * U) {
        key[e] = n;
        return;
    }
    const uint32_t row = e < U ? uu[e] : vv[e - U];
    key[e] = row;
    atomicAdd(deg + row, 1);
}

__global__ void adj_emit_kernel(int64_t m, const int32_t *__restrict__ count, const uint32_t *__restrict__ order,
                                const uint32_t *__restrict__ uu, const uint32_t *__restrict__ vv,
                                const int32_t *__restrict__ ww, int32_t *__restrict__ adjncy,
                                int32_t *__restrict__ eweights) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    const int64_t U = *count;
    if (j >= 2 * U) return;
    const uint32_t e = order[j];
    const bool first = e < U;
    const uint32_t s = first ? e : e - (uint32_t)U;
    adjncy[j] = (int32_t)(first ? vv[s] : uu[s]);
    eweights[j] = ww[s];
}

struct AdjWs {
    uint32_t *ku, *kv, *ka, *kb, *va, *vb, *head, *seg, *uu, *vv, *hist, *partials;
    int32_t *ww, *deg, *deg_partials;
};

AdjWs carve_adj(void *base, size_t cap, int64_t m, int64_t n, size_t *used) {
    Carver c(base, cap);
    AdjWs w;
    const int64_t m2 = 2 * m > 1 ? 2 * m : 1;
    w.ku = c.take<uint32_t>(m);
    w.kv = c.take<uint32_t>(m);
    w.ka = c.take<uint32_t>(m2);
    w.kb = c.take<uint32_t>(m2);
    w.va = c.take<uint32_t>(m2);
    w.vb = c.take<uint32_t>(m2);
    w.head = c.take<uint32_t>(m + 1);
    w.seg = c.take<uint32_t>(m + 1);
    w.uu = c.take<uint32_t>(m);
    w.vv = c.take<uint32_t>(m);
    w.ww = c.take<int32_t>(m);
    w.hist = c.take<uint32_t>(256 * radix_tiles(m2));
    w.partials = c.take<uint32_t>(scan_partials_count(256 * radix_tiles(m2) > m + 1 ? 256 * radix_tiles(m2) : m + 1) + 1);
    w.deg = c.take<int32_t>(n + 1);
    w.deg_partials = c.take<int32_t>(scan_partials_count(n + 1) + 1);
    *used = c.used;
    return w;
}

// ---------------------------------------------------------------------------------------------
// halo merge
// ---------------------------------------------------------------------------------------------
__global__ void halo_mark_kernel(int64_t p, int64_t n, const int64_t *__restrict__ part, const int32_t *__restrict__ xadj,
                                 int32_t *__restrict__ member, int64_t *__restrict__ deg, int32_t *__restrict__ bad) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i >= p) return;
    const int64_t x = part[i];
    if (x < 0 || x >= n) {
        atomicAdd(bad, 1);
        deg[i] = 0;
        return;
    }
    member[x] = 1;
    deg[i] = xadj[x + 1] - xadj[x];
}

__global__ void sum_i64_kernel(int64_t p, const int64_t *__restrict__ deg, const int64_t *__restrict__ off,
                               int64_t *__restrict__ total) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *total = p > 0 ? off[p - 1] + deg[p - 1] : 0;
}

// One warp per window node i (in the window's order): its neighbour list in CSR order, entry
// position off[i] + j.  External neighbours keep their id as sort key, members get key n.
__global__ void halo_expand_kernel(int64_t p, uint32_t n, const int64_t *__restrict__ part,
                                   const int32_t *__restrict__ xadj, const int32_t *__restrict__ adjncy,
                                   const int32_t *__restrict__ eweights, const int32_t *__restrict__ member,
                                   const int64_t *__restrict__ off, uint32_t *__restrict__ key,
                                   uint32_t *__restrict__ pos, int32_t *__restrict__ wpos) {
    const int64_t i = ((int64_t)blockIdx.x * kT + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= p) return;
    const int64_t x = part[i];
    if (x < 0 || x >= (int64_t)n) return;
    const int64_t b = xadj[x], d = xadj[x + 1] - b, o = off[i];
    for (int64_t j = lane; j < d; j += 32) {
        const int32_t nb = adjncy[b + j];
        const bool ext = nb >= 0 && (uint32_t)nb < n && member[nb] == 0;
        key[o + j] = ext ? (uint32_t)nb : n;
        pos[o + j] = (uint32_t)(o + j);
        wpos[o + j] = eweights[b + j];
    }
}

__global__ void halo_heads_kernel(int64_t t, uint32_t n, const uint32_t *__restrict__ key, uint32_t *__restrict__ head) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j > t) return;
    head[j] = (j < t && key[j] != n && (j == 0 || key[j] != key[j - 1])) ? 1u : 0u;
}

// Weights in sorted order (0 for members) for a prefix sum, and the end of each external
// neighbour's run of entries, written by the run's last entry.
__global__ void halo_runs_kernel(int64_t t, uint32_t n, const uint32_t *__restrict__ key,
                                 const uint32_t *__restrict__ pos, const int32_t *__restrict__ wpos,
                                 const uint32_t *__restrict__ head, const uint32_t *__restrict__ seg,
                                 int64_t *__restrict__ wsorted, uint32_t *__restrict__ seg_end) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j > t) return;
    if (j == t) {
        wsorted[j] = 0;
        return;
    }
    const bool ext = key[j] != n;
    wsorted[j] = ext ? (int64_t)wpos[pos[j]] : 0;
    // seg is the exclusive scan of the run heads, so entry j belongs to run seg[j] + head[j] - 1
    if (ext && (j + 1 == t || key[j + 1] != key[j])) seg_end[seg[j] + head[j] - 1] = (uint32_t)(j + 1);
}

// Per external neighbour: total weight (integer sum, from the prefix sum of the sorted weights)
// and first-encounter position (the head's position: the sort is stable and positions increase
// with the input index).
__global__ void halo_segments_kernel(int64_t t, uint32_t n, const uint32_t *__restrict__ key,
                                     const uint32_t *__restrict__ pos, const int64_t *__restrict__ wscan,
                                     const uint32_t *__restrict__ seg_end,
                                     const uint32_t *__restrict__ head, const uint32_t *__restrict__ seg,
                                     uint32_t *__restrict__ seg_nb, uint32_t *__restrict__ first_key,
                                     uint32_t *__restrict__ invw_key, uint32_t *__restrict__ sidx) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j >= t) return;
    const uint32_t s_total = seg[t - 1] + head[t - 1];
    // padding so that the two sorts below can run over t entries: keys past the segments last
    if (j >= s_total) {
        first_key[j] = 0xFFFFFFFFu;
        invw_key[j] = 0xFFFFFFFFu;
        sidx[j] = (uint32_t)j;
    }
    if (!head[j]) return;
    const uint32_t s = seg[j];
    const int64_t w = wscan[seg_end[s]] - wscan[j];
    seg_nb[s] = key[j];
    first_key[s] = pos[j];
    invw_key[s] = 0xFFFFFFFEu - (uint32_t)(w < 0 ? 0 : (w > 0xFFFFFFFEll ? 0xFFFFFFFEll : w));
    sidx[s] = s;
}

// n_select = externals * percent / 100 (Python's len * topk_percent // 100 on non-negatives);
// counts[0] = merged size, counts[1] = n_select, counts[2] = distinct external neighbours.
__global__ void halo_select_kernel(int64_t t, int64_t p, int percent, const uint32_t *__restrict__ head,
                                   const uint32_t *__restrict__ seg, int64_t *__restrict__ counts) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int64_t ext = t > 0 ? (int64_t)(seg[t - 1] + head[t - 1]) : 0;
    const int64_t sel = percent > 0 ? ext * percent / 100 : 0;
    counts[0] = p + sel;
    counts[1] = sel;
    counts[2] = ext;
}

// union = window nodes then the selected externals, padded with key n to p + t entries
__global__ void halo_union_kernel(int64_t p, int64_t t, uint32_t n, const int64_t *__restrict__ part,
                                  const uint32_t *__restrict__ order, const uint32_t *__restrict__ seg_nb,
                                  const int64_t *__restrict__ counts, uint32_t *__restrict__ key,
                                  uint32_t *__restrict__ idx) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j >= p + t) return;
    const int64_t sel = counts[1];
    uint32_t k = n;
    if (j < p) {
        const int64_t x = part[j];
        k = (x >= 0 && x < (int64_t)n) ? (uint32_t)x : n;
    } else if (j - p < sel) {
        k = seg_nb[order[j - p]];
    }
    key[j] = k;
    idx[j] = (uint32_t)j;
}

__global__ void halo_out_kernel(int64_t cap, const uint32_t *__restrict__ key, const int64_t *__restrict__ counts,
                                int64_t *__restrict__ out) {
    const int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (j < cap && j < counts[0]) out[j] = (int64_t)key[j];
}

struct HaloWs {
    int32_t *member, *bad, *wpos;
    int64_t *deg, *off, *off_partials, *total, *wsorted, *wscan, *w_partials;
    uint32_t *ka, *kb, *va, *vb, *head, *seg, *seg_nb, *seg_end, *fk, *wk, *hist, *partials;
};

HaloWs carve_halo(void *base, size_t cap, int64_t n, int64_t p, int64_t t, size_t *used) {
    Carver c(base, cap);
    HaloWs w;
    const int64_t big = (p + t) > 1 ? p + t : 1;
    w.member = c.take<int32_t>(n);
    w.bad = c.take<int32_t>(1);
    w.deg = c.take<int64_t>(p + 1);
    w.off = c.take<int64_t>(p + 1);
    w.off_partials = c.take<int64_t>(scan_partials_count(p + 1) + 1);
    w.total = c.take<int64_t>(1);
    w.wpos = c.take<int32_t>(t + 1);
    w.ka = c.take<uint32_t>(big);
    w.kb = c.take<uint32_t>(big);
    w.va = c.take<uint32_t>(big);
    w.vb = c.take<uint32_t>(big);
    w.head = c.take<uint32_t>(t + 1);
    w.seg = c.take<uint32_t>(t + 1);
    w.seg_nb = c.take<uint32_t>(t + 1);
    w.seg_end = c.take<uint32_t>(t + 1);
    w.wsorted = c.take<int64_t>(t + 1);
    w.wscan = c.take<int64_t>(t + 1);
    w.w_partials = c.take<int64_t>(scan_partials_count(t + 1) + 1);
    w.fk = c.take<uint32_t>(t + 1);
    w.wk = c.take<uint32_t>(t + 1);
    const int64_t hist_n = 256 * radix_tiles(big);
    w.hist = c.take<uint32_t>(hist_n);
    w.partials = c.take<uint32_t>(scan_partials_count(hist_n > t + 1 ? hist_n : t + 1) + 1);
    *used = c.used;
    return w;
}

// ---------------------------------------------------------------------------------------------
// duplicate-first ordering
// ---------------------------------------------------------------------------------------------
__global__ void dup_count_kernel(int64_t total, int64_t n, const int64_t *__restrict__ nodes, int32_t *__restrict__ cnt,
                                 int32_t *__restrict__ bad) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i >= total) return;
    const int64_t x = nodes[i];
    if (x < 0 || x >= n) {
        atomicAdd(bad, 1);
        return;
    }
    atomicAdd(cnt + x, 1);
}

__global__ void dup_flag_kernel(int64_t total, int64_t n, const int64_t *__restrict__ nodes,
                                const int32_t *__restrict__ cnt, int64_t *__restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i > total) return;
    if (i == total) {
        flag[i] = 0;
        return;
    }
    const int64_t x = nodes[i];
    flag[i] = (x >= 0 && x < n && cnt[x] >= 2) ? 1 : 0;
}

// Stable partition of each window: its duplicated nodes first, then the others, each in the
// window's order.  fs = exclusive scan of the flags over all windows (total + 1 entries).
__global__ void dup_place_kernel(int64_t total, int parts, const int64_t *__restrict__ offsets,
                                 const int64_t *__restrict__ nodes, const int64_t *__restrict__ flag,
                                 const int64_t *__restrict__ fs, int64_t *__restrict__ out,
                                 int64_t *__restrict__ dup_counts) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i < parts) dup_counts[i] = fs[offsets[i + 1]] - fs[offsets[i]];
    if (i >= total) return;
    int lo = 0, hi = parts - 1;   // window k with offsets[k] <= i < offsets[k + 1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= i) lo = mid;
        else hi = mid - 1;
    }
    const int64_t ok = offsets[lo];
    const int64_t before = fs[i] - fs[ok];
    const int64_t ndup = fs[offsets[lo + 1]] - fs[ok];
    const int64_t at = flag[i] ? before : ndup + (i - ok) - before;
    out[ok + at] = nodes[i];
}

// ---------------------------------------------------------------------------------------------
// random connections of isolated nodes
// ---------------------------------------------------------------------------------------------
// SplitMix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number generators",
// OOPSLA 2014): a counter-based generator, so pair (a, b) gets the same draw on any thread.
__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Bernoulli draw of pair (isolated index a, other index b): top 32 bits of the hash below the
// threshold floor(p * 2^32).
__device__ __forceinline__ bool connect_draw(uint64_t seed, int64_t a, int64_t b, uint64_t threshold) {
    const uint64_t h = splitmix64(seed ^ splitmix64(((uint64_t)a << 32) ^ (uint64_t)b));
    return (h >> 32) < threshold;
}

__global__ void iso_mark_kernel(int64_t m, const int64_t *__restrict__ ei, int64_t n, int32_t *__restrict__ seen,
                                int32_t *__restrict__ bad) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i >= 2 * m) return;
    const int64_t x = ei[i];
    if (x < 0 || x >= n) {
        atomicAdd(bad, 1);
        return;
    }
    seen[x] = 1;
}

__global__ void iso_flags_kernel(int64_t n, const int32_t *__restrict__ seen, int64_t *__restrict__ iso,
                                 int64_t *__restrict__ non) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i > n) return;
    iso[i] = (i < n && !seen[i]) ? 1 : 0;
    non[i] = (i < n && seen[i]) ? 1 : 0;
}

// ascending lists of isolated and of appeared nodes (torch.arange(n)[mask] order)
__global__ void iso_compact_kernel(int64_t n, const int32_t *__restrict__ seen, const int64_t *__restrict__ iso_pos,
                                   const int64_t *__restrict__ non_pos, int64_t *__restrict__ iso_list,
                                   int64_t *__restrict__ non_list, int64_t *__restrict__ counts) {
    const int64_t i = (int64_t)blockIdx.x * kT + threadIdx.x;
    if (i == 0) {
        counts[0] = iso_pos[n];
        counts[1] = non_pos[n];
    }
    if (i >= n) return;
    if (seen[i]) non_list[non_pos[i]] = i;
    else iso_list[iso_pos[i]] = i;
}

// one block per isolated node a: how many of the appeared nodes it connects to
__global__ void __launch_bounds__(kT) iso_row_count_kernel(const int64_t *__restrict__ counts, uint64_t seed,
                                                           uint64_t threshold, int64_t *__restrict__ rowcnt) {
    const int64_t ni = counts[0], nn = counts[1];
    __shared__ int64_t part[kT / 32];
    for (int64_t a = blockIdx.x; a < ni; a += gridDim.x) {
        int64_t c = 0;
        for (int64_t b = threadIdx.x; b < nn; b += kT) c += connect_draw(seed, a, b, threshold) ? 1 : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
        __syncthreads();
        if (threadIdx.x == 0) {
            int64_t t = 0;
            for (int w = 0; w < kT / 32; w++) t += part[w];
            rowcnt[a] = t;
        }
        __syncthreads();
    }
}

__global__ void iso_total_kernel(const int64_t *__restrict__ rowcnt, const int64_t *__restrict__ rowoff,
                                 int64_t *__restrict__ counts) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const int64_t ni = counts[0];
        counts[2] = ni > 0 ? rowoff[ni - 1] + rowcnt[ni - 1] : 0;
    }
}

// row a's pairs in column order (torch.where order on the dense mask)
__global__ void __launch_bounds__(kT) iso_fill_kernel(const int64_t *__restrict__ counts, uint64_t seed,
                                                      uint64_t threshold, const int64_t *__restrict__ rowoff,
                                                      const int64_t *__restrict__ iso_list,
                                                      const int64_t *__restrict__ non_list, int64_t e_new,
                                                      int64_t *__restrict__ out) {
    const int64_t ni = counts[0], nn = counts[1];
    __shared__ int wsum[kT / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t a = blockIdx.x; a < ni; a += gridDim.x) {
        int64_t base = rowoff[a];
        for (int64_t b0 = 0; b0 < nn; b0 += kT) {
            const int64_t b = b0 + threadIdx.x;
            const bool hit = b < nn && connect_draw(seed, a, b, threshold);
            const uint32_t bal = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) wsum[warp] = __popc(bal);
            __syncthreads();
            int before = 0, all = 0;
            for (int w = 0; w < kT / 32; w++) {
                if (w < warp) before += wsum[w];
                all += wsum[w];
            }
            if (hit) {
                const int64_t at = base + before + __popc(bal & ((1u << lane) - 1u));
                if (at < e_new) {
                    out[at] = iso_list[a];
                    out[e_new + at] = non_list[b];
                }
            }
            base += all;
            __syncthreads();
        }
    }
}

}  // namespace
}  // namespace ngt

using namespace ngt;

// ---------------------------------------------------------------------------------------------
extern "C" int ngt_ppr_adjacency_workspace_size(int64_t m, int64_t n, size_t *bytes) {
    if (!bytes || m < 0 || n < 0) return NGT_ERR_INVALID_ARGUMENT;
    if (m >= ((int64_t)1 << 30) || n >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    carve_adj(nullptr, 0, m, n, bytes);
    return NGT_OK;
}

extern "C" int ngt_ppr_adjacency(int64_t m, int64_t n, const int64_t *edge_index, const float *values,
                                 int32_t *xadj, int32_t *adjncy, int32_t *eweights, int32_t *info, void *workspace,
                                 size_t workspace_bytes, ngt_stream_t stream) {
    if (m < 0 || n < 0 || !xadj || !info) return NGT_ERR_INVALID_ARGUMENT;
    if (m > 0 && (!edge_index || !values || !adjncy || !eweights)) return NGT_ERR_INVALID_ARGUMENT;
    if (m >= ((int64_t)1 << 30) || n >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    size_t need = 0;
    AdjWs w = carve_adj(workspace, workspace_bytes, m, n, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(info, 0, 2 * sizeof(int32_t), st);      // [bad entries, unique undirected edges]
    cudaMemsetAsync(w.deg, 0, sizeof(int32_t) * (size_t)(n + 1), st);
    if (m > 0) {
        const int kbits = bits_for(n > 0 ? n - 1 : 0);
        adj_keys_kernel<<<grid_for(m), kT, 0, st>>>(m, n, edge_index, w.ku, w.kv, w.va, info);
        // stable sort by (u, v): v first, then u
        cudaMemcpyAsync(w.ka, w.kv, sizeof(uint32_t) * (size_t)m, cudaMemcpyDeviceToDevice, st);
        int where = 0;
        int rc = radix_sort_pairs(w.ka, w.va, w.kb, w.vb, m, kbits, w.hist, w.partials, st, &where);
        if (rc) return rc;
        uint32_t *perm1 = where ? w.vb : w.va;
        uint32_t *other = where ? w.va : w.vb;
        gather_u32_kernel<<<grid_for(m), kT, 0, st>>>(m, perm1, w.ku, w.ka);
        cudaMemcpyAsync(other, perm1, sizeof(uint32_t) * (size_t)m, cudaMemcpyDeviceToDevice, st);
        rc = radix_sort_pairs(w.ka, other, w.kb, perm1, m, kbits, w.hist, w.partials, st, &where);
        if (rc) return rc;
        uint32_t *perm = where ? perm1 : other;
        adj_heads_kernel<<<grid_for(m + 1), kT, 0, st>>>(m, perm, w.ku, w.kv, w.head);
        rc = exclusive_scan<uint32_t>(w.head, w.seg, m + 1, w.partials, st);
        if (rc) return rc;
        adj_segments_kernel<<<grid_for(m), kT, 0, st>>>(m, perm, w.ku, w.kv, values, w.head, w.seg, w.uu, w.vv, w.ww,
                                                         info + 1);
        // rows of the symmetric list, stable by row
        adj_sym_kernel<<<grid_for(2 * m), kT, 0, st>>>(m, (uint32_t)n, info + 1, w.uu, w.vv, w.ka, w.va, w.deg);
        rc = radix_sort_pairs(w.ka, w.va, w.kb, w.vb, 2 * m, bits_for(n), w.hist, w.partials, st, &where);
        if (rc) return rc;
        adj_emit_kernel<<<grid_for(2 * m), kT, 0, st>>>(m, info + 1, where ? w.vb : w.va, w.uu, w.vv, w.ww, adjncy,
                                                        eweights);
    }
    int rc = exclusive_scan<int32_t>(w.deg, xadj, n + 1, w.deg_partials, st);
    if (rc) return rc;
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// ---------------------------------------------------------------------------------------------
extern "C" int ngt_halo_degree(int64_t n, const int32_t *xadj, int64_t p, const int64_t *part, int64_t *total,
                               void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || p < 0 || !total || (p > 0 && (!xadj || !part))) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    size_t need = 0;
    HaloWs w = carve_halo(workspace, workspace_bytes, n, p, 0, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(w.member, 0, sizeof(int32_t) * (size_t)n, st);
    cudaMemsetAsync(w.bad, 0, sizeof(int32_t), st);
    if (p == 0) {
        cudaMemsetAsync(total, 0, sizeof(int64_t), st);
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    halo_mark_kernel<<<grid_for(p), kT, 0, st>>>(p, n, part, xadj, w.member, w.deg, w.bad);
    int rc = exclusive_scan<int64_t>(w.deg, w.off, p, w.off_partials, st);
    if (rc) return rc;
    sum_i64_kernel<<<1, 32, 0, st>>>(p, w.deg, w.off, total);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_halo_merge_workspace_size(int64_t n, int64_t p, int64_t total, size_t *bytes) {
    if (!bytes || n < 0 || p < 0 || total < 0) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || p + total >= (int64_t)UINT32_MAX) return NGT_ERR_TOO_LARGE;
    carve_halo(nullptr, 0, n, p, total, bytes);
    return NGT_OK;
}

extern "C" int ngt_halo_merge(int64_t n, const int32_t *xadj, const int32_t *adjncy, const int32_t *eweights,
                              int64_t p, const int64_t *part, int64_t total, int32_t topk_percent, int64_t *out,
                              int64_t *counts, void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || p < 0 || total < 0 || topk_percent < 0 || !counts || (p + total > 0 && !out))
        return NGT_ERR_INVALID_ARGUMENT;
    if (p > 0 && (!xadj || !part)) return NGT_ERR_INVALID_ARGUMENT;
    if (total > 0 && (!adjncy || !eweights)) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || p + total >= (int64_t)UINT32_MAX) return NGT_ERR_TOO_LARGE;
    size_t need = 0;
    HaloWs w = carve_halo(workspace, workspace_bytes, n, p, total, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // membership and offsets again (the workspace may have been reused since ngt_halo_degree)
    cudaMemsetAsync(w.member, 0, sizeof(int32_t) * (size_t)n, st);
    cudaMemsetAsync(w.bad, 0, sizeof(int32_t), st);
    if (p > 0) {
        halo_mark_kernel<<<grid_for(p), kT, 0, st>>>(p, n, part, xadj, w.member, w.deg, w.bad);
        int rc = exclusive_scan<int64_t>(w.deg, w.off, p, w.off_partials, st);
        if (rc) return rc;
    }
    const uint32_t un = (uint32_t)n;
    int where = 0;
    uint32_t *order = w.va;
    if (total > 0) {
        halo_expand_kernel<<<grid_for(32 * p), kT, 0, st>>>(p, un, part, xadj, adjncy, eweights, w.member, w.off, w.ka,
                                                            w.va, w.wpos);
        int rc = radix_sort_pairs(w.ka, w.va, w.kb, w.vb, total, bits_for(n), w.hist, w.partials, st, &where);
        if (rc) return rc;
        uint32_t *skey = where ? w.kb : w.ka, *spos = where ? w.vb : w.va;
        halo_heads_kernel<<<grid_for(total + 1), kT, 0, st>>>(total, un, skey, w.head);
        rc = exclusive_scan<uint32_t>(w.head, w.seg, total + 1, w.partials, st);
        if (rc) return rc;
        // free buffers for the segment sort: the one not holding (skey, spos)
        uint32_t *ska = where ? w.ka : w.kb, *sva = where ? w.va : w.vb;
        halo_runs_kernel<<<grid_for(total + 1), kT, 0, st>>>(total, un, skey, spos, w.wpos, w.head, w.seg,
                                                              w.wsorted, w.seg_end);
        rc = exclusive_scan<int64_t>(w.wsorted, w.wscan, total + 1, w.w_partials, st);
        if (rc) return rc;
        halo_segments_kernel<<<grid_for(total), kT, 0, st>>>(total, un, skey, spos, w.wscan, w.seg_end, w.head, w.seg,
                                                              w.seg_nb, w.fk, w.wk, sva);
        halo_select_kernel<<<1, 32, 0, st>>>(total, p, topk_percent, w.head, w.seg, counts);
        // order the externals by (weight desc, first encounter asc): stable sort by position, then
        // stable sort by inverted weight (the other key buffers are free now)
        rc = radix_sort_pairs(w.fk, sva, ska, spos, total, 32, w.hist, w.partials, st, &where);
        if (rc) return rc;
        uint32_t *p1 = where ? spos : sva, *p1_free = where ? sva : spos;
        gather_u32_kernel<<<grid_for(total), kT, 0, st>>>(total, p1, w.wk, ska);
        cudaMemcpyAsync(p1_free, p1, sizeof(uint32_t) * (size_t)total, cudaMemcpyDeviceToDevice, st);
        rc = radix_sort_pairs(ska, p1_free, w.fk, p1, total, 32, w.hist, w.partials, st, &where);
        if (rc) return rc;
        order = where ? p1 : p1_free;
        // the union goes into the buffers that do not hold `order`: (w.kb or w.ka) pair chosen below
    } else {
        halo_select_kernel<<<1, 32, 0, st>>>(0, p, topk_percent, w.head, w.seg, counts);
    }
    // union buffers: any two key and two value buffers of p + total entries not aliasing `order`
    uint32_t *bufs[4] = {w.ka, w.kb, w.va, w.vb};
    uint32_t *free_b[4];
    int nf = 0;
    for (int i = 0; i < 4; i++)
        if (bufs[i] != order) free_b[nf++] = bufs[i];
    const int64_t cap = p + total;
    if (cap > 0) {
        halo_union_kernel<<<grid_for(cap), kT, 0, st>>>(p, total, un, part, order, w.seg_nb, counts, free_b[0],
                                                       free_b[1]);
        int rc = radix_sort_pairs(free_b[0], free_b[1], free_b[2], order, cap, bits_for(n), w.hist, w.partials, st,
                                  &where);
        if (rc) return rc;
        halo_out_kernel<<<grid_for(cap), kT, 0, st>>>(cap, where ? free_b[2] : free_b[0], counts, out);
    }
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// ---------------------------------------------------------------------------------------------
extern "C" int ngt_duplicate_rerange_workspace_size(int64_t n, int64_t total, size_t *bytes) {
    if (!bytes || n < 0 || total < 0) return NGT_ERR_INVALID_ARGUMENT;
    Carver c(nullptr, 0);
    c.take<int32_t>(n);
    c.take<int32_t>(1);
    c.take<int64_t>(total + 1);
    c.take<int64_t>(total + 1);
    c.take<int64_t>(scan_partials_count(total + 1) + 1);
    *bytes = c.used;
    return NGT_OK;
}

extern "C" int ngt_duplicate_rerange(int64_t n, int32_t parts, const int64_t *offsets, const int64_t *nodes,
                                     int64_t total, int64_t *out_nodes, int64_t *dup_counts, int32_t *bad,
                                     void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || parts < 0 || total < 0 || !bad) return NGT_ERR_INVALID_ARGUMENT;
    if (parts > 0 && (!offsets || !dup_counts)) return NGT_ERR_INVALID_ARGUMENT;
    if (total > 0 && (!nodes || !out_nodes)) return NGT_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    ngt_duplicate_rerange_workspace_size(n, total, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    Carver c(workspace, workspace_bytes);
    int32_t *cnt = c.take<int32_t>(n);
    c.take<int32_t>(1);
    int64_t *flag = c.take<int64_t>(total + 1);
    int64_t *fs = c.take<int64_t>(total + 1);
    int64_t *partials = c.take<int64_t>(scan_partials_count(total + 1) + 1);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(bad, 0, sizeof(int32_t), st);
    if (n > 0) cudaMemsetAsync(cnt, 0, sizeof(int32_t) * (size_t)n, st);
    if (parts == 0) {
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    if (total > 0) dup_count_kernel<<<grid_for(total), kT, 0, st>>>(total, n, nodes, cnt, bad);
    dup_flag_kernel<<<grid_for(total + 1), kT, 0, st>>>(total, n, nodes, cnt, flag);
    int rc = exclusive_scan<int64_t>(flag, fs, total + 1, partials, st);
    if (rc) return rc;
    const int64_t g = total > parts ? total : parts;
    dup_place_kernel<<<grid_for(g), kT, 0, st>>>(total, parts, offsets, nodes, flag, fs, out_nodes, dup_counts);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// ---------------------------------------------------------------------------------------------
namespace {
struct IsoWs {
    int32_t *seen, *bad;
    int64_t *iso, *non, *iso_pos, *non_pos, *partials, *iso_list, *non_list, *rowcnt, *rowoff, *row_partials;
};
IsoWs carve_iso(void *base, size_t cap, int64_t n, size_t *used) {
    Carver c(base, cap);
    IsoWs w;
    w.seen = c.take<int32_t>(n + 1);
    w.bad = c.take<int32_t>(1);
    w.iso = c.take<int64_t>(n + 1);
    w.non = c.take<int64_t>(n + 1);
    w.iso_pos = c.take<int64_t>(n + 1);
    w.non_pos = c.take<int64_t>(n + 1);
    w.partials = c.take<int64_t>(scan_partials_count(n + 1) + 1);
    w.iso_list = c.take<int64_t>(n + 1);
    w.non_list = c.take<int64_t>(n + 1);
    w.rowcnt = c.take<int64_t>(n + 1);
    w.rowoff = c.take<int64_t>(n + 1);
    w.row_partials = c.take<int64_t>(scan_partials_count(n + 1) + 1);
    *used = c.used;
    return w;
}
uint64_t prob_threshold(double p) {
    if (!(p > 0.0)) return 0;
    if (p >= 1.0) return (uint64_t)1 << 32;
    return (uint64_t)(p * 4294967296.0);
}
}  // namespace

extern "C" int ngt_isolated_connections_workspace_size(int64_t n, size_t *bytes) {
    if (!bytes || n < 0) return NGT_ERR_INVALID_ARGUMENT;
    carve_iso(nullptr, 0, n, bytes);
    return NGT_OK;
}

extern "C" int ngt_isolated_connections_count(int64_t n, int64_t m_ppr, const int64_t *ppr_edge_index,
                                              int64_t m_graph, const int64_t *graph_edge_index, double connect_prob,
                                              uint64_t seed, int64_t *counts, int32_t *bad, void *workspace,
                                              size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || m_ppr < 0 || m_graph < 0 || !counts || !bad) return NGT_ERR_INVALID_ARGUMENT;
    if ((m_ppr > 0 && !ppr_edge_index) || (m_graph > 0 && !graph_edge_index)) return NGT_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    IsoWs w = carve_iso(workspace, workspace_bytes, n, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(counts, 0, 3 * sizeof(int64_t), st);
    cudaMemsetAsync(bad, 0, sizeof(int32_t), st);
    cudaMemsetAsync(w.seen, 0, sizeof(int32_t) * (size_t)(n + 1), st);
    if (m_ppr > 0) iso_mark_kernel<<<grid_for(2 * m_ppr), kT, 0, st>>>(m_ppr, ppr_edge_index, n, w.seen, bad);
    if (m_graph > 0) iso_mark_kernel<<<grid_for(2 * m_graph), kT, 0, st>>>(m_graph, graph_edge_index, n, w.seen, bad);
    iso_flags_kernel<<<grid_for(n + 1), kT, 0, st>>>(n, w.seen, w.iso, w.non);
    int rc = exclusive_scan<int64_t>(w.iso, w.iso_pos, n + 1, w.partials, st);
    if (rc) return rc;
    rc = exclusive_scan<int64_t>(w.non, w.non_pos, n + 1, w.partials, st);
    if (rc) return rc;
    iso_compact_kernel<<<grid_for(n > 0 ? n : 1), kT, 0, st>>>(n, w.seen, w.iso_pos, w.non_pos, w.iso_list, w.non_list,
                                                              counts);
    const uint64_t thr = prob_threshold(connect_prob);
    if (n > 0) {
        cudaMemsetAsync(w.rowcnt, 0, sizeof(int64_t) * (size_t)(n + 1), st);
        iso_row_count_kernel<<<1184, kT, 0, st>>>(counts, seed, thr, w.rowcnt);
        rc = exclusive_scan<int64_t>(w.rowcnt, w.rowoff, n + 1, w.row_partials, st);
        if (rc) return rc;
        iso_total_kernel<<<1, 32, 0, st>>>(w.rowcnt, w.rowoff, counts);
    }
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_isolated_connections_fill(int64_t n, double connect_prob, uint64_t seed, const int64_t *counts,
                                             int64_t e_new, int64_t *new_edge_index, void *workspace,
                                             size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || e_new < 0 || !counts || (e_new > 0 && !new_edge_index)) return NGT_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    IsoWs w = carve_iso(workspace, workspace_bytes, n, &need);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    if (e_new == 0 || n == 0) return NGT_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    iso_fill_kernel<<<1184, kT, 0, st>>>(counts, seed, prob_threshold(connect_prob), w.rowoff, w.iso_list, w.non_list,
                                         e_new, new_edge_index);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}
