// Window edge list -> destination/source-major CSR, and the window subgraph (sm_100a).
//
// ngt_edge_csr_build: the reference gathers and scatters by edge_index on every call
// (NeutronGT/models/gt_dist_node_level_single_window.py:130-131, 161-178).  The kernels
// here read two CSR views instead, built once per window: the edge list is validated,
// then stably radix-sorted by destination and by source (edge ids as values), and the
// row pointers come from a per-row count and an exclusive scan.
//
// ngt_window_subgraph_*: `_subgraph_from_csr`
// (NeutronGT/core/node_level_pipeline/window_state.py:92-119) on the device.  A global ->
// window-position map is scattered once; one warp per window node counts (pass 1) and
// then compacts in CSR order with a ballot (pass 2), so the output order equals the
// reference's: window order for the source, CSR order within a source.
#include "scan_sort.cuh"

namespace ngt {
namespace {

constexpr int kThreads = 256;

// ---------------- edge list -> CSR ----------------
__global__ void extract_edges(int64_t e, int64_t n, const int64_t *__restrict__ ei,
                              uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                              uint32_t *__restrict__ eid, int32_t *__restrict__ dst_count,
                              int32_t *__restrict__ src_count, int32_t *__restrict__ info) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= e) return;
    int64_t s = ei[i], d = ei[e + i];
    if (s < 0 || s >= n || d < 0 || d >= n) {
        atomicAdd(info, 1);
        s = 0;  // keep every later access in bounds; the caller sees info[0] != 0
        d = 0;
    }
    src[i] = (uint32_t)s;
    dst[i] = (uint32_t)d;
    eid[i] = (uint32_t)i;
    atomicAdd(dst_count + d, 1);
    atomicAdd(src_count + s, 1);
    atomicMax(info + 1, (int32_t)d);
}

__global__ void init_info(int32_t *info) {
    info[0] = 0;
    info[1] = -1;
}

__global__ void gather_u32(int64_t e, const uint32_t *__restrict__ perm,
                           const uint32_t *__restrict__ from, int32_t *__restrict__ to) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < e) to[i] = (int32_t)from[perm[i]];
}

__global__ void iota_u32(int64_t e, uint32_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < e) out[i] = (uint32_t)i;
}

__global__ void invert_perm(int64_t e, const uint32_t *__restrict__ perm, uint32_t *__restrict__ inv) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < e) inv[perm[i]] = (uint32_t)i;
}

struct CsrWs {
    uint32_t *src, *dst, *keys_a, *vals_a, *keys_b, *vals_b, *pos_in_dst, *hist, *partials;
    int32_t *counts_d, *counts_s, *rp_partials;
};

CsrWs carve_csr(void *base, size_t cap, int64_t n, int64_t e, size_t *used) {
    Carver c(base, cap);
    CsrWs w;
    w.src = c.take<uint32_t>(e);
    w.dst = c.take<uint32_t>(e);
    w.keys_a = c.take<uint32_t>(e);
    w.vals_a = c.take<uint32_t>(e);
    w.keys_b = c.take<uint32_t>(e);
    w.vals_b = c.take<uint32_t>(e);
    w.pos_in_dst = c.take<uint32_t>(e);
    const int64_t nh = 256 * radix_tiles(e > 0 ? e : 1);
    w.hist = c.take<uint32_t>(nh);
    w.partials = c.take<uint32_t>(scan_partials_count(nh) + 1);
    w.counts_d = c.take<int32_t>(n + 1);
    w.counts_s = c.take<int32_t>(n + 1);
    w.rp_partials = c.take<int32_t>(scan_partials_count(n + 1) + 1);
    *used = c.used;
    return w;
}

// ---------------- window subgraph ----------------
__global__ void map_nodes(int64_t w, int64_t num_global, const int64_t *__restrict__ nodes,
                          int32_t *__restrict__ map, int32_t *__restrict__ info) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= w) return;
    const int64_t g = nodes[i];
    if (g < 0 || g >= num_global) {
        atomicAdd(info, 1);
        return;
    }
    const int32_t prev = atomicExch(map + g, (int32_t)i);
    if (prev != -1) atomicAdd(info, 1);  // repeated window node
}

__global__ void subgraph_count(int64_t w, const int64_t *__restrict__ rowptr,
                               const int64_t *__restrict__ col, const int64_t *__restrict__ nodes,
                               const int32_t *__restrict__ map, int64_t num_global,
                               int64_t *__restrict__ counts) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= w) return;
    const int64_t g = nodes[row];
    int64_t cnt = 0;
    if (g >= 0 && g < num_global) {
        const int64_t b = rowptr[g], en = rowptr[g + 1];
        for (int64_t p = b + lane; p < en; p += 32) {
            const int64_t c = col[p];
            cnt += (c >= 0 && c < num_global && map[c] >= 0) ? 1 : 0;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
    if (lane == 0) counts[row] = cnt;
}

__global__ void subgraph_fill(int64_t w, const int64_t *__restrict__ rowptr,
                              const int64_t *__restrict__ col, const int64_t *__restrict__ nodes,
                              const int32_t *__restrict__ map, int64_t num_global,
                              const int64_t *__restrict__ out_rowptr, int64_t total,
                              int64_t *__restrict__ out) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= w) return;
    const int64_t g = nodes[row];
    if (g < 0 || g >= num_global) return;
    int64_t pos = out_rowptr[row];
    const int64_t b = rowptr[g], en = rowptr[g + 1];
    for (int64_t p0 = b; p0 < en; p0 += 32) {
        const int64_t p = p0 + lane;
        int32_t loc = -1;
        if (p < en) {
            const int64_t c = col[p];
            if (c >= 0 && c < num_global) loc = map[c];
        }
        const uint32_t ball = __ballot_sync(0xffffffffu, loc >= 0);
        if (loc >= 0) {
            const int64_t o = pos + __popc(ball & ((1u << lane) - 1u));
            if (o < total) {
                out[o] = row;
                out[total + o] = loc;
            }
        }
        pos += __popc(ball);
    }
}

struct SubWs {
    int32_t *map;
    int64_t *counts, *partials;
};

SubWs carve_sub(void *base, size_t cap, int64_t num_global, int64_t w, size_t *used) {
    Carver c(base, cap);
    SubWs s;
    s.map = c.take<int32_t>(num_global);
    s.counts = c.take<int64_t>(w + 1);
    s.partials = c.take<int64_t>(scan_partials_count(w + 1) + 1);
    *used = c.used;
    return s;
}

// Upper bound on the segments of one view: each heavy row has more than seg_edges entries, so
// sum ceil(d / seg_edges) <= e / seg_edges + (heavy rows) <= 2 e / seg_edges.
int64_t segment_capacity(int64_t e, int seg_edges) { return 2 * ((e + seg_edges - 1) / seg_edges) + 1; }

// Heavy-row segments of both CSR views.  Thread i < n handles destination row i, thread n + i
// source row i.  A row of degree d > seg_edges gets ceil(d / seg_edges) consecutive segment
// numbers from its view's counter (their position among rows depends on scheduling; the rows a
// segment covers and the order its partial sums are combined in do not); other rows get -1.
__global__ void csr_segments_kernel(int n, const int32_t *__restrict__ dst_rowptr,
                                    const int32_t *__restrict__ src_rowptr, int seg_edges, int64_t cap,
                                    int32_t *__restrict__ seg_first, int32_t *__restrict__ seg_row,
                                    int32_t *__restrict__ counts) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 2 * (int64_t)n) return;
    const int view = i >= n;
    const int r = (int)(view ? i - n : i);
    const int32_t *rp = view ? src_rowptr : dst_rowptr;
    const int deg = rp[r + 1] - rp[r];
    if (deg <= seg_edges) {
        seg_first[i] = -1;
        return;
    }
    const int ns = (deg + seg_edges - 1) / seg_edges;
    const int s0 = atomicAdd(counts + view, ns);
    seg_first[i] = s0;
    for (int j = 0; j < ns; j++)
        if (s0 + j < cap) seg_row[(size_t)view * cap + s0 + j] = r;
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_edge_csr_segment_capacity(int64_t e, int32_t seg_edges, int64_t *cap) {
    if (e < 0 || seg_edges <= 0 || !cap) return NGT_ERR_INVALID_ARGUMENT;
    *cap = segment_capacity(e, seg_edges);
    return NGT_OK;
}

extern "C" int ngt_edge_csr_segments(int64_t n, int64_t e, const int32_t *dst_rowptr, const int32_t *src_rowptr,
                                     int32_t seg_edges, int32_t *seg_first, int32_t *seg_row, int32_t *counts,
                                     ngt_stream_t stream) {
    if (n < 0 || e < 0 || seg_edges <= 0 || !counts) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || e >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(counts, 0, 2 * sizeof(int32_t), st);
    if (n > 0) {
        if (!dst_rowptr || !src_rowptr || !seg_first || (e > 0 && !seg_row)) return NGT_ERR_INVALID_ARGUMENT;
        const int64_t cap = segment_capacity(e, seg_edges);
        const unsigned g = (unsigned)((2 * n + kThreads - 1) / kThreads);
        csr_segments_kernel<<<g, kThreads, 0, st>>>((int)n, dst_rowptr, src_rowptr, seg_edges, cap, seg_first,
                                                    seg_row, counts);
    }
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_edge_csr_workspace_size(int64_t n, int64_t e, size_t *bytes) {
    if (n < 0 || e < 0 || !bytes) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || e >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    carve_csr(nullptr, 0, n, e, bytes);
    return NGT_OK;
}

extern "C" int ngt_edge_csr_build(int64_t n, int64_t e, const int64_t *edge_index,
                                  int32_t *dst_rowptr, int32_t *dst_src, int32_t *src_rowptr,
                                  int32_t *src_dst, int32_t *src_to_dst_slot, int32_t *info,
                                  void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (n < 0 || e < 0 || !dst_rowptr || !src_rowptr || !info) return NGT_ERR_INVALID_ARGUMENT;
    if (e > 0 && (!edge_index || !dst_src || !src_dst)) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || e >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    size_t need = 0;
    CsrWs w = carve_csr(workspace, workspace_bytes, n, e, &need);
    if (workspace == nullptr || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    init_info<<<1, 1, 0, st>>>(info);
    cudaMemsetAsync(w.counts_d, 0, sizeof(int32_t) * (size_t)(n + 1), st);
    cudaMemsetAsync(w.counts_s, 0, sizeof(int32_t) * (size_t)(n + 1), st);
    const unsigned ge = (unsigned)((e + kThreads - 1) / kThreads);
    if (e > 0)
        extract_edges<<<ge, kThreads, 0, st>>>(e, n, edge_index, w.src, w.dst, w.vals_a,
                                               w.counts_d, w.counts_s, info);
    NGT_CHECK_LAUNCH();
    int rc = exclusive_scan<int32_t>(w.counts_d, dst_rowptr, n + 1, w.rp_partials, st);
    if (rc) return rc;
    rc = exclusive_scan<int32_t>(w.counts_s, src_rowptr, n + 1, w.rp_partials, st);
    if (rc) return rc;
    if (e == 0) return NGT_OK;
    const int bits = bits_for(n > 0 ? n - 1 : 0);

    // destination-major: keys = dst, values = edge id (w.vals_a holds 0..e-1)
    cudaMemcpyAsync(w.keys_a, w.dst, sizeof(uint32_t) * (size_t)e, cudaMemcpyDeviceToDevice, st);
    int where = 0;
    rc = radix_sort_pairs(w.keys_a, w.vals_a, w.keys_b, w.vals_b, e, bits, w.hist, w.partials, st, &where);
    if (rc) return rc;
    uint32_t *perm_d = where ? w.vals_b : w.vals_a;
    gather_u32<<<ge, kThreads, 0, st>>>(e, perm_d, w.src, dst_src);
    if (src_to_dst_slot) invert_perm<<<ge, kThreads, 0, st>>>(e, perm_d, w.pos_in_dst);
    NGT_CHECK_LAUNCH();

    // source-major: keys = src, values = edge id
    iota_u32<<<ge, kThreads, 0, st>>>(e, w.vals_a);
    cudaMemcpyAsync(w.keys_a, w.src, sizeof(uint32_t) * (size_t)e, cudaMemcpyDeviceToDevice, st);
    rc = radix_sort_pairs(w.keys_a, w.vals_a, w.keys_b, w.vals_b, e, bits, w.hist, w.partials, st, &where);
    if (rc) return rc;
    uint32_t *perm_s = where ? w.vals_b : w.vals_a;
    gather_u32<<<ge, kThreads, 0, st>>>(e, perm_s, w.dst, src_dst);
    if (src_to_dst_slot) gather_u32<<<ge, kThreads, 0, st>>>(e, perm_s, w.pos_in_dst, src_to_dst_slot);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_window_subgraph_workspace_size(int64_t num_global_nodes, int64_t window_nodes,
                                                  size_t *bytes) {
    if (num_global_nodes < 0 || window_nodes < 0 || !bytes) return NGT_ERR_INVALID_ARGUMENT;
    if (window_nodes >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    carve_sub(nullptr, 0, num_global_nodes, window_nodes, bytes);
    return NGT_OK;
}

extern "C" int ngt_window_subgraph_count(int64_t num_global_nodes, const int64_t *rowptr,
                                         const int64_t *col, const int64_t *nodes,
                                         int64_t window_nodes, int64_t *out_rowptr, int32_t *info,
                                         void *workspace, size_t workspace_bytes,
                                         ngt_stream_t stream) {
    if (num_global_nodes < 0 || window_nodes < 0 || !rowptr || !out_rowptr || !info)
        return NGT_ERR_INVALID_ARGUMENT;
    if (window_nodes > 0 && (!nodes || !col)) return NGT_ERR_INVALID_ARGUMENT;
    if (window_nodes >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    size_t need = 0;
    SubWs w = carve_sub(workspace, workspace_bytes, num_global_nodes, window_nodes, &need);
    if (workspace == nullptr || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaMemsetAsync(info, 0, sizeof(int32_t), st);
    cudaMemsetAsync(w.map, 0xff, sizeof(int32_t) * (size_t)num_global_nodes, st);
    cudaMemsetAsync(w.counts, 0, sizeof(int64_t) * (size_t)(window_nodes + 1), st);
    if (window_nodes > 0) {
        const unsigned g = (unsigned)((window_nodes + kThreads - 1) / kThreads);
        map_nodes<<<g, kThreads, 0, st>>>(window_nodes, num_global_nodes, nodes, w.map, info);
        const unsigned gw = (unsigned)((window_nodes * 32 + kThreads - 1) / kThreads);
        subgraph_count<<<gw, kThreads, 0, st>>>(window_nodes, rowptr, col, nodes, w.map,
                                                num_global_nodes, w.counts);
        NGT_CHECK_LAUNCH();
    }
    return exclusive_scan<int64_t>(w.counts, out_rowptr, window_nodes + 1, w.partials, st);
}

extern "C" int ngt_window_subgraph_fill(int64_t num_global_nodes, const int64_t *rowptr,
                                        const int64_t *col, const int64_t *nodes,
                                        int64_t window_nodes, const int64_t *out_rowptr,
                                        int64_t *out_edge_index, int64_t num_edges,
                                        void *workspace, size_t workspace_bytes,
                                        ngt_stream_t stream) {
    if (num_global_nodes < 0 || window_nodes < 0 || num_edges < 0 || !rowptr || !out_rowptr)
        return NGT_ERR_INVALID_ARGUMENT;
    if (num_edges > 0 && (!out_edge_index || !nodes || !col)) return NGT_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    SubWs w = carve_sub(workspace, workspace_bytes, num_global_nodes, window_nodes, &need);
    if (workspace == nullptr || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    if (window_nodes == 0 || num_edges == 0) return NGT_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const unsigned gw = (unsigned)((window_nodes * 32 + kThreads - 1) / kThreads);
    subgraph_fill<<<gw, kThreads, 0, st>>>(window_nodes, rowptr, col, nodes, w.map, num_global_nodes,
                                           out_rowptr, num_edges, out_edge_index);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}
