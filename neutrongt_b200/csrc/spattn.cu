// Graph-sparse window attention: fused forward and atomic-free backward (sm_100a).
//
// Forward replaces `CoreAttention.sparse_attention_bias`
// (NeutronGT/models/gt_dist_node_level_single_window.py:112-179).  The reference builds
// about eight [E, H, D] tensors per layer (gathers, products, exp, messages) and three
// atomic scatters; here one warp owns one destination row, walks its in-edges from the
// dst-major CSR, and keeps the score, exp, normaliser and weighted sum in registers, so
// per-edge values never reach HBM.  HBM traffic per edge is one gathered K row and one
// gathered V row (plus a 4-byte column index); per row, one Q row in and one output row
// out.
//
// Backward is the reference's autograd graph written out (see oracle/attention.py for the
// formulas).  It runs as two launches: a per-row delta = <dout, out> pass, then one launch
// whose first half of blocks walks the dst-major CSR (dq) and whose second half walks the
// src-major CSR (dk, dv), recomputing scores instead of storing them.  Every output row is
// written by exactly one warp, so no atomics and no zero-fill are needed, and reruns are
// bitwise identical.
//
// Lane layout of the vector path: a row of H*D elements is ROW_VECS 16-byte vectors.  A
// group of G = min(ROW_VECS, 32) lanes cooperates on one edge (lane gl owns vectors
// gl + G*t), so a warp keeps 32/G edges of the same row in flight, times UNROLL.  A head
// spans HEAD_VECS consecutive lanes; its dot product is reduced with xor shuffles.  Rows of 128
// elements run separate packed-math kernels: spattn_*_r128 (bf16, the 65,536-token workload) and
// spattn_*_f128 (fp32, the GT model).
#include <mutex>

#include "common.cuh"

namespace ngt {
namespace {

constexpr float kClamp = 5.0f;
constexpr float kEps = 1e-6f;
constexpr int kBlock = 256;
constexpr int kWarpsPerBlock = kBlock / kWarp;

template <typename T, int HEAD_VECS, int ROW_VECS>
struct VecLayout {
    static constexpr int G = ROW_VECS < 32 ? ROW_VECS : 32;
    static constexpr int VPL = ROW_VECS / G;
    static constexpr int EPW = 32 / G;
    static constexpr int VE = Elem<T>::kPerVec;
    static constexpr int UNROLL = VPL >= 4 ? 1 : 4 / VPL;
    static_assert(ROW_VECS % G == 0, "row vectors must tile the lane group");
    static_assert(G % HEAD_VECS == 0, "a head must not straddle lane groups");
};

template <int HEAD_VECS>
__device__ __forceinline__ float head_reduce(float x) {
#pragma unroll
    for (int off = 1; off < HEAD_VECS; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

// Sum over the EPW edge slots of a warp (lanes with equal gl in different groups).
template <int G>
__device__ __forceinline__ float slot_reduce(float x) {
#pragma unroll
    for (int off = G; off < 32; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

// Heavy-row segments of one CSR view (all null / 0: every row is one warp's work).  A row with
// more than `edges` entries is split into consecutive segments of `edges` entries; segment s
// covers entries [rowptr[row[s]] + (s - first[row[s]]) * edges, +edges) of row row[s].  Its warp
// writes partial sums to part[s]; a finish pass adds a row's partials in segment order.
struct SegView {
    int edges;
    const int32_t *first;   // [n] first segment of a heavy row, -1 for other rows
    const int32_t *row;     // [nseg] row of each segment
    int nseg;
    float *part;            // [nseg][record]
};

__host__ __device__ inline int fwd_record(int heads, int row_floats) { return row_floats + ((heads + 3) & ~3); }

// ------------------------------------------------------------------------------------
// forward (vector path)
// ------------------------------------------------------------------------------------
// Output row, Z and node score of a finished row (acc and zs complete in every lane group).
template <typename T, int HEAD_VECS, int ROW_VECS>
__device__ __forceinline__ void fwd_finish(int row, int heads, const float (&acc)[VecLayout<T, HEAD_VECS, ROW_VECS>::VPL][VecLayout<T, HEAD_VECS, ROW_VECS>::VE],
                                           const float (&zs)[VecLayout<T, HEAD_VECS, ROW_VECS>::VPL], T *__restrict__ out,
                                           float *__restrict__ z, float *__restrict__ node_scores, int ns_len) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, VE = L::VE;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    if (sub == 0) {
        Vec16 *ov = reinterpret_cast<Vec16 *>(out) + (size_t)row * ROW_VECS + gl;
#pragma unroll
        for (int t = 0; t < VPL; t++) {
            const float inv = 1.0f / (zs[t] + kEps);
            float o[VE];
#pragma unroll
            for (int i = 0; i < VE; i++) o[i] = acc[t][i] * inv;
            st16(ov + G * t, Elem<T>::pack(o));
            if (z != nullptr && (gl % HEAD_VECS) == 0) z[(size_t)row * heads + (gl + G * t) / HEAD_VECS] = zs[t];
        }
    }
    // node score: head mean of Z (one lane per head contributes through the xor tree)
    float hs = 0.f;
#pragma unroll
    for (int t = 0; t < VPL; t++) hs += zs[t];
#pragma unroll
    for (int off = HEAD_VECS; off < G; off <<= 1) hs += __shfl_xor_sync(0xffffffffu, hs, off);
    if (lane == 0 && row < ns_len) node_scores[row] = hs / (float)heads;
}

template <typename T, int HEAD_VECS, int ROW_VECS>
__global__ void __launch_bounds__(kBlock)
    spattn_fwd_vec(int n, int heads, float scale_inv, const T *__restrict__ q,
                   const T *__restrict__ k, const T *__restrict__ v,
                   const int *__restrict__ rowptr, const int *__restrict__ col,
                   const float *__restrict__ bias, T *__restrict__ out, float *__restrict__ z,
                   float *__restrict__ node_scores, int ns_len, int row_blocks, SegView sg) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, EPW = L::EPW, VE = L::VE, UNROLL = L::UNROLL;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    const int wid = threadIdx.x >> 5;
    // blocks [0, row_blocks): one warp per row; after them: one warp per heavy-row segment
    int row, beg, end, seg = -1;
    if ((int)blockIdx.x < row_blocks) {
        row = blockIdx.x * kWarpsPerBlock + wid;
        if (row >= n) return;
        if (sg.first != nullptr && __ldg(sg.first + row) >= 0) return;   // done by its segments
        beg = __ldg(rowptr + row);
        end = __ldg(rowptr + row + 1);
    } else {
        seg = ((int)blockIdx.x - row_blocks) * kWarpsPerBlock + wid;
        if (seg >= sg.nseg) return;
        row = __ldg(sg.row + seg);
        beg = __ldg(rowptr + row) + (seg - __ldg(sg.first + row)) * sg.edges;
        end = min(__ldg(rowptr + row + 1), beg + sg.edges);
    }

    const Vec16 *qv = reinterpret_cast<const Vec16 *>(q) + (size_t)row * ROW_VECS + gl;
    const Vec16 *kv = reinterpret_cast<const Vec16 *>(k) + gl;
    const Vec16 *vv = reinterpret_cast<const Vec16 *>(v) + gl;

    float qf[VPL][VE];
#pragma unroll
    for (int t = 0; t < VPL; t++) Elem<T>::unpack(ldg16(qv + G * t), qf[t]);
    float acc[VPL][VE];
    float zs[VPL];
#pragma unroll
    for (int t = 0; t < VPL; t++) {
        zs[t] = 0.f;
#pragma unroll
        for (int i = 0; i < VE; i++) acc[t][i] = 0.f;
    }

    for (int e0 = beg; e0 < end; e0 += EPW * UNROLL) {
        int src[UNROLL];
        bool ok[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int e = e0 + sub + EPW * u;
            ok[u] = e < end;
            src[u] = ok[u] ? __ldg(col + e) : 0;
        }
        Vec16 kr[UNROLL][VPL], vr[UNROLL][VPL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
#pragma unroll
            for (int t = 0; t < VPL; t++) {
                kr[u][t] = ldg16(kv + (size_t)src[u] * ROW_VECS + G * t);
                vr[u][t] = ldg16(vv + (size_t)src[u] * ROW_VECS + G * t);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int e = e0 + sub + EPW * u;
#pragma unroll
            for (int t = 0; t < VPL; t++) {
                float kf[VE], vf[VE];
                Elem<T>::unpack(kr[u][t], kf);
                float d = 0.f;
#pragma unroll
                for (int i = 0; i < VE; i++) d = fmaf(kf[i], qf[t][i], d);
                d = head_reduce<HEAD_VECS>(d);
                float s = fminf(fmaxf(d * scale_inv, -kClamp), kClamp);
                if (bias != nullptr && ok[u]) s += __ldg(bias + (size_t)e * heads + (gl + G * t) / HEAD_VECS);
                const float p = ok[u] ? expf(s) : 0.f;
                zs[t] += p;
                Elem<T>::unpack(vr[u][t], vf);
#pragma unroll
                for (int i = 0; i < VE; i++) acc[t][i] = fmaf(p, vf[i], acc[t][i]);
            }
        }
    }
    if (EPW > 1) {
#pragma unroll
        for (int t = 0; t < VPL; t++) {
            zs[t] = slot_reduce<G>(zs[t]);
#pragma unroll
            for (int i = 0; i < VE; i++) acc[t][i] = slot_reduce<G>(acc[t][i]);
        }
    }
    if (seg >= 0) {      // partial sums of the segment: acc in row layout, then Z per head
        if (sub == 0) {
            float *rec = sg.part + (size_t)seg * fwd_record(heads, ROW_VECS * VE);
#pragma unroll
            for (int t = 0; t < VPL; t++) {
#pragma unroll
                for (int i = 0; i < VE; i += 4)
                    *reinterpret_cast<float4 *>(rec + (gl + G * t) * VE + i) =
                        make_float4(acc[t][i], acc[t][i + 1], acc[t][i + 2], acc[t][i + 3]);
                if ((gl % HEAD_VECS) == 0) rec[ROW_VECS * VE + (gl + G * t) / HEAD_VECS] = zs[t];
            }
        }
        return;
    }
    fwd_finish<T, HEAD_VECS, ROW_VECS>(row, heads, acc, zs, out, z, node_scores, ns_len);
}

// One warp per heavy row (the warp of its first segment): adds the row's segment partials in
// segment order and finishes the row.
template <typename T, int HEAD_VECS, int ROW_VECS>
__global__ void __launch_bounds__(kBlock)
    spattn_fwd_seg_finish(int heads, const int *__restrict__ rowptr, T *__restrict__ out, float *__restrict__ z,
                          float *__restrict__ node_scores, int ns_len, SegView sg) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, VE = L::VE;
    const int seg = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    if (seg >= sg.nseg) return;
    const int row = __ldg(sg.row + seg);
    if (seg != __ldg(sg.first + row)) return;
    const int gl = lane_id() % G;
    const int cnt = (__ldg(rowptr + row + 1) - __ldg(rowptr + row) + sg.edges - 1) / sg.edges;
    const int rs = fwd_record(heads, ROW_VECS * VE);
    float acc[VPL][VE], zs[VPL];
#pragma unroll
    for (int t = 0; t < VPL; t++) {
        zs[t] = 0.f;
#pragma unroll
        for (int i = 0; i < VE; i++) acc[t][i] = 0.f;
    }
    for (int j = 0; j < cnt; j++) {
        const float *rec = sg.part + (size_t)(seg + j) * rs;
#pragma unroll
        for (int t = 0; t < VPL; t++) {
#pragma unroll
            for (int i = 0; i < VE; i += 4) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(rec + (gl + G * t) * VE + i));
                acc[t][i] += a.x;
                acc[t][i + 1] += a.y;
                acc[t][i + 2] += a.z;
                acc[t][i + 3] += a.w;
            }
            zs[t] += __ldg(rec + ROW_VECS * VE + (gl + G * t) / HEAD_VECS);
        }
    }
    fwd_finish<T, HEAD_VECS, ROW_VECS>(row, heads, acc, zs, out, z, node_scores, ns_len);
}

// ------------------------------------------------------------------------------------
// backward (vector path)
// ------------------------------------------------------------------------------------
template <typename T, int HEAD_VECS, int ROW_VECS>
__global__ void __launch_bounds__(kBlock)
    spattn_delta_vec(int n, int heads, const T *__restrict__ out, const T *__restrict__ dout,
                     float *__restrict__ delta) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, EPW = L::EPW, VE = L::VE;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    const int row = (blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5)) * EPW + sub;
    const bool valid = row < n;
    const size_t base = (size_t)(valid ? row : 0) * ROW_VECS + gl;
#pragma unroll
    for (int t = 0; t < VPL; t++) {
        float a[VE], b[VE];
        Elem<T>::unpack(ldg16(reinterpret_cast<const Vec16 *>(out) + base + G * t), a);
        Elem<T>::unpack(ldg16(reinterpret_cast<const Vec16 *>(dout) + base + G * t), b);
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < VE; i++) d = fmaf(a[i], b[i], d);
        d = head_reduce<HEAD_VECS>(d);
        if (valid && (gl % HEAD_VECS) == 0) delta[(size_t)row * heads + (gl + G * t) / HEAD_VECS] = d;
    }
}

// Blocks [0, blocks_a) : one warp per destination row -> dq.
// Blocks [blocks_a, .) : one warp per source row      -> dk, dv.
template <typename T, int HEAD_VECS, int ROW_VECS>
__global__ void __launch_bounds__(kBlock)
    spattn_bwd_vec(int n, int heads, float scale_inv, int blocks_a, const T *__restrict__ q,
                   const T *__restrict__ k, const T *__restrict__ v, const T *__restrict__ dout,
                   const float *__restrict__ z, const float *__restrict__ delta,
                   const int *__restrict__ dst_rowptr, const int *__restrict__ dst_src,
                   const int *__restrict__ src_rowptr, const int *__restrict__ src_dst,
                   const int *__restrict__ src_to_dst_slot, const float *__restrict__ bias,
                   T *__restrict__ dq, T *__restrict__ dk, T *__restrict__ dv,
                   float *__restrict__ dbias, SegView sgd, SegView sgs) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, EPW = L::EPW, VE = L::VE, UNROLL = L::UNROLL;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    const int wid = threadIdx.x >> 5;
    const int b = blockIdx.x;
    // blocks: [0, blocks_a) destination rows, [blocks_a, 2 blocks_a) source rows, then the
    // destination-view segments and the source-view segments of heavy rows
    const int seg_blocks_d = (sgd.nseg + kWarpsPerBlock - 1) / kWarpsPerBlock;
    bool role_a;
    int row, beg, end, seg = -1;
    if (b < 2 * blocks_a) {
        role_a = b < blocks_a;
        row = (role_a ? b : b - blocks_a) * kWarpsPerBlock + wid;
        if (row >= n) return;
        const int32_t *first = role_a ? sgd.first : sgs.first;
        if (first != nullptr && __ldg(first + row) >= 0) return;   // done by its segments
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        beg = __ldg(rp + row);
        end = __ldg(rp + row + 1);
    } else {
        const int sb = b - 2 * blocks_a;
        role_a = sb < seg_blocks_d;
        seg = (role_a ? sb : sb - seg_blocks_d) * kWarpsPerBlock + wid;
        if (seg >= (role_a ? sgd.nseg : sgs.nseg)) return;
        row = __ldg((role_a ? sgd.row : sgs.row) + seg);
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        const int edges = role_a ? sgd.edges : sgs.edges;
        beg = __ldg(rp + row) + (seg - __ldg((role_a ? sgd.first : sgs.first) + row)) * edges;
        end = min(__ldg(rp + row + 1), beg + edges);
    }
    const Vec16 *Q = reinterpret_cast<const Vec16 *>(q) + gl;
    const Vec16 *K = reinterpret_cast<const Vec16 *>(k) + gl;
    const Vec16 *V = reinterpret_cast<const Vec16 *>(v) + gl;
    const Vec16 *DO = reinterpret_cast<const Vec16 *>(dout) + gl;
    const size_t rbase = (size_t)row * ROW_VECS;
    int head[VPL];
#pragma unroll
    for (int t = 0; t < VPL; t++) head[t] = (gl + G * t) / HEAD_VECS;

    if (role_a) {
        // ---- dq for destination row `row` ----
        float qf[VPL][VE], gf[VPL][VE], inv[VPL], dl[VPL], acc[VPL][VE];
#pragma unroll
        for (int t = 0; t < VPL; t++) {
            Elem<T>::unpack(ldg16(Q + rbase + G * t), qf[t]);
            Elem<T>::unpack(ldg16(DO + rbase + G * t), gf[t]);
            inv[t] = 1.0f / (__ldg(z + (size_t)row * heads + head[t]) + kEps);
            dl[t] = __ldg(delta + (size_t)row * heads + head[t]);
#pragma unroll
            for (int i = 0; i < VE; i++) acc[t][i] = 0.f;
        }
        for (int e0 = beg; e0 < end; e0 += EPW * UNROLL) {
            int src[UNROLL];
            bool ok[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const int e = e0 + sub + EPW * u;
                ok[u] = e < end;
                src[u] = ok[u] ? __ldg(dst_src + e) : 0;
            }
            Vec16 kr[UNROLL][VPL], vr[UNROLL][VPL];
#pragma unroll
            for (int u = 0; u < UNROLL; u++)
#pragma unroll
                for (int t = 0; t < VPL; t++) {
                    kr[u][t] = ldg16(K + (size_t)src[u] * ROW_VECS + G * t);
                    vr[u][t] = ldg16(V + (size_t)src[u] * ROW_VECS + G * t);
                }
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const int e = e0 + sub + EPW * u;
#pragma unroll
                for (int t = 0; t < VPL; t++) {
                    float kf[VE], vf[VE];
                    Elem<T>::unpack(kr[u][t], kf);
                    Elem<T>::unpack(vr[u][t], vf);
                    float dqk = 0.f, dgv = 0.f;
#pragma unroll
                    for (int i = 0; i < VE; i++) {
                        dqk = fmaf(kf[i], qf[t][i], dqk);
                        dgv = fmaf(gf[t][i], vf[i], dgv);
                    }
                    dqk = head_reduce<HEAD_VECS>(dqk);
                    dgv = head_reduce<HEAD_VECS>(dgv);
                    const float s = dqk * scale_inv;
                    const bool inside = s >= -kClamp && s <= kClamp;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    if (bias != nullptr && ok[u]) sc += __ldg(bias + (size_t)e * heads + head[t]);
                    const float p = expf(sc);
                    const float dpre = (dgv - dl[t]) * inv[t] * p;
                    const float ds = (ok[u] && inside) ? dpre : 0.f;
                    if (dbias != nullptr && ok[u] && (gl % HEAD_VECS) == 0) dbias[(size_t)e * heads + head[t]] = dpre;
#pragma unroll
                    for (int i = 0; i < VE; i++) acc[t][i] = fmaf(ds, kf[i], acc[t][i]);
                }
            }
        }
        if (EPW > 1) {
#pragma unroll
            for (int t = 0; t < VPL; t++)
#pragma unroll
                for (int i = 0; i < VE; i++) acc[t][i] = slot_reduce<G>(acc[t][i]);
        }
        if (seg >= 0) {   // segment partial of dq (before the 1/sqrt(D) scale)
            if (sub == 0) {
                float *rec = sgd.part + (size_t)seg * ROW_VECS * VE;
#pragma unroll
                for (int t = 0; t < VPL; t++)
#pragma unroll
                    for (int i = 0; i < VE; i += 4)
                        *reinterpret_cast<float4 *>(rec + (gl + G * t) * VE + i) =
                            make_float4(acc[t][i], acc[t][i + 1], acc[t][i + 2], acc[t][i + 3]);
            }
            return;
        }
        if (sub == 0) {
            Vec16 *o = reinterpret_cast<Vec16 *>(dq) + rbase + gl;
#pragma unroll
            for (int t = 0; t < VPL; t++) {
                float r[VE];
#pragma unroll
                for (int i = 0; i < VE; i++) r[i] = acc[t][i] * scale_inv;
                st16(o + G * t, Elem<T>::pack(r));
            }
        }
    } else {
        // ---- dk, dv for source row `row` ----
        float kf[VPL][VE], vf[VPL][VE], ak[VPL][VE], av[VPL][VE];
#pragma unroll
        for (int t = 0; t < VPL; t++) {
            Elem<T>::unpack(ldg16(K + rbase + G * t), kf[t]);
            Elem<T>::unpack(ldg16(V + rbase + G * t), vf[t]);
#pragma unroll
            for (int i = 0; i < VE; i++) ak[t][i] = av[t][i] = 0.f;
        }
        for (int e0 = beg; e0 < end; e0 += EPW * UNROLL) {
            int dst[UNROLL];
            bool ok[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const int e = e0 + sub + EPW * u;
                ok[u] = e < end;
                dst[u] = ok[u] ? __ldg(src_dst + e) : 0;
            }
            Vec16 qr[UNROLL][VPL], gr[UNROLL][VPL];
            float zr[UNROLL][VPL], dr[UNROLL][VPL];
#pragma unroll
            for (int u = 0; u < UNROLL; u++)
#pragma unroll
                for (int t = 0; t < VPL; t++) {
                    qr[u][t] = ldg16(Q + (size_t)dst[u] * ROW_VECS + G * t);
                    gr[u][t] = ldg16(DO + (size_t)dst[u] * ROW_VECS + G * t);
                    zr[u][t] = __ldg(z + (size_t)dst[u] * heads + head[t]);
                    dr[u][t] = __ldg(delta + (size_t)dst[u] * heads + head[t]);
                }
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const int e = e0 + sub + EPW * u;
#pragma unroll
                for (int t = 0; t < VPL; t++) {
                    float qf[VE], gf[VE];
                    Elem<T>::unpack(qr[u][t], qf);
                    Elem<T>::unpack(gr[u][t], gf);
                    float dqk = 0.f, dgv = 0.f;
#pragma unroll
                    for (int i = 0; i < VE; i++) {
                        dqk = fmaf(kf[t][i], qf[i], dqk);
                        dgv = fmaf(gf[i], vf[t][i], dgv);
                    }
                    dqk = head_reduce<HEAD_VECS>(dqk);
                    dgv = head_reduce<HEAD_VECS>(dgv);
                    const float s = dqk * scale_inv;
                    const bool inside = s >= -kClamp && s <= kClamp;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    if (bias != nullptr && ok[u])
                        sc += __ldg(bias + (size_t)__ldg(src_to_dst_slot + e) * heads + head[t]);
                    const float p = ok[u] ? expf(sc) : 0.f;
                    const float inv = 1.0f / (zr[u][t] + kEps);
                    const float a = p * inv;
                    const float dpre = (dgv - dr[u][t]) * inv * p;
                    const float ds = inside ? dpre : 0.f;
#pragma unroll
                    for (int i = 0; i < VE; i++) {
                        av[t][i] = fmaf(a, gf[i], av[t][i]);
                        ak[t][i] = fmaf(ds, qf[i], ak[t][i]);
                    }
                }
            }
        }
        if (EPW > 1) {
#pragma unroll
            for (int t = 0; t < VPL; t++)
#pragma unroll
                for (int i = 0; i < VE; i++) {
                    ak[t][i] = slot_reduce<G>(ak[t][i]);
                    av[t][i] = slot_reduce<G>(av[t][i]);
                }
        }
        if (seg >= 0) {   // segment partials of dk (unscaled) and dv
            if (sub == 0) {
                float *rec = sgs.part + (size_t)seg * 2 * ROW_VECS * VE;
#pragma unroll
                for (int t = 0; t < VPL; t++)
#pragma unroll
                    for (int i = 0; i < VE; i += 4) {
                        *reinterpret_cast<float4 *>(rec + (gl + G * t) * VE + i) =
                            make_float4(ak[t][i], ak[t][i + 1], ak[t][i + 2], ak[t][i + 3]);
                        *reinterpret_cast<float4 *>(rec + ROW_VECS * VE + (gl + G * t) * VE + i) =
                            make_float4(av[t][i], av[t][i + 1], av[t][i + 2], av[t][i + 3]);
                    }
            }
            return;
        }
        if (sub == 0) {
            Vec16 *ok_ = reinterpret_cast<Vec16 *>(dk) + rbase + gl;
            Vec16 *ov = reinterpret_cast<Vec16 *>(dv) + rbase + gl;
#pragma unroll
            for (int t = 0; t < VPL; t++) {
                float r[VE];
#pragma unroll
                for (int i = 0; i < VE; i++) r[i] = ak[t][i] * scale_inv;
                st16(ok_ + G * t, Elem<T>::pack(r));
                st16(ov + G * t, Elem<T>::pack(av[t]));
            }
        }
    }
}

// e^s of a clamped edge score as 2^(s log2 e) on the MUFU unit (ex2.approx: relative error
// ~2^-22, plus ~2^-21 from rounding s log2 e), and 1 / x as rcp.approx (<= 1 ulp for the normal
// x = Z + 1e-6 here): both far inside the parity tolerances.
constexpr float kLog2e = 1.44269504088896341f;
__device__ __forceinline__ float mufu_exp(float s) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s * kLog2e));
    return y;
}
__device__ __forceinline__ float mufu_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------------------------
// bf16 rows of 128 elements (16 vectors of 16 B): packed-math kernels
// ------------------------------------------------------------------------------------
// The 65,536-token workload's row shape (H * D = 128, bf16) with its own forward and backward.
// Lane groups of 16 lanes hold one row (one 16-byte vector of eight bf16 per lane): two edges per
// warp instruction, UNROLL pairs in flight.  Dot products run as fma.rn.f32.bf16 straight on the
// packed words (a bf16 x bf16 product is exact in f32, so every step equals fmaf of the widened
// values), in an even and an odd chain added at the end; weighted sums run as packed f32x2 FMAs on
// the widened vector; exponentials and the source role's reciprocal on the MUFU unit.  The
// segment records are laid out as in the general kernels, so the same finish kernels serve both.
namespace r128 {
constexpr int G = 16;
constexpr int RV = 16;

// Read-only 16-byte load that the compiler may schedule freely (the tensors are not written by
// the kernels that read them).
__device__ __forceinline__ uint4 ld16(const uint4 *p) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ void fma_pair(float &d0, float &d1, uint32_t a, uint32_t b) {
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "r"(a), "r"(b));
}

// sum_i a_i b_i over the eight bf16 of two vectors (even and odd elements in separate chains).
__device__ __forceinline__ float dot8(const uint4 &a, const uint4 &b) {
    float d0 = 0.f, d1 = 0.f;
    fma_pair(d0, d1, a.x, b.x);
    fma_pair(d0, d1, a.y, b.y);
    fma_pair(d0, d1, a.z, b.z);
    fma_pair(d0, d1, a.w, b.w);
    return d0 + d1;
}

__device__ __forceinline__ float2 widen(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// acc[j] += s * (elements 2j, 2j + 1 of x)
__device__ __forceinline__ void axpy8(float2 (&acc)[4], float s, const uint4 &x) {
    const float2 ss = make_float2(s, s);
    acc[0] = __ffma2_rn(ss, widen(x.x), acc[0]);
    acc[1] = __ffma2_rn(ss, widen(x.y), acc[1]);
    acc[2] = __ffma2_rn(ss, widen(x.z), acc[2]);
    acc[3] = __ffma2_rn(ss, widen(x.w), acc[3]);
}

// Adds the two edge slots of a warp (lane groups 0 and 1).
__device__ __forceinline__ void slot_sum(float2 (&acc)[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        acc[j].x += __shfl_xor_sync(0xffffffffu, acc[j].x, G);
        acc[j].y += __shfl_xor_sync(0xffffffffu, acc[j].y, G);
    }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ uint4 pack8(const float2 (&acc)[4], float s) {
    return make_uint4(pack2(acc[0].x * s, acc[0].y * s), pack2(acc[1].x * s, acc[1].y * s),
                      pack2(acc[2].x * s, acc[2].y * s), pack2(acc[3].x * s, acc[3].y * s));
}

__device__ __forceinline__ void store_rec(float *rec, const float2 (&acc)[4]) {
    *reinterpret_cast<float4 *>(rec) = make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y);
    *reinterpret_cast<float4 *>(rec + 4) = make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y);
}
}  // namespace r128

// PAIRS (HEAD_VECS = 2): the two lanes of a head finish different edges of an edge pair and
// exchange the exponentials (as spattn_bwd_r128 below); the same results as without pairs.
// NB: launched without an edge bias (and, in the backward, without its gradient), so the per-edge
// bias tests compile away.
template <int HEAD_VECS, int UNROLL, int MIN_BLOCKS = 4, bool PAIRS = false, bool PF = false, bool NB = false>
__global__ void __launch_bounds__(kBlock, MIN_BLOCKS)
    spattn_fwd_r128(int n, int heads, float scale_inv, const __nv_bfloat16 *__restrict__ q,
                    const __nv_bfloat16 *__restrict__ k, const __nv_bfloat16 *__restrict__ v,
                    const int *__restrict__ rowptr, const int *__restrict__ col,
                    const float *__restrict__ bias, __nv_bfloat16 *__restrict__ out, float *__restrict__ z,
                    float *__restrict__ node_scores, int ns_len, int row_blocks, SegView sg) {
    using namespace r128;
    constexpr int EPW = 32 / G;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    const int wid = threadIdx.x >> 5;
    int row, beg, end, seg = -1;
    if ((int)blockIdx.x < row_blocks) {
        row = blockIdx.x * kWarpsPerBlock + wid;
        if (row >= n) return;
        if (sg.first != nullptr && __ldg(sg.first + row) >= 0) return;   // done by its segments
        beg = __ldg(rowptr + row);
        end = __ldg(rowptr + row + 1);
    } else {
        seg = ((int)blockIdx.x - row_blocks) * kWarpsPerBlock + wid;
        if (seg >= sg.nseg) return;
        row = __ldg(sg.row + seg);
        beg = __ldg(rowptr + row) + (seg - __ldg(sg.first + row)) * sg.edges;
        end = min(__ldg(rowptr + row + 1), beg + sg.edges);
    }
    const int head = gl / HEAD_VECS;
    const uint4 *K = reinterpret_cast<const uint4 *>(k) + gl;
    const uint4 *V = reinterpret_cast<const uint4 *>(v) + gl;
    const uint4 qw = ld16(reinterpret_cast<const uint4 *>(q) + (size_t)row * RV + gl);
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float zs = 0.f;
    // PF: the next batch's column indices are loaded while this batch computes, so only the row
    // gathers wait on L2 at the top of a batch
    int nxt[UNROLL];
    if constexpr (PF) {
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int e = beg + sub + EPW * u;
            nxt[u] = e < end ? __ldg(col + e) : 0;
        }
    }
    for (int e0 = beg; e0 < end; e0 += EPW * UNROLL) {
        int src[UNROLL];
        bool ok[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int e = e0 + sub + EPW * u;
            ok[u] = e < end;
            if constexpr (PF) src[u] = nxt[u];
            else src[u] = ok[u] ? __ldg(col + e) : 0;
        }
        uint4 kr[UNROLL], vr[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            kr[u] = ld16(K + (size_t)src[u] * RV);
            vr[u] = ld16(V + (size_t)src[u] * RV);
        }
        if constexpr (PF) {
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const int e = e0 + EPW * UNROLL + sub + EPW * u;
                nxt[u] = e < end ? __ldg(col + e) : 0;
            }
        }
        if constexpr (PAIRS) {
            static_assert(HEAD_VECS == 2 && UNROLL % 2 == 0, "pairs of edges, two lanes per head");
            const bool odd = (gl & 1) != 0;   // this lane finishes edge u + 1 of each pair
#pragma unroll
            for (int u = 0; u < UNROLL; u += 2) {
                const float d0 = dot8(kr[u], qw), d1 = dot8(kr[u + 1], qw);
                const float d = (odd ? d1 : d0) + __shfl_xor_sync(0xffffffffu, odd ? d0 : d1, 1);
                const bool okm = odd ? ok[u + 1] : ok[u];
                float s = fminf(fmaxf(d * scale_inv, -kClamp), kClamp);
                if (!NB && bias != nullptr && okm)
                    s += __ldg(bias + (size_t)(e0 + sub + EPW * u + (odd ? EPW : 0)) * heads + head);
                const float p = okm ? mufu_exp(s) : 0.f;
                const float pp = __shfl_xor_sync(0xffffffffu, p, 1);
                const float p0 = odd ? pp : p, p1 = odd ? p : pp;
                zs += p0;
                axpy8(acc, p0, vr[u]);
                zs += p1;
                axpy8(acc, p1, vr[u + 1]);
            }
        } else {
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                const float d = head_reduce<HEAD_VECS>(dot8(kr[u], qw));
                float s = fminf(fmaxf(d * scale_inv, -kClamp), kClamp);
                if (!NB && bias != nullptr && ok[u]) s += __ldg(bias + (size_t)(e0 + sub + EPW * u) * heads + head);
                const float p = ok[u] ? mufu_exp(s) : 0.f;
                zs += p;
                axpy8(acc, p, vr[u]);
            }
        }
    }
    zs += __shfl_xor_sync(0xffffffffu, zs, G);
    slot_sum(acc);
    if (seg >= 0) {   // partial sums of the segment: acc in row layout, then Z per head
        if (sub == 0) {
            float *rec = sg.part + (size_t)seg * fwd_record(heads, RV * 8);
            store_rec(rec + gl * 8, acc);
            if ((gl % HEAD_VECS) == 0) rec[RV * 8 + head] = zs;
        }
        return;
    }
    if (sub == 0) {
        const float inv = 1.0f / (zs + kEps);
        *(reinterpret_cast<uint4 *>(out) + (size_t)row * RV + gl) = pack8(acc, inv);
        if (z != nullptr && (gl % HEAD_VECS) == 0) z[(size_t)row * heads + head] = zs;
    }
    // node score: head mean of Z (lane groups of one head hold equal values)
    float hs = zs;
#pragma unroll
    for (int off = HEAD_VECS; off < G; off <<= 1) hs += __shfl_xor_sync(0xffffffffu, hs, off);
    if (lane == 0 && row < ns_len) node_scores[row] = hs / (float)heads;
}

// PAIRS (two lanes per head, HEAD_VECS = 2): the two lanes of a head finish different edges of an
// edge pair.  Each sends the partner the partial dot product of the partner's edge, runs the score,
// exponential and gradient arithmetic once for its own edge, and hands back the two scalars the
// weighted sums need, instead of both lanes repeating that arithmetic for every edge.  The sums
// are added in the same order as without pairs, so the results are identical.
template <int HEAD_VECS, int UNROLL_A, int UNROLL_B, int MIN_BLOCKS = 4, bool PAIRS = false, bool PF = false,
          bool NB = false>
__global__ void __launch_bounds__(kBlock, MIN_BLOCKS)
    spattn_bwd_r128(int n, int heads, float scale_inv, int blocks_a, const __nv_bfloat16 *__restrict__ q,
                    const __nv_bfloat16 *__restrict__ k, const __nv_bfloat16 *__restrict__ v,
                    const __nv_bfloat16 *__restrict__ dout, const float *__restrict__ z,
                    const float *__restrict__ delta, const int *__restrict__ dst_rowptr,
                    const int *__restrict__ dst_src, const int *__restrict__ src_rowptr,
                    const int *__restrict__ src_dst, const int *__restrict__ src_to_dst_slot,
                    const float *__restrict__ bias, __nv_bfloat16 *__restrict__ dq,
                    __nv_bfloat16 *__restrict__ dk, __nv_bfloat16 *__restrict__ dv, float *__restrict__ dbias,
                    SegView sgd, SegView sgs) {
    using namespace r128;
    constexpr int EPW = 32 / G;
    const int lane = lane_id();
    const int sub = lane / G;
    const int gl = lane % G;
    const int wid = threadIdx.x >> 5;
    const int b = blockIdx.x;
    // blocks: [0, blocks_a) destination rows, [blocks_a, 2 blocks_a) source rows, then the
    // destination-view segments and the source-view segments of heavy rows
    const int seg_blocks_d = (sgd.nseg + kWarpsPerBlock - 1) / kWarpsPerBlock;
    bool role_a;
    int row, beg, end, seg = -1;
    if (b < 2 * blocks_a) {
        role_a = b < blocks_a;
        row = (role_a ? b : b - blocks_a) * kWarpsPerBlock + wid;
        if (row >= n) return;
        const int32_t *first = role_a ? sgd.first : sgs.first;
        if (first != nullptr && __ldg(first + row) >= 0) return;   // done by its segments
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        beg = __ldg(rp + row);
        end = __ldg(rp + row + 1);
    } else {
        const int sb = b - 2 * blocks_a;
        role_a = sb < seg_blocks_d;
        seg = (role_a ? sb : sb - seg_blocks_d) * kWarpsPerBlock + wid;
        if (seg >= (role_a ? sgd.nseg : sgs.nseg)) return;
        row = __ldg((role_a ? sgd.row : sgs.row) + seg);
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        const int edges = role_a ? sgd.edges : sgs.edges;
        beg = __ldg(rp + row) + (seg - __ldg((role_a ? sgd.first : sgs.first) + row)) * edges;
        end = min(__ldg(rp + row + 1), beg + edges);
    }
    const uint4 *Q = reinterpret_cast<const uint4 *>(q) + gl;
    const uint4 *K = reinterpret_cast<const uint4 *>(k) + gl;
    const uint4 *V = reinterpret_cast<const uint4 *>(v) + gl;
    const uint4 *DO = reinterpret_cast<const uint4 *>(dout) + gl;
    const size_t rbase = (size_t)row * RV;
    const int head = gl / HEAD_VECS;
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};

    if (role_a) {
        // ---- dq for destination row `row` ----
        const uint4 qw = ld16(Q + rbase), gw = ld16(DO + rbase);
        const float inv = 1.0f / (__ldg(z + (size_t)row * heads + head) + kEps);
        const float dl = __ldg(delta + (size_t)row * heads + head);
        int nxt[UNROLL_A];
        if constexpr (PF) {
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                const int e = beg + sub + EPW * u;
                nxt[u] = e < end ? __ldg(dst_src + e) : 0;
            }
        }
        for (int e0 = beg; e0 < end; e0 += EPW * UNROLL_A) {
            int src[UNROLL_A];
            bool ok[UNROLL_A];
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                const int e = e0 + sub + EPW * u;
                ok[u] = e < end;
                if constexpr (PF) src[u] = nxt[u];
                else src[u] = ok[u] ? __ldg(dst_src + e) : 0;
            }
            uint4 kr[UNROLL_A], vr[UNROLL_A];
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                kr[u] = ld16(K + (size_t)src[u] * RV);
                vr[u] = ld16(V + (size_t)src[u] * RV);
            }
            if constexpr (PF) {
#pragma unroll
                for (int u = 0; u < UNROLL_A; u++) {
                    const int e = e0 + EPW * UNROLL_A + sub + EPW * u;
                    nxt[u] = e < end ? __ldg(dst_src + e) : 0;
                }
            }
            if constexpr (PAIRS) {
                static_assert(HEAD_VECS == 2 && UNROLL_A % 2 == 0, "pairs of edges, two lanes per head");
                const bool odd = (gl & 1) != 0;   // this lane finishes edge u + 1 of each pair
#pragma unroll
                for (int u = 0; u < UNROLL_A; u += 2) {
                    const float q0 = dot8(kr[u], qw), q1 = dot8(kr[u + 1], qw);
                    const float g0 = dot8(vr[u], gw), g1 = dot8(vr[u + 1], gw);
                    const float dqk = (odd ? q1 : q0) + __shfl_xor_sync(0xffffffffu, odd ? q0 : q1, 1);
                    const float dgv = (odd ? g1 : g0) + __shfl_xor_sync(0xffffffffu, odd ? g0 : g1, 1);
                    const bool okm = odd ? ok[u + 1] : ok[u];
                    const int e = e0 + sub + EPW * u + (odd ? EPW : 0);
                    const float s = dqk * scale_inv;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                    if (!NB && bias != nullptr && okm) sc += __ldg(bias + (size_t)e * heads + head);
                    const float p = mufu_exp(sc);
                    const float dpre = (dgv - dl) * inv * p;
                    const float ds = (okm && inside) ? dpre : 0.f;
                    if (!NB && dbias != nullptr && okm) dbias[(size_t)e * heads + head] = dpre;
                    const float dsp = __shfl_xor_sync(0xffffffffu, ds, 1);
                    axpy8(acc, odd ? dsp : ds, kr[u]);
                    axpy8(acc, odd ? ds : dsp, kr[u + 1]);
                }
            } else {
#pragma unroll
                for (int u = 0; u < UNROLL_A; u++) {
                    const int e = e0 + sub + EPW * u;
                    const float dqk = head_reduce<HEAD_VECS>(dot8(kr[u], qw));
                    const float dgv = head_reduce<HEAD_VECS>(dot8(vr[u], gw));
                    const float s = dqk * scale_inv;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                    if (!NB && bias != nullptr && ok[u]) sc += __ldg(bias + (size_t)e * heads + head);
                    const float p = mufu_exp(sc);
                    const float dpre = (dgv - dl) * inv * p;
                    const float ds = (ok[u] && inside) ? dpre : 0.f;
                    if (!NB && dbias != nullptr && ok[u] && (gl % HEAD_VECS) == 0) dbias[(size_t)e * heads + head] = dpre;
                    axpy8(acc, ds, kr[u]);
                }
            }
        }
        slot_sum(acc);
        if (seg >= 0) {   // segment partial of dq (before the 1/sqrt(D) scale)
            if (sub == 0) store_rec(sgd.part + (size_t)seg * RV * 8 + gl * 8, acc);
            return;
        }
        if (sub == 0) *(reinterpret_cast<uint4 *>(dq) + rbase + gl) = pack8(acc, scale_inv);
    } else {
        // ---- dk, dv for source row `row` ----
        const uint4 kw = ld16(K + rbase), vw = ld16(V + rbase);
        float2 av[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        int nxt[UNROLL_B];
        if constexpr (PF) {
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                const int e = beg + sub + EPW * u;
                nxt[u] = e < end ? __ldg(src_dst + e) : 0;
            }
        }
        for (int e0 = beg; e0 < end; e0 += EPW * UNROLL_B) {
            int dst[UNROLL_B];
            bool ok[UNROLL_B];
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                const int e = e0 + sub + EPW * u;
                ok[u] = e < end;
                if constexpr (PF) dst[u] = nxt[u];
                else dst[u] = ok[u] ? __ldg(src_dst + e) : 0;
            }
            uint4 qr[UNROLL_B], gr[UNROLL_B];
            float zr[UNROLL_B], dr[UNROLL_B];
            const bool odd = (gl & 1) != 0;
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                qr[u] = ld16(Q + (size_t)dst[u] * RV);
                gr[u] = ld16(DO + (size_t)dst[u] * RV);
                if constexpr (PAIRS) {   // Z and delta of the edge this lane finishes
                    if (u % 2 == 0) {
                        const int dm = odd ? dst[u + 1] : dst[u];
                        zr[u] = __ldg(z + (size_t)dm * heads + head);
                        dr[u] = __ldg(delta + (size_t)dm * heads + head);
                    }
                } else {
                    zr[u] = __ldg(z + (size_t)dst[u] * heads + head);
                    dr[u] = __ldg(delta + (size_t)dst[u] * heads + head);
                }
            }
            if constexpr (PF) {
#pragma unroll
                for (int u = 0; u < UNROLL_B; u++) {
                    const int e = e0 + EPW * UNROLL_B + sub + EPW * u;
                    nxt[u] = e < end ? __ldg(src_dst + e) : 0;
                }
            }
            if constexpr (PAIRS) {
                static_assert(HEAD_VECS == 2 && UNROLL_B % 2 == 0, "pairs of edges, two lanes per head");
#pragma unroll
                for (int u = 0; u < UNROLL_B; u += 2) {
                    const float q0 = dot8(qr[u], kw), q1 = dot8(qr[u + 1], kw);
                    const float g0 = dot8(gr[u], vw), g1 = dot8(gr[u + 1], vw);
                    const float dqk = (odd ? q1 : q0) + __shfl_xor_sync(0xffffffffu, odd ? q0 : q1, 1);
                    const float dgv = (odd ? g1 : g0) + __shfl_xor_sync(0xffffffffu, odd ? g0 : g1, 1);
                    const bool okm = odd ? ok[u + 1] : ok[u];
                    const int e = e0 + sub + EPW * u + (odd ? EPW : 0);
                    const float s = dqk * scale_inv;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                    if (!NB && bias != nullptr && okm)
                        sc += __ldg(bias + (size_t)__ldg(src_to_dst_slot + e) * heads + head);
                    const float p = okm ? mufu_exp(sc) : 0.f;
                    const float inv = mufu_rcp(zr[u] + kEps);
                    const float a = p * inv;
                    const float dpre = (dgv - dr[u]) * inv * p;
                    const float ds = inside ? dpre : 0.f;
                    const float ap = __shfl_xor_sync(0xffffffffu, a, 1);
                    const float dsp = __shfl_xor_sync(0xffffffffu, ds, 1);
                    axpy8(av, odd ? ap : a, gr[u]);
                    axpy8(acc, odd ? dsp : ds, qr[u]);
                    axpy8(av, odd ? a : ap, gr[u + 1]);
                    axpy8(acc, odd ? ds : dsp, qr[u + 1]);
                }
            } else {
#pragma unroll
                for (int u = 0; u < UNROLL_B; u++) {
                    const int e = e0 + sub + EPW * u;
                    const float dqk = head_reduce<HEAD_VECS>(dot8(qr[u], kw));
                    const float dgv = head_reduce<HEAD_VECS>(dot8(gr[u], vw));
                    const float s = dqk * scale_inv;
                    float sc = fminf(fmaxf(s, -kClamp), kClamp);
                    const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                    if (!NB && bias != nullptr && ok[u])
                        sc += __ldg(bias + (size_t)__ldg(src_to_dst_slot + e) * heads + head);
                    const float p = ok[u] ? mufu_exp(sc) : 0.f;
                    const float inv = mufu_rcp(zr[u] + kEps);
                    const float a = p * inv;
                    const float dpre = (dgv - dr[u]) * inv * p;
                    const float ds = inside ? dpre : 0.f;
                    axpy8(av, a, gr[u]);
                    axpy8(acc, ds, qr[u]);
                }
            }
        }
        slot_sum(acc);
        slot_sum(av);
        if (seg >= 0) {   // segment partials of dk (unscaled) and dv
            if (sub == 0) {
                float *rec = sgs.part + (size_t)seg * 2 * RV * 8;
                store_rec(rec + gl * 8, acc);
                store_rec(rec + RV * 8 + gl * 8, av);
            }
            return;
        }
        if (sub == 0) {
            *(reinterpret_cast<uint4 *>(dk) + rbase + gl) = pack8(acc, scale_inv);
            *(reinterpret_cast<uint4 *>(dv) + rbase + gl) = pack8(av, 1.0f);
        }
    }
}

// ------------------------------------------------------------------------------------
// fp32 rows of 128 elements (32 vectors of 16 B): packed-math kernels
// ------------------------------------------------------------------------------------
// The GT model's row shape (fp32, H * D = 128; D = 4, 8, 16 or 32).  A warp holds one row, one
// 16-byte vector of four floats per lane, one edge per warp instruction, UNROLL edges in flight,
// and the next batch's column indices loaded ahead.  Dot products and weighted sums run as packed
// f32x2 FMAs, exponentials and the source role's reciprocal on the MUFU unit (`ex2.approx`, relative
// error ~2^-22, inside the fp32 parity tolerance).  NB: launched without an edge bias (nor its
// gradient), the per-edge bias tests compiled out.  Segment records are laid out as in the general
// kernels, so the same finish kernels serve both.
namespace f128 {
constexpr int RV = 32;

__device__ __forceinline__ float2 lo(const uint4 &x) { return make_float2(__uint_as_float(x.x), __uint_as_float(x.y)); }
__device__ __forceinline__ float2 hi(const uint4 &x) { return make_float2(__uint_as_float(x.z), __uint_as_float(x.w)); }

// sum of the four products of a gathered vector and a row-constant one (pairs, then the halves)
__device__ __forceinline__ float dot4(const uint4 &a, float2 b0, float2 b1) {
    const float2 d = __ffma2_rn(hi(a), b1, __fmul2_rn(lo(a), b0));
    return d.x + d.y;
}

__device__ __forceinline__ void axpy4(float2 &a0, float2 &a1, float s, const uint4 &x) {
    const float2 ss = make_float2(s, s);
    a0 = __ffma2_rn(ss, lo(x), a0);
    a1 = __ffma2_rn(ss, hi(x), a1);
}
}  // namespace f128

template <int HEAD_VECS, int UNROLL, int MIN_BLOCKS = 4, bool NB = false>
__global__ void __launch_bounds__(kBlock, MIN_BLOCKS)
    spattn_fwd_f128(int n, int heads, float scale_inv, const float *__restrict__ q, const float *__restrict__ k,
                    const float *__restrict__ v, const int *__restrict__ rowptr, const int *__restrict__ col,
                    const float *__restrict__ bias, float *__restrict__ out, float *__restrict__ z,
                    float *__restrict__ node_scores, int ns_len, int row_blocks, SegView sg) {
    using namespace f128;
    const int lane = lane_id();
    const int wid = threadIdx.x >> 5;
    int row, beg, end, seg = -1;
    if ((int)blockIdx.x < row_blocks) {
        row = blockIdx.x * kWarpsPerBlock + wid;
        if (row >= n) return;
        if (sg.first != nullptr && __ldg(sg.first + row) >= 0) return;   // done by its segments
        beg = __ldg(rowptr + row);
        end = __ldg(rowptr + row + 1);
    } else {
        seg = ((int)blockIdx.x - row_blocks) * kWarpsPerBlock + wid;
        if (seg >= sg.nseg) return;
        row = __ldg(sg.row + seg);
        beg = __ldg(rowptr + row) + (seg - __ldg(sg.first + row)) * sg.edges;
        end = min(__ldg(rowptr + row + 1), beg + sg.edges);
    }
    const int head = lane / HEAD_VECS;
    const uint4 *K = reinterpret_cast<const uint4 *>(k) + lane;
    const uint4 *V = reinterpret_cast<const uint4 *>(v) + lane;
    const uint4 qv = r128::ld16(reinterpret_cast<const uint4 *>(q) + (size_t)row * RV + lane);
    const float2 q0 = lo(qv), q1 = hi(qv);
    float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
    float zs = 0.f;
    int nxt[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; u++) nxt[u] = beg + u < end ? __ldg(col + beg + u) : 0;
    for (int e0 = beg; e0 < end; e0 += UNROLL) {
        int src[UNROLL];
        bool ok[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            ok[u] = e0 + u < end;
            src[u] = nxt[u];
        }
        uint4 kr[UNROLL], vr[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            kr[u] = r128::ld16(K + (size_t)src[u] * RV);
            vr[u] = r128::ld16(V + (size_t)src[u] * RV);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int e = e0 + UNROLL + u;
            nxt[u] = e < end ? __ldg(col + e) : 0;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const float d = head_reduce<HEAD_VECS>(dot4(kr[u], q0, q1));
            float s = fminf(fmaxf(d * scale_inv, -kClamp), kClamp);
            if (!NB && bias != nullptr && ok[u]) s += __ldg(bias + (size_t)(e0 + u) * heads + head);
            const float p = ok[u] ? mufu_exp(s) : 0.f;
            zs += p;
            axpy4(a0, a1, p, vr[u]);
        }
    }
    if (seg >= 0) {   // partial sums of the segment: acc in row layout, then Z per head
        float *rec = sg.part + (size_t)seg * fwd_record(heads, RV * 4);
        *reinterpret_cast<float4 *>(rec + lane * 4) = make_float4(a0.x, a0.y, a1.x, a1.y);
        if ((lane % HEAD_VECS) == 0) rec[RV * 4 + head] = zs;
        return;
    }
    const float inv = 1.0f / (zs + kEps);
    *(reinterpret_cast<float4 *>(out) + (size_t)row * RV + lane) = make_float4(a0.x * inv, a0.y * inv, a1.x * inv, a1.y * inv);
    if (z != nullptr && (lane % HEAD_VECS) == 0) z[(size_t)row * heads + head] = zs;
    // node score: head mean of Z (lanes of one head hold equal values)
    float hs = zs;
#pragma unroll
    for (int off = HEAD_VECS; off < 32; off <<= 1) hs += __shfl_xor_sync(0xffffffffu, hs, off);
    if (lane == 0 && row < ns_len) node_scores[row] = hs / (float)heads;
}

template <int HEAD_VECS, int UNROLL_A, int UNROLL_B, int MIN_BLOCKS = 4, bool NB = false>
__global__ void __launch_bounds__(kBlock, MIN_BLOCKS)
    spattn_bwd_f128(int n, int heads, float scale_inv, int blocks_a, const float *__restrict__ q,
                    const float *__restrict__ k, const float *__restrict__ v, const float *__restrict__ dout,
                    const float *__restrict__ z, const float *__restrict__ delta, const int *__restrict__ dst_rowptr,
                    const int *__restrict__ dst_src, const int *__restrict__ src_rowptr,
                    const int *__restrict__ src_dst, const int *__restrict__ src_to_dst_slot,
                    const float *__restrict__ bias, float *__restrict__ dq, float *__restrict__ dk,
                    float *__restrict__ dv, float *__restrict__ dbias, SegView sgd, SegView sgs) {
    using namespace f128;
    const int lane = lane_id();
    const int wid = threadIdx.x >> 5;
    const int b = blockIdx.x;
    // blocks: [0, blocks_a) destination rows, [blocks_a, 2 blocks_a) source rows, then the
    // destination-view segments and the source-view segments of heavy rows
    const int seg_blocks_d = (sgd.nseg + kWarpsPerBlock - 1) / kWarpsPerBlock;
    bool role_a;
    int row, beg, end, seg = -1;
    if (b < 2 * blocks_a) {
        role_a = b < blocks_a;
        row = (role_a ? b : b - blocks_a) * kWarpsPerBlock + wid;
        if (row >= n) return;
        const int32_t *first = role_a ? sgd.first : sgs.first;
        if (first != nullptr && __ldg(first + row) >= 0) return;   // done by its segments
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        beg = __ldg(rp + row);
        end = __ldg(rp + row + 1);
    } else {
        const int sb = b - 2 * blocks_a;
        role_a = sb < seg_blocks_d;
        seg = (role_a ? sb : sb - seg_blocks_d) * kWarpsPerBlock + wid;
        if (seg >= (role_a ? sgd.nseg : sgs.nseg)) return;
        row = __ldg((role_a ? sgd.row : sgs.row) + seg);
        const int *rp = role_a ? dst_rowptr : src_rowptr;
        const int edges = role_a ? sgd.edges : sgs.edges;
        beg = __ldg(rp + row) + (seg - __ldg((role_a ? sgd.first : sgs.first) + row)) * edges;
        end = min(__ldg(rp + row + 1), beg + edges);
    }
    const uint4 *Q = reinterpret_cast<const uint4 *>(q) + lane;
    const uint4 *K = reinterpret_cast<const uint4 *>(k) + lane;
    const uint4 *V = reinterpret_cast<const uint4 *>(v) + lane;
    const uint4 *DO = reinterpret_cast<const uint4 *>(dout) + lane;
    const size_t rbase = (size_t)row * RV;
    const int head = lane / HEAD_VECS;
    float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);

    if (role_a) {
        // ---- dq for destination row `row` ----
        const uint4 qv = r128::ld16(Q + rbase), gv = r128::ld16(DO + rbase);
        const float2 q0 = lo(qv), q1 = hi(qv), g0 = lo(gv), g1 = hi(gv);
        const float inv = 1.0f / (__ldg(z + (size_t)row * heads + head) + kEps);
        const float dl = __ldg(delta + (size_t)row * heads + head);
        int nxt[UNROLL_A];
#pragma unroll
        for (int u = 0; u < UNROLL_A; u++) nxt[u] = beg + u < end ? __ldg(dst_src + beg + u) : 0;
        for (int e0 = beg; e0 < end; e0 += UNROLL_A) {
            int src[UNROLL_A];
            bool ok[UNROLL_A];
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                ok[u] = e0 + u < end;
                src[u] = nxt[u];
            }
            uint4 kr[UNROLL_A], vr[UNROLL_A];
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                kr[u] = r128::ld16(K + (size_t)src[u] * RV);
                vr[u] = r128::ld16(V + (size_t)src[u] * RV);
            }
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                const int e = e0 + UNROLL_A + u;
                nxt[u] = e < end ? __ldg(dst_src + e) : 0;
            }
#pragma unroll
            for (int u = 0; u < UNROLL_A; u++) {
                const int e = e0 + u;
                const float dqk = head_reduce<HEAD_VECS>(dot4(kr[u], q0, q1));
                const float dgv = head_reduce<HEAD_VECS>(dot4(vr[u], g0, g1));
                const float s = dqk * scale_inv;
                float sc = fminf(fmaxf(s, -kClamp), kClamp);
                const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                if (!NB && bias != nullptr && ok[u]) sc += __ldg(bias + (size_t)e * heads + head);
                const float p = mufu_exp(sc);
                const float dpre = (dgv - dl) * inv * p;
                const float ds = (ok[u] && inside) ? dpre : 0.f;
                if (!NB && dbias != nullptr && ok[u] && (lane % HEAD_VECS) == 0) dbias[(size_t)e * heads + head] = dpre;
                axpy4(a0, a1, ds, kr[u]);
            }
        }
        if (seg >= 0) {   // segment partial of dq (before the 1/sqrt(D) scale)
            *reinterpret_cast<float4 *>(sgd.part + (size_t)seg * RV * 4 + lane * 4) = make_float4(a0.x, a0.y, a1.x, a1.y);
            return;
        }
        *(reinterpret_cast<float4 *>(dq) + rbase + lane) =
            make_float4(a0.x * scale_inv, a0.y * scale_inv, a1.x * scale_inv, a1.y * scale_inv);
    } else {
        // ---- dk, dv for source row `row` ----
        const uint4 kv = r128::ld16(K + rbase), vv = r128::ld16(V + rbase);
        const float2 k0 = lo(kv), k1 = hi(kv), v0 = lo(vv), v1 = hi(vv);
        float2 b0 = make_float2(0.f, 0.f), b1 = make_float2(0.f, 0.f);
        int nxt[UNROLL_B];
#pragma unroll
        for (int u = 0; u < UNROLL_B; u++) nxt[u] = beg + u < end ? __ldg(src_dst + beg + u) : 0;
        for (int e0 = beg; e0 < end; e0 += UNROLL_B) {
            int dst[UNROLL_B];
            bool ok[UNROLL_B];
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                ok[u] = e0 + u < end;
                dst[u] = nxt[u];
            }
            uint4 qr[UNROLL_B], gr[UNROLL_B];
            float zr[UNROLL_B], dr[UNROLL_B];
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                qr[u] = r128::ld16(Q + (size_t)dst[u] * RV);
                gr[u] = r128::ld16(DO + (size_t)dst[u] * RV);
                zr[u] = __ldg(z + (size_t)dst[u] * heads + head);
                dr[u] = __ldg(delta + (size_t)dst[u] * heads + head);
            }
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                const int e = e0 + UNROLL_B + u;
                nxt[u] = e < end ? __ldg(src_dst + e) : 0;
            }
#pragma unroll
            for (int u = 0; u < UNROLL_B; u++) {
                const int e = e0 + u;
                const float dqk = head_reduce<HEAD_VECS>(dot4(qr[u], k0, k1));
                const float dgv = head_reduce<HEAD_VECS>(dot4(gr[u], v0, v1));
                const float s = dqk * scale_inv;
                float sc = fminf(fmaxf(s, -kClamp), kClamp);
                const bool inside = sc == s;   // -kClamp <= s <= kClamp (false for NaN)
                if (!NB && bias != nullptr && ok[u])
                    sc += __ldg(bias + (size_t)__ldg(src_to_dst_slot + e) * heads + head);
                const float p = ok[u] ? mufu_exp(sc) : 0.f;
                const float inv = mufu_rcp(zr[u] + kEps);
                const float a = p * inv;
                const float dpre = (dgv - dr[u]) * inv * p;
                const float ds = inside ? dpre : 0.f;
                axpy4(b0, b1, a, gr[u]);    // dv
                axpy4(a0, a1, ds, qr[u]);   // dk
            }
        }
        if (seg >= 0) {   // segment partials of dk (unscaled) and dv
            float *rec = sgs.part + (size_t)seg * 2 * RV * 4;
            *reinterpret_cast<float4 *>(rec + lane * 4) = make_float4(a0.x, a0.y, a1.x, a1.y);
            *reinterpret_cast<float4 *>(rec + RV * 4 + lane * 4) = make_float4(b0.x, b0.y, b1.x, b1.y);
            return;
        }
        *(reinterpret_cast<float4 *>(dk) + rbase + lane) =
            make_float4(a0.x * scale_inv, a0.y * scale_inv, a1.x * scale_inv, a1.y * scale_inv);
        *(reinterpret_cast<float4 *>(dv) + rbase + lane) = make_float4(b0.x, b0.y, b1.x, b1.y);
    }
}

// One warp per heavy row and view (the warp of its first segment): adds the segment partials in
// segment order and writes dq (destination view) or dk, dv (source view).
template <typename T, int HEAD_VECS, int ROW_VECS>
__global__ void __launch_bounds__(kBlock)
    spattn_bwd_seg_finish(float scale_inv, const int *__restrict__ dst_rowptr, const int *__restrict__ src_rowptr,
                          T *__restrict__ dq, T *__restrict__ dk, T *__restrict__ dv, SegView sgd, SegView sgs) {
    using L = VecLayout<T, HEAD_VECS, ROW_VECS>;
    constexpr int G = L::G, VPL = L::VPL, VE = L::VE, RF = ROW_VECS * VE;
    const int seg_blocks_d = (sgd.nseg + kWarpsPerBlock - 1) / kWarpsPerBlock;
    const bool role_a = (int)blockIdx.x < seg_blocks_d;
    const int seg = ((int)blockIdx.x - (role_a ? 0 : seg_blocks_d)) * kWarpsPerBlock + (threadIdx.x >> 5);
    if (seg >= (role_a ? sgd.nseg : sgs.nseg)) return;
    const int row = __ldg((role_a ? sgd.row : sgs.row) + seg);
    if (seg != __ldg((role_a ? sgd.first : sgs.first) + row)) return;
    const int lane = lane_id(), sub = lane / G, gl = lane % G;
    const int *rp = role_a ? dst_rowptr : src_rowptr;
    const int edges = role_a ? sgd.edges : sgs.edges;
    const int cnt = (__ldg(rp + row + 1) - __ldg(rp + row) + edges - 1) / edges;
    const int parts = role_a ? 1 : 2;
    const float *base = (role_a ? sgd.part : sgs.part) + (size_t)seg * parts * RF;
    float a0[VPL][VE], a1[VPL][VE];
#pragma unroll
    for (int t = 0; t < VPL; t++)
#pragma unroll
        for (int i = 0; i < VE; i++) a0[t][i] = a1[t][i] = 0.f;
    for (int j = 0; j < cnt; j++) {
        const float *rec = base + (size_t)j * parts * RF;
#pragma unroll
        for (int t = 0; t < VPL; t++)
#pragma unroll
            for (int i = 0; i < VE; i += 4) {
                const float4 x = __ldg(reinterpret_cast<const float4 *>(rec + (gl + G * t) * VE + i));
                a0[t][i] += x.x;
                a0[t][i + 1] += x.y;
                a0[t][i + 2] += x.z;
                a0[t][i + 3] += x.w;
                if (!role_a) {
                    const float4 y = __ldg(reinterpret_cast<const float4 *>(rec + RF + (gl + G * t) * VE + i));
                    a1[t][i] += y.x;
                    a1[t][i + 1] += y.y;
                    a1[t][i + 2] += y.z;
                    a1[t][i + 3] += y.w;
                }
            }
    }
    if (sub != 0) return;
    const size_t rbase = (size_t)row * ROW_VECS + gl;
#pragma unroll
    for (int t = 0; t < VPL; t++) {
        float r[VE];
#pragma unroll
        for (int i = 0; i < VE; i++) r[i] = a0[t][i] * scale_inv;
        if (role_a) {
            st16(reinterpret_cast<Vec16 *>(dq) + rbase + G * t, Elem<T>::pack(r));
        } else {
            st16(reinterpret_cast<Vec16 *>(dk) + rbase + G * t, Elem<T>::pack(r));
            st16(reinterpret_cast<Vec16 *>(dv) + rbase + G * t, Elem<T>::pack(a1[t]));
        }
    }
}

// ------------------------------------------------------------------------------------
// generic scalar path: one thread per (row, head); any head_dim in the instantiated set,
// any alignment.  Used for shapes the vector layout does not cover (e.g. head_dim 24).
// ------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kBlock)
    spattn_fwd_scalar(int n, int heads, float scale_inv, const T *__restrict__ q,
                      const T *__restrict__ k, const T *__restrict__ v,
                      const int *__restrict__ rowptr, const int *__restrict__ col,
                      const float *__restrict__ bias, T *__restrict__ out, float *__restrict__ z) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)n * heads) return;
    const int row = (int)(gid / heads), h = (int)(gid % heads);
    const size_t rs = (size_t)heads * D;
    float qf[D], acc[D];
#pragma unroll
    for (int i = 0; i < D; i++) {
        qf[i] = Elem<T>::load1(q + row * rs + h * D + i);
        acc[i] = 0.f;
    }
    float zs = 0.f;
    for (int e = rowptr[row]; e < rowptr[row + 1]; e++) {
        const int s_ = col[e];
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < D; i++) d = fmaf(Elem<T>::load1(k + s_ * rs + h * D + i), qf[i], d);
        float s = fminf(fmaxf(d * scale_inv, -kClamp), kClamp);
        if (bias != nullptr) s += bias[(size_t)e * heads + h];
        const float p = expf(s);
        zs += p;
#pragma unroll
        for (int i = 0; i < D; i++) acc[i] = fmaf(p, Elem<T>::load1(v + s_ * rs + h * D + i), acc[i]);
    }
    const float inv = 1.0f / (zs + kEps);
#pragma unroll
    for (int i = 0; i < D; i++) Elem<T>::store1(out + row * rs + h * D + i, acc[i] * inv);
    z[(size_t)row * heads + h] = zs;
}

__global__ void node_scores_from_z(int n, int heads, const float *__restrict__ z,
                                   float *__restrict__ node_scores, int ns_len) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n || row >= ns_len) return;
    float s = 0.f;
    for (int h = 0; h < heads; h++) s += z[(size_t)row * heads + h];
    node_scores[row] = s / (float)heads;
}

template <typename T, int D>
__global__ void __launch_bounds__(kBlock)
    spattn_delta_scalar(int n, int heads, const T *__restrict__ out, const T *__restrict__ dout,
                        float *__restrict__ delta) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)n * heads) return;
    const size_t base = (size_t)gid * D;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < D; i++) d = fmaf(Elem<T>::load1(out + base + i), Elem<T>::load1(dout + base + i), d);
    delta[gid] = d;
}

template <typename T, int D>
__global__ void __launch_bounds__(kBlock)
    spattn_bwd_scalar(int n, int heads, float scale_inv, const T *__restrict__ q,
                      const T *__restrict__ k, const T *__restrict__ v, const T *__restrict__ dout,
                      const float *__restrict__ z, const float *__restrict__ delta,
                      const int *__restrict__ dst_rowptr, const int *__restrict__ dst_src,
                      const int *__restrict__ src_rowptr, const int *__restrict__ src_dst,
                      const int *__restrict__ src_to_dst_slot, const float *__restrict__ bias,
                      T *__restrict__ dq, T *__restrict__ dk, T *__restrict__ dv,
                      float *__restrict__ dbias) {
    const int64_t total = (int64_t)n * heads;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool role_a = gid < total;
    if (!role_a) gid -= total;
    if (gid >= total) return;
    const int row = (int)(gid / heads), h = (int)(gid % heads);
    const size_t rs = (size_t)heads * D;
    const size_t me = row * rs + h * D;
    if (role_a) {
        float qf[D], gf[D], acc[D];
#pragma unroll
        for (int i = 0; i < D; i++) {
            qf[i] = Elem<T>::load1(q + me + i);
            gf[i] = Elem<T>::load1(dout + me + i);
            acc[i] = 0.f;
        }
        const float inv = 1.0f / (z[gid] + kEps), dl = delta[gid];
        for (int e = dst_rowptr[row]; e < dst_rowptr[row + 1]; e++) {
            const size_t o = (size_t)dst_src[e] * rs + h * D;
            float dqk = 0.f, dgv = 0.f;
#pragma unroll
            for (int i = 0; i < D; i++) {
                dqk = fmaf(Elem<T>::load1(k + o + i), qf[i], dqk);
                dgv = fmaf(gf[i], Elem<T>::load1(v + o + i), dgv);
            }
            const float s = dqk * scale_inv;
            float sc = fminf(fmaxf(s, -kClamp), kClamp);
            if (bias != nullptr) sc += bias[(size_t)e * heads + h];
            const float p = expf(sc);
            const float dpre = (dgv - dl) * inv * p;
            if (dbias != nullptr) dbias[(size_t)e * heads + h] = dpre;
            const float ds = (s >= -kClamp && s <= kClamp) ? dpre : 0.f;
#pragma unroll
            for (int i = 0; i < D; i++) acc[i] = fmaf(ds, Elem<T>::load1(k + o + i), acc[i]);
        }
#pragma unroll
        for (int i = 0; i < D; i++) Elem<T>::store1(dq + me + i, acc[i] * scale_inv);
    } else {
        float kf[D], vf[D], ak[D], av[D];
#pragma unroll
        for (int i = 0; i < D; i++) {
            kf[i] = Elem<T>::load1(k + me + i);
            vf[i] = Elem<T>::load1(v + me + i);
            ak[i] = av[i] = 0.f;
        }
        for (int e = src_rowptr[row]; e < src_rowptr[row + 1]; e++) {
            const int d_ = src_dst[e];
            const size_t o = (size_t)d_ * rs + h * D;
            float dqk = 0.f, dgv = 0.f;
#pragma unroll
            for (int i = 0; i < D; i++) {
                dqk = fmaf(kf[i], Elem<T>::load1(q + o + i), dqk);
                dgv = fmaf(Elem<T>::load1(dout + o + i), vf[i], dgv);
            }
            const float s = dqk * scale_inv;
            float sc = fminf(fmaxf(s, -kClamp), kClamp);
            if (bias != nullptr) sc += bias[(size_t)src_to_dst_slot[e] * heads + h];
            const float p = expf(sc);
            const float inv = 1.0f / (z[(size_t)d_ * heads + h] + kEps);
            const float a = p * inv;
            const float dpre = (dgv - delta[(size_t)d_ * heads + h]) * inv * p;
            const float ds = (s >= -kClamp && s <= kClamp) ? dpre : 0.f;
#pragma unroll
            for (int i = 0; i < D; i++) {
                const float gq = Elem<T>::load1(q + o + i), gd = Elem<T>::load1(dout + o + i);
                av[i] = fmaf(a, gd, av[i]);
                ak[i] = fmaf(ds, gq, ak[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < D; i++) {
            Elem<T>::store1(dk + me + i, ak[i] * scale_inv);
            Elem<T>::store1(dv + me + i, av[i]);
        }
    }
}

// ------------------------------------------------------------------------------------
// dispatch
// ------------------------------------------------------------------------------------
struct Shape {
    int head_vecs = 0, row_vecs = 0;
};

template <typename T>
Shape vec_shape(int heads, int head_dim) {
    Shape s;
    const int hb = head_dim * (int)sizeof(T);
    if (hb % 16 != 0) return s;
    const int hv = hb / 16;
    const int rv = hv * heads;
    auto pow2 = [](int x) { return x > 0 && (x & (x - 1)) == 0; };
    if (!pow2(hv) || hv > 8 || !pow2(rv) || rv < 2 || rv > 128) return s;
    s.head_vecs = hv;
    s.row_vecs = rv;
    return s;
}

#define NGT_VEC_CASES(MACRO)                                                                   \
    MACRO(1, 2) MACRO(1, 4) MACRO(1, 8) MACRO(1, 16) MACRO(1, 32) MACRO(1, 64) MACRO(1, 128)  \
    MACRO(2, 2) MACRO(2, 4) MACRO(2, 8) MACRO(2, 16) MACRO(2, 32) MACRO(2, 64) MACRO(2, 128)  \
    MACRO(4, 4) MACRO(4, 8) MACRO(4, 16) MACRO(4, 32) MACRO(4, 64) MACRO(4, 128)               \
    MACRO(8, 8) MACRO(8, 16) MACRO(8, 32) MACRO(8, 64) MACRO(8, 128)

#define NGT_SCALAR_DIMS(MACRO) MACRO(4) MACRO(8) MACRO(12) MACRO(16) MACRO(24) MACRO(32) MACRO(48) MACRO(64)

// bf16 128-element rows: edge pairs and index prefetch where a head spans two lanes (D = 16); the
// per-edge bias tests compiled away when the call has no edge bias (nor its gradient).
template <int HV>
void launch_fwd_r128(unsigned grid, cudaStream_t st, int n, int heads, float scale_inv, const void *q, const void *k,
                     const void *v, const int32_t *rowptr, const int32_t *col, const float *bias, void *out, float *z,
                     float *ns, int ns_len, int row_blocks, SegView sg) {
    constexpr int U = HV == 2 ? 2 : 4;
    constexpr bool P = HV == 2;
    using B = __nv_bfloat16;
    if (bias != nullptr)
        spattn_fwd_r128<HV, U, 4, P, P, false><<<grid, kBlock, 0, st>>>(n, heads, scale_inv, (const B *)q, (const B *)k,
                                                                       (const B *)v, rowptr, col, bias, (B *)out, z,
                                                                       ns, ns_len, row_blocks, sg);
    else
        spattn_fwd_r128<HV, U, 4, P, P, true><<<grid, kBlock, 0, st>>>(n, heads, scale_inv, (const B *)q, (const B *)k,
                                                                      (const B *)v, rowptr, col, nullptr, (B *)out, z,
                                                                      ns, ns_len, row_blocks, sg);
}

template <int HV>
void launch_bwd_r128(unsigned grid, cudaStream_t st, int n, int heads, float scale_inv, int blocks_a, const void *q,
                     const void *k, const void *v, const void *dout, const float *z, const float *delta,
                     const int32_t *dst_rowptr, const int32_t *dst_src, const int32_t *src_rowptr,
                     const int32_t *src_dst, const int32_t *s2d, const float *bias, void *dq, void *dk, void *dv,
                     float *dbias, SegView sgd, SegView sgs) {
    constexpr int UA = HV == 2 ? 2 : 3;
    constexpr bool P = HV == 2;
    using B = __nv_bfloat16;
    if (bias != nullptr || dbias != nullptr)
        spattn_bwd_r128<HV, UA, 2, 4, P, P, false><<<grid, kBlock, 0, st>>>(
            n, heads, scale_inv, blocks_a, (const B *)q, (const B *)k, (const B *)v, (const B *)dout, z, delta,
            dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias, (B *)dq, (B *)dk, (B *)dv, dbias, sgd, sgs);
    else
        spattn_bwd_r128<HV, UA, 2, 4, P, P, true><<<grid, kBlock, 0, st>>>(
            n, heads, scale_inv, blocks_a, (const B *)q, (const B *)k, (const B *)v, (const B *)dout, z, delta,
            dst_rowptr, dst_src, src_rowptr, src_dst, s2d, nullptr, (B *)dq, (B *)dk, (B *)dv, nullptr, sgd, sgs);
}

// fp32 128-element rows, with the bias tests compiled out when the call has no edge bias.
template <int HV>
void launch_fwd_f128(unsigned grid, cudaStream_t st, int n, int heads, float scale_inv, const void *q, const void *k,
                     const void *v, const int32_t *rowptr, const int32_t *col, const float *bias, void *out, float *z,
                     float *ns, int ns_len, int row_blocks, SegView sg) {
    const float *Q = (const float *)q, *K = (const float *)k, *V = (const float *)v;
    if (bias != nullptr)
        spattn_fwd_f128<HV, 4, 4, false><<<grid, kBlock, 0, st>>>(n, heads, scale_inv, Q, K, V, rowptr, col, bias,
                                                                   (float *)out, z, ns, ns_len, row_blocks, sg);
    else
        spattn_fwd_f128<HV, 4, 4, true><<<grid, kBlock, 0, st>>>(n, heads, scale_inv, Q, K, V, rowptr, col, nullptr,
                                                                  (float *)out, z, ns, ns_len, row_blocks, sg);
}

template <int HV>
void launch_bwd_f128(unsigned grid, cudaStream_t st, int n, int heads, float scale_inv, int blocks_a, const void *q,
                     const void *k, const void *v, const void *dout, const float *z, const float *delta,
                     const int32_t *dst_rowptr, const int32_t *dst_src, const int32_t *src_rowptr,
                     const int32_t *src_dst, const int32_t *s2d, const float *bias, void *dq, void *dk, void *dv,
                     float *dbias, SegView sgd, SegView sgs) {
    const float *Q = (const float *)q, *K = (const float *)k, *V = (const float *)v, *G = (const float *)dout;
    if (bias != nullptr || dbias != nullptr)
        spattn_bwd_f128<HV, 3, 2, 4, false><<<grid, kBlock, 0, st>>>(
            n, heads, scale_inv, blocks_a, Q, K, V, G, z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias,
            (float *)dq, (float *)dk, (float *)dv, dbias, sgd, sgs);
    else
        spattn_bwd_f128<HV, 3, 2, 4, true><<<grid, kBlock, 0, st>>>(
            n, heads, scale_inv, blocks_a, Q, K, V, G, z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, nullptr,
            (float *)dq, (float *)dk, (float *)dv, nullptr, sgd, sgs);
}

template <typename T>
int forward_t(int64_t n, int heads, int head_dim, const void *q, const void *k, const void *v,
              const int32_t *rowptr, const int32_t *col, const float *bias, void *out, float *z,
              float *ns, int64_t ns_len, SegView sg, cudaStream_t st) {
    const float scale_inv = 1.0f / sqrtf((float)head_dim);
    const Shape sh = vec_shape<T>(heads, head_dim);
    const bool al = aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out);
    if (n == 0) return NGT_OK;
    if (sh.head_vecs && al) {
        const int row_blocks = ceil_div_i(n, kWarpsPerBlock);
        const int seg_blocks = ceil_div_i(sg.nseg, kWarpsPerBlock);
#define NGT_FWD(HV, RV)                                                                          \
    if (sh.head_vecs == HV && sh.row_vecs == RV) {                                               \
        if constexpr (sizeof(T) == 2 && RV == 16)                                                \
            launch_fwd_r128<HV>(row_blocks + seg_blocks, st, (int)n, heads, scale_inv, q, k, v,      \
                                rowptr, col, bias, out, z, ns, (int)ns_len, row_blocks, sg);     \
        else if constexpr (sizeof(T) == 4 && RV == 32)                                           \
            launch_fwd_f128<HV>(row_blocks + seg_blocks, st, (int)n, heads, scale_inv, q, k, v,      \
                                rowptr, col, bias, out, z, ns, (int)ns_len, row_blocks, sg);     \
        else                                                                                     \
            spattn_fwd_vec<T, HV, RV><<<row_blocks + seg_blocks, kBlock, 0, st>>>(               \
                (int)n, heads, scale_inv, (const T *)q, (const T *)k, (const T *)v, rowptr, col, \
                bias, (T *)out, z, ns, (int)ns_len, row_blocks, sg);                             \
        NGT_CHECK_LAUNCH();                                                                      \
        if (sg.nseg > 0)                                                                         \
            spattn_fwd_seg_finish<T, HV, RV><<<seg_blocks, kBlock, 0, st>>>(heads, rowptr, (T *)out, z, ns, \
                                                                            (int)ns_len, sg);    \
        NGT_CHECK_LAUNCH();                                                                      \
        return NGT_OK;                                                                           \
    }
        NGT_VEC_CASES(NGT_FWD)
#undef NGT_FWD
    }
    if (z == nullptr) return NGT_ERR_INVALID_ARGUMENT;  // the scalar path derives scores from z
    const int grid = ceil_div_i(n * heads, kBlock);
#define NGT_FWDS(DD)                                                                                 \
    if (head_dim == DD) {                                                                            \
        spattn_fwd_scalar<T, DD><<<grid, kBlock, 0, st>>>((int)n, heads, scale_inv, (const T *)q,    \
                                                          (const T *)k, (const T *)v, rowptr, col,   \
                                                          bias, (T *)out, z);                        \
        NGT_CHECK_LAUNCH();                                                                          \
        node_scores_from_z<<<ceil_div_i(n, kBlock), kBlock, 0, st>>>((int)n, heads, z, ns, (int)ns_len); \
        NGT_CHECK_LAUNCH();                                                                          \
        return NGT_OK;                                                                               \
    }
    NGT_SCALAR_DIMS(NGT_FWDS)
#undef NGT_FWDS
    return NGT_ERR_UNSUPPORTED;
}

template <typename T>
int backward_t(int64_t n, int heads, int head_dim, const void *q, const void *k, const void *v,
               const void *out, const void *dout, const float *z, const int32_t *dst_rowptr,
               const int32_t *dst_src, const int32_t *src_rowptr, const int32_t *src_dst,
               const int32_t *s2d, const float *bias, float *delta, void *dq, void *dk, void *dv,
               float *dbias, SegView sgd, SegView sgs, cudaStream_t st) {
    const float scale_inv = 1.0f / sqrtf((float)head_dim);
    if (n == 0) return NGT_OK;
    const Shape sh = vec_shape<T>(heads, head_dim);
    const bool al = aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
                    aligned16(dout) && aligned16(dq) && aligned16(dk) && aligned16(dv);
    if (sh.head_vecs && al) {
        const int blocks_a = ceil_div_i(n, kWarpsPerBlock);
        const int seg_blocks = ceil_div_i(sgd.nseg, kWarpsPerBlock) + ceil_div_i(sgs.nseg, kWarpsPerBlock);
#define NGT_BWD(HV, RV)                                                                           \
    if (sh.head_vecs == HV && sh.row_vecs == RV) {                                                \
        using Lay = VecLayout<T, HV, RV>;                                                         \
        spattn_delta_vec<T, HV, RV><<<ceil_div_i(n, (int64_t)kWarpsPerBlock * Lay::EPW), kBlock, 0, st>>>( \
            (int)n, heads, (const T *)out, (const T *)dout, delta);                               \
        NGT_CHECK_LAUNCH();                                                                       \
        if constexpr (sizeof(T) == 2 && RV == 16)                                                 \
            launch_bwd_r128<HV>(2 * blocks_a + seg_blocks, st, (int)n, heads, scale_inv, blocks_a, q, k, v, \
                                dout, z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias, dq,  \
                                dk, dv, dbias, sgd, sgs);                                          \
        else if constexpr (sizeof(T) == 4 && RV == 32)                                            \
            launch_bwd_f128<HV>(2 * blocks_a + seg_blocks, st, (int)n, heads, scale_inv, blocks_a, q, k, v, \
                                dout, z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias, dq,  \
                                dk, dv, dbias, sgd, sgs);                                          \
        else                                                                                      \
            spattn_bwd_vec<T, HV, RV><<<2 * blocks_a + seg_blocks, kBlock, 0, st>>>(              \
                (int)n, heads, scale_inv, blocks_a, (const T *)q, (const T *)k, (const T *)v,     \
                (const T *)dout, z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias,   \
                (T *)dq, (T *)dk, (T *)dv, dbias, sgd, sgs);                                      \
        NGT_CHECK_LAUNCH();                                                                       \
        if (seg_blocks > 0)                                                                       \
            spattn_bwd_seg_finish<T, HV, RV><<<seg_blocks, kBlock, 0, st>>>(                      \
                scale_inv, dst_rowptr, src_rowptr, (T *)dq, (T *)dk, (T *)dv, sgd, sgs);          \
        NGT_CHECK_LAUNCH();                                                                       \
        return NGT_OK;                                                                            \
    }
        NGT_VEC_CASES(NGT_BWD)
#undef NGT_BWD
    }
    const int grid1 = ceil_div_i(n * heads, kBlock);
#define NGT_BWDS(DD)                                                                              \
    if (head_dim == DD) {                                                                         \
        spattn_delta_scalar<T, DD><<<grid1, kBlock, 0, st>>>((int)n, heads, (const T *)out,       \
                                                             (const T *)dout, delta);             \
        NGT_CHECK_LAUNCH();                                                                       \
        spattn_bwd_scalar<T, DD><<<2 * grid1, kBlock, 0, st>>>(                                   \
            (int)n, heads, scale_inv, (const T *)q, (const T *)k, (const T *)v, (const T *)dout,  \
            z, delta, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, bias, (T *)dq, (T *)dk,      \
            (T *)dv, dbias);                                                                      \
        NGT_CHECK_LAUNCH();                                                                       \
        return NGT_OK;                                                                            \
    }
    NGT_SCALAR_DIMS(NGT_BWDS)
#undef NGT_BWDS
    return NGT_ERR_UNSUPPORTED;
}

int check_common(int dtype, int64_t n, int64_t e, int heads, int head_dim) {
    if (n < 0 || e < 0 || heads <= 0 || head_dim <= 0) return NGT_ERR_INVALID_ARGUMENT;
    if (dtype != NGT_F32 && dtype != NGT_BF16) return NGT_ERR_INVALID_ARGUMENT;
    if (n >= (int64_t)INT32_MAX || e >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if (n * heads >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    return NGT_OK;
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_spattn_forward(int dtype, int64_t n, int64_t e, int heads, int head_dim,
                                  const void *q, const void *k, const void *v,
                                  const int32_t *dst_rowptr, const int32_t *dst_src,
                                  const float *edge_bias, void *out, float *z, float *node_scores,
                                  int64_t node_scores_len, ngt_stream_t stream) {
    int rc = check_common(dtype, n, e, heads, head_dim);
    if (rc != NGT_OK) return rc;
    if (n > 0 && (!q || !k || !v || !dst_rowptr || !out)) return NGT_ERR_INVALID_ARGUMENT;
    if (e > 0 && !dst_src) return NGT_ERR_INVALID_ARGUMENT;
    if (node_scores_len < 0 || node_scores_len > n || (node_scores_len > 0 && !node_scores))
        return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const SegView none{0, nullptr, nullptr, 0, nullptr};
    if (dtype == NGT_F32)
        return forward_t<float>(n, heads, head_dim, q, k, v, dst_rowptr, dst_src, edge_bias, out, z,
                                node_scores, node_scores_len, none, st);
    return forward_t<__nv_bfloat16>(n, heads, head_dim, q, k, v, dst_rowptr, dst_src, edge_bias, out,
                                    z, node_scores, node_scores_len, none, st);
}

namespace {
// Segment tables of one view as the kernels take them; a view without segments is all null.
int seg_view(int64_t n, int32_t seg_edges, const int32_t *first, const int32_t *row, int64_t nseg, float *part,
             SegView *out) {
    *out = SegView{0, nullptr, nullptr, 0, nullptr};
    if (nseg < 0) return NGT_ERR_INVALID_ARGUMENT;
    if (nseg == 0 || n == 0) return NGT_OK;
    if (seg_edges <= 0 || !first || !row || !part) return NGT_ERR_INVALID_ARGUMENT;
    if (nseg >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if ((reinterpret_cast<uintptr_t>(part) & 15u) != 0) return NGT_ERR_MISALIGNED;
    *out = SegView{seg_edges, first, row, (int)nseg, part};
    return NGT_OK;
}
}  // namespace

extern "C" int ngt_spattn_seg_part_size(int pass, int heads, int head_dim, int64_t dst_nseg, int64_t src_nseg,
                                        size_t *bytes) {
    if (!bytes || heads <= 0 || head_dim <= 0 || dst_nseg < 0 || src_nseg < 0 || (pass != 0 && pass != 1))
        return NGT_ERR_INVALID_ARGUMENT;
    const size_t hd = (size_t)heads * head_dim;
    *bytes = sizeof(float) * (pass == 0 ? (size_t)dst_nseg * fwd_record(heads, (int)hd)
                                        : (size_t)dst_nseg * hd + (size_t)src_nseg * 2 * hd);
    return NGT_OK;
}

extern "C" int ngt_spattn_forward_seg(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                                      const void *k, const void *v, const int32_t *dst_rowptr,
                                      const int32_t *dst_src, const float *edge_bias, void *out, float *z,
                                      float *node_scores, int64_t node_scores_len, int32_t seg_edges,
                                      const int32_t *dst_seg_first, const int32_t *dst_seg_row, int64_t dst_nseg,
                                      float *seg_part, ngt_stream_t stream) {
    int rc = check_common(dtype, n, e, heads, head_dim);
    if (rc != NGT_OK) return rc;
    if (n > 0 && (!q || !k || !v || !dst_rowptr || !out)) return NGT_ERR_INVALID_ARGUMENT;
    if (e > 0 && !dst_src) return NGT_ERR_INVALID_ARGUMENT;
    if (node_scores_len < 0 || node_scores_len > n || (node_scores_len > 0 && !node_scores))
        return NGT_ERR_INVALID_ARGUMENT;
    SegView sg;
    rc = seg_view(n, seg_edges, dst_seg_first, dst_seg_row, dst_nseg, seg_part, &sg);
    if (rc != NGT_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == NGT_F32)
        return forward_t<float>(n, heads, head_dim, q, k, v, dst_rowptr, dst_src, edge_bias, out, z,
                                node_scores, node_scores_len, sg, st);
    return forward_t<__nv_bfloat16>(n, heads, head_dim, q, k, v, dst_rowptr, dst_src, edge_bias, out,
                                    z, node_scores, node_scores_len, sg, st);
}

extern "C" int ngt_spattn_backward(int dtype, int64_t n, int64_t e, int heads, int head_dim,
                                   const void *q, const void *k, const void *v, const void *out,
                                   const void *dout, const float *z, const int32_t *dst_rowptr,
                                   const int32_t *dst_src, const int32_t *src_rowptr,
                                   const int32_t *src_dst, const int32_t *src_to_dst_slot,
                                   const float *edge_bias, float *delta, void *dq, void *dk,
                                   void *dv, float *dedge_bias, ngt_stream_t stream) {
    int rc = check_common(dtype, n, e, heads, head_dim);
    if (rc != NGT_OK) return rc;
    if (n > 0 && (!q || !k || !v || !out || !dout || !z || !dst_rowptr || !src_rowptr || !delta ||
                  !dq || !dk || !dv))
        return NGT_ERR_INVALID_ARGUMENT;
    if (e > 0 && (!dst_src || !src_dst)) return NGT_ERR_INVALID_ARGUMENT;
    if (edge_bias != nullptr && e > 0 && src_to_dst_slot == nullptr) return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const SegView none{0, nullptr, nullptr, 0, nullptr};
    if (dtype == NGT_F32)
        return backward_t<float>(n, heads, head_dim, q, k, v, out, dout, z, dst_rowptr, dst_src,
                                 src_rowptr, src_dst, src_to_dst_slot, edge_bias, delta, dq, dk, dv,
                                 dedge_bias, none, none, st);
    return backward_t<__nv_bfloat16>(n, heads, head_dim, q, k, v, out, dout, z, dst_rowptr, dst_src,
                                     src_rowptr, src_dst, src_to_dst_slot, edge_bias, delta, dq, dk,
                                     dv, dedge_bias, none, none, st);
}

extern "C" int ngt_spattn_backward_seg(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                                       const void *k, const void *v, const void *out, const void *dout,
                                       const float *z, const int32_t *dst_rowptr, const int32_t *dst_src,
                                       const int32_t *src_rowptr, const int32_t *src_dst,
                                       const int32_t *src_to_dst_slot, const float *edge_bias, float *delta,
                                       void *dq, void *dk, void *dv, float *dedge_bias, int32_t seg_edges,
                                       const int32_t *dst_seg_first, const int32_t *dst_seg_row,
                                       int64_t dst_nseg, const int32_t *src_seg_first,
                                       const int32_t *src_seg_row, int64_t src_nseg, float *seg_part,
                                       ngt_stream_t stream) {
    int rc = check_common(dtype, n, e, heads, head_dim);
    if (rc != NGT_OK) return rc;
    if (n > 0 && (!q || !k || !v || !out || !dout || !z || !dst_rowptr || !src_rowptr || !delta ||
                  !dq || !dk || !dv))
        return NGT_ERR_INVALID_ARGUMENT;
    if (e > 0 && (!dst_src || !src_dst)) return NGT_ERR_INVALID_ARGUMENT;
    if (edge_bias != nullptr && e > 0 && src_to_dst_slot == nullptr) return NGT_ERR_INVALID_ARGUMENT;
    SegView sgd, sgs;
    rc = seg_view(n, seg_edges, dst_seg_first, dst_seg_row, dst_nseg, seg_part, &sgd);
    if (rc != NGT_OK) return rc;
    float *src_part = seg_part ? seg_part + (size_t)dst_nseg * heads * head_dim : nullptr;
    rc = seg_view(n, seg_edges, src_seg_first, src_seg_row, src_nseg, src_part, &sgs);
    if (rc != NGT_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == NGT_F32)
        return backward_t<float>(n, heads, head_dim, q, k, v, out, dout, z, dst_rowptr, dst_src,
                                 src_rowptr, src_dst, src_to_dst_slot, edge_bias, delta, dq, dk, dv,
                                 dedge_bias, sgd, sgs, st);
    return backward_t<__nv_bfloat16>(n, heads, head_dim, q, k, v, out, dout, z, dst_rowptr, dst_src,
                                     src_rowptr, src_dst, src_to_dst_slot, edge_bias, delta, dq, dk,
                                     dv, dedge_bias, sgd, sgs, st);
}

// ------------------------------------------------------------------------------------
// Backward without any allocation: the per-row delta scratch lives in a fixed
// file-scope device array instead of a caller buffer.  For callers that cannot call
// cudaMalloc (or a caching allocator) at the point where they run the backward.
// ------------------------------------------------------------------------------------
namespace {

// n * heads floats of delta scratch; every GPU that loads the library keeps this much
// (8 MiB) reserved until the process exits.
static __device__ __align__(256) float g_noalloc_delta[NGT_NOALLOC_MAX_ROWS_X_HEADS];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float *g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_delta on the current device.  The host-side name is only a
// stand-in for the symbol, so the address is looked up once per device, with that device
// current, and cached.
int noalloc_delta(float **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NGT_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return NGT_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_delta) != cudaSuccess || p == nullptr) return NGT_ERR_CUDA;
        g_noalloc_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return NGT_OK;
}

}  // namespace

extern "C" int ngt_spattn_backward_noalloc(int dtype, int64_t n, int64_t e, int heads, int head_dim,
                                           const void *q, const void *k, const void *v,
                                           const void *out, const void *dout, const float *z,
                                           const int32_t *dst_rowptr, const int32_t *dst_src,
                                           const int32_t *src_rowptr, const int32_t *src_dst,
                                           const int32_t *src_to_dst_slot, const float *edge_bias,
                                           void *dq, void *dk, void *dv, float *dedge_bias,
                                           ngt_stream_t stream) {
    int rc = check_common(dtype, n, e, heads, head_dim);
    if (rc != NGT_OK) return rc;
    if (n * (int64_t)heads > (int64_t)NGT_NOALLOC_MAX_ROWS_X_HEADS) return NGT_ERR_TOO_LARGE;
    float *delta = nullptr;
    rc = noalloc_delta(&delta);
    if (rc != NGT_OK) return rc;
    return ngt_spattn_backward(dtype, n, e, heads, head_dim, q, k, v, out, dout, z, dst_rowptr, dst_src,
                               src_rowptr, src_dst, src_to_dst_slot, edge_bias, delta, dq, dk, dv,
                               dedge_bias, stream);
}
