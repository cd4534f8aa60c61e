// Dense full-attention windows on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Replaces `CoreAttention.full_attention`
// (NeutronGT/models/gt_dist_node_level_single_window.py:56-109; graphormer_dist_node_level.py:42-65):
//     S = (q * sqrt(D)) k^T          (the reference multiplies by sqrt(D); kept as is)
//     P = softmax(S), dropout(P), X = P v
//     node_scores[j] = sum_i mean_h |S[h, i, j]|      (raw S, before softmax)
// The reference materialises [H, s, s]; here each CTA owns 128 queries of one head and
// streams 128-key blocks:
//   * Q, K, V tiles are staged in shared memory in the no-swizzle core-matrix layout
//     (8 rows x 16 B), head_dim zero-padded to a multiple of 16;
//   * S = Q K^T and O += P V run as tcgen05.mma (bf16 in, fp32 accumulate in TMEM);
//     V is read as an MN-major operand, so it is staged exactly like K;
//   * online softmax (base-2, one TMEM lane = one query row per thread) rescales O in TMEM;
//   * the node-score column sums sum_i |S_ij| run on the tensor core as |S|^T * ones (|S|
//     written once to shared memory and read as an MN-major operand), one atomic add per key;
//   * two CTAs share an SM and the next K/V block is prefetched into registers during the
//     current block's MMA and softmax.
// Every mbarrier wait is bounded; on timeout the CTA records a status, waits (bounded) for
// its own MMAs, frees its TMEM and exits.
#include "dense_tma.h"
#include "tc.cuh"

namespace ngt {
namespace {

constexpr int BM = 128;          // queries per CTA (one TMEM lane each)
constexpr int BN = 128;          // keys per block
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kWaitLimit = 1u << 20;
constexpr float kLn2 = 0.69314718055994531f;
constexpr float kLog2e = 1.44269504088896341f;

// Byte offset of (row r, 16-byte chunk c) in a core-matrix tile with `row_chunks` chunks per row.
__device__ __forceinline__ uint32_t core_off(int r, int c, int row_chunks) {
    return (uint32_t)((r >> 3) * (row_chunks * 128) + c * 128 + (r & 7) * 16);
}

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Keep decision of attention dropout for (head, query, key): a counter-based hash, so the
// backward regenerates the same mask.
__device__ __forceinline__ bool keep_elem(uint32_t seed, int h, int i, int j, uint32_t threshold) {
    const uint32_t x = mix32(seed ^ mix32((uint32_t)i * 0x9E3779B1u + (uint32_t)h * 0x85EBCA77u) ^ ((uint32_t)j * 0xC2B2AE3Du));
    return x >= threshold;
}

template <int DP>
struct FwdSmem {
    static constexpr int CH = DP / 8;
    static constexpr int kOnesRows = 16;
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kK = kQ + BM * DP * 2;
    static constexpr uint32_t kV = kK + BN * DP * 2;
    static constexpr uint32_t kP = kV + BN * DP * 2;
    static constexpr uint32_t kAbs = kP + BM * BN * 2;
    static constexpr uint32_t kOnes = kAbs + BM * BN * 2;
    static constexpr uint32_t kBar = kOnes + kOnesRows * BM * 2;
    static constexpr uint32_t kTmemSlot = kBar + 16;
    static constexpr uint32_t kBytes = kTmemSlot + 16;
};

// Two CTAs share an SM (<= 113 KiB shared memory and 256 TMEM columns each), so one CTA's
// softmax overlaps the other's tensor-core work.
// BIAS: an additive fp32 bias joins the scores before the softmax, X = S + bias[h, i, j] (bias
// element (h, i, j) at h * bias_hs + i * s + j; bias_hs = 0 shares one [s, s] matrix over the
// heads); -inf entries (masked keys) take no weight.  The node scores stay those of the raw S.
template <int DP, bool BIAS = false>
__global__ void __launch_bounds__(kThreads, 2)
    dense_fwd_kernel(int s, int H, int D, float scale, float score_scale, float drop_p, uint32_t seed,
                     const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                     const __nv_bfloat16 *__restrict__ v, __nv_bfloat16 *__restrict__ out,
                     float *__restrict__ lse, float *__restrict__ node_scores, int *__restrict__ status,
                     const float *__restrict__ bias, int64_t bias_hs) {
    using L = FwdSmem<DP>;
    constexpr int CH = L::CH;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kTmemSlot);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int q0 = blockIdx.x * BM, h = blockIdx.y;
    const size_t rs = (size_t)H * D;

    if (warp == 0) tc::tmem_alloc(tmem_slot, kTmemCols);
    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::mbar_init_fence();
    }
    {   // Q row `tid` (zero padded) and the 16 x 128 all-ones operand of the column sums
        const int qi = q0 + tid;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            uint4 val = make_uint4(0, 0, 0, 0);
            if (qi < s && c * 8 < D) val = *reinterpret_cast<const uint4 *>(q + qi * rs + (size_t)h * D + c * 8);
            *reinterpret_cast<uint4 *>(smem + L::kQ + core_off(tid, c, CH)) = val;
        }
        if (tid < L::kOnesRows) {
            const uint4 ones = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
#pragma unroll
            for (int c = 0; c < BM / 8; c++) *reinterpret_cast<uint4 *>(smem + L::kOnes + core_off(tid, c, BM / 8)) = ones;
        }
    }
    // first K/V block in registers; every later block is prefetched during the previous one
    uint4 nk[CH], nv[CH];
    auto fetch_kv = [&](int k0) {
        const int kj = k0 + tid;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            nk[c] = make_uint4(0, 0, 0, 0);
            nv[c] = make_uint4(0, 0, 0, 0);
            if (kj < s && c * 8 < D) {
                nk[c] = *reinterpret_cast<const uint4 *>(k + kj * rs + (size_t)h * D + c * 8);
                nv[c] = *reinterpret_cast<const uint4 *>(v + kj * rs + (size_t)h * D + c * 8);
            }
        }
    };
    fetch_kv(0);
    tc::fence_smem_for_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + BN;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t aQ = tc::smem_addr(smem + L::kQ), aK = tc::smem_addr(smem + L::kK),
                   aV = tc::smem_addr(smem + L::kV), aP = tc::smem_addr(smem + L::kP),
                   aAbs = tc::smem_addr(smem + L::kAbs), aOnes = tc::smem_addr(smem + L::kOnes);
    constexpr uint32_t idesc_s = tc::idesc_bf16(BM, BN, false, false);
    constexpr uint32_t idesc_pv = tc::idesc_bf16(BM, DP, false, true);
    constexpr uint32_t idesc_c = tc::idesc_bf16(BN, L::kOnesRows, true, false);
    const float sl2 = scale * kLog2e;
    const float col_scale = scale * score_scale;
    const uint32_t drop_threshold = drop_p > 0.f ? (uint32_t)fminf(drop_p * 4294967296.0f, 4294967295.0f) : 0u;
    const float keep_scale = drop_p > 0.f ? 1.0f / (1.0f - drop_p) : 1.0f;
    const int qi = q0 + tid;
    const bool row_ok = qi < s;

    float m2 = -INFINITY, l = 0.f;
    uint32_t phase = 0;
    int failed = 0;
    const int nkb = (s + BN - 1) / BN;
    for (int kb = 0; kb < nkb; kb++) {
        const int k0 = kb * BN;
#pragma unroll
        for (int c = 0; c < CH; c++) {   // the previous block's MMAs are complete: reuse the tiles
            *reinterpret_cast<uint4 *>(smem + L::kK + core_off(tid, c, CH)) = nk[c];
            *reinterpret_cast<uint4 *>(smem + L::kV + core_off(tid, c, CH)) = nv[c];
        }
        tc::fence_smem_for_async();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < DP / 16; kk++)
                tc::mma_bf16(tS, tc::smem_desc(aQ + kk * 256, 128, CH * 128), tc::smem_desc(aK + kk * 256, 128, CH * 128),
                             idesc_s, kk > 0);
            tc::commit(bar);
        }
        if (kb + 1 < nkb) fetch_kv(k0 + BN);   // global loads overlap the MMA and the softmax
        if (tc::mbar_wait_bounded(bar, phase, kWaitLimit)) phase ^= 1;
        else failed = 1;
        failed = __syncthreads_or(failed);
        if (failed) break;
        tc::fence_after_sync();

        const bool full_block = k0 + BN <= s;   // every key of the block is real
        // the row's bias for this key block (BIAS only; rows past s read none)
        const float *brow = BIAS && row_ok ? bias + (size_t)h * bias_hs + (size_t)qi * s + k0 : nullptr;
        // pass 1: row max of the raw scores (scale > 0, so the max commutes with scaling); with a
        // bias, the max of the biased scores in log2 units
        float mraw = -INFINITY, mb2 = -INFINITY;
#pragma unroll 1
        for (int c4 = 0; c4 < BN / 32; c4++) {
            float t[32];
            tc::ld32(tS + lane_off + c4 * 32, t);
            if constexpr (BIAS) {
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (k0 + c4 * 32 + i < s) mb2 = fmaxf(mb2, fmaf(t[i], sl2, brow[c4 * 32 + i] * kLog2e));
                }
            } else if (full_block) {
#pragma unroll
                for (int i = 0; i < 32; i++) mraw = fmaxf(mraw, t[i]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++)
                    if (k0 + c4 * 32 + i < s) mraw = fmaxf(mraw, t[i]);
            }
        }
        const float m_new = fmaxf(m2, BIAS ? mb2 : mraw * sl2);
        const float alpha = (m_new == -INFINITY) ? 1.f : tc::ex2(m2 - m_new);
        l *= alpha;
        m2 = m_new;
        // pass 2: probabilities (dropout applied to what multiplies V, not to the normaliser)
        // and |S| in natural units for the node scores
#pragma unroll 1
        for (int c4 = 0; c4 < BN / 32; c4++) {
            float t[32];
            tc::ld32(tS + lane_off + c4 * 32, t);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t pw[4], aw[4];
                if (!BIAS && full_block && row_ok && !drop_threshold) {   // common case: no checks per element
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const float p0 = tc::ex2(fmaf(t[c * 8 + e], sl2, -m_new));
                        const float p1 = tc::ex2(fmaf(t[c * 8 + e + 1], sl2, -m_new));
                        l += p0 + p1;
                        pw[e / 2] = tc::pack_bf16(p0, p1);
                        aw[e / 2] = tc::pack_bf16(fabsf(t[c * 8 + e]), fabsf(t[c * 8 + e + 1]));
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        float pv[2], av[2];
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const int jj = c * 8 + e + u;
                            const int key = k0 + c4 * 32 + jj;
                            const bool ok = key < s;
                            float p;
                            if constexpr (BIAS) {
                                // a key whose biased score is -inf (or a row with none finite yet) takes no weight
                                const float x2 = ok && row_ok ? fmaf(t[jj], sl2, brow[c4 * 32 + jj] * kLog2e) : -INFINITY;
                                p = (x2 == -INFINITY || m_new == -INFINITY) ? 0.f : tc::ex2(x2 - m_new);
                            } else {
                                p = ok ? tc::ex2(fmaf(t[jj], sl2, -m_new)) : 0.f;
                            }
                            l += p;
                            float pd = p;
                            if (drop_threshold) pd = keep_elem(seed, h, qi, key, drop_threshold) ? p * keep_scale : 0.f;
                            pv[u] = pd;
                            av[u] = (ok && row_ok) ? fabsf(t[jj]) : 0.f;
                        }
                        pw[e / 2] = tc::pack_bf16(pv[0], pv[1]);
                        aw[e / 2] = tc::pack_bf16(av[0], av[1]);
                    }
                }
                const int chunk = c4 * 4 + c;
                *reinterpret_cast<uint4 *>(smem + L::kP + core_off(tid, chunk, BN / 8)) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
                *reinterpret_cast<uint4 *>(smem + L::kAbs + core_off(tid, chunk, BN / 8)) = make_uint4(aw[0], aw[1], aw[2], aw[3]);
            }
        }
        if (kb > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {   // rescale O by exp(m_old - m_new)
#pragma unroll
            for (int c4 = 0; c4 < DP / 32; c4++) {
                float o[32];
                tc::ld32(tO + lane_off + c4 * 32, o);
#pragma unroll
                for (int i = 0; i < 32; i++) o[i] *= alpha;
                tc::st32(tO + lane_off + c4 * 32, o);
            }
        }
        tc::fence_smem_for_async();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < BN / 16; kk++)   // O += P V   (V as an MN-major operand)
                tc::mma_bf16(tO, tc::smem_desc(aP + kk * 256, 128, (BN / 8) * 128),
                             tc::smem_desc(aV + kk * 2 * CH * 128, CH * 128, 128), idesc_pv, (kb > 0 || kk > 0));
#pragma unroll
            for (int kk = 0; kk < BM / 16; kk++)   // C = |S|^T ones: row j of C = sum_i |S_ij| (|S| read MN-major)
                tc::mma_bf16(tS, tc::smem_desc(aAbs + kk * 2 * (BN / 8) * 128, (BN / 8) * 128, 128),
                             tc::smem_desc(aOnes + kk * 256, 128, (BM / 8) * 128), idesc_c, kk > 0);
            tc::commit(bar);
        }
        if (tc::mbar_wait_bounded(bar, phase, kWaitLimit)) phase ^= 1;
        else failed = 1;
        failed = __syncthreads_or(failed);
        if (failed) break;
        tc::fence_after_sync();
        {   // lane `tid` of C holds the column sum of key k0 + tid
            float cs[32];
            tc::ld32(tS + lane_off, cs);
            const int key = k0 + tid;
            if (key < s) atomicAdd(node_scores + key, cs[0] * col_scale);   // |S| was staged unscaled
        }
        tc::fence_before_sync();
        __syncthreads();
    }
    if (!failed) {
        tc::fence_after_sync();
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c4 = 0; c4 < DP / 32; c4++) {
            float o[32];
            tc::ld32(tO + lane_off + c4 * 32, o);
            if (row_ok) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int d0 = c4 * 32 + c * 8;
                    if (d0 < D) {
                        uint4 w = make_uint4(tc::pack_bf16(o[c * 8] * inv, o[c * 8 + 1] * inv),
                                             tc::pack_bf16(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv),
                                             tc::pack_bf16(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv),
                                             tc::pack_bf16(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv));
                        *reinterpret_cast<uint4 *>(out + qi * rs + (size_t)h * D + d0) = w;
                    }
                }
            }
        }
        if (row_ok) lse[(size_t)h * s + qi] = (m2 + __log2f(l)) * kLn2;
    } else {
        tc::mbar_wait_bounded(bar, phase, kWaitLimit);   // let this CTA's own MMAs drain
        if (tid == 0) atomicExch(status, 1);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

template <int DP, bool BIAS = false>
int launch_fwd(int64_t s, int heads, int head_dim, float scale, float score_scale, float drop_p, uint32_t seed,
               const void *q, const void *k, const void *v, void *out, float *lse, float *ns, int *status,
               cudaStream_t st, const float *bias = nullptr, int64_t bias_hs = 0) {
    using L = FwdSmem<DP>;
    auto fn = dense_fwd_kernel<DP, BIAS>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes) != cudaSuccess)
        return NGT_ERR_CUDA;
    dim3 grid((unsigned)((s + BM - 1) / BM), (unsigned)heads);
    fn<<<grid, kThreads, L::kBytes, st>>>((int)s, heads, head_dim, scale, score_scale, drop_p, seed,
                                          (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k,
                                          (const __nv_bfloat16 *)v, (__nv_bfloat16 *)out, lse, ns, status, bias,
                                          bias_hs);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_dense_attn_forward(int64_t s, int heads, int head_dim, float scale, float score_scale,
                                      float dropout_p, uint64_t seed, const void *q, const void *k, const void *v,
                                      void *out, float *lse, float *node_scores, int32_t *status,
                                      ngt_stream_t stream) {
    if (s < 0 || heads <= 0 || head_dim <= 0 || !status) return NGT_ERR_INVALID_ARGUMENT;
    if (s > 0 && (!q || !k || !v || !out || !lse || !node_scores)) return NGT_ERR_INVALID_ARGUMENT;
    if (head_dim % 8 != 0 || head_dim > 64) return NGT_ERR_UNSUPPORTED;
    if (!(dropout_p >= 0.f && dropout_p < 1.f) || !(scale > 0.f)) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return NGT_ERR_MISALIGNED;
    if (s * (int64_t)heads * head_dim >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if (s == 0) return NGT_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t sd = (uint32_t)(seed ^ (seed >> 32));
    if (head_dim <= 32)   // warp-specialised TMA kernel
        return dense_fwd_tma(s, heads, head_dim, scale, score_scale, dropout_p, sd, q, k, v, out, lse, node_scores,
                             status, st);
    return launch_fwd<64>(s, heads, head_dim, scale, score_scale, dropout_p, sd, q, k, v, out, lse, node_scores,
                          status, st);
}

// ------------------------------------------------------------------------------------
// Backward.  One CTA per (128-key block, head), looping over 128-query blocks:
//   S^T = K Q^T, dP^T = V dO^T                       (tensor core, fp32 in TMEM)
//   P = exp(scale*S - lse), dP <- dP * dropout mask, dS = P (dP - delta)   (registers)
//   dV += (P*mask)^T dO, dK += dS^T Q, dQ_part = dS K (tensor core; the dS^T tile is read
//   K-major for dK and MN-major for dQ, so no transpose is written)
// dQ partials of every key block are added in fp32 with atomics; the gradients carry the
// forward's scale (d/dq of scale*q k^T).
// ------------------------------------------------------------------------------------
namespace ngt {
namespace {

constexpr uint32_t kBwdTmemCols = 256;   // two CTAs per SM

template <int DP>
struct BwdSmem {
    static constexpr int CH = DP / 8;
    static constexpr uint32_t kK = 0;
    static constexpr uint32_t kV = kK + BN * DP * 2;
    static constexpr uint32_t kQ = kV + BN * DP * 2;
    static constexpr uint32_t kDO = kQ + BM * DP * 2;
    static constexpr uint32_t kPt = kDO + BM * DP * 2;
    static constexpr uint32_t kDSt = kPt + BN * BM * 2;
    static constexpr uint32_t kLse = kDSt + BN * BM * 2;
    static constexpr uint32_t kDelta = kLse + BM * 4;
    static constexpr uint32_t kBar = kDelta + BM * 4;
    static constexpr uint32_t kTmemSlot = kBar + 16;
    static constexpr uint32_t kBytes = kTmemSlot + 16;
};

// Four fp32 additions to consecutive, 16-byte aligned global addresses in one reduction.
__device__ __forceinline__ void red_add_v4(float *p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__device__ __forceinline__ void stage_rows(uint8_t *dst, const __nv_bfloat16 *src, int row0, int s, size_t rs,
                                           int h, int D, int CH, int tid) {
    const int r = row0 + tid;
    for (int c = 0; c < CH; c++) {
        uint4 val = make_uint4(0, 0, 0, 0);
        if (r < s && c * 8 < D) val = *reinterpret_cast<const uint4 *>(src + r * rs + (size_t)h * D + c * 8);
        *reinterpret_cast<uint4 *>(dst + core_off(tid, c, CH)) = val;
    }
}

// BIAS: the forward's additive bias (same layout) is added to the recomputed scores, and the
// gradient of the biased scores, dX = P (dP - delta) (zero at -inf entries), is written to
// dbias [H, s, s] when it is not null.
template <int DP, bool BIAS = false>
__global__ void __launch_bounds__(kThreads, 2)
    dense_bwd_kernel(int s, int H, int D, float scale, float drop_p, uint32_t seed,
                     const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                     const __nv_bfloat16 *__restrict__ v, const __nv_bfloat16 *__restrict__ dout,
                     const float *__restrict__ lse, const float *__restrict__ delta,
                     float *__restrict__ dq_acc, __nv_bfloat16 *__restrict__ dk, __nv_bfloat16 *__restrict__ dv,
                     int *__restrict__ status, const float *__restrict__ bias, int64_t bias_hs,
                     float *__restrict__ dbias) {
    using L = BwdSmem<DP>;
    constexpr int CH = L::CH;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kTmemSlot);
    float *s_lse = reinterpret_cast<float *>(smem + L::kLse);
    float *s_delta = reinterpret_cast<float *>(smem + L::kDelta);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int k0 = blockIdx.x * BN, h = blockIdx.y;
    const size_t rs = (size_t)H * D;

    if (warp == 0) tc::tmem_alloc(tmem_slot, kBwdTmemCols);
    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::mbar_init_fence();
    }
    stage_rows(smem + L::kK, k, k0, s, rs, h, D, CH, tid);
    stage_rows(smem + L::kV, v, k0, s, rs, h, D, CH, tid);
    tc::fence_smem_for_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // TMEM: S and dP of one 64-query half side by side, then the dV and dK accumulators;
    // the dQ partial reuses the S/dP columns once both halves have been read
    constexpr int QH = BM / 2;
    const uint32_t tS = tmem, tDP = tmem + QH, tDV = tmem + 2 * QH, tDK = tmem + 2 * QH + DP, tDQ = tmem;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t aK = tc::smem_addr(smem + L::kK), aV = tc::smem_addr(smem + L::kV),
                   aQ = tc::smem_addr(smem + L::kQ), aDO = tc::smem_addr(smem + L::kDO),
                   aPt = tc::smem_addr(smem + L::kPt), aDSt = tc::smem_addr(smem + L::kDSt);
    constexpr uint32_t idesc_sq = tc::idesc_bf16(BN, QH, false, false);      // [keys x 64 queries], K-major
    constexpr uint32_t idesc_acc = tc::idesc_bf16(BN, DP, false, true);      // [keys x d], B MN-major
    constexpr uint32_t idesc_dq = tc::idesc_bf16(BM, DP, true, true);        // [queries x d], A and B MN-major
    const float sl2 = scale * kLog2e;
    const uint32_t drop_threshold = drop_p > 0.f ? (uint32_t)fminf(drop_p * 4294967296.0f, 4294967295.0f) : 0u;
    const float keep_scale = drop_p > 0.f ? 1.0f / (1.0f - drop_p) : 1.0f;
    const int kj = k0 + tid;
    const bool key_ok = kj < s;

    uint32_t phase = 0;
    int failed = 0;
    const int nqb = (s + BM - 1) / BM;
    // the next query block's rows are fetched into registers while the current one is processed
    uint4 nq[CH], ndo[CH];
    float nlse = INFINITY, ndl = 0.f;
    auto fetch_q = [&](int q0) {
        const int qi = q0 + tid;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            nq[c] = make_uint4(0, 0, 0, 0);
            ndo[c] = make_uint4(0, 0, 0, 0);
            if (qi < s && c * 8 < D) {
                nq[c] = *reinterpret_cast<const uint4 *>(q + qi * rs + (size_t)h * D + c * 8);
                ndo[c] = *reinterpret_cast<const uint4 *>(dout + qi * rs + (size_t)h * D + c * 8);
            }
        }
        nlse = qi < s ? lse[(size_t)h * s + qi] * kLog2e : INFINITY;   // invalid query -> P = 0
        ndl = qi < s ? delta[(size_t)h * s + qi] : 0.f;
    };
    fetch_q(0);
    for (int qb = 0; qb < nqb && !failed; qb++) {
        const int q0 = qb * BM;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            *reinterpret_cast<uint4 *>(smem + L::kQ + core_off(tid, c, CH)) = nq[c];
            *reinterpret_cast<uint4 *>(smem + L::kDO + core_off(tid, c, CH)) = ndo[c];
        }
        s_lse[tid] = nlse;
        s_delta[tid] = ndl;
        tc::fence_smem_for_async();
        tc::fence_before_sync();
        __syncthreads();
        if (qb + 1 < nqb) fetch_q(q0 + BM);
        for (int half = 0; half < 2; half++) {
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t qoff = half * (QH / 8) * CH * 128;   // 8 row groups of 8 queries
#pragma unroll
                for (int kk = 0; kk < DP / 16; kk++) {
                    tc::mma_bf16(tS, tc::smem_desc(aK + kk * 256, 128, CH * 128),
                                 tc::smem_desc(aQ + qoff + kk * 256, 128, CH * 128), idesc_sq, kk > 0);
                    tc::mma_bf16(tDP, tc::smem_desc(aV + kk * 256, 128, CH * 128),
                                 tc::smem_desc(aDO + qoff + kk * 256, 128, CH * 128), idesc_sq, kk > 0);
                }
                tc::commit(bar);
            }
            if (tc::mbar_wait_bounded(bar, phase, kWaitLimit)) phase ^= 1;
            else failed = 1;
            failed = __syncthreads_or(failed);
        if (failed) break;
            tc::fence_after_sync();
#pragma unroll 1
            for (int c4 = 0; c4 < QH / 32; c4++) {
                float sv[32], dp[32];
                tc::ld32(tS + lane_off + c4 * 32, sv);
                tc::ld32(tDP + lane_off + c4 * 32, dp);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint32_t pw[4], dw[4];
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        float pv[2], dv2[2];
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const int j = c * 8 + e + u;                   // query within the 32-chunk
                            const int qq = half * QH + c4 * 32 + j;        // query within the block
                            float p;
                            if constexpr (BIAS) {
                                const int qg = q0 + qq;
                                const float l2 = s_lse[qq];
                                const float x2 = key_ok && qg < s
                                                     ? fmaf(sv[j], sl2, bias[(size_t)h * bias_hs + (size_t)qg * s + kj] * kLog2e)
                                                     : -INFINITY;
                                p = (x2 == -INFINITY || l2 == -INFINITY) ? 0.f : tc::ex2(x2 - l2);
                            } else {
                                p = key_ok ? tc::ex2(fmaf(sv[j], sl2, -s_lse[qq])) : 0.f;
                            }
                            float g = dp[j];
                            float pd = p;
                            if (drop_threshold) {
                                const bool keep = keep_elem(seed, h, q0 + qq, kj, drop_threshold);
                                pd = keep ? p * keep_scale : 0.f;
                                g = keep ? g * keep_scale : 0.f;
                            }
                            pv[u] = pd;
                            dv2[u] = p * (g - s_delta[qq]);
                            if (BIAS && dbias != nullptr && key_ok && q0 + qq < s)
                                dbias[(size_t)h * s * s + (size_t)(q0 + qq) * s + kj] = dv2[u];
                        }
                        pw[e / 2] = tc::pack_bf16(pv[0], pv[1]);
                        dw[e / 2] = tc::pack_bf16(dv2[0], dv2[1]);
                    }
                    const int chunk = half * (QH / 8) + c4 * 4 + c;
                    *reinterpret_cast<uint4 *>(smem + L::kPt + core_off(tid, chunk, BM / 8)) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
                    *reinterpret_cast<uint4 *>(smem + L::kDSt + core_off(tid, chunk, BM / 8)) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
                }
            }
            tc::fence_before_sync();
            __syncthreads();   // S/dP of this half read by every thread before they are overwritten
        }
        if (failed) break;
        tc::fence_smem_for_async();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < BM / 16; kk++) {
                const uint64_t a_pt = tc::smem_desc(aPt + kk * 256, 128, (BM / 8) * 128);
                const uint64_t a_dst = tc::smem_desc(aDSt + kk * 256, 128, (BM / 8) * 128);
                const uint64_t b_do = tc::smem_desc(aDO + kk * 2 * CH * 128, CH * 128, 128);
                const uint64_t b_q = tc::smem_desc(aQ + kk * 2 * CH * 128, CH * 128, 128);
                tc::mma_bf16(tDV, a_pt, b_do, idesc_acc, (qb > 0 || kk > 0));
                tc::mma_bf16(tDK, a_dst, b_q, idesc_acc, (qb > 0 || kk > 0));
            }
#pragma unroll
            for (int kk = 0; kk < BN / 16; kk++)   // dQ_part = dS K: dS^T read MN-major, K read MN-major
                tc::mma_bf16(tDQ, tc::smem_desc(aDSt + kk * 2 * (BM / 8) * 128, (BM / 8) * 128, 128),
                             tc::smem_desc(aK + kk * 2 * CH * 128, CH * 128, 128), idesc_dq, kk > 0);
            tc::commit(bar);
        }
        if (tc::mbar_wait_bounded(bar, phase, kWaitLimit)) phase ^= 1;
        else failed = 1;
        failed = __syncthreads_or(failed);
        if (failed) break;
        tc::fence_after_sync();
        {   // this thread's lane is query q0 + tid for the dQ partial
            const int qi = q0 + tid;
#pragma unroll
            for (int c4 = 0; c4 < DP / 32; c4++) {
                float g[32];
                tc::ld32(tDQ + lane_off + c4 * 32, g);
                if (qi < s) {   // dq_acc rows are 16-byte aligned: D % 8 == 0 and fp32
                    float *dst = dq_acc + qi * rs + (size_t)h * D + c4 * 32;
#pragma unroll
                    for (int d = 0; d < 32; d += 4)
                        if (c4 * 32 + d < D)
                            red_add_v4(dst + d, g[d] * scale, g[d + 1] * scale, g[d + 2] * scale, g[d + 3] * scale);
                }
            }
        }
        tc::fence_before_sync();
        __syncthreads();
    }
    if (!failed) {
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < DP / 32; c4++) {
            float gv[32], gk[32];
            tc::ld32(tDV + lane_off + c4 * 32, gv);
            tc::ld32(tDK + lane_off + c4 * 32, gk);
            if (key_ok) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int d0 = c4 * 32 + c * 8;
                    if (d0 < D) {
                        uint4 wv = make_uint4(tc::pack_bf16(gv[c * 8], gv[c * 8 + 1]), tc::pack_bf16(gv[c * 8 + 2], gv[c * 8 + 3]),
                                              tc::pack_bf16(gv[c * 8 + 4], gv[c * 8 + 5]), tc::pack_bf16(gv[c * 8 + 6], gv[c * 8 + 7]));
                        uint4 wk = make_uint4(tc::pack_bf16(gk[c * 8] * scale, gk[c * 8 + 1] * scale),
                                              tc::pack_bf16(gk[c * 8 + 2] * scale, gk[c * 8 + 3] * scale),
                                              tc::pack_bf16(gk[c * 8 + 4] * scale, gk[c * 8 + 5] * scale),
                                              tc::pack_bf16(gk[c * 8 + 6] * scale, gk[c * 8 + 7] * scale));
                        *reinterpret_cast<uint4 *>(dv + kj * rs + (size_t)h * D + d0) = wv;
                        *reinterpret_cast<uint4 *>(dk + kj * rs + (size_t)h * D + d0) = wk;
                    }
                }
            }
        }
    } else {
        tc::mbar_wait_bounded(bar, phase, kWaitLimit);
        if (tid == 0) atomicExch(status, 1);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kBwdTmemCols);
}

// delta[h, i] = <dout[i, h, :], out[i, h, :]>
__global__ void dense_delta_kernel(int s, int H, int D, const __nv_bfloat16 *__restrict__ out,
                                   const __nv_bfloat16 *__restrict__ dout, float *__restrict__ delta) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)s * H) return;
    const int i = (int)(gid / H), h = (int)(gid % H);
    const size_t base = (size_t)i * H * D + (size_t)h * D;
    float acc = 0.f;
    for (int d = 0; d < D; d++) acc = fmaf(__bfloat162float(out[base + d]), __bfloat162float(dout[base + d]), acc);
    delta[(size_t)h * s + i] = acc;
}

__global__ void dense_dq_cast_kernel(int64_t n, const float *__restrict__ acc, __nv_bfloat16 *__restrict__ dq) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dq[i] = __float2bfloat16_rn(acc[i]);
}

template <int DP>
int launch_bwd(int64_t s, int heads, int head_dim, float scale, float drop_p, uint32_t seed, const void *q,
               const void *k, const void *v, const void *out, const void *dout, const float *lse, float *delta,
               float *dq_acc, void *dq, void *dk, void *dv, int *status, cudaStream_t st) {
    using L = BwdSmem<DP>;
    const int64_t n = s * heads * head_dim;
    cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)n, st);
    dense_delta_kernel<<<(unsigned)((s * heads + 255) / 256), 256, 0, st>>>(
        (int)s, heads, head_dim, (const __nv_bfloat16 *)out, (const __nv_bfloat16 *)dout, delta);
    if constexpr (DP == 32) {   // head_dim <= 32: the warp-specialised TMA kernel
        const int rc = dense_bwd_tma(s, heads, head_dim, scale, drop_p, seed, q, k, v, dout, lse, delta, dq_acc, dk,
                                     dv, status, st);
        if (rc != NGT_OK) return rc;
    } else {
        auto fn = dense_bwd_kernel<DP>;
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes) != cudaSuccess)
            return NGT_ERR_CUDA;
        dim3 grid((unsigned)((s + BN - 1) / BN), (unsigned)heads);
        fn<<<grid, kThreads, L::kBytes, st>>>((int)s, heads, head_dim, scale, drop_p, seed, (const __nv_bfloat16 *)q,
                                              (const __nv_bfloat16 *)k, (const __nv_bfloat16 *)v,
                                              (const __nv_bfloat16 *)dout, lse, delta, dq_acc, (__nv_bfloat16 *)dk,
                                              (__nv_bfloat16 *)dv, status, nullptr, 0, nullptr);
    }
    dense_dq_cast_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(n, dq_acc, (__nv_bfloat16 *)dq);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

}  // namespace
}  // namespace ngt

extern "C" int ngt_dense_attn_backward(int64_t s, int heads, int head_dim, float scale, float dropout_p,
                                       uint64_t seed, const void *q, const void *k, const void *v,
                                       const void *out, const void *dout, const float *lse, float *delta,
                                       float *dq_accum, void *dq, void *dk, void *dv, int32_t *status,
                                       ngt_stream_t stream) {
    if (s < 0 || heads <= 0 || head_dim <= 0 || !status) return NGT_ERR_INVALID_ARGUMENT;
    if (s > 0 && (!q || !k || !v || !out || !dout || !lse || !delta || !dq_accum || !dq || !dk || !dv))
        return NGT_ERR_INVALID_ARGUMENT;
    if (head_dim % 8 != 0 || head_dim > 64) return NGT_ERR_UNSUPPORTED;
    if (!(dropout_p >= 0.f && dropout_p < 1.f)) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dk) || !aligned16(dv)) return NGT_ERR_MISALIGNED;
    if (s * (int64_t)heads * head_dim >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if (s == 0) return NGT_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t sd = (uint32_t)(seed ^ (seed >> 32));
    if (head_dim <= 32)
        return launch_bwd<32>(s, heads, head_dim, scale, dropout_p, sd, q, k, v, out, dout, lse, delta, dq_accum, dq,
                              dk, dv, status, st);
    return launch_bwd<64>(s, heads, head_dim, scale, dropout_p, sd, q, k, v, out, dout, lse, delta, dq_accum, dq, dk,
                          dv, status, st);
}

// ------------------------------------------------------------------------------------
// Dense attention with an additive bias (attn_bias + pruning_mask, masked keys at -inf): the
// single-role kernels above with BIAS set, for any head_dim <= 64 (padded to 32 or 64).
// ------------------------------------------------------------------------------------
namespace ngt {
namespace {

template <int DP>
int launch_bwd_bias(int64_t s, int heads, int head_dim, float scale, float drop_p, uint32_t seed, const void *q,
                    const void *k, const void *v, const void *out, const void *dout, const float *lse,
                    const float *bias, int64_t bias_hs, float *delta, float *dq_acc, void *dq, void *dk, void *dv,
                    float *dbias, int *status, cudaStream_t st) {
    using L = BwdSmem<DP>;
    const int64_t n = s * heads * head_dim;
    if (cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)n, st) != cudaSuccess) return NGT_ERR_CUDA;
    dense_delta_kernel<<<(unsigned)((s * heads + 255) / 256), 256, 0, st>>>(
        (int)s, heads, head_dim, (const __nv_bfloat16 *)out, (const __nv_bfloat16 *)dout, delta);
    auto fn = dense_bwd_kernel<DP, true>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes) != cudaSuccess)
        return NGT_ERR_CUDA;
    dim3 grid((unsigned)((s + BN - 1) / BN), (unsigned)heads);
    fn<<<grid, kThreads, L::kBytes, st>>>((int)s, heads, head_dim, scale, drop_p, seed, (const __nv_bfloat16 *)q,
                                          (const __nv_bfloat16 *)k, (const __nv_bfloat16 *)v,
                                          (const __nv_bfloat16 *)dout, lse, delta, dq_acc, (__nv_bfloat16 *)dk,
                                          (__nv_bfloat16 *)dv, status, bias, bias_hs, dbias);
    dense_dq_cast_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(n, dq_acc, (__nv_bfloat16 *)dq);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

int check_bias_args(int64_t s, int heads, int64_t bias_hs, const float *bias) {
    if (!bias) return NGT_ERR_INVALID_ARGUMENT;
    if (bias_hs != 0 && bias_hs != s * s) return NGT_ERR_INVALID_ARGUMENT;
    if (s * s * (int64_t)heads >= ((int64_t)1 << 40)) return NGT_ERR_TOO_LARGE;
    return NGT_OK;
}

}  // namespace
}  // namespace ngt

extern "C" int ngt_dense_attn_forward_bias(int64_t s, int heads, int head_dim, float scale, float score_scale,
                                           float dropout_p, uint64_t seed, const void *q, const void *k, const void *v,
                                           const float *bias, int64_t bias_head_stride, void *out, float *lse,
                                           float *node_scores, int32_t *status, ngt_stream_t stream) {
    if (s < 0 || heads <= 0 || head_dim <= 0 || !status) return NGT_ERR_INVALID_ARGUMENT;
    if (s > 0 && (!q || !k || !v || !out || !lse || !node_scores)) return NGT_ERR_INVALID_ARGUMENT;
    if (head_dim % 8 != 0 || head_dim > 64) return NGT_ERR_UNSUPPORTED;
    if (!(dropout_p >= 0.f && dropout_p < 1.f) || !(scale > 0.f)) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return NGT_ERR_MISALIGNED;
    if (s * (int64_t)heads * head_dim >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if (s == 0) return NGT_OK;
    int rc = check_bias_args(s, heads, bias_head_stride, bias);
    if (rc != NGT_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t sd = (uint32_t)(seed ^ (seed >> 32));
    if (head_dim <= 32)
        return launch_fwd<32, true>(s, heads, head_dim, scale, score_scale, dropout_p, sd, q, k, v, out, lse,
                                    node_scores, status, st, bias, bias_head_stride);
    return launch_fwd<64, true>(s, heads, head_dim, scale, score_scale, dropout_p, sd, q, k, v, out, lse, node_scores,
                                status, st, bias, bias_head_stride);
}

extern "C" int ngt_dense_attn_backward_bias(int64_t s, int heads, int head_dim, float scale, float dropout_p,
                                            uint64_t seed, const void *q, const void *k, const void *v, const void *out,
                                            const void *dout, const float *lse, const float *bias,
                                            int64_t bias_head_stride, float *delta, float *dq_accum, void *dq, void *dk,
                                            void *dv, float *dbias, int32_t *status, ngt_stream_t stream) {
    if (s < 0 || heads <= 0 || head_dim <= 0 || !status) return NGT_ERR_INVALID_ARGUMENT;
    if (s > 0 && (!q || !k || !v || !out || !dout || !lse || !delta || !dq_accum || !dq || !dk || !dv))
        return NGT_ERR_INVALID_ARGUMENT;
    if (head_dim % 8 != 0 || head_dim > 64) return NGT_ERR_UNSUPPORTED;
    if (!(dropout_p >= 0.f && dropout_p < 1.f)) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dk) || !aligned16(dv)) return NGT_ERR_MISALIGNED;
    if (s * (int64_t)heads * head_dim >= (int64_t)INT32_MAX) return NGT_ERR_TOO_LARGE;
    if (s == 0) return NGT_OK;
    int rc = check_bias_args(s, heads, bias_head_stride, bias);
    if (rc != NGT_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t sd = (uint32_t)(seed ^ (seed >> 32));
    if (head_dim <= 32)
        return launch_bwd_bias<32>(s, heads, head_dim, scale, dropout_p, sd, q, k, v, out, dout, lse, bias,
                                   bias_head_stride, delta, dq_accum, dq, dk, dv, dbias, status, st);
    return launch_bwd_bias<64>(s, heads, head_dim, scale, dropout_p, sd, q, k, v, out, dout, lse, bias,
                               bias_head_stride, delta, dq_accum, dq, dk, dv, dbias, status, st);
}
