// Warp-specialised dense full-attention windows for head_dim <= 32 (TMA + tcgen05 + TMEM).
//
// Same contract as the kernels of dense_attn.cu (which keep head_dim 33..64):
//   forward   S = (q * scale) k^T, P = softmax(S) (+ dropout), X = P v, lse, and the node-score
//             column sums sum_i |S_ij| (times score_scale) added into node_scores;
//   backward  dQ (fp32 partials, added by TMA reduce-add), dK, dV.
// Reference: CoreAttention.full_attention, NeutronGT/models/gt_dist_node_level_single_window.py:56-109.
//
// Q, K, V and dO tiles arrive by cp.async.bulk.tensor from a 4-D tensor map over the [s, H, D]
// bf16 tensor, dims (8 elements, rows, D/8 chunks, heads) and box (8, 128, 4, 1): the box is
// written to shared memory element-fastest, then rows, then chunks, which is exactly the
// no-swizzle core-matrix layout (8 rows x 16 B = 128 contiguous bytes) the tensor core reads.
// TMA zero-fills head_dim 24 -> 32, rows past s and the ragged last block.  One tile can be
// read K-major (rows = M/N, chunks along K) and MN-major (rows along K) without a transpose.
//
// Roles in a CTA of 16 warps:
//   warp 0        producer: TMA loads into a ring of stages, guarded by full/empty mbarriers;
//   warp 1        one thread issues every tcgen05.mma and tcgen05.commit;
//   warps 4..7    softmax warpgroup 0 and warps 8..11 softmax warpgroup 1, each owning one
//                 TMEM accumulator set, so one group's exponentials overlap the other's MMAs;
//   warps 12..15  epilogue: node-score column sums (forward) or dQ reductions (backward).
// Every wait is bounded; a timeout sets a shared abort flag and the device status word, every
// role leaves its loop, the producer waits (bounded) for its own copies in flight, the MMA
// thread for its own MMAs, and the TMEM is freed.
#include <cuda.h>

#include <mutex>

#include "dense_tma.h"
#include "tc.cuh"

namespace ngt {
namespace dtma {
namespace {

constexpr int DP = 32;                                // padded head_dim
constexpr int TILE = 128;                             // rows of a TMA tile / TMEM lanes
constexpr uint32_t kTileBytes = TILE * DP * 2;        // 8 KiB, box (8, 128, 4, 1)
constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr float kLn2 = 0.69314718055994531f;
constexpr float kLog2e = 1.44269504088896341f;

// Descriptors of a TMA-written tile (row r, chunk c at c * 2048 + r * 16).
__device__ __forceinline__ uint64_t kmajor_tma(uint32_t a) { return tc::smem_desc(a, 2048, 128); }
__device__ __forceinline__ uint64_t mnmajor_tma(uint32_t a) { return tc::smem_desc(a, 128, 2048); }
// Thread-written 128 x 128 bf16 tiles: (row r, chunk c) at (r / 8) * 2048 + c * 128 + (r % 8) * 16.
__device__ __forceinline__ uint32_t sq_off(int r, int c) {
    return (uint32_t)((r >> 3) * 2048 + c * 128 + (r & 7) * 16);
}
__device__ __forceinline__ uint64_t kmajor_sq(uint32_t a) { return tc::smem_desc(a, 128, 2048); }
__device__ __forceinline__ uint64_t mnmajor_sq(uint32_t a) { return tc::smem_desc(a, 2048, 128); }

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}
// Dropout keep decision of (head, query, key); identical to dense_attn.cu's.
__device__ __forceinline__ bool keep_elem(uint32_t seed, int h, int i, int j, uint32_t threshold) {
    const uint32_t x = mix32(seed ^ mix32((uint32_t)i * 0x9E3779B1u + (uint32_t)h * 0x85EBCA77u) ^ ((uint32_t)j * 0xC2B2AE3Du));
    return x >= threshold;
}

__device__ __forceinline__ void st16(uint8_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4 *>(p) = make_uint4(a, b, c, d);
}


// Abort flag in shared memory plus the device status word.
struct Abort {
    uint32_t flag;   // shared-memory address
    int *status;
    __device__ void raise() const {
        asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(flag), "r"(1) : "memory");
        atomicExch(status, 1);
    }
    __device__ bool set() const {
        uint32_t v;
        asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(flag) : "memory");
        return v != 0;
    }
};

// try_wait with a suspend-time hint: a waiting warp sleeps instead of taking issue slots from
// the warps that compute, and wakes when the phase completes.
__device__ __forceinline__ bool try_wait_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(tc::smem_addr(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSleepPolls = 1u << 21;   // x <= 1 us each: a bound of ~2 s

// Warp-uniform wait: every lane polls (its own acquire), one vote decides for the warp.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, const Abort &ab) {
    bool ok = false;
    for (uint32_t i = 0; i < kSleepPolls; i++)
        if (try_wait_sleep(bar, parity)) {
            ok = true;
            break;
        }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && (threadIdx.x & 31) == 0) ab.raise();
    return ok;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes' worth of work).
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(f32x2 v, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 ffma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ f32x2 fadd2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 fmul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for x <= 0 on the FMA pipe, for a share of the scores so that the MUFU unit is not the only
// exponential unit: Cody-Waite reduction x = n + r with n = round(x) (added through the 1.5 * 2^23
// shifter), 2^r on [-0.5, 0.5] by a degree-3 polynomial whose coefficients were fitted here
// (relative-error least squares on Chebyshev nodes; max relative error 7.8e-5, below bf16's 2^-9
// rounding of P), and 2^n added into the exponent field.  x is clamped at -126: p(r) has a biased
// exponent of 126 or 127, so n >= -126 keeps the sum a non-negative (possibly subnormal) float.
__device__ __forceinline__ void exp2_poly(float x0, float x1, float &y0, float &y1) {
    const float kShift = 12582912.0f;   // 1.5 * 2^23
    const f32x2 x = pk(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
    const f32x2 t = fadd2(x, pk(kShift, kShift));
    const f32x2 n = fadd2(t, pk(-kShift, -kShift));
    float n0, n1;
    upk(n, n0, n1);
    const f32x2 r = fadd2(x, pk(-n0, -n1));
    f32x2 p = ffma2(pk(0.055088773f, 0.055088773f), r, pk(0.24260406f, 0.24260406f));
    p = ffma2(p, r, pk(0.69327623f, 0.69327623f));
    p = ffma2(p, r, pk(0.99992895f, 0.99992895f));
    float p0, p1, t0, t1;
    upk(p, p0, p1);
    upk(t, t0, t1);
    y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
    y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// 32 scores of one row (all keys real, no dropout): P = 2^(s * scale * log2e - mu) and |s| as bf16
// into the row's next four 16-byte chunks of the P and |S| tiles (chunk stride 128 bytes); one pair
// in four takes the polynomial exp2, the rest the MUFU unit.  |s| is the packed bf16 pair with its
// sign bits cleared (bf16 rounding is symmetric, so |bf16(s)| = bf16(|s|)).
template <bool PT>
__device__ __forceinline__ void chunk_fast(const float (&v)[32], f32x2 sl2x2, f32x2 nmu, f32x2 &l2, uint8_t *prow,
                                           uint8_t *arow, uint32_t (&pt)[16]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t pw[4], aw[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const f32x2 x = ffma2(pk(v[c * 8 + e], v[c * 8 + e + 1]), sl2x2, nmu);
            float x0, x1, p0, p1;
            upk(x, x0, x1);
            if (e == 0) {
                exp2_poly(x0, x1, p0, p1);
            } else {
                p0 = tc::ex2(x0);
                p1 = tc::ex2(x1);
            }
            l2 = fadd2(l2, pk(p0, p1));
            pw[e / 2] = tc::pack_bf16(p0, p1);
            aw[e / 2] = tc::pack_bf16(v[c * 8 + e], v[c * 8 + e + 1]) & 0x7FFF7FFFu;
        }
        if constexpr (PT) {
#pragma unroll
            for (int i = 0; i < 4; i++) pt[c * 4 + i] = pw[i];
        } else {
            st16(prow + c * 128, pw[0], pw[1], pw[2], pw[3]);
        }
        st16(arow + c * 128, aw[0], aw[1], aw[2], aw[3]);
    }
}

// ------------------------------------------------------------------------------------
// Forward: one CTA = one head x two 128-query tiles; tile t has its own softmax warpgroup and
// its own MMA-issuing warp, so the two tiles never wait for each other.  Keys stream in 64-key
// sub-blocks j (TMA stages hold 128-key blocks kb = j / 2):
//   S_t(j) = Q_t K_j^T into TMEM buffer j % 2 of tile t (double-buffered: the tensor core
//   computes S_t(j + 2) while the warpgroup exponentiates S_t(j + 1));
//   P_t(j) (bf16) and |S_t(j)| into shared memory; O_t += P_t(j) V_j in TMEM;
//   per 128-key block, C_t = |S_t|^T ones (two buffers per tile) gives the node-score column
//   sums, which the epilogue warps add over both tiles.
// The running max is raised only when a row's max grows by more than 2^8 (P <= 256 in between,
// exact after the final 1 / l), so O is rarely rescaled.
// ------------------------------------------------------------------------------------
template <bool PT>
struct FwdL {
    static constexpr int NKV = PT ? 3 : 2;                // K/V stages (128-key blocks)
    static constexpr int SUB = 64;                        // keys per sub-block
    static constexpr uint32_t kQ = 0;                     // 2 query tiles
    static constexpr uint32_t kKV = kQ + 2 * kTileBytes;  // NKV x {K, V}
    static constexpr uint32_t kP = kKV + NKV * 2 * kTileBytes;   // 2 tiles x P [128 q x 64 keys] bf16
    static constexpr uint32_t kPBytes = TILE * SUB * 2;
    static constexpr uint32_t kAbs = kP + (PT ? 0 : 2 * kPBytes);   // 2 tiles x 2 blocks x |S| [128 q x 128 keys]
    static constexpr uint32_t kAbsBytes = TILE * TILE * 2;
    static constexpr uint32_t kOnes = kAbs + 4 * kAbsBytes;      // 16 x 128 ones
    static constexpr int kOnesRows = 16;
    static constexpr uint32_t kBars = kOnes + kOnesRows * TILE * 2;
    enum {
        QF = 0,
        KVF = 1,
        KVE = KVF + NKV,   // count 2: both tiles' MMAs that read the stage issued
        SF = KVE + NKV,    // [tile][buffer] S_t in TMEM buffer
        PF = SF + 4,       // [tile] S buffer read, P and |S| staged, O rescaled
        OV = PF + 2,       // [tile] O_t += P_t V done
        CF = OV + 2,       // [tile][block parity] column sums in TMEM
        CE = CF + 4,       // [block parity] column sums of both tiles read
        OF = CE + 2,       // [tile] all MMAs of the tile done
        NB = OF + 2
    };
    static constexpr uint32_t kSlot = kBars + NB * 8;
    static constexpr uint32_t kAbort = kSlot + 4;
    static constexpr uint32_t kBytes = kAbort + 4;
};
static_assert(FwdL<false>::kKV % 1024 == 0 && FwdL<false>::kP % 1024 == 0 && FwdL<false>::kAbs % 1024 == 0,
              "1 KiB alignment");
static_assert(FwdL<true>::kAbs % 1024 == 0 && FwdL<true>::kOnes % 1024 == 0, "1 KiB alignment");
static_assert(FwdL<false>::kBytes <= 232448 && FwdL<true>::kBytes <= 232448, "shared memory");

// (row r, 16-byte chunk c) of a [128 x 64] bf16 tile: 8 chunks per row
__device__ __forceinline__ uint32_t sub_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + c * 128 + (r & 7) * 16);
}

// PT: P_t(j) goes back into tensor memory over the 32 first columns of its S buffer (bf16 pairs)
// and O_t += P_t V reads it from there as the A operand, so a warpgroup writes P_t(j) as soon as
// S_t(j) is in (the MMAs of buffer j % 2 run in issue order: S(j) completing means PV(j - 2),
// the last reader of that buffer, and the column sums of block kb - 2 have completed), and waits
// for O_t += P_t(j - 1) V only before it may rescale O_t.  Without PT, P_t is staged in shared memory.
template <bool PT>
__global__ void __launch_bounds__(kThreads, 1)
    dense_fwd_tma_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, int s, int H, int D, float scale,
                         float score_scale, float drop_p, uint32_t seed, __nv_bfloat16 *__restrict__ out,
                         float *__restrict__ lse, float *__restrict__ node_scores, int *__restrict__ status) {
    using L = FwdL<PT>;
    constexpr int SUB = L::SUB;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBars);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kSlot);
    const Abort ab{tc::smem_addr(smem + L::kAbort), status};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * 2 * TILE, h = blockIdx.y;
    const int nkb = (s + TILE - 1) / TILE;
    const int nsb = (s + SUB - 1) / SUB;
    const bool two_tiles = q0 + TILE < s;

    if (warp == 0) tc::tmem_alloc(tmem_slot, kTmemCols);
    if (tid == 32) {
        tc::mbar_init(&bars[L::QF], 2);
        for (int i = 0; i < L::NKV; i++) {
            tc::mbar_init(&bars[L::KVF + i], 1);
            tc::mbar_init(&bars[L::KVE + i], 2);
        }
        for (int i = 0; i < 4; i++) {
            tc::mbar_init(&bars[L::SF + i], 1);
            tc::mbar_init(&bars[L::CF + i], 1);
        }
        for (int t = 0; t < 2; t++) {
            tc::mbar_init(&bars[L::PF + t], 4);
            tc::mbar_init(&bars[L::OV + t], 1);
            tc::mbar_init(&bars[L::CE + t], 4);
            tc::mbar_init(&bars[L::OF + t], 1);
        }
        *reinterpret_cast<volatile int *>(smem + L::kAbort) = 0;
        tc::mbar_init_fence();
    }
    if (tid >= 64 && tid < 64 + L::kOnesRows) {   // the all-ones operand of the column sums
        const uint4 ones = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
        const int r = tid - 64;
#pragma unroll
        for (int c = 0; c < TILE / 8; c++) *reinterpret_cast<uint4 *>(smem + L::kOnes + sq_off(r, c)) = ones;
        tc::fence_smem_for_async();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns: S_t buffer u at t * 128 + u * 64, O_t at 256 + t * 32, C_{t,c} at 320 + (2t + c) * 16
    const uint32_t tO0 = tmem + 256, tC0 = tmem + 320;

    if (warp == 0) {
        // ---------------- producer ----------------
        int issued = 0;
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(&bars[L::QF], (two_tiles ? 2 : 1) * kTileBytes);
            tc::tma_load_4d(smem + L::kQ, &tm_q, 0, q0, 0, h, &bars[L::QF]);
            if (two_tiles) tc::tma_load_4d(smem + L::kQ + kTileBytes, &tm_q, 0, q0 + TILE, 0, h, &bars[L::QF]);
        }
        if (!two_tiles) {   // the second tile lies wholly past s: zeros, written here
            for (int i = lane; i < (int)(kTileBytes / 16); i += 32)
                *reinterpret_cast<uint4 *>(smem + L::kQ + kTileBytes + i * 16) = make_uint4(0, 0, 0, 0);
            tc::fence_smem_for_async();
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[L::QF]);
        for (int kb = 0; kb < nkb; kb++) {
            if (ab.set()) break;
            const int st = kb % L::NKV;
            if (!warp_wait(&bars[L::KVE + st], ((kb / L::NKV) & 1) ^ 1, ab)) break;
            if (lane == 0) {
                uint8_t *dst = smem + L::kKV + st * 2 * kTileBytes;
                tc::mbar_arrive_expect_tx(&bars[L::KVF + st], 2 * kTileBytes);
                tc::tma_load_4d(dst, &tm_k, 0, kb * TILE, 0, h, &bars[L::KVF + st]);
                tc::tma_load_4d(dst + kTileBytes, &tm_v, 0, kb * TILE, 0, h, &bars[L::KVF + st]);
            }
            issued = kb + 1;
        }
        if (lane == 0) {   // every copy this warp started has landed before the CTA can exit
            tc::mbar_wait_bounded(&bars[L::QF], 0, kWaitLimit);
            for (int kb = issued - L::NKV < 0 ? 0 : issued - L::NKV; kb < issued; kb++)
                tc::mbar_wait_bounded(&bars[L::KVF + kb % L::NKV], (kb / L::NKV) & 1, kWaitLimit);
        }
    } else if (warp == 1 || warp == 2) {
        // ---------------- MMA issuer of tile t (the warp waits, lane 0 issues) ----------------
        const int t = warp - 1;
        constexpr uint32_t idesc_s = tc::idesc_bf16(TILE, SUB, false, false);
        constexpr uint32_t idesc_pv = tc::idesc_bf16(TILE, DP, false, true);
        constexpr uint32_t idesc_c = tc::idesc_bf16(TILE, L::kOnesRows, true, false);
        const uint32_t aq = tc::smem_addr(smem + L::kQ) + t * kTileBytes, aKV = tc::smem_addr(smem + L::kKV),
                       ap = tc::smem_addr(smem + L::kP) + t * L::kPBytes,
                       aAbs = tc::smem_addr(smem + L::kAbs) + t * 2 * L::kAbsBytes,
                       aOnes = tc::smem_addr(smem + L::kOnes);
        const uint32_t tS = tmem + t * TILE, tO = tO0 + t * DP;
        const bool leader = lane == 0;
        auto issue_s = [&](int j) {   // S_t(j) = Q_t K_j^T into buffer j % 2
            if (leader) {
                const int u = j & 1;
                const uint32_t aK = aKV + ((j >> 1) % L::NKV) * 2 * kTileBytes + u * SUB * 16;
#pragma unroll
                for (int kk = 0; kk < DP / 16; kk++)
                    tc::mma_bf16(tS + u * SUB, kmajor_tma(aq + kk * 4096), kmajor_tma(aK + kk * 4096), idesc_s, kk > 0);
                tc::commit(&bars[L::SF + t * 2 + u]);
            }
            __syncwarp();
        };
        bool ok = warp_wait(&bars[L::QF], 0, ab) && warp_wait(&bars[L::KVF], 0, ab);
        if (ok) {
            tc::fence_after_sync();
            issue_s(0);
            if (nsb > 1) issue_s(1);
        }
        for (int j = 0; ok && j < nsb; j++) {
            const int kb = j >> 1, u = j & 1, st = kb % L::NKV;
            const uint32_t aV = aKV + st * 2 * kTileBytes + kTileBytes;
            const bool next_s = j + 2 < nsb, last_of_block = u == 1 || j == nsb - 1;
            if (!(ok = warp_wait(&bars[L::PF + t], j & 1, ab))) break;
            tc::fence_after_sync();
            if (leader) {   // first what the warpgroup waits for, then what is needed later
#pragma unroll
                for (int kk = 0; kk < SUB / 16; kk++) {   // O_t += P_t V_j   (V read MN-major)
                    if constexpr (PT)
                        tc::mma_bf16_ts(tO, tS + u * SUB + kk * 8, mnmajor_tma(aV + (u * SUB + kk * 16) * 16), idesc_pv,
                                        (j > 0 || kk > 0));
                    else
                        tc::mma_bf16(tO, tc::smem_desc(ap + kk * 256, 128, 1024),
                                     mnmajor_tma(aV + (u * SUB + kk * 16) * 16), idesc_pv, (j > 0 || kk > 0));
                }
                tc::commit(&bars[L::OV + t]);
                if (last_of_block) tc::commit(&bars[L::KVE + st]);   // every MMA reading this stage issued
            }
            __syncwarp();
            if (last_of_block) {   // column sums of block kb
                const int cb = kb & 1;
                if (!(ok = warp_wait(&bars[L::CE + cb], ((kb >> 1) & 1) ^ 1, ab))) break;
                tc::fence_after_sync();
                if (leader) {
                    const uint32_t aa = aAbs + cb * L::kAbsBytes;
#pragma unroll
                    for (int kk = 0; kk < TILE / 16; kk++)   // C_t = |S_t|^T ones  (|S_t| read MN-major)
                        tc::mma_bf16(tC0 + (t * 2 + cb) * L::kOnesRows, mnmajor_sq(aa + kk * 4096),
                                     kmajor_sq(aOnes + kk * 256), idesc_c, kk > 0);
                    tc::commit(&bars[L::CF + t * 2 + cb]);
                }
                __syncwarp();
            }
            if (next_s) {
                if (u == 0 && !(ok = warp_wait(&bars[L::KVF + (kb + 1) % L::NKV], ((kb + 1) / L::NKV) & 1, ab)))
                    break;   // S(j + 2) reads the next block's K
                tc::fence_after_sync();
                issue_s(j + 2);
            }
        }
        if (leader) {
            tc::commit(&bars[L::OF + t]);
            tc::mbar_wait_bounded(&bars[L::OF + t], 0, kWaitLimit);   // own MMAs drained
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 12) {
        // ---------------- softmax warpgroups: tile t, query row r ----------------
        const int t = (warp - 4) >> 2, r = tid & 127;
        const int qi = q0 + t * TILE + r;
        const bool row_ok = qi < s;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tO = tO0 + t * DP;
        uint8_t *pt = smem + L::kP + t * L::kPBytes;
        uint8_t *at0 = smem + L::kAbs + t * 2 * L::kAbsBytes;
        const float sl2 = scale * kLog2e;
        const uint32_t thr = drop_p > 0.f ? (uint32_t)fminf(drop_p * 4294967296.0f, 4294967295.0f) : 0u;
        const float keep_scale = drop_p > 0.f ? 1.0f / (1.0f - drop_p) : 1.0f;
        const f32x2 sl2x2 = pk(sl2, sl2);
        float mu = -INFINITY;   // max used for the exponentials (log2 units)
        f32x2 l2 = pk(0.f, 0.f);
        bool ok = true;
        for (int j = 0; j < nsb; j++) {
            const int kb = j >> 1, u = j & 1, k0 = j * SUB;
            const uint32_t tS = tmem + t * TILE + u * SUB + lane_off;
            uint8_t *at = at0 + (kb & 1) * L::kAbsBytes;
            if (ab.set() || !warp_wait(&bars[L::SF + t * 2 + u], kb & 1, ab)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const bool full = k0 + SUB <= s;
            float mraw = -INFINITY;
            if (full) {
                static_assert(SUB == 64, "one paired load covers the sub-block");
                float v[32], w[32];
                tc::ld32_pair(tS, v, tS + 32, w);
                float a = max3(v[0], v[1], v[2]), b = max3(v[3], v[4], v[5]), c = max3(w[0], w[1], w[2]),
                      d = max3(w[3], w[4], w[5]);
#pragma unroll
                for (int i = 6; i < 30; i += 4) {
                    a = max3(a, v[i], v[i + 1]);
                    b = max3(b, v[i + 2], v[i + 3]);
                    c = max3(c, w[i], w[i + 1]);
                    d = max3(d, w[i + 2], w[i + 3]);
                }
                a = max3(a, v[30], v[31]);
                c = max3(c, w[30], w[31]);
                mraw = max3(max3(a, b, c), d, mraw);
            } else {
#pragma unroll 1
                for (int c4 = 0; c4 < SUB / 32; c4++) {
                    float v[32];
                    tc::ld32(tS + c4 * 32, v);
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (k0 + c4 * 32 + i < s) mraw = fmaxf(mraw, v[i]);
                }
            }
            // raise the running max only when it grows by more than 2^8
            const float mcand = mraw * sl2;
            float alpha = 1.f;
            if (mcand > mu + 8.f) {
                alpha = (mu == -INFINITY) ? 0.f : tc::ex2(mu - mcand);
                mu = mcand;
                l2 = fmul2(l2, pk(alpha, alpha));
            }
            // O_t += P_t(j - 1) V done: P_t free, O_t current, and (issued before it) the column sums
            // of block kb - 2, the last reader of this |S| buffer (with PT, S_t(j) completing covers
            // both buffers, and this wait moves below, before the rescale of O_t)
            if constexpr (!PT) {
                if (j > 0 && !warp_wait(&bars[L::OV + t], (j - 1) & 1, ab)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
            }
            const f32x2 nmu = pk(-mu, -mu);
            uint32_t pwords[16];   // with PT: 32 P values of this row as bf16 pairs, for TMEM
            if (full && !thr) {   // every key real, no dropout: the common case
#pragma unroll 1
                for (int c4 = 0; c4 < SUB / 32; c4++) {
                    float v[32];
                    tc::ld32(tS + c4 * 32, v);
                    chunk_fast<PT>(v, sl2x2, nmu, l2, pt + sub_off(r, c4 * 4), at + sq_off(r, u * (SUB / 8) + c4 * 4),
                                   pwords);
                    if constexpr (PT) tc::st16_nowait(tS + c4 * 16, pwords);   // S columns already read
                }
            } else {
#pragma unroll 1
                for (int c4 = 0; c4 < SUB / 32; c4++) {
                    float v[32];
                    tc::ld32(tS + c4 * 32, v);
                    float lsum = 0.f;
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t pw[4], aw[4];
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            float pv[2], av[2];
#pragma unroll
                            for (int w = 0; w < 2; w++) {
                                const int key = k0 + c4 * 32 + c * 8 + e + w;
                                const bool kok = key < s;
                                const float p = kok ? tc::ex2(fmaf(v[c * 8 + e + w], sl2, -mu)) : 0.f;
                                lsum += p;
                                pv[w] = (thr && !keep_elem(seed, h, qi, key, thr)) ? 0.f : p * keep_scale;
                                av[w] = kok ? v[c * 8 + e + w] : 0.f;
                            }
                            pw[e / 2] = tc::pack_bf16(pv[0], pv[1]);
                            aw[e / 2] = tc::pack_bf16(av[0], av[1]) & 0x7FFF7FFFu;
                        }
                        if constexpr (PT) {
#pragma unroll
                            for (int i = 0; i < 4; i++) pwords[c * 4 + i] = pw[i];
                        } else {
                            st16(pt + sub_off(r, c4 * 4 + c), pw[0], pw[1], pw[2], pw[3]);
                        }
                        st16(at + sq_off(r, u * (SUB / 8) + c4 * 4 + c), aw[0], aw[1], aw[2], aw[3]);
                    }
                    if constexpr (PT) tc::st16_nowait(tS + c4 * 16, pwords);
                    l2 = fadd2(l2, pk(lsum, 0.f));
                }
            }
            if constexpr (PT) {
                tc::wait_st();   // P_t(j) is in TMEM
                if (j > 0 && !warp_wait(&bars[L::OV + t], (j - 1) & 1, ab)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
            }
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {   // O_t *= 2^(mu_old - mu_new)
                float o[32];
                tc::ld32(tO + lane_off, o);
#pragma unroll
                for (int i = 0; i < 32; i++) o[i] *= alpha;
                tc::st32(tO + lane_off, o);
            }
            tc::fence_smem_for_async();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[L::PF + t]);
        }
        if (ok && warp_wait(&bars[L::OF + t], 0, ab) && !ab.set()) {
            tc::fence_after_sync();
            float o[32];
            tc::ld32(tO + lane_off, o);
            float l0, l1;
            upk(l2, l0, l1);
            const float l = l0 + l1;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            if (row_ok) {
                __nv_bfloat16 *dst = out + (size_t)qi * H * D + (size_t)h * D;
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (c * 8 < D)
                        st16(reinterpret_cast<uint8_t *>(dst + c * 8), tc::pack_bf16(o[c * 8] * inv, o[c * 8 + 1] * inv),
                             tc::pack_bf16(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv),
                             tc::pack_bf16(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv),
                             tc::pack_bf16(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv));
                lse[(size_t)h * s + qi] = (mu + __log2f(l)) * kLn2;
            }
        }
    } else if (warp >= 12) {
        // ---------------- column sums of both tiles -> node scores (lane = key) ----------------
        const int r = tid & 127;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const float col_scale = scale * score_scale;
        for (int kb = 0; kb < nkb; kb++) {
            const int cb = kb & 1;
            if (ab.set() || !warp_wait(&bars[L::CF + cb], (kb >> 1) & 1, ab) ||
                !warp_wait(&bars[L::CF + 2 + cb], (kb >> 1) & 1, ab))
                break;
            tc::fence_after_sync();
            const float c = tc::ld1(tC0 + cb * L::kOnesRows + lane_off) + tc::ld1(tC0 + (2 + cb) * L::kOnesRows + lane_off);
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[L::CE + cb]);
            const int key = kb * TILE + r;
            if (key < s) atomicAdd(node_scores + key, c * col_scale);   // |S| was staged unscaled
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------------------
// Backward: one CTA = one head x one 128-key tile; loops over 128-query blocks qb.  Lanes are
// queries (so lse and delta are per-thread constants), the key tile is split in two 64-key
// halves, each with its own softmax warpgroup and its own S / dP MMA warp; a third MMA warp
// accumulates once both halves of a query block are staged:
//   S_b = Q K_b^T, dP_b = dO V_b^T                    (TMEM, lanes = queries)
//   P = 2^(S * scale * log2e - lse * log2e), dS = P (dP - delta)   (registers -> shared memory)
//   dV += P^T dO, dK += dS^T Q   (P, dS read MN-major: lanes = keys)
//   dQ(qb) = dS K                 (TMEM, two buffers) -> shared memory -> one TMA reduce-add of
//                                 the [128 x D] fp32 partial into dq_acc per query block
// ------------------------------------------------------------------------------------
struct BwdL {
    static constexpr int NST = 3;   // Q / dO / lse / delta stages
    static constexpr uint32_t kK = 0;
    static constexpr uint32_t kV = kK + kTileBytes;
    static constexpr uint32_t kStage = kV + kTileBytes;
    static constexpr uint32_t kStageBytes = 2 * kTileBytes + 2 * TILE * 4;   // Q, dO, -lse*log2e, -delta
    static constexpr uint32_t kPS = kStage + NST * kStageBytes;              // 2 x {P, dS} [128 q x 128 keys]
    static constexpr uint32_t kPSBytes = 2 * TILE * TILE * 2;
    static constexpr uint32_t kDQS = kPS + 2 * kPSBytes;                     // dQ partial [128 q x D] fp32
    static constexpr uint32_t kDQSBytes = TILE * DP * 4;
    static constexpr uint32_t kBars = kDQS + kDQSBytes;
    enum {
        KVF = 0,
        QF = 1,
        QE = QF + NST,   // count 11: three MMA warps' commits + the 8 softmax warps
        SF = QE + NST,   // [half] S_b, dP_b in TMEM
        SR = SF + 2,     // [half] S_b, dP_b read from TMEM (the buffer may be overwritten)
        DS = SR + 2,     // [parity] P / dS of both halves staged (count 8)
        PE = DS + 2,     // [parity] P / dS buffer read by the accumulating MMAs
        DQF = PE + 2,    // [parity] dQ partial in TMEM
        DQE = DQF + 2,   // [parity] dQ partial read
        ACC = DQE + 2,   // [3] each MMA warp's MMAs done
        NB = ACC + 3
    };
    static constexpr uint32_t kSlot = kBars + NB * 8;
    static constexpr uint32_t kAbort = kSlot + 4;
    static constexpr uint32_t kBytes = kAbort + 4;
};
static_assert(BwdL::kStage % 1024 == 0 && BwdL::kStageBytes % 1024 == 0 && BwdL::kPS % 1024 == 0,
              "TMA destinations 1 KiB aligned");
static_assert(BwdL::kBytes <= 232448, "shared memory");

// 32 keys of one query row (no dropout): P = 2^(s * sl2 + nl), dS = P (dp + nd) with the row's
// nl = -lse * log2e and nd = -delta; P and dS as bf16 into the row's next four 16-byte chunks
// (chunk stride 128 bytes).  One pair in four takes the polynomial exp2.
__device__ __forceinline__ void bwd_chunk_fast(const float (&sv)[32], const float (&dp)[32], f32x2 sl2x2, f32x2 nl2,
                                               f32x2 nd2, uint8_t *prow, uint8_t *drow) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t pw[4], dw[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const f32x2 x = ffma2(pk(sv[c * 8 + e], sv[c * 8 + e + 1]), sl2x2, nl2);
            float x0, x1, p0, p1;
            upk(x, x0, x1);
            if (e == 0) {
                exp2_poly(x0, x1, p0, p1);
            } else {
                p0 = tc::ex2(x0);
                p1 = tc::ex2(x1);
            }
            const f32x2 ds = fmul2(pk(p0, p1), fadd2(pk(dp[c * 8 + e], dp[c * 8 + e + 1]), nd2));
            float d0, d1;
            upk(ds, d0, d1);
            pw[e / 2] = tc::pack_bf16(p0, p1);
            dw[e / 2] = tc::pack_bf16(d0, d1);
        }
        st16(prow + c * 128, pw[0], pw[1], pw[2], pw[3]);
        st16(drow + c * 128, dw[0], dw[1], dw[2], dw[3]);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    dense_bwd_tma_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                         const __grid_constant__ CUtensorMap tm_dq, int s,
                         int H, int D, float scale, float drop_p, uint32_t seed, const float *__restrict__ lse,
                         const float *__restrict__ delta, float *__restrict__ dq_acc, __nv_bfloat16 *__restrict__ dk,
                         __nv_bfloat16 *__restrict__ dv, int *__restrict__ status) {
    using L = BwdL;
    constexpr int NST = L::NST;
    constexpr int KH = TILE / 2;   // keys per half
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBars);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kSlot);
    const Abort ab{tc::smem_addr(smem + L::kAbort), status};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = blockIdx.x * TILE, h = blockIdx.y;
    const int nqb = (s + TILE - 1) / TILE;

    if (warp == 0) tc::tmem_alloc(tmem_slot, kTmemCols);
    if (tid == 32) {
        tc::mbar_init(&bars[L::KVF], 1);
        for (int i = 0; i < NST; i++) {
            tc::mbar_init(&bars[L::QF + i], 2);
            tc::mbar_init(&bars[L::QE + i], 3 + 8);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&bars[L::SF + b], 1);
            tc::mbar_init(&bars[L::SR + b], 4);
            tc::mbar_init(&bars[L::DS + b], 8);
            tc::mbar_init(&bars[L::PE + b], 1);
            tc::mbar_init(&bars[L::DQF + b], 1);
            tc::mbar_init(&bars[L::DQE + b], 4);
        }
        for (int i = 0; i < 3; i++) tc::mbar_init(&bars[L::ACC + i], 1);
        *reinterpret_cast<volatile int *>(smem + L::kAbort) = 0;
        tc::mbar_init_fence();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns: S_b at b * 128, dP_b at b * 128 + 64 (lanes = queries); dV at 256, dK at 288
    // (lanes = keys); dQ_c at 320 + c * 32 (lanes = queries)
    const uint32_t tDV = tmem + 256, tDK = tmem + 256 + DP, tDQ0 = tmem + 256 + 2 * DP;

    if (warp == 0) {
        // ---------------- producer ----------------
        int issued = 0;
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(&bars[L::KVF], 2 * kTileBytes);
            tc::tma_load_4d(smem + L::kK, &tm_k, 0, k0, 0, h, &bars[L::KVF]);
            tc::tma_load_4d(smem + L::kV, &tm_v, 0, k0, 0, h, &bars[L::KVF]);
        }
        // lse and delta of a query block are read one block ahead, so their global-load latency
        // overlaps the wait for a free stage; rows past s get P = 0
        float nl4[TILE / 32], nd4[TILE / 32];
        auto load_rows = [&](int q0) {
#pragma unroll
            for (int k = 0; k < TILE / 32; k++) {
                const int qi = q0 + lane + 32 * k;
                nl4[k] = qi < s ? -lse[(size_t)h * s + qi] * kLog2e : -INFINITY;
                nd4[k] = qi < s ? -delta[(size_t)h * s + qi] : 0.f;
            }
        };
        load_rows(0);
        for (int qb = 0; qb < nqb; qb++) {
            if (ab.set()) break;
            const int st = qb % NST, q0 = qb * TILE;
            if (!warp_wait(&bars[L::QE + st], ((qb / NST) & 1) ^ 1, ab)) break;
            uint8_t *sb = smem + L::kStage + st * L::kStageBytes;
            if (lane == 0) {
                tc::mbar_arrive_expect_tx(&bars[L::QF + st], 2 * kTileBytes);
                tc::tma_load_4d(sb, &tm_q, 0, q0, 0, h, &bars[L::QF + st]);
                tc::tma_load_4d(sb + kTileBytes, &tm_do, 0, q0, 0, h, &bars[L::QF + st]);
            }
            float *nl = reinterpret_cast<float *>(sb + 2 * kTileBytes), *nd = nl + TILE;
#pragma unroll
            for (int k = 0; k < TILE / 32; k++) {
                nl[lane + 32 * k] = nl4[k];
                nd[lane + 32 * k] = nd4[k];
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[L::QF + st]);
            issued = qb + 1;
            if (qb + 1 < nqb) load_rows(q0 + TILE);
        }
        if (lane == 0) {
            tc::mbar_wait_bounded(&bars[L::KVF], 0, kWaitLimit);
            for (int qb = issued - NST < 0 ? 0 : issued - NST; qb < issued; qb++)
                tc::mbar_wait_bounded(&bars[L::QF + qb % NST], (qb / NST) & 1, kWaitLimit);
        }
    } else if (warp == 1 || warp == 2) {
        // ---------------- S / dP MMA warp of key half b ----------------
        const int b = warp - 1;
        constexpr uint32_t idesc_s = tc::idesc_bf16(TILE, KH, false, false);   // [queries x 64 keys]
        const uint32_t aK = tc::smem_addr(smem + L::kK) + b * KH * 16, aV = tc::smem_addr(smem + L::kV) + b * KH * 16,
                       aSt = tc::smem_addr(smem + L::kStage);
        const uint32_t tS = tmem + b * TILE;
        const bool leader = lane == 0;
        auto issue_sdp = [&](int qb) {   // S_b(qb), dP_b(qb); the stage's Q / dO reads end with them
            if (leader) {
                const uint32_t aq = aSt + (qb % NST) * L::kStageBytes, ado = aq + kTileBytes;
#pragma unroll
                for (int kk = 0; kk < DP / 16; kk++) {
                    tc::mma_bf16(tS, kmajor_tma(aq + kk * 4096), kmajor_tma(aK + kk * 4096), idesc_s, kk > 0);
                    tc::mma_bf16(tS + KH, kmajor_tma(ado + kk * 4096), kmajor_tma(aV + kk * 4096), idesc_s, kk > 0);
                }
                tc::commit(&bars[L::SF + b]);
                tc::commit(&bars[L::QE + qb % NST]);
            }
            __syncwarp();
        };
        bool ok = warp_wait(&bars[L::KVF], 0, ab) && warp_wait(&bars[L::QF], 0, ab);
        if (ok) {
            tc::fence_after_sync();
            issue_sdp(0);
        }
        for (int qb = 0; ok && qb + 1 < nqb; qb++) {
            if (!(ok = warp_wait(&bars[L::SR + b], qb & 1, ab))) break;
            if (!(ok = warp_wait(&bars[L::QF + (qb + 1) % NST], ((qb + 1) / NST) & 1, ab))) break;
            tc::fence_after_sync();
            issue_sdp(qb + 1);
        }
        if (leader) {
            tc::commit(&bars[L::ACC + b]);
            tc::mbar_wait_bounded(&bars[L::ACC + b], 0, kWaitLimit);   // own MMAs drained
        }
        __syncwarp();
    } else if (warp == 3) {
        // ---------------- accumulating MMA warp: dV, dK, dQ ----------------
        constexpr uint32_t idesc_kv = tc::idesc_bf16(TILE, DP, true, true);    // [keys x d], P / dS read MN-major
        constexpr uint32_t idesc_dq = tc::idesc_bf16(TILE, DP, false, true);   // [queries x d]
        const uint32_t aK = tc::smem_addr(smem + L::kK), aSt = tc::smem_addr(smem + L::kStage),
                       aPS = tc::smem_addr(smem + L::kPS);
        const bool leader = lane == 0;
        bool ok = warp_wait(&bars[L::KVF], 0, ab);
        for (int qb = 0; ok && qb < nqb; qb++) {
            const int st = qb % NST, par = qb & 1;
            if (!(ok = warp_wait(&bars[L::DS + par], (qb >> 1) & 1, ab))) break;
            if (!(ok = warp_wait(&bars[L::QF + st], (qb / NST) & 1, ab))) break;
            if (!(ok = warp_wait(&bars[L::DQE + par], ((qb >> 1) & 1) ^ 1, ab))) break;
            tc::fence_after_sync();
            if (leader) {
                const uint32_t aq = aSt + st * L::kStageBytes, ado = aq + kTileBytes;
                const uint32_t ap = aPS + par * L::kPSBytes, ads = ap + TILE * TILE * 2;
#pragma unroll
                for (int kk = 0; kk < TILE / 16; kk++) {   // K = 128 queries
                    const uint32_t acc = (qb > 0 || kk > 0);
                    tc::mma_bf16(tDV, mnmajor_sq(ap + kk * 4096), mnmajor_tma(ado + kk * 256), idesc_kv, acc);
                    tc::mma_bf16(tDK, mnmajor_sq(ads + kk * 4096), mnmajor_tma(aq + kk * 256), idesc_kv, acc);
                }
#pragma unroll
                for (int kk = 0; kk < TILE / 16; kk++)   // K = 128 keys: dS read K-major, K read MN-major
                    tc::mma_bf16(tDQ0 + par * DP, kmajor_sq(ads + kk * 256), mnmajor_tma(aK + kk * 256), idesc_dq,
                                 kk > 0);
                tc::commit(&bars[L::DQF + par]);
                tc::commit(&bars[L::PE + par]);
                tc::commit(&bars[L::QE + st]);
            }
            __syncwarp();
        }
        if (leader) {
            tc::commit(&bars[L::ACC + 2]);
            tc::mbar_wait_bounded(&bars[L::ACC + 2], 0, kWaitLimit);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 12) {
        // ---------------- softmax warpgroups: key half b, query row r ----------------
        const int b = (warp - 4) >> 2, r = tid & 127;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + b * TILE + lane_off, tDP = tS + KH;
        const float sl2 = scale * kLog2e;
        const f32x2 sl2x2 = pk(sl2, sl2);
        const uint32_t thr = drop_p > 0.f ? (uint32_t)fminf(drop_p * 4294967296.0f, 4294967295.0f) : 0u;
        const float keep_scale = drop_p > 0.f ? 1.0f / (1.0f - drop_p) : 1.0f;
        auto release_s = [&](int half) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[L::SR + half]);
        };
        for (int qb = 0; qb < nqb; qb++) {
            const int st = qb % NST, par = qb & 1;
            if (ab.set()) break;
            if (!warp_wait(&bars[L::SF + b], qb & 1, ab)) break;
            if (!warp_wait(&bars[L::QF + st], (qb / NST) & 1, ab)) break;   // lse / delta visible
            if (!warp_wait(&bars[L::PE + par], ((qb >> 1) & 1) ^ 1, ab)) break;
            tc::fence_after_sync();
            const float *sl = reinterpret_cast<const float *>(smem + L::kStage + st * L::kStageBytes + 2 * kTileBytes);
            const float nl = sl[r], nd = sl[TILE + r];
            uint8_t *pt = smem + L::kPS + par * L::kPSBytes, *dst = pt + TILE * TILE * 2;
            const int qi = qb * TILE + r;
            if (!thr) {
                const f32x2 nl2 = pk(nl, nl), nd2 = pk(nd, nd);
#pragma unroll 1
                for (int c4 = 0; c4 < KH / 32; c4++) {
                    float sv[32], dp[32];
                    tc::ld32_pair(tS + c4 * 32, sv, tDP + c4 * 32, dp);
                    if (c4 == KH / 32 - 1) release_s(b);   // the next S_b, dP_b may overwrite the buffer
                    const int chunk = b * (KH / 8) + c4 * 4;
                    bwd_chunk_fast(sv, dp, sl2x2, nl2, nd2, pt + sq_off(r, chunk), dst + sq_off(r, chunk));
                }
            } else {   // attention dropout: P and dP masked by the forward's keep decisions
#pragma unroll 1
                for (int c4 = 0; c4 < KH / 32; c4++) {
                    float sv[32], dp[32];
                    tc::ld32_pair(tS + c4 * 32, sv, tDP + c4 * 32, dp);
                    if (c4 == KH / 32 - 1) release_s(b);
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        float pv[8], dsv[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const int j = c * 8 + e;
                            const float p = tc::ex2(fmaf(sv[j], sl2, nl));
                            const bool keep = keep_elem(seed, h, qi, k0 + b * KH + c4 * 32 + j, thr);
                            pv[e] = keep ? p * keep_scale : 0.f;
                            dsv[e] = p * ((keep ? dp[j] * keep_scale : 0.f) + nd);
                        }
                        const int chunk = b * (KH / 8) + c4 * 4 + c;
                        st16(pt + sq_off(r, chunk), tc::pack_bf16(pv[0], pv[1]), tc::pack_bf16(pv[2], pv[3]),
                             tc::pack_bf16(pv[4], pv[5]), tc::pack_bf16(pv[6], pv[7]));
                        st16(dst + sq_off(r, chunk), tc::pack_bf16(dsv[0], dsv[1]), tc::pack_bf16(dsv[2], dsv[3]),
                             tc::pack_bf16(dsv[4], dsv[5]), tc::pack_bf16(dsv[6], dsv[7]));
                    }
                }
            }
            tc::fence_smem_for_async();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&bars[L::DS + par]);
                tc::mbar_arrive(&bars[L::QE + st]);
            }
        }
    } else if (warp >= 12) {
        // ---------------- dQ partials (lane = query), then dK / dV (lane = key) ----------------
        // Per query block the four warps stage the [128 x D] partial in shared memory and thread
        // 384 adds it to dq_acc with one TMA reduce-add (rows past s are clipped by the tensor
        // map).  Barrier 1 (these 128 threads) orders the stage's reuse and makes every exit
        // decision collective, so no warp waits at a barrier that another warp has left.
        constexpr int kDqBar = 1;
        const int r = tid & 127;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const size_t rs = (size_t)H * D;
        float *stage = reinterpret_cast<float *>(smem + L::kDQS);
        bool ok = true;
        for (int qb = 0; qb < nqb; qb++) {
            const int par = qb & 1;
            const bool fail = ab.set() || !warp_wait(&bars[L::DQF + par], (qb >> 1) & 1, ab);
            if (tc::bar_red_or(kDqBar, 128, fail)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            float g[32];
            tc::ld32(tDQ0 + par * DP + lane_off, g);
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[L::DQE + par]);
            if (r == 0) tc::bulk_wait_read_all();   // the previous block's reduce has read the stage
            tc::bar_sync(kDqBar, 128);
            float *row = stage + r * D;            // D % 8 == 0: 16-byte aligned rows
#pragma unroll
            for (int d = 0; d < DP; d += 4)
                if (d < D)
                    *reinterpret_cast<float4 *>(row + d) =
                        make_float4(g[d] * scale, g[d + 1] * scale, g[d + 2] * scale, g[d + 3] * scale);
            tc::fence_smem_for_async();
            tc::bar_sync(kDqBar, 128);
            if (r == 0) {
                tc::tma_reduce_add_2d(&tm_dq, h * D, qb * TILE, stage);
                tc::bulk_commit();
            }
        }
        if (r == 0) tc::bulk_wait_all();
        if (ok && warp_wait(&bars[L::ACC + 2], 0, ab) && !ab.set()) {
            tc::fence_after_sync();
            const int kj = k0 + r;
#pragma unroll 1
            for (int which = 0; which < 2; which++) {   // dV, then dK * scale
                float g[32];
                tc::ld32((which ? tDK : tDV) + lane_off, g);
                const float f = which ? scale : 1.f;
                __nv_bfloat16 *dst = (which ? dk : dv) + (size_t)kj * rs + (size_t)h * D;
                if (kj < s) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        if (c * 8 >= D) continue;
                        st16(reinterpret_cast<uint8_t *>(dst + c * 8), tc::pack_bf16(g[c * 8] * f, g[c * 8 + 1] * f),
                             tc::pack_bf16(g[c * 8 + 2] * f, g[c * 8 + 3] * f),
                             tc::pack_bf16(g[c * 8 + 4] * f, g[c * 8 + 5] * f),
                             tc::pack_bf16(g[c * 8 + 6] * f, g[c * 8 + 7] * f));
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------------------
// Host side: tensor maps
// ------------------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// The encoder is a driver call: it needs the device's primary context current in the calling
// thread, which a thread that has only made runtime calls (autograd's device threads) may lack.
void bind_primary_context() {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
}

// [s, H, D] bf16 rows viewed as (8 elements, s rows, D / 8 chunks, H heads); box (8, 128, 4, 1).
int rows_map(CUtensorMap *m, const void *base, int64_t s, int H, int D) {
    bind_primary_context();
    EncodeTiled enc = encoder();
    if (!enc) return NGT_ERR_CUDA;
    const cuuint64_t dims[4] = {8, (cuuint64_t)s, (cuuint64_t)(D / 8), (cuuint64_t)H};
    const cuuint64_t strides[3] = {(cuuint64_t)H * D * 2, 16, (cuuint64_t)D * 2};
    const cuuint32_t box[4] = {8, TILE, DP / 8, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NGT_OK : NGT_ERR_CUDA;
}

// dq_acc [s, H * D] fp32 as 2-D (H * D columns, s rows); box (D, 128): one head's D columns of a
// 128-row query block.  Column coordinate h * D: h * D * 4 bytes is a multiple of 16 (D % 8 == 0).
int dq_map(CUtensorMap *m, float *base, int64_t s, int H, int D) {
    bind_primary_context();
    EncodeTiled enc = encoder();
    if (!enc) return NGT_ERR_CUDA;
    const cuuint64_t dims[2] = {(cuuint64_t)H * D, (cuuint64_t)s};
    const cuuint64_t strides[1] = {(cuuint64_t)H * D * 4};
    const cuuint32_t box[2] = {(cuuint32_t)D, TILE};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NGT_OK : NGT_ERR_CUDA;
}

}  // namespace
}  // namespace dtma

template <bool PT>
int dense_fwd_tma_t(int64_t s, int heads, int head_dim, float scale, float score_scale, float drop_p, uint32_t seed,
                    const void *q, const void *k, const void *v, void *out, float *lse, float *ns, int *status,
                    cudaStream_t st) {
    using namespace dtma;
    CUtensorMap mq, mk, mv;
    int rc;
    if ((rc = rows_map(&mq, q, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = rows_map(&mk, k, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = rows_map(&mv, v, s, heads, head_dim)) != NGT_OK) return rc;
    if (cudaFuncSetAttribute(dense_fwd_tma_kernel<PT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)FwdL<PT>::kBytes) != cudaSuccess)
        return NGT_ERR_CUDA;
    dim3 grid((unsigned)((s + 2 * TILE - 1) / (2 * TILE)), (unsigned)heads);
    dense_fwd_tma_kernel<PT><<<grid, kThreads, FwdL<PT>::kBytes, st>>>(mq, mk, mv, (int)s, heads, head_dim, scale,
                                                                   score_scale, drop_p, seed, (__nv_bfloat16 *)out,
                                                                   lse, ns, status);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

int dense_fwd_tma(int64_t s, int heads, int head_dim, float scale, float score_scale, float drop_p, uint32_t seed,
                  const void *q, const void *k, const void *v, void *out, float *lse, float *ns, int *status,
                  cudaStream_t st) {
    return dense_fwd_tma_t<true>(s, heads, head_dim, scale, score_scale, drop_p, seed, q, k, v, out, lse, ns, status,
                                 st);
}

int dense_bwd_tma(int64_t s, int heads, int head_dim, float scale, float drop_p, uint32_t seed, const void *q,
                  const void *k, const void *v, const void *dout, const float *lse, const float *delta, float *dq_acc,
                  void *dk, void *dv, int *status, cudaStream_t st) {
    using namespace dtma;
    CUtensorMap mq, mk, mv, mdo, mdq;
    int rc;
    if ((rc = rows_map(&mq, q, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = rows_map(&mk, k, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = rows_map(&mv, v, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = rows_map(&mdo, dout, s, heads, head_dim)) != NGT_OK) return rc;
    if ((rc = dq_map(&mdq, dq_acc, s, heads, head_dim)) != NGT_OK) return rc;
    if (cudaFuncSetAttribute(dense_bwd_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BwdL::kBytes) !=
        cudaSuccess)
        return NGT_ERR_CUDA;
    dim3 grid((unsigned)((s + TILE - 1) / TILE), (unsigned)heads);
    dense_bwd_tma_kernel<<<grid, kThreads, BwdL::kBytes, st>>>(mq, mk, mv, mdo, mdq, (int)s, heads, head_dim, scale, drop_p,
                                                               seed, lse, delta, dq_acc, (__nv_bfloat16 *)dk,
                                                               (__nv_bfloat16 *)dv, status);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

}  // namespace ngt
