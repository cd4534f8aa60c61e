// fp32 Linear GEMMs (forward y = x W^T + b, input grad dx = dy W) on the tcgen05 tensor cores
// with split TF32 operands.
//
// Every fp32 operand element a is split into hi = tf32_rn(a) and lo = tf32_rn(a - hi) (a - hi is
// exact in fp32); a b is then hi_a hi_b + hi_a lo_b + lo_a hi_b, three kind::tf32 MMAs per k-step
// into one fp32 TMEM accumulator.  The dropped lo_a lo_b and the rounding of lo leave a relative
// error per product near 2^-21, the size of fp32's own rounding in a sum of 10^2 products, so the
// result keeps the precision of torch's fp32 Linear (no TF32 loss), at tensor-core speed.
//
// Tiling: one CTA = 128 rows (the 128 TMEM lanes, MMA M = 128) x `ncta` output columns (MMA N,
// padded to a multiple of 16, <= 256), the reduction dimension streamed in slices of 16 elements.
// One producer thread keeps STAGES - 1 slices in flight with 2-D TMA boxes of 64-byte rows: A as
// [128 rows][16] (64-byte swizzle), the forward's weight as [np rows][16], the input grad's weight
// (W [out, in], reduced over `out`) as [16 k][np n], transposed by the threads.  512 splitter
// threads (16 warps) split a landed slice: A's hi / lo go to TMEM with tcgen05.st (A is the MMA's
// TMEM operand: 32 columns per slice after the accumulator, four buffers), B's to one of four
// shared-memory operand buffers in the no-swizzle K-major core-matrix layout (row r, 16-byte chunk
// c at c * LBO + r * 16, LBO = rows * 16 + 32, so the eight 16-byte stores of a quarter-warp hit
// distinct banks).  The producer issues the slice's 6 MMAs (A from TMEM, B from shared memory) and
// commits them to the buffer's mbarrier.  TMA writes through the async proxy, so the splitters'
// proxy fence before the MMAs waits only for their own stores, never for loads in flight.  The
// epilogue reads the accumulator with tcgen05.ld (warp w: lanes 32 (w % 4).., column groups dealt
// round-robin over the warps of a lane quarter) into a shared-memory tile; one warp per row then
// stores it (coalesced) with the bias.
//
// Per-CTA clock traces of the 14,252 x 128 -> 128 forward: a slice costs ~1,100-1,600 cycles, set by
// the splitters on the SM sub-partition that also runs the producer (its four splitter warps
// finish last); hence the cheap split (cvt.rna, split4) and the producer's precomputed
// descriptors.  A in TMEM halves the MMAs' shared-memory reads but measured no faster by itself.
//
// Every wait is bounded; a timeout is counted in a device word (ngt_linear_status), the CTA waits
// (bounded) for its MMAs in flight, frees its TMEM and returns without storing.
//
// Reference layers: the models' nn.Linear (NeutronGT/models/gt_dist_node_level_single_window.py:
// 235-237, 313-318, 361; graphormer_dist_node_level.py:179, 183, 286).
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "linear_tc.h"
#include "tc.cuh"

namespace ngt {

__device__ int g_linear_tc_timeouts = 0;

namespace {

constexpr int kM = 128;                        // rows per CTA = TMEM lanes = MMA M
constexpr int kKS = 16;                        // reduction elements per slice (4 chunks of 16 B)
constexpr int kThreads = 4 * kM;               // splitter / epilogue threads: one per A row and 4-wide k chunk
constexpr int kThreadsAll = kThreads + 32;     // + one warp: its lane 0 issues the TMA loads and MMAs
constexpr int kBufs = 4;                       // operand buffers (A in TMEM, B in shared memory)
constexpr int kColParts = kThreads / kM;       // splitter threads per A row (the weight grad's column sums)
constexpr uint32_t kARaw = kM * kKS * 4;       // bytes of one A slice (raw, hi or lo): 8 KiB
constexpr uint32_t kPolls = 1u << 26;
constexpr int kMaxN = 256;                     // widest CTA output tile (the row stores take <= 64 vectors)
constexpr uint32_t kSmemPerSm = 233472;        // 228 KiB per SM, 1 KiB of it reserved per CTA
constexpr uint32_t kSmemPerCta = 232448;       // 227 KiB: the most one CTA may request
constexpr int kMaxStages = 8;

struct TcArgs {
    int64_t M;
    int K, N;          // reduction length, output columns (row stride of C)
    int ncta, np;      // columns per CTA, padded to the MMA N
    uint32_t tmem_cols;
    int trans;         // 0: B(n, k) = W[n * K + k];  1: B(n, k) = W[k * N + n]
    int trans_a;       // 0: A(m, k) = A[m * K + k];  1: A(m, k) = A[k * M + m] (weight grad: A = dy)
    int db;            // 1: also store the sums of A over the CTA's k range at C + M * N + m
    int64_t k_per_cta; // reduction elements per blockIdx.z (a multiple of kKS unless it is all of K)
    int64_t c_stride;  // floats between the outputs of consecutive blockIdx.z
    const float *bias;
    float *C;
};

// Shared memory: STAGES raw slices (A, then B), two B operand buffers (B hi, B lo), then the mbarriers
// (STAGES "slice landed", 2 "MMAs done", 2 "operands split") and the TMEM address.  A's hi / lo
// operands live in TMEM: two buffers of 32 columns (hi k 0..15, lo k 0..15) after the accumulator.
__host__ __device__ constexpr uint32_t raw_bytes(int np) { return kARaw + (uint32_t)np * 64u; }
// Operand tiles: K-chunk stride (LBO) rows * 16 + 32 bytes; a tile spans 3 LBO + rows * 16 bytes.
__host__ __device__ constexpr uint32_t op_lbo(int rows) { return (uint32_t)rows * 16u + 32u; }
__host__ __device__ constexpr uint32_t op_tile(int rows) { return 3 * op_lbo(rows) + (uint32_t)rows * 16u; }
__host__ __device__ constexpr uint32_t op_bytes(int np) { return 2 * op_tile(np); }
__host__ __device__ constexpr uint32_t a_col(int np) { return (uint32_t)(np + 31) / 32u * 32u; }
__host__ __device__ constexpr uint32_t smem_bytes(int np, int stages) {
    return (uint32_t)stages * raw_bytes(np) + kBufs * op_bytes(np) + 8 * (uint32_t)(stages + 2 * kBufs) + 16;
}

// hi = x rounded to the nearest tf32 (ties away from zero; 10 mantissa bits), lo = x - hi (exact);
// the tensor core reads lo as tf32 too, which costs at most 2^-11 of |lo| <= 2^-22 |x|.
// Within 2^-11 of FLT_MAX the rounding would carry into the exponent (hi = inf, lo = -inf, a NaN
// product); there hi is truncated instead, and lo stays exact.  Non-finite x: hi = x, lo = 0.
__device__ __forceinline__ void split1(float x, uint32_t &hi, float &lo) {
    const uint32_t b = __float_as_uint(x);
    const bool fin = (b & 0x7F800000u) != 0x7F800000u;
    uint32_t r = (b + 0x1000u) & 0xFFFFE000u;
    if ((r & 0x7F800000u) == 0x7F800000u) r = b & 0xFFFFE000u;
    hi = fin ? r : b;
    lo = fin ? x - __uint_as_float(hi) : 0.f;
}
__device__ __forceinline__ uint32_t tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// split1 of four values.  While all four are below 0x7F7FF000 in magnitude (so none is within
// 2^-11 of FLT_MAX or infinite), hi is cvt.rna.tf32 — the same round-to-nearest, ties away, as
// split1's bit arithmetic — and lo = x - hi: two instructions per value instead of split1's ten.
// (A NaN among finite values takes the short path too; its hi and lo are NaN, as is its product.)
__device__ __forceinline__ void split4(const float4 v, uint4 &h, float4 &l) {
    const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    if (__float_as_uint(m) < 0x7F7FF000u) {
        h = make_uint4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        l = make_float4(v.x - __uint_as_float(h.x), v.y - __uint_as_float(h.y), v.z - __uint_as_float(h.z),
                        v.w - __uint_as_float(h.w));
    } else {
        split1(v.x, h.x, l.x);
        split1(v.y, h.y, l.y);
        split1(v.z, h.z, l.z);
        split1(v.w, h.w, l.w);
    }
}
__device__ __forceinline__ void split_store(float4 v, uint8_t *hi, uint8_t *lo) {
    uint4 h;
    float4 l;
    split4(v, h, l);
    *reinterpret_cast<uint4 *>(hi) = h;
    *reinterpret_cast<float4 *>(lo) = l;
}

// Splits a landed slice: A into the TMEM buffer at column `ta` of this thread's lane quarter, B
// into shared operand buffer `op`.  A: thread (m = tid % 128, c = tid / 128) takes row m's four
// reduction elements 4c .. 4c + 3 (warp tid / 32 sits on lane quarter m / 32 as tcgen05.st needs):
// hi to columns 4c.., lo to 16 + 4c..  The forward / input-grad raw A slice is [128 rows][16] with
// the TMA's 64-byte swizzle (chunk c of row m at chunk c ^ ((m >> 1) & 3), so the eight rows of a
// quarter-warp's 16-byte loads hit distinct banks); the weight grad's is row-major [16 k][128 m]
// (thread tid always takes column m = tid % 128) and its four values are also added into `asum` in
// a fixed order (the bias gradient of the weight-grad GEMM).  B: raw rows are 64 bytes (item idx =
// row idx / 4, chunk idx % 4, at idx * 16: consecutive threads read consecutive bytes); operand
// chunk (r, c) goes to c * LBO + r * 16.
__device__ __forceinline__ void split_slice(const TcArgs &p, const uint8_t *raw, uint8_t *op, uint32_t ta,
                                            float &asum) {
    const int tid = threadIdx.x;
    const uint8_t *rb = raw + kARaw;
    const uint32_t lbb = op_lbo(p.np);
    uint8_t *b_hi = op, *b_lo = op + op_tile(p.np);
    {
        const int m = tid % kM, c = tid / kM;
        float4 v;
        if (!p.trans_a) {
            v = *reinterpret_cast<const float4 *>(raw + m * 64 + ((c ^ ((m >> 1) & 3)) << 4));
        } else {
            const float *colp = reinterpret_cast<const float *>(raw) + (4 * c) * kM + m;
            v = make_float4(colp[0], colp[kM], colp[2 * kM], colp[3 * kM]);
            asum += ((v.x + v.y) + v.z) + v.w;
        }
        uint4 h;
        float4 l;
        split4(v, h, l);
        tc::st4_nowait(ta + 4 * c, h.x, h.y, h.z, h.w);
        tc::st4_nowait(ta + 16 + 4 * c, __float_as_uint(l.x), __float_as_uint(l.y), __float_as_uint(l.z),
                       __float_as_uint(l.w));
    }
    const int items = p.np * 4;
    for (int idx = tid; idx < items; idx += kThreads) {
        float4 v;
        uint32_t o;
        if (!p.trans) {
            v = *reinterpret_cast<const float4 *>(rb + idx * 16);
            o = (uint32_t)(idx & 3) * lbb + (uint32_t)(idx >> 2) * 16u;
        } else {   // raw row-major [16 k][np n]: column n, rows 4c .. 4c + 3
            const int n = idx % p.np, c = idx / p.np;
            const float *col = reinterpret_cast<const float *>(rb) + (4 * c) * p.np + n;
            v = make_float4(col[0], col[p.np], col[2 * p.np], col[3 * p.np]);
            o = (uint32_t)c * lbb + (uint32_t)n * 16u;
        }
        split_store(v, b_hi + o, b_lo + o);
    }
}

template <int STAGES>
__global__ void __launch_bounds__(kThreadsAll, 2)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                     const TcArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t m0 = (int64_t)blockIdx.x * kM;
    const int n0 = blockIdx.y * p.ncta;
    const int64_t kb = (int64_t)blockIdx.z * p.k_per_cta;            // this CTA's reduction range
    const int64_t kc = p.K - kb < p.k_per_cta ? p.K - kb : p.k_per_cta;
    float *const C = p.C + (int64_t)blockIdx.z * p.c_stride;
    const uint32_t rawb = raw_bytes(p.np), opb = op_bytes(p.np);
    uint8_t *ops = smem + STAGES * rawb;
    uint64_t *full = reinterpret_cast<uint64_t *>(ops + kBufs * opb);   // [STAGES] slice landed (TMA bytes)
    uint64_t *done = full + STAGES;                                  // [2] MMAs of an operand buffer done
    uint64_t *ready = done + kBufs;                                  // [kBufs] operand buffer split (kThreads arrivals)
    uint32_t *slot = reinterpret_cast<uint32_t *>(ready + kBufs);
    const int ns = (int)((kc + kKS - 1) / kKS);
    const bool producer = tid == kThreads;                           // last warp, lane 0

    auto load = [&](int j) {   // slice j into stage j % STAGES
        uint8_t *raw = smem + (j % STAGES) * rawb;
        uint64_t *bar = &full[j % STAGES];
        const int k = (int)(kb + (int64_t)j * kKS);
        tc::mbar_arrive_expect_tx(bar, rawb);
        if (!p.trans_a)
            tc::tma_load_2d(raw, &tm_a, k, (int)m0, bar);
        else
            tc::tma_load_2d(raw, &tm_a, (int)m0, k, bar);
        if (!p.trans)
            tc::tma_load_2d(raw + kARaw, &tm_w, k, n0, bar);
        else
            tc::tma_load_2d(raw + kARaw, &tm_w, n0, k, bar);
    };

    int loaded = 0, issued = 0;   // producer's counts
    if (producer) {
        for (int st = 0; st < STAGES; st++) tc::mbar_init(&full[st], 1);
        for (int b = 0; b < kBufs; b++) {
            tc::mbar_init(&done[b], 1);
            tc::mbar_init(&ready[b], kThreads);
        }
        tc::mbar_init_fence();
        for (; loaded < STAGES - 1 && loaded < ns; loaded++) load(loaded);
    }
    if (warp == 0) tc::tmem_alloc(slot, p.tmem_cols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *slot;

    bool ok = true;
    float asum = 0.f;   // splitter thread's sum of A over its column (db only)
    if (producer) {
        // Slice s - 1's stage is free once every splitter arrived on ready for slice s - 1 (waited
        // below in the previous iteration), so slice s + STAGES - 1 can take it.
        const uint32_t idesc = tc::idesc_tf32(kM, p.np);
        const uint32_t b_lbo = op_lbo(p.np);
        // B descriptors: buffer 0's hi tile once; the others differ only in the start-address field
        // (address >> 4, far below its 14-bit limit), so one 64-bit add selects buffer, lo / hi and k step.
        const uint64_t desc0 = tc::smem_desc(tc::smem_addr(ops), b_lbo, 128);
        const uint64_t step_buf = opb >> 4, step_lo = op_tile(p.np) >> 4, step_k = (2u * b_lbo) >> 4;
        for (int s = 0; s < ns; s++) {
            if (loaded < ns) load(loaded++);
            if (!tc::mbar_wait_bounded(&ready[s % kBufs], (uint32_t)(s / kBufs) & 1u, kPolls)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t a_hi = tmem + a_col(p.np) + 32u * (uint32_t)(s % kBufs), a_lo = a_hi + 16u;
            const uint64_t dbuf = desc0 + (uint64_t)(s % kBufs) * step_buf;
#pragma unroll
            for (int kk = 0; kk < kKS / 8; kk++) {   // K = 8 tf32 = 8 TMEM columns of A, two 16-byte chunks of B
                const uint64_t dbh = dbuf + (uint64_t)kk * step_k, dbl = dbh + step_lo;
                tc::mma_tf32_ts(tmem, a_lo + 8u * kk, dbh, idesc, (s > 0 || kk > 0) ? 1u : 0u);
                tc::mma_tf32_ts(tmem, a_hi + 8u * kk, dbl, idesc, 1u);
                tc::mma_tf32_ts(tmem, a_hi + 8u * kk, dbh, idesc, 1u);
            }
            tc::commit(&done[s % kBufs]);
            issued = s + 1;
        }
    } else if (tid < kThreads) {   // splitters: no CTA-wide barrier per slice
        const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + a_col(p.np);   // A buffer 0, my lanes
        for (int s = 0; s < ns; s++) {
            const int b = s % kBufs;
            bool w = tc::mbar_wait_bounded(&full[s % STAGES], (uint32_t)(s / STAGES) & 1u, kPolls);
            if (w && s >= kBufs)   // operand buffer b was last read by the MMAs of slice s - kBufs
                w = tc::mbar_wait_bounded(&done[b], (uint32_t)((s - kBufs) / kBufs) & 1u, kPolls);
            if (!__all_sync(0xffffffffu, w)) {   // warp-uniform: tcgen05.st below is .sync.aligned
                ok = false;
                break;
            }
            split_slice(p, smem + (s % STAGES) * rawb, ops + b * opb, ta + 32u * (uint32_t)b, asum);
            tc::wait_st();                 // A's TMEM stores done,
            tc::fence_smem_for_async();    // B's shared stores visible to the MMAs,
            tc::fence_before_sync();       // ordered before the arrival
            tc::mbar_arrive(&ready[b]);
        }
    }
    {
        const int last = ns - 1;
        const bool w = ok && tc::mbar_wait_bounded(&done[last % kBufs], (uint32_t)(last / kBufs) & 1u, kPolls);
        ok = !__syncthreads_or(!w);
    }
    if (!ok) {
        if (producer) {
            atomicAdd(&g_linear_tc_timeouts, 1);
            // slices loaded - STAGES .. loaded - 1 may still be landing: slice s's stage was only
            // known free (its splitters arrived on ready) up to slice s - 1 when the loop stopped
            for (int j = loaded - STAGES < 0 ? 0 : loaded - STAGES; j < loaded; j++)
                tc::mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, kPolls);   // TMA in flight
            if (issued > 0)   // and the MMAs in flight end before the TMEM is freed (bounded)
                tc::mbar_wait_bounded(&done[(issued - 1) % kBufs], (uint32_t)((issued - 1) / kBufs) & 1u, kPolls);
        }
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (warp == 0) tc::tmem_dealloc(tmem, p.tmem_cols);
        return;
    }
    tc::fence_after_sync();

    // Epilogue: accumulator -> shared tile [128 rows][ldt floats] (the raw stages and operand
    // buffers are all consumed; ldt = 32 k + 4, so rows sit 16 bytes apart modulo 128 and a
    // quarter-warp's 16-byte stores hit distinct banks), then coalesced row stores with the bias.
    const int q = warp & 3;
    const int nv = min(p.ncta, p.N - n0);
    const int ngrp = (nv + 31) / 32;
    const int ldt = ngrp * 32 + 4;
    float *tile = reinterpret_cast<float *>(smem);
    float *sdb = tile + kM * ldt;   // [kThreads] splitter sums of A (db only)
    if (p.db && tid < kThreads) sdb[tid] = asum;
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    for (int g = warp >> 2; warp < kThreads / 32 && g < ngrp; g += kThreads / 128) {
        float v[32];
        tc::ld32(taddr + (uint32_t)(g * 32), v);
        float4 *dst = reinterpret_cast<float4 *>(tile + (q * 32 + lane) * ldt + g * 32);
#pragma unroll
        for (int j = 0; j < 8; j++) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    tc::fence_before_sync();
    __syncthreads();
    // Row stores: warp w takes rows w, w + 9, ...; lane l the row's 16-byte vectors l and l + 32
    // (nv <= 256), with the bias for those columns held in registers.
    const int vpr = nv / 4;   // 16-byte vectors per output row (N % 4 == 0)
    const int rows_here = (int)(p.M - m0 < kM ? p.M - m0 : kM);
    float4 bias0 = make_float4(0.f, 0.f, 0.f, 0.f), bias1 = bias0;
    if (p.bias) {
        if (lane < vpr) bias0 = __ldg(reinterpret_cast<const float4 *>(p.bias + n0) + lane);
        if (lane + 32 < vpr) bias1 = __ldg(reinterpret_cast<const float4 *>(p.bias + n0) + lane + 32);
    }
    for (int rr = warp; rr < rows_here; rr += kThreadsAll / 32) {
        const float4 *trow = reinterpret_cast<const float4 *>(tile + rr * ldt);
        float4 *crow = reinterpret_cast<float4 *>(C + (m0 + rr) * p.N + n0);
        if (lane < vpr) {
            float4 o = trow[lane];
            o.x += bias0.x;
            o.y += bias0.y;
            o.z += bias0.z;
            o.w += bias0.w;
            crow[lane] = o;
        }
        if (lane + 32 < vpr) {
            float4 o = trow[lane + 32];
            o.x += bias1.x;
            o.y += bias1.y;
            o.z += bias1.z;
            o.w += bias1.w;
            crow[lane + 32] = o;
        }
    }
    if (p.db && tid < kM && m0 + tid < p.M) {   // column m's partial sums: threads tid + j * 128
        float t = sdb[tid];
#pragma unroll
        for (int j = 1; j < kColParts; j++) t += sdb[tid + j * kM];
        C[p.M * (int64_t)p.N + m0 + tid] = t;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, p.tmem_cols);
}

// ------------------------------------------------------------------------------------
// Host side
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

// Row-major fp32 [rows, cols] (cols % 4 == 0) as a 2-D map with box (box_cols, box_rows).
int map2d(CUtensorMap *m, const float *base, int64_t rows, int cols, int box_cols, int box_rows,
          CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    EncodeTiled enc = encoder();
    if (!enc) return NGT_ERR_CUDA;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NGT_OK : NGT_ERR_CUDA;
}

int sm_count_tc() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

// TMEM: the accumulator (np columns) and A's two 32-column operand buffers, as a power of two.
uint32_t tmem_cols_for(int np) {
    uint32_t c = 32;
    while (c < a_col(np) + 32u * kBufs) c <<= 1;
    return c;
}

struct TcPlan {
    int split, stages;
};

// Raw-stage depth (3..8 slices; STAGES - 1 in flight): all CTAs resident in one wave where possible
// (two CTAs per SM need <= 113 KiB of shared memory each), deeper first.  One CTA covers all N
// columns of its 128 rows: splitting the columns over two CTAs (so that 10^4-row windows fill more
// SMs) measured equal or slower for every model shape — the block scheduler packs the halves two
// per SM, and each half loads and splits the whole A tile again.
TcPlan tc_plan(int64_t gm, int N, int sms) {
    const int np = (N + 15) / 16 * 16;
    const uint32_t tmem_per_sm = 512u / tmem_cols_for(np);
    for (int stages = kMaxStages; stages >= 3; stages--) {
        uint32_t per_sm = kSmemPerSm / (smem_bytes(np, stages) + 1024);
        if (per_sm > tmem_per_sm) per_sm = tmem_per_sm;
        if (per_sm >= 1 && gm <= (int64_t)sms * (per_sm > 2 ? 2 : per_sm)) return {1, stages};
    }
    return {1, 3};
}

template <int STAGES>
int launch_stages(const CUtensorMap &ma, const CUtensorMap &mw, const TcArgs &p, dim3 grid, cudaStream_t st) {
    // The attribute is set once per device to the largest size this instantiation can take, under a
    // lock, so concurrent host threads never leave it below what a later launch needs.
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NGT_ERR_CUDA;
    const uint32_t need = smem_bytes(p.np, STAGES);
    if (need > kSmemPerCta) return NGT_ERR_UNSUPPORTED;
    {
        const uint32_t most = smem_bytes(kMaxN, STAGES) < kSmemPerCta ? smem_bytes(kMaxN, STAGES) : kSmemPerCta;
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            if (cudaFuncSetAttribute(linear_tc_kernel<STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)most) != cudaSuccess)
                return NGT_ERR_CUDA;
            if (dev >= 0 && dev < 64) attr_set[dev] = true;
        }
    }
    linear_tc_kernel<STAGES><<<grid, kThreadsAll, need, st>>>(ma, mw, p);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// The epilogue's output tile (and the splitter sums) reuse the stages and operand buffers.
int launch_plan(const CUtensorMap &ma, const CUtensorMap &mw, const TcArgs &p, dim3 grid, int stages,
                cudaStream_t st) {
    if ((size_t)kM * (((p.ncta + 31) / 32) * 32 + 4) * 4 + (size_t)kThreads * 4 >
        (size_t)stages * raw_bytes(p.np) + kBufs * op_bytes(p.np))
        return NGT_ERR_UNSUPPORTED;
    switch (stages) {
    case 8: return launch_stages<8>(ma, mw, p, grid, st);
    case 7: return launch_stages<7>(ma, mw, p, grid, st);
    case 6: return launch_stages<6>(ma, mw, p, grid, st);
    case 5: return launch_stages<5>(ma, mw, p, grid, st);
    case 4: return launch_stages<4>(ma, mw, p, grid, st);
    default: return launch_stages<3>(ma, mw, p, grid, st);
    }
}

}  // namespace

bool linear_tc_supported(int K, int N) { return K > 0 && N > 0 && N <= kMaxN && K % 4 == 0 && N % 4 == 0; }

int launch_linear_tc(int64_t M, int K, int N, const float *A, const float *W, bool trans_w, const float *bias,
                     float *C, cudaStream_t st) {
    const int64_t gm = (M + kM - 1) / kM;
    if (M > 0x7fffffffLL - kM) return NGT_ERR_UNSUPPORTED;   // TMA row coordinates are 32-bit signed
    const TcPlan plan = tc_plan(gm, N, sm_count_tc());
    TcArgs p;
    p.M = M;
    p.K = K;
    p.N = N;
    p.ncta = (N + plan.split - 1) / plan.split;
    p.np = (p.ncta + 15) / 16 * 16;
    p.tmem_cols = tmem_cols_for(p.np);
    p.trans = trans_w ? 1 : 0;
    p.trans_a = 0;
    p.db = 0;
    p.k_per_cta = K;
    p.c_stride = 0;
    p.bias = bias;
    p.C = C;
    CUtensorMap ma, mw;
    bind_primary_context();
    int rc = map2d(&ma, A, M, K, kKS, kM, CU_TENSOR_MAP_SWIZZLE_64B);   // [128 rows][16] boxes, 64-byte swizzle
    if (rc == NGT_OK)                                            // [16 k][np n] or [np rows][16]
        rc = trans_w ? map2d(&mw, W, K, N, p.np, kKS) : map2d(&mw, W, N, K, kKS, p.np);
    if (rc != NGT_OK) return rc;
    const dim3 grid((unsigned)gm, (unsigned)plan.split);
    return launch_plan(ma, mw, p, grid, plan.stages, st);
}

bool wgrad_tc_supported(int in_features, int out_features) {
    return in_features > 0 && out_features > 0 && in_features <= kMaxN && in_features % 4 == 0 &&
           out_features % 4 == 0;
}

int launch_wgrad_tc(int64_t rows, int in_features, int out_features, const float *x, const float *dy, float *part,
                    int64_t splits, int64_t rows_per_split, cudaStream_t st) {
    if (rows <= 0 || rows > 0x7fffffffLL - kM || splits < 1 || rows_per_split % kKS != 0 ||
        splits * rows_per_split < rows || (splits - 1) * rows_per_split >= rows)
        return NGT_ERR_UNSUPPORTED;
    const int64_t gm = (out_features + kM - 1) / kM;
    const TcPlan plan = tc_plan(gm * splits, in_features, sm_count_tc());
    TcArgs p;
    p.M = out_features;            // rows of dW
    p.K = rows;                    // reduced over the rows of x and dy
    p.N = in_features;             // columns of dW
    p.ncta = in_features;
    p.np = (in_features + 15) / 16 * 16;
    p.tmem_cols = tmem_cols_for(p.np);
    p.trans = 1;                   // B(n, k) = x[k * in + n]
    p.trans_a = 1;                 // A(m, k) = dy[k * out + m]
    p.db = 1;
    p.k_per_cta = rows_per_split;
    p.c_stride = (int64_t)in_features * out_features + out_features;
    p.bias = nullptr;
    p.C = part;
    CUtensorMap ma, mw;
    bind_primary_context();
    int rc = map2d(&ma, dy, rows, out_features, kM, kKS);        // [16 k][128 m] boxes
    if (rc == NGT_OK) rc = map2d(&mw, x, rows, in_features, p.np, kKS);   // [16 k][np n] boxes
    if (rc != NGT_OK) return rc;
    const dim3 grid((unsigned)gm, 1u, (unsigned)splits);
    return launch_plan(ma, mw, p, grid, plan.stages, st);
}

int linear_tc_timeouts(int *count) {
    if (cudaMemcpyFromSymbol(count, g_linear_tc_timeouts, sizeof(int)) != cudaSuccess) return NGT_ERR_CUDA;
    return NGT_OK;
}

}  // namespace ngt
