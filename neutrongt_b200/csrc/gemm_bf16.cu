// bf16 Linear layers of the large model on the tcgen05 tensor cores (sm_100a).
//
// Replaces the torch Linear GEMMs of GPH_Large's projections (NeutronGT/models/
// gt_dist_node_level_single_window.py:235-237 linear_q/k/v, :313-318 output and FFN layers;
// graphormer_dist_node_level.py:139, 179, 183): y = x W^T + b, its input gradient dy W and its
// weight gradient dy^T x (+ the bias gradient, column sums of dy), bf16 operands with fp32
// accumulation in TMEM.
//
// One kernel computes D[M, N] = sum_k A(m, k) B(n, k) for any major-ness of A and B:
//   forward      A = x  [rows, in]   (K-major)   B = W [out, in]   (K-major)
//   input grad   A = dy [rows, out]  (K-major)   B(n=in, k=out) = W[out, in]   (MN-major)
//   weight grad  A(m=out, k=row) = dy (MN-major) B(n=in, k=row) = x  (MN-major), split over rows
// Operands arrive by TMA in 128-byte-swizzled tiles (64 bf16 per swizzle row), which the MMA
// reads directly through swizzled shared-memory descriptors, so no thread touches an operand.
//
// Persistent, warp-specialised CTA (one per SM, 192 threads):
//   warp 0      lane 0 issues the TMA loads into a ring of kStages stages (full/empty mbarriers)
//   warp 1      lane 0 issues the MMAs (BM=128 x BN x 16 per instruction) into one of two TMEM
//               accumulators and commits each stage back to the producer
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (TMEM lane = output row), bias, bf16
//               conversion and row stores, then the accumulator is handed back to the MMA warp,
//               so tile i's epilogue overlaps tile i+1's MMAs
// Every wait is bounded; a CTA whose wait runs out counts a timeout (ngt_linear_status), waits
// (bounded) for its own copies and MMAs in flight, frees its TMEM and exits.
#include <cuda.h>

#include <mutex>

#include "gemm_bf16.h"
#include "tc.cuh"

namespace ngt {

__device__ int g_gemm_bf16_timeouts = 0;

namespace {

constexpr int BM = 128;                      // tile rows = TMEM lanes = MMA M
constexpr int BK = 64;                       // reduction elements per stage (one swizzle row)
constexpr int kThreads = 192;
constexpr uint32_t kPolls = 1u << 26;
constexpr uint32_t kAtom = 1024;             // 8 rows x 128 bytes: one swizzle atom

struct GemmArgs {
    int64_t M;              // output rows (A's m extent)
    int N, K;               // output columns (B's n extent), reduction length
    int a_mn, b_mn;         // 1: operand is MN-major (m / n contiguous in global memory)
    int tiles_m, tiles_n, splits, kb_total, kb_per_split;
    const __nv_bfloat16 *bias;   // [N] or null (forward only)
    void *out;              // bf16 [M, N] (mode 0) or fp32 partials [splits][M][N] (mode 1)
    int mode;
    int bias_vec;           // 1: bias is 16-byte aligned, read as 16-byte vectors
};

// Shared-memory descriptor of a 128-byte-swizzled operand tile (layout type 2 in bits 61-63).
// K-major: rows of 128 bytes (64 elements of k), 8-row atoms `sbo` apart.  MN-major: rows of 128
// bytes along m / n, one per k, 8-k atoms `sbo` apart, 64-element m / n groups `lbo` apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ __forceinline__ void st_v4(void *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int BN, int kStages>
struct Smem {
    static constexpr uint32_t kA = BM * BK * 2;            // 16 KiB
    static constexpr uint32_t kB = BN * BK * 2;
    static constexpr uint32_t kStage = kA + kB;
    static constexpr uint32_t kBars = kStages * kStage;    // full[S], empty[S], acc_full[2], acc_empty[2]
    static constexpr uint32_t kSlot = kBars + (2 * kStages + 4) * 8;
    static constexpr uint32_t kAbort = kSlot + 4;
    static constexpr uint32_t kBytes = kAbort + 4 + 1024;  // + alignment slack for the 1 KiB atoms
    static constexpr uint32_t kTmemCols = 2 * BN;
};

// Bounded wait that gives up early once another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort) {
    for (uint32_t i = 0; i < kPolls; i++) {
        if (tc::mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort) return false;
    }
    return false;
}

__device__ __forceinline__ void raise_abort(volatile int *abort) {
    if (atomicExch(const_cast<int *>(abort), 1) == 0) atomicAdd(&g_gemm_bf16_timeouts, 1);
}

template <int BN, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const GemmArgs p) {
    using L = Smem<BN, kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBars);
    uint64_t *empty = full + kStages;
    uint64_t *acc_full = empty + kStages;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::kSlot);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbort);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = p.tiles_m * p.tiles_n * p.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            tc::mbar_init(&acc_full[a], 1);
            tc::mbar_init(&acc_empty[a], 4);   // one arrival per epilogue warp
        }
        *abort = 0;
        tc::mbar_init_fence();
    }
    if (warp == 1) tc::tmem_alloc(slot, L::kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *slot;

    // tile t -> (split, m tile, n tile); n fastest, so CTAs running together share A rows
    auto tile_coords = [&](int t, int &sp, int &mt, int &nt) {
        nt = t % p.tiles_n;
        const int r = t / p.tiles_n;
        mt = r % p.tiles_m;
        sp = r / p.tiles_m;
    };
    auto kb_range = [&](int sp, int &kb0, int &kb1) {
        kb0 = sp * p.kb_per_split;
        kb1 = min(p.kb_total, kb0 + p.kb_per_split);
    };

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            uint32_t g = 0;           // stages issued so far (all tiles)
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int sp, mt, nt, kb0, kb1;
                tile_coords(t, sp, mt, nt);
                kb_range(sp, kb0, kb1);
                const int m0 = mt * BM, n0 = nt * BN;
                for (int kb = kb0; kb < kb1; kb++, g++) {
                    const uint32_t s = g % kStages;
                    if (!wait_or_abort(&empty[s], ((g / kStages) & 1u) ^ 1u, abort)) {
                        raise_abort(abort);
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + s * L::kStage, *sb = sa + L::kA;
                    tc::mbar_arrive_expect_tx(&full[s], L::kStage);
                    const int k0 = kb * BK;
                    if (!p.a_mn) {
                        tc::tma_load_2d(sa, &tm_a, k0, m0, &full[s]);
                    } else {
#pragma unroll
                        for (int j = 0; j < BM / 64; j++)
                            tc::tma_load_2d(sa + j * (BK * 128), &tm_a, m0 + 64 * j, k0, &full[s]);
                    }
                    if (!p.b_mn) {
                        tc::tma_load_2d(sb, &tm_b, k0, n0, &full[s]);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 64; j++)
                            tc::tma_load_2d(sb + j * (BK * 128), &tm_b, n0 + 64 * j, k0, &full[s]);
                    }
                }
            }
            if (!ok) {   // the copies issued last may still be landing: wait for them (bounded)
                for (uint32_t j = g > (uint32_t)kStages ? g - kStages : 0u; j < g; j++)
                    tc::mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1u, kPolls);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(BM, BN, p.a_mn != 0, p.b_mn != 0);
            // K-major: 16 elements = 32 bytes along the swizzled row per MMA; MN-major: 16 k = two atoms
            const uint32_t a_step = p.a_mn ? 2 * kAtom : 32, b_step = p.b_mn ? 2 * kAtom : 32;
            const uint32_t a_lbo = p.a_mn ? BK * 128 : 16, b_lbo = p.b_mn ? BK * 128 : 16;
            uint32_t g = 0, it = 0;
            bool ok = true, any = false;
            uint64_t *last = nullptr;
            uint32_t last_par = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, it++) {
                int sp, mt, nt, kb0, kb1;
                tile_coords(t, sp, mt, nt);
                kb_range(sp, kb0, kb1);
                const uint32_t a = it & 1u;
                if (!wait_or_abort(&acc_empty[a], ((it >> 1) & 1u) ^ 1u, abort)) {
                    raise_abort(abort);
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t tacc = tmem + a * BN;
                for (int kb = kb0; kb < kb1; kb++, g++) {
                    const uint32_t s = g % kStages;
                    if (!wait_or_abort(&full[s], (g / kStages) & 1u, abort)) {
                        raise_abort(abort);
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t sa = tc::smem_addr(smem + s * L::kStage), sb = sa + L::kA;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint64_t da = desc_sw128(sa + kk * a_step, a_lbo, kAtom);
                        const uint64_t db = desc_sw128(sb + kk * b_step, b_lbo, kAtom);
                        tc::mma_bf16(tacc, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                    }
                    tc::commit(&empty[s]);   // the stage is free once these MMAs have read it
                    last = &empty[s];
                    last_par = (g / kStages) & 1u;
                    any = true;
                }
                if (!ok) break;
                tc::commit(&acc_full[a]);   // every split holds at least one block, so D was written
                last = &acc_full[a];
                last_par = (it >> 1) & 1u;
            }
            if (!ok && any) tc::mbar_wait_bounded(last, last_par, kPolls);   // own MMAs drain
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        const int quarter = warp & 3;                     // TMEM lanes 32 * quarter ...
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
            int sp, mt, nt;
            tile_coords(t, sp, mt, nt);
            const uint32_t a = it & 1u;
            if (!wait_or_abort(&acc_full[a], (it >> 1) & 1u, abort)) {
                raise_abort(abort);
                break;
            }
            tc::fence_after_sync();
            const int64_t row = (int64_t)mt * BM + quarter * 32 + lane;
            const bool row_ok = row < p.M;
            const int n0 = nt * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                float v[32];
                tc::ld32(tmem + a * BN + lane_base + c * 32, v);
                const int col0 = n0 + c * 32;
                if (!row_ok || col0 >= p.N) continue;
                const int ncols = min(32, p.N - col0);
                if (p.mode == 0) {
                    if (p.bias != nullptr && p.bias_vec && ncols == 32) {
                        // the chunk's 32 bias values as four 16-byte loads (one address for the warp)
                        const uint4 *bp = reinterpret_cast<const uint4 *>(p.bias + col0);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const uint4 b = __ldg(bp + j);
                            const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                v[8 * j + 2 * i] += __uint_as_float(w[i] << 16);
                                v[8 * j + 2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
                            }
                        }
                    } else if (p.bias != nullptr) {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (i < ncols) v[i] += __bfloat162float(p.bias[col0 + i]);
                    }
                    __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.out) + row * p.N + col0;
                    if (ncols == 32) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            st_v4(dst + 8 * j, tc::pack_bf16(v[8 * j], v[8 * j + 1]),
                                  tc::pack_bf16(v[8 * j + 2], v[8 * j + 3]), tc::pack_bf16(v[8 * j + 4], v[8 * j + 5]),
                                  tc::pack_bf16(v[8 * j + 6], v[8 * j + 7]));
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (i < ncols) dst[i] = __float2bfloat16_rn(v[i]);
                    }
                } else {
                    float *dst = reinterpret_cast<float *>(p.out) + ((int64_t)sp * p.M + row) * p.N + col0;
                    if (ncols == 32) {
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            st_v4(dst + 4 * j, __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                  __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (i < ncols) dst[i] = v[i];
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acc_empty[a]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 1) tc::tmem_dealloc(tmem, L::kTmemCols);
}

// Sums the fp32 split partials [splits][rows][cols] in split order (bitwise reproducible) and
// writes bf16 [rows][cols]; four columns per thread.
__global__ void split_sum_bf16_kernel(int splits, int64_t count4, int64_t stride, const float *__restrict__ part,
                                      __nv_bfloat16 *__restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 acc = __ldg(reinterpret_cast<const float4 *>(part) + i);
        for (int s = 1; s < splits; s++) {
            const float4 x = __ldg(reinterpret_cast<const float4 *>(part + s * stride) + i);
            acc.x += x.x;
            acc.y += x.y;
            acc.z += x.z;
            acc.w += x.w;
        }
        uint2 w;
        w.x = tc::pack_bf16(acc.x, acc.y);
        w.y = tc::pack_bf16(acc.z, acc.w);
        reinterpret_cast<uint2 *>(out)[i] = w;
    }
}

// Column sums of a bf16 [rows, cols] matrix (the bias gradient): thread column c of block row y
// sums the y-th chunk of rows in row order into part[y][c]; colsum_finish_kernel adds the chunks
// in chunk order, so the result is bitwise reproducible.
__global__ void colsum_part_kernel(int64_t rows, int cols, int64_t rows_per_chunk, const __nv_bfloat16 *__restrict__ x,
                                   float *__restrict__ part) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const int64_t r0 = blockIdx.y * rows_per_chunk;
    const int64_t r1 = min(rows, r0 + rows_per_chunk);
    float acc = 0.f;
    for (int64_t r = r0; r < r1; r++) acc += __bfloat162float(x[r * cols + c]);
    part[(int64_t)blockIdx.y * cols + c] = acc;
}

__global__ void colsum_finish_kernel(int chunks, int cols, const float *__restrict__ part,
                                     __nv_bfloat16 *__restrict__ out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    float acc = 0.f;
    for (int j = 0; j < chunks; j++) acc += part[(int64_t)j * cols + c];
    out[c] = __float2bfloat16_rn(acc);
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

// Row-major bf16 [rows, cols] as a 2-D map, box (64 columns, box_rows), 128-byte swizzle; reads past
// the edges fill zeros.
int map_bf16(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return NGT_ERR_CUDA;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);   // the driver call needs a current context
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NGT_OK : NGT_ERR_CUDA;
}

int sm_count() {
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

template <int BN, int kStages>
int launch(const CUtensorMap &ma, const CUtensorMap &mb, const GemmArgs &p, cudaStream_t st) {
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NGT_ERR_CUDA;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            if (cudaFuncSetAttribute(gemm_bf16_kernel<BN, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Smem<BN, kStages>::kBytes) != cudaSuccess)
                return NGT_ERR_CUDA;
            if (dev >= 0 && dev < 64) attr_set[dev] = true;
        }
    }
    const int tiles = p.tiles_m * p.tiles_n * p.splits;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_bf16_kernel<BN, kStages><<<grid, kThreads, Smem<BN, kStages>::kBytes, st>>>(ma, mb, p);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

// BN = 256 unless the output has at most 128 columns (narrow heads, class layers).
int run(GemmArgs p, const void *a, int64_t a_rows, int64_t a_cols, const void *b, int64_t b_rows, int64_t b_cols,
        cudaStream_t st) {
    const int bn = p.N <= 128 ? 128 : 256;
    p.tiles_m = (int)((p.M + BM - 1) / BM);
    p.tiles_n = (p.N + bn - 1) / bn;
    CUtensorMap ma, mb;
    int rc = map_bf16(&ma, a, a_rows, a_cols, p.a_mn ? BK : BM);
    if (rc == NGT_OK) rc = map_bf16(&mb, b, b_rows, b_cols, p.b_mn ? BK : bn);
    if (rc != NGT_OK) return rc;
    return bn == 128 ? launch<128, 4>(ma, mb, p, st) : launch<256, 4>(ma, mb, p, st);
}

bool shape_ok(int64_t rows, int in_f, int out_f) {
    return rows >= 0 && in_f > 0 && out_f > 0 && in_f % 8 == 0 && out_f % 8 == 0 && rows < (int64_t)INT32_MAX;
}

// Weight-gradient plan: rows cut into `splits` ranges of whole 64-row blocks so that the
// (out / 128) x (in / BN) tiles times the splits fill the SMs about twice; `chunks` row chunks for
// the bias gradient.
void wgrad_plan(int64_t rows, int in_f, int out_f, int sms, int *splits, int *kb_per, int *chunks) {
    const int bn = in_f <= 128 ? 128 : 256;
    const int tiles = ((out_f + BM - 1) / BM) * ((in_f + bn - 1) / bn);
    const int kb_total = (int)((rows + BK - 1) / BK);
    int s = (2 * sms + tiles - 1) / tiles;
    if (s > kb_total) s = kb_total;
    if (s < 1) s = 1;
    const int per = (kb_total + s - 1) / s;
    s = (kb_total + per - 1) / per;   // every split holds at least one block
    *splits = s;
    *kb_per = per;
    const int c = (int)((rows + 511) / 512);
    *chunks = c < 1 ? 1 : (c > 256 ? 256 : c);
}

}  // namespace

int gemm_bf16_timeouts(int *count) {
    if (cudaMemcpyFromSymbol(count, g_gemm_bf16_timeouts, sizeof(int)) != cudaSuccess) return NGT_ERR_CUDA;
    return NGT_OK;
}

}  // namespace ngt

using namespace ngt;

extern "C" int ngt_linear_bf16_forward(int64_t rows, int in_features, int out_features, const void *x,
                                       const void *weight, const void *bias, void *y, ngt_stream_t stream) {
    if (!shape_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    if (rows == 0) return NGT_OK;
    if (!x || !weight || !y) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(weight) || !aligned16(y)) return NGT_ERR_MISALIGNED;
    GemmArgs p{};
    p.M = rows;
    p.N = out_features;
    p.K = in_features;
    p.kb_total = (in_features + BK - 1) / BK;
    p.kb_per_split = p.kb_total;
    p.splits = 1;
    p.bias = static_cast<const __nv_bfloat16 *>(bias);
    p.bias_vec = bias != nullptr && aligned16(bias);
    p.out = y;
    p.mode = 0;
    return run(p, x, rows, in_features, weight, out_features, in_features, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ngt_linear_bf16_backward_input(int64_t rows, int in_features, int out_features, const void *dy,
                                              const void *weight, void *dx, ngt_stream_t stream) {
    if (!shape_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    if (rows == 0) return NGT_OK;
    if (!dy || !weight || !dx) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(dy) || !aligned16(weight) || !aligned16(dx)) return NGT_ERR_MISALIGNED;
    GemmArgs p{};
    p.M = rows;
    p.N = in_features;
    p.K = out_features;
    p.b_mn = 1;
    p.kb_total = (out_features + BK - 1) / BK;
    p.kb_per_split = p.kb_total;
    p.splits = 1;
    p.out = dx;
    p.mode = 0;
    // B(n = input feature, k = output feature) = W[k, n]: the weight as [out rows, in columns]
    return run(p, dy, rows, out_features, weight, out_features, in_features, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ngt_linear_bf16_weight_workspace_size(int64_t rows, int in_features, int out_features, size_t *bytes) {
    if (!bytes || !shape_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    int splits, per, chunks;
    wgrad_plan(rows < 1 ? 1 : rows, in_features, out_features, sm_count(), &splits, &per, &chunks);
    *bytes = sizeof(float) * ((size_t)splits * out_features * in_features + (size_t)chunks * out_features);
    return NGT_OK;
}

extern "C" int ngt_linear_bf16_backward_weight(int64_t rows, int in_features, int out_features, const void *x,
                                               const void *dy, void *dweight, void *dbias, void *workspace,
                                               size_t workspace_bytes, ngt_stream_t stream) {
    if (!shape_ok(rows, in_features, out_features) || !dweight) return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (rows == 0) {   // no rows: zero gradients
        if (cudaMemsetAsync(dweight, 0, (size_t)in_features * out_features * 2, st) != cudaSuccess) return NGT_ERR_CUDA;
        if (dbias && cudaMemsetAsync(dbias, 0, (size_t)out_features * 2, st) != cudaSuccess) return NGT_ERR_CUDA;
        return NGT_OK;
    }
    if (!x || !dy) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(dy) || !aligned16(dweight) || !aligned16(workspace)) return NGT_ERR_MISALIGNED;
    int splits, per, chunks;
    wgrad_plan(rows, in_features, out_features, sm_count(), &splits, &per, &chunks);
    const size_t need = sizeof(float) * ((size_t)splits * out_features * in_features + (size_t)chunks * out_features);
    if (!workspace || workspace_bytes < need) return NGT_ERR_WORKSPACE;
    float *part = static_cast<float *>(workspace);
    GemmArgs p{};
    p.M = out_features;
    p.N = in_features;
    p.K = (int)rows;
    p.a_mn = 1;
    p.b_mn = 1;
    p.kb_total = (int)((rows + BK - 1) / BK);
    p.kb_per_split = per;
    p.splits = splits;
    p.out = part;
    p.mode = 1;
    // A(m = output feature, k = row) = dy[row, m]; B(n = input feature, k = row) = x[row, n]
    int rc = run(p, dy, rows, out_features, x, rows, in_features, st);
    if (rc != NGT_OK) return rc;
    const int64_t count4 = (int64_t)out_features * in_features / 4;
    const int64_t blocks = (count4 + 255) / 256 < 4096 ? (count4 + 255) / 256 : 4096;
    split_sum_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(splits, count4, (int64_t)out_features * in_features, part,
                                                            static_cast<__nv_bfloat16 *>(dweight));
    NGT_CHECK_LAUNCH();
    if (dbias) {
        float *cpart = part + (size_t)splits * out_features * in_features;
        const int64_t per_chunk = (rows + chunks - 1) / chunks;
        colsum_part_kernel<<<dim3((out_features + 255) / 256, chunks), 256, 0, st>>>(
            rows, out_features, per_chunk, static_cast<const __nv_bfloat16 *>(dy), cpart);
        NGT_CHECK_LAUNCH();
        colsum_finish_kernel<<<(out_features + 255) / 256, 256, 0, st>>>(chunks, out_features, cpart,
                                                                         static_cast<__nv_bfloat16 *>(dbias));
        NGT_CHECK_LAUNCH();
    }
    return NGT_OK;
}
