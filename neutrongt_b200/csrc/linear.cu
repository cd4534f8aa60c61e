// fp32 Linear layers of the GT / Graphormer models: entry points, and the CUDA-core kernels (sm_100a):
//   forward       y  = x W^T + b               x [rows, in], W [out, in], y [rows, out]
//   input grad    dx = dy W                    dy [rows, out], dx [rows, in]
//   weight grad   dW = dy^T x, db = sum dy     dW [out, in], db [out]
//
// The models' windows are thin GEMMs: rows ~ 10^4, in / out 32..256.  The whole weight fits in
// shared memory and there are only ~70 rows per SM, so library tiles of 64..128 rows leave SMs
// idle, and the weight gradient (a 128 x 128 output reduced over 10^4 rows) runs on a handful of
// CTAs.  Both kernels here size their work to the SM count instead:
//
//  * row GEMM (forward, input grad): one CTA of 8 warps per SM and 128-column tile keeps the
//    tile's weight slice resident in shared memory and owns 16 * TR consecutive rows, TR chosen so
//    the rows spread evenly over the SMs.  Warps w and w + 4 (one SM sub-partition)
//    share columns 32w..32w+31 and split the 8-row slots between them; lane (rg, cg) computes
//    row rg of each of its slots x 8 columns.  The A operand streams through a 3-stage cp.async
//    ring of 32-wide k slices (rows padded to 36 floats so the 8 row groups hit distinct banks).
//  * weight grad: the rows are cut into one chunk per SM (per 128 x 128 output tile); a CTA's
//    256 threads each accumulate an 8 x 8 block of dW over the chunk (rows streamed through a
//    2-stage cp.async ring of 16-row slabs), and a share of db.  Per-chunk partials are summed in chunk order by
//    a second kernel, so dW and db are bitwise reproducible.
//
// fp32 FFMA throughout (no TF32), the precision of torch's fp32 Linear.  The forward and input
// grad with both dimensions <= 256 go to the split-TF32 tensor-core kernel of linear_tc.cu (same
// precision); the row GEMM keeps the wider outputs.  Reference layers: the
// models' nn.Linear (NeutronGT/models/gt_dist_node_level_single_window.py:235-237, 313-318, 361;
// graphormer_dist_node_level.py:179, 183, 286).
#include "chunk_sum.cuh"
#include "common.cuh"
#include "gemm_bf16.h"
#include "linear_tc.h"

namespace ngt {
namespace {

constexpr int kTileN = 128;        // output columns per CTA tile
constexpr int kSlice = 32;         // k columns per staged slice of the row GEMM
constexpr int kAStride = 36;       // padded row stride (floats) of a staged slice
constexpr int kStages = 3;         // cp.async ring depth of the row GEMM
// Row GEMM: two groups of 4 warps, so each SM sub-partition runs 2 warps.  (One group with up to
// 12 rows per lane balances shared-memory and FFMA cycles better on paper, but with one warp per
// sub-partition nothing hides the operand latency, and 2 CTAs no longer fit for 256-wide outputs;
// measured slower.)
constexpr int kHalves = 2;
constexpr int kRowThreads = 128 * kHalves;
constexpr int kMaxTR = 9;           // row GEMM: rows per lane
constexpr int kMaxInner = 256;     // row GEMM: inner dimension kept resident in shared memory
constexpr int kWgThreads = 256;    // weight grad: 16 x 16 threads, 8 x 8 outputs each
constexpr int kWgSlab = 16;        // rows per staged slab (weight grad); 2 x 2 x 8 KB static smem
#ifndef NGT_WGRAD_CTAS_PER_SM
#define NGT_WGRAD_CTAS_PER_SM 1
#endif
constexpr int kWgCtasPerSm = NGT_WGRAD_CTAS_PER_SM;   // row chunks per SM and output tile

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int src_bytes = valid ? 16 : 0;     // 0: zero-fill the 16 bytes, read nothing
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// acc[0..3] (as pairs) += a * (b0, b1): packed f32x2 FMAs, each lane rounded like fmaf
__device__ __forceinline__ void fma4x2(float2 (&acc)[4], float a, const float4 &b0, const float4 &b1) {
    const float2 aa = make_float2(a, a);
    acc[0] = __ffma2_rn(aa, make_float2(b0.x, b0.y), acc[0]);
    acc[1] = __ffma2_rn(aa, make_float2(b0.z, b0.w), acc[1]);
    acc[2] = __ffma2_rn(aa, make_float2(b1.x, b1.y), acc[2]);
    acc[3] = __ffma2_rn(aa, make_float2(b1.z, b1.w), acc[3]);
}

__device__ __forceinline__ float comp(const float4 &v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// ---------------------------------------------------------------------------------------------
// Row GEMM: C[M, N] = A[M, K] B[K, N] (+ bias).
//  TRANS (forward): B = W^T with W [N, K]; W's 128-row slice stays in its own layout in shared
//    memory, rows padded to kpad + 4 floats, and lane (rg, cg) of warp w owns the interleaved
//    columns 32w + cg + 4j (j < 8): for each j the 4 lanes of a row group read 4 consecutive W
//    rows, which the padding puts in distinct banks.  Stores are per column (the lane's columns
//    are not contiguous).
//  !TRANS (input grad): B = W with W [K, N]; slice [kpad][128], lane owns columns 32w + 8cg ..+7.
// Then kStages slices of A [16 * TR][kAStride].  During a CTA's first row tile the weight
// slice arrives k slice by k slice in the same cp.async groups as A, so the first FFMAs wait for
// 32 k rows of it, not all of it.  Inside a slice the k loop is rolled, one 4-wide k group per
// iteration, so the loop body stays in the instruction cache.
// ---------------------------------------------------------------------------------------------
template <bool TRANS>
__host__ __device__ constexpr int b_floats(int kpad) {
    return TRANS ? kTileN * (kpad + 4) : kpad * kTileN;
}

// Operands of one 4-wide k group: a[i] = A[row i][k..k+3]; TRANS: w[j] = W[col + 4j][k..k+3];
// !TRANS: w[2j], w[2j+1] = W[k + j][col..col+7].
template <int TRH, bool TRANS>
__device__ __forceinline__ void load_group(float4 (&a)[TRH], float4 (&w)[8], const float *as, const float *bsrc,
                                           int g, int wst) {
#pragma unroll
    for (int i = 0; i < TRH; i++) a[i] = *reinterpret_cast<const float4 *>(as + 8 * kHalves * i * kAStride + 4 * g);
    if (TRANS) {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = *reinterpret_cast<const float4 *>(bsrc + 4 * j * wst + 4 * g);
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            w[2 * j] = *reinterpret_cast<const float4 *>(bsrc + (4 * g + j) * kTileN);
            w[2 * j + 1] = *reinterpret_cast<const float4 *>(bsrc + (4 * g + j) * kTileN + 4);
        }
    }
}

template <int TRH, bool TRANS>
__device__ __forceinline__ void fma_group(float2 (&acc)[TRH][4], const float4 (&a)[TRH], const float4 (&w)[8]) {
    // acc[i][jp] holds the lane's columns 2jp, 2jp + 1.  The input-grad layout has column pairs
    // adjacent in w, so it uses packed f32x2 FMAs (each lane rounded like fmaf); the forward's
    // pairs would need repacking per k, which costs more than it saves, so it stays scalar.
    if (TRANS) {
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
#pragma unroll
            for (int i = 0; i < TRH; i++)
#pragma unroll
                for (int jp = 0; jp < 4; jp++) {
                    acc[i][jp].x = fmaf(comp(a[i], kk), comp(w[2 * jp], kk), acc[i][jp].x);
                    acc[i][jp].y = fmaf(comp(a[i], kk), comp(w[2 * jp + 1], kk), acc[i][jp].y);
                }
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int i = 0; i < TRH; i++) fma4x2(acc[i], comp(a[i], j), w[2 * j], w[2 * j + 1]);
    }
}

struct RowGemmArgs {
    int64_t M;
    int K, N;
    const float *A, *W, *bias;
    float *C;
};

// One row tile; lane rows r0 + rg + 8 * (half + kHalves * i), i < TRH.
template <int TRH, bool TRANS>
__device__ __forceinline__ void row_tile(const RowGemmArgs &p, float *Bs, float *As, int64_t r0, int RT, int n0,
                                         bool load_b, int half) {
    const int kpad = (p.K + kSlice - 1) / kSlice * kSlice;
    const int wst = kpad + 4;
    const int nk = kpad / kSlice;
    const int tid = threadIdx.x, warp = (tid >> 5) & 3, lane = tid & 31;
    const int rg = lane >> 2, cg = lane & 3;
    const int col = TRANS ? 32 * warp + cg : 32 * warp + 8 * cg;

    auto issue = [&](int kb) {
        if (kb < nk) {
            float *dst = As + (size_t)(kb % kStages) * RT * kAStride;
            for (int idx = tid; idx < RT * (kSlice / 4); idx += kRowThreads) {
                const int r = idx / (kSlice / 4), c = 4 * (idx % (kSlice / 4));
                const int64_t row = r0 + r;
                const int k = kb * kSlice + c;
                const bool ok = row < p.M && k < p.K;
                cp_async16(dst + r * kAStride + c, ok ? p.A + row * p.K + k : p.A, ok);
            }
            if (load_b) {   // the weight slice's k rows kb * 32 .. + 31, zero beyond K and N
                if (TRANS) {
                    for (int idx = tid; idx < kTileN * (kSlice / 4); idx += kRowThreads) {
                        const int n = idx / (kSlice / 4), k = kb * kSlice + 4 * (idx % (kSlice / 4));
                        const bool ok = n0 + n < p.N && k < p.K;
                        cp_async16(Bs + (size_t)n * wst + k, ok ? p.W + (size_t)(n0 + n) * p.K + k : p.W, ok);
                    }
                } else {
                    for (int idx = tid; idx < kSlice * (kTileN / 4); idx += kRowThreads) {
                        const int k = kb * kSlice + idx / (kTileN / 4), c = 4 * (idx % (kTileN / 4));
                        const bool ok = k < p.K && n0 + c < p.N;
                        cp_async16(Bs + (size_t)k * kTileN + c, ok ? p.W + (size_t)k * p.N + n0 + c : p.W, ok);
                    }
                }
            }
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);
    float2 acc[TRH > 0 ? TRH : 1][4];
#pragma unroll
    for (int i = 0; i < (TRH > 0 ? TRH : 1); i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = make_float2(0.f, 0.f);

    for (int kb = 0; kb < nk; kb++) {
        issue(kb + 2);
        cp_async_wait<2>();      // slice kb of A (and of the weight slice) have landed
        __syncthreads();
        if constexpr (TRH > 0) {
            const float *as = As + (size_t)(kb % kStages) * RT * kAStride + (rg + 8 * half) * kAStride;
            const float *bsrc = TRANS ? Bs + (size_t)col * wst + kb * kSlice : Bs + (size_t)kb * kSlice * kTileN + col;
#pragma unroll 1
            for (int g = 0; g < kSlice / 4; g++) {
                float4 a0[TRH], w0[8];
                load_group<TRH, TRANS>(a0, w0, as, bsrc, g, wst);
                fma_group<TRH, TRANS>(acc, a0, w0);
            }
        }
        __syncthreads();         // the stage is refilled two slices later
    }

    if constexpr (TRH > 0) {
        if (TRANS) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int c = n0 + col + 4 * j;
                if (c >= p.N) continue;
                const float bj = p.bias ? __ldg(p.bias + c) : 0.f;
#pragma unroll
                for (int i = 0; i < TRH; i++) {
                    const int64_t row = r0 + rg + 8 * (half + kHalves * i);
                    if (row < p.M) p.C[row * p.N + c] = ((j & 1) ? acc[i][j >> 1].y : acc[i][j >> 1].x) + bj;
                }
            }
        } else {
            const int c = n0 + col;
            float4 bb0 = make_float4(0.f, 0.f, 0.f, 0.f), bb1 = bb0;
            if (p.bias) {
                if (c < p.N) bb0 = __ldg(reinterpret_cast<const float4 *>(p.bias + c));
                if (c + 4 < p.N) bb1 = __ldg(reinterpret_cast<const float4 *>(p.bias + c + 4));
            }
#pragma unroll
            for (int i = 0; i < TRH; i++) {
                const int64_t row = r0 + rg + 8 * (half + kHalves * i);
                if (row >= p.M) continue;
                float *cr = p.C + row * p.N + c;
                if (c < p.N)
                    *reinterpret_cast<float4 *>(cr) = make_float4(acc[i][0].x + bb0.x, acc[i][0].y + bb0.y,
                                                                  acc[i][1].x + bb0.z, acc[i][1].y + bb0.w);
                if (c + 4 < p.N)
                    *reinterpret_cast<float4 *>(cr + 4) = make_float4(acc[i][2].x + bb1.x, acc[i][2].y + bb1.y,
                                                                      acc[i][3].x + bb1.z, acc[i][3].y + bb1.w);
            }
        }
    }
}

// A CTA owns RT = 8 * kHalves * TR rows per row tile; warp group h (warps 4h..4h+3) takes the
// 8-row slots h, h + kHalves, ... (TR each, so all groups run one code path).
template <int TR, bool TRANS>
__global__ void __launch_bounds__(kRowThreads, 1)
    row_gemm_kernel(RowGemmArgs p, int col_tiles, int64_t row_tiles) {
    extern __shared__ __align__(16) float smem[];
    const int kpad = (p.K + kSlice - 1) / kSlice * kSlice;
    float *Bs = smem;
    float *As = smem + b_floats<TRANS>(kpad);
    const int half = threadIdx.x >> 7;
    const int ct = blockIdx.x % col_tiles;
    const int64_t slot = blockIdx.x / col_tiles, nslots = gridDim.x / col_tiles;
    const int n0 = ct * kTileN;
    const int RT = 8 * kHalves * TR;
    bool load_b = true;
    for (int64_t t = slot; t < row_tiles; t += nslots) {
        row_tile<TR, TRANS>(p, Bs, As, t * RT, RT, n0, load_b, half);
        load_b = false;
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------------------------------------
// Weight grad, pass 1: part[chunk] = (dy^T x over the chunk's rows, sum of dy over those rows).
// part layout per chunk: [N * K] dW partial, then [N] db partial.  Thread (ty, tx) of 16 x 16
// owns dW rows n0 + {4ty..4ty+3, 64+4ty..64+4ty+3} x columns k0 + {4tx.., 64+4tx..}; threads
// with tx < 8 also sum dy column n0 + (tx < 4 ? 4ty + tx : 60 + 4ty + tx) for db.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kWgThreads, kWgCtasPerSm)
    wgrad_partial_kernel(int64_t M, int K, int N, const float *__restrict__ x, const float *__restrict__ dy,
                         float *__restrict__ part, int64_t rows_per_chunk, int k_tiles) {
    __shared__ __align__(16) float Gs[2][kWgSlab][kTileN];
    __shared__ __align__(16) float Xs[2][kWgSlab][kTileN];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int chunk = blockIdx.x;
    const int nt = blockIdx.y / k_tiles, kt = blockIdx.y % k_tiles;
    const int n0 = nt * kTileN, k0 = kt * kTileN;
    const int64_t rb = (int64_t)chunk * rows_per_chunk;
    const int64_t re = rb + rows_per_chunk < M ? rb + rows_per_chunk : M;
    const int nslabs = (int)((re - rb + kWgSlab - 1) / kWgSlab);

    auto issue = [&](int s) {
        if (s < nslabs) {
            const int b = s & 1;
            for (int idx = tid; idx < 2 * kWgSlab * (kTileN / 4); idx += kWgThreads) {
                const int m = idx / (kWgSlab * (kTileN / 4));
                const int rem = idx % (kWgSlab * (kTileN / 4));
                const int r = rem / (kTileN / 4), c = 4 * (rem % (kTileN / 4));
                const int64_t row = rb + (int64_t)s * kWgSlab + r;
                if (m == 0) {
                    const bool ok = row < re && n0 + c < N;
                    cp_async16(&Gs[b][r][c], ok ? dy + row * N + n0 + c : dy, ok);
                } else {
                    const bool ok = row < re && k0 + c < K;
                    cp_async16(&Xs[b][r][c], ok ? x + row * K + k0 + c : x, ok);
                }
            }
        }
        cp_async_commit();
    };

    float2 acc[8][4];     // acc[i][jp] = dW entries (i, 2jp) and (i, 2jp + 1) of the thread's 8 x 8 block
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = make_float2(0.f, 0.f);
    float dbacc = 0.f;
    const bool db_lane = kt == 0 && tx < 8;
    const int db_col = (tx & 7) < 4 ? 4 * ty + (tx & 7) : 60 + 4 * ty + (tx & 7);   // tx >= 8: a db lane's column

    issue(0);
    for (int s = 0; s < nslabs; s++) {
        issue(s + 1);
        cp_async_wait<1>();
        __syncthreads();
        const int b = s & 1;
        const int64_t left = re - (rb + (int64_t)s * kWgSlab);
        const int nrows = left < kWgSlab ? (int)left : kWgSlab;
        // two register sets ping-pong: row r + 1's operands load while row r's FFMAs run.  An odd
        // row count processes one zero-filled row (past the chunk end) as the pair's second row.
        float4 ga0, ga1, xa0, xa1, gb0, gb1, xb0, xb1;
        float gda, gdb;
        auto load_row = [&](int r, float4 &g0, float4 &g1, float4 &x0, float4 &x1, float &gd) {
            g0 = *reinterpret_cast<const float4 *>(&Gs[b][r][4 * ty]);
            g1 = *reinterpret_cast<const float4 *>(&Gs[b][r][64 + 4 * ty]);
            x0 = *reinterpret_cast<const float4 *>(&Xs[b][r][4 * tx]);
            x1 = *reinterpret_cast<const float4 *>(&Xs[b][r][64 + 4 * tx]);
            gd = Gs[b][r][db_col];
        };
        auto fma_row = [&](const float4 &g0, const float4 &g1, const float4 &x0, const float4 &x1) {
            fma4x2(acc[0], g0.x, x0, x1);
            fma4x2(acc[1], g0.y, x0, x1);
            fma4x2(acc[2], g0.z, x0, x1);
            fma4x2(acc[3], g0.w, x0, x1);
            fma4x2(acc[4], g1.x, x0, x1);
            fma4x2(acc[5], g1.y, x0, x1);
            fma4x2(acc[6], g1.z, x0, x1);
            fma4x2(acc[7], g1.w, x0, x1);
        };
        load_row(0, ga0, ga1, xa0, xa1, gda);
#pragma unroll 1
        for (int r = 0; r < nrows; r += 2) {
            load_row(r + 1, gb0, gb1, xb0, xb1, gdb);
            fma_row(ga0, ga1, xa0, xa1);
            dbacc += gda;                         // kept only by the db lanes
            load_row(r + 2 < kWgSlab ? r + 2 : r + 1, ga0, ga1, xa0, xa1, gda);
            fma_row(gb0, gb1, xb0, xb1);
            dbacc += gdb;
        }
        __syncthreads();
    }
    cp_async_wait<0>();

    float *p = part + (size_t)chunk * ((size_t)N * K + N);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int n = n0 + (i < 4 ? 4 * ty + i : 60 + 4 * ty + i);
        if (n >= N) continue;
        float *pr = p + (size_t)n * K + k0;
        if (k0 + 4 * tx < K)
            *reinterpret_cast<float4 *>(pr + 4 * tx) = make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
        if (k0 + 64 + 4 * tx < K)
            *reinterpret_cast<float4 *>(pr + 64 + 4 * tx) =
                make_float4(acc[i][2].x, acc[i][2].y, acc[i][3].x, acc[i][3].y);
    }
    if (db_lane && n0 + db_col < N) p[(size_t)N * K + n0 + db_col] = dbacc;
}

int sm_count() {
    static int count[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        count[dev] = n;
    }
    return count[dev];
}

template <bool TRANS>
size_t row_gemm_smem(int slots, int K) {
    const int kpad = (K + kSlice - 1) / kSlice * kSlice;
    return sizeof(float) * ((size_t)b_floats<TRANS>(kpad) + (size_t)kStages * 8 * slots * kAStride);
}

template <int TR, bool TRANS>
int launch_row_gemm_t(int64_t M, int K, int N, const float *A, const float *W, const float *bias, float *C,
                      cudaStream_t st) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = row_gemm_smem<TRANS>(kHalves * TR, kMaxInner);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(row_gemm_kernel<TR, TRANS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return NGT_ERR_CUDA;
        attr_set[dev] = true;
    }
    const int col_tiles = (N + kTileN - 1) / kTileN;
    const int64_t rt = 8 * kHalves * TR;
    const int64_t row_tiles = (M + rt - 1) / rt;
    int64_t ctas = sm_count() / col_tiles;
    if (ctas < 1) ctas = 1;
    if (ctas > row_tiles) ctas = row_tiles;
    const unsigned grid = (unsigned)(ctas * col_tiles);
    RowGemmArgs p{M, K, N, A, W, bias, C};
    row_gemm_kernel<TR, TRANS><<<grid, kRowThreads, row_gemm_smem<TRANS>(kHalves * TR, K), st>>>(p, col_tiles,
                                                                                              row_tiles);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

template <bool TRANS>
int launch_row_gemm(int64_t M, int K, int N, const float *A, const float *W, const float *bias, float *C,
                    cudaStream_t st) {
    // 8-row slots per CTA: spread M over one CTA per SM (col_tiles CTAs share a row range), at
    // most kMaxTR rows per lane (then CTAs loop over row tiles)
    const int col_tiles = (N + kTileN - 1) / kTileN;
    int64_t ctas = sm_count() / col_tiles;
    if (ctas < 1) ctas = 1;
    const int64_t per_cta = (M + ctas - 1) / ctas;
    int tr = (int)((per_cta + 8 * kHalves - 1) / (8 * kHalves));     // rows per lane
    tr = tr < 1 ? 1 : tr > kMaxTR ? kMaxTR : tr;
    switch (tr) {
    case 1: return launch_row_gemm_t<1, TRANS>(M, K, N, A, W, bias, C, st);
    case 2: return launch_row_gemm_t<2, TRANS>(M, K, N, A, W, bias, C, st);
    case 3: return launch_row_gemm_t<3, TRANS>(M, K, N, A, W, bias, C, st);
    case 4: return launch_row_gemm_t<4, TRANS>(M, K, N, A, W, bias, C, st);
    case 5: return launch_row_gemm_t<5, TRANS>(M, K, N, A, W, bias, C, st);
    case 6: return launch_row_gemm_t<6, TRANS>(M, K, N, A, W, bias, C, st);
    case 7: return launch_row_gemm_t<7, TRANS>(M, K, N, A, W, bias, C, st);
    case 8: return launch_row_gemm_t<8, TRANS>(M, K, N, A, W, bias, C, st);
    default: return launch_row_gemm_t<9, TRANS>(M, K, N, A, W, bias, C, st);
    }
}

struct WgradPlan {
    int64_t chunks, rows_per_chunk;
    int n_tiles, k_tiles;
};

WgradPlan wgrad_plan(int64_t rows, int in_features, int out_features) {
    WgradPlan p;
    p.n_tiles = (out_features + kTileN - 1) / kTileN;
    p.k_tiles = (in_features + kTileN - 1) / kTileN;
    int64_t chunks = (int64_t)sm_count() * kWgCtasPerSm / (p.n_tiles * p.k_tiles);
    const int64_t max_chunks = (rows + kWgSlab - 1) / kWgSlab;
    if (chunks > max_chunks) chunks = max_chunks;
    if (chunks < 1) chunks = 1;
    p.rows_per_chunk = (rows + chunks - 1) / chunks;
    if (p.rows_per_chunk < 1) p.rows_per_chunk = 1;
    p.chunks = (rows + p.rows_per_chunk - 1) / p.rows_per_chunk;
    if (p.chunks < 1) p.chunks = 1;
    return p;
}

// Row ranges of the tensor-core weight grad: a multiple of 16 rows each, about one CTA per four SMs
// and output tile (the weight grads run on a side stream beside the input-grad chain, where fewer,
// longer CTAs overlap it best: GT epoch 28.0 ms with one CTA per SM, 27.0-27.1 with one per four,
// 27.5 with one per two, 30.0 with one per eight), at least 64 rows, and at most 512 rows so that no
// range accumulates a long chain of products in one fp32 accumulator (the ranges are summed in a
// fixed order afterwards).
struct TcWgradPlan {
    int64_t splits, rows_per_split;
};

TcWgradPlan tc_wgrad_plan(int64_t rows, int out_features) {
    const int64_t m_tiles = (out_features + 127) / 128;
    int64_t splits = sm_count() / (4 * m_tiles);
    if (splits > rows / 64) splits = rows / 64;
    if (splits < (rows + 511) / 512) splits = (rows + 511) / 512;
    if (splits < 1) splits = 1;
    TcWgradPlan p;
    p.rows_per_split = ((rows + splits - 1) / splits + 15) / 16 * 16;
    p.splits = (rows + p.rows_per_split - 1) / p.rows_per_split;
    return p;
}

bool use_tc_wgrad(int64_t rows, int in_features, int out_features) {
    return rows >= 64 && wgrad_tc_supported(in_features, out_features);
}

bool dims_ok(int64_t rows, int in_features, int out_features) {
    return rows >= 0 && rows < ((int64_t)1 << 40) && in_features > 0 && out_features > 0 && in_features % 4 == 0 &&
           out_features % 4 == 0;
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_linear_forward(int64_t rows, int in_features, int out_features, const float *x,
                                  const float *weight, const float *bias, float *y, ngt_stream_t stream) {
    if (!dims_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    if (in_features > kMaxInner) return NGT_ERR_UNSUPPORTED;
    if (rows == 0) return NGT_OK;
    if (!x || !weight || !y) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(weight) || !aligned16(y) || (bias && !aligned16(bias))) return NGT_ERR_MISALIGNED;
    if (linear_tc_supported(in_features, out_features))
        return launch_linear_tc(rows, in_features, out_features, x, weight, false, bias, y,
                                reinterpret_cast<cudaStream_t>(stream));
    return launch_row_gemm<true>(rows, in_features, out_features, x, weight, bias, y,
                                 reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ngt_linear_backward_input(int64_t rows, int in_features, int out_features, const float *dy,
                                         const float *weight, float *dx, ngt_stream_t stream) {
    if (!dims_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    if (out_features > kMaxInner) return NGT_ERR_UNSUPPORTED;
    if (rows == 0) return NGT_OK;
    if (!dy || !weight || !dx) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(dy) || !aligned16(weight) || !aligned16(dx)) return NGT_ERR_MISALIGNED;
    if (linear_tc_supported(out_features, in_features))
        return launch_linear_tc(rows, out_features, in_features, dy, weight, true, nullptr, dx,
                                reinterpret_cast<cudaStream_t>(stream));
    return launch_row_gemm<false>(rows, out_features, in_features, dy, weight, nullptr, dx,
                                  reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ngt_linear_weight_workspace_size(int64_t rows, int in_features, int out_features, size_t *bytes) {
    if (!bytes || !dims_ok(rows, in_features, out_features)) return NGT_ERR_INVALID_ARGUMENT;
    const WgradPlan p = wgrad_plan(rows, in_features, out_features);
    int64_t parts = p.chunks;
    if (use_tc_wgrad(rows, in_features, out_features)) {
        const TcWgradPlan t = tc_wgrad_plan(rows, out_features);
        if (t.splits > parts) parts = t.splits;
    }
    *bytes = sizeof(float) * (size_t)parts * ((size_t)in_features * out_features + out_features);
    return NGT_OK;
}

extern "C" int ngt_linear_backward_weight(int64_t rows, int in_features, int out_features, const float *x,
                                          const float *dy, float *dweight, float *dbias, void *workspace,
                                          size_t workspace_bytes, ngt_stream_t stream) {
    if (!dims_ok(rows, in_features, out_features) || !dweight) return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t nk = (int64_t)in_features * out_features;
    if (rows == 0) {
        cudaMemsetAsync(dweight, 0, sizeof(float) * nk, st);
        if (dbias) cudaMemsetAsync(dbias, 0, sizeof(float) * out_features, st);
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    if (!x || !dy || !workspace) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(dy) || !aligned16(dweight) || !aligned16(workspace) ||
        (dbias && !aligned16(dbias)))
        return NGT_ERR_MISALIGNED;
    size_t need = 0;
    ngt_linear_weight_workspace_size(rows, in_features, out_features, &need);
    if (workspace_bytes < need) return NGT_ERR_WORKSPACE;
    const WgradPlan p = wgrad_plan(rows, in_features, out_features);
    float *part = static_cast<float *>(workspace);
    if (use_tc_wgrad(rows, in_features, out_features)) {   // split-TF32 tensor-core GEMM per row range
        const TcWgradPlan t = tc_wgrad_plan(rows, out_features);
        const int rc = launch_wgrad_tc(rows, in_features, out_features, x, dy, part, t.splits, t.rows_per_split, st);
        if (rc != NGT_OK) return rc;
        launch_chunk_sum((int)t.splits, nk, nk + out_features, part, dweight, dbias, st);
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    wgrad_partial_kernel<<<dim3((unsigned)p.chunks, (unsigned)(p.n_tiles * p.k_tiles)), kWgThreads, 0, st>>>(
        rows, in_features, out_features, x, dy, part, p.rows_per_chunk, p.k_tiles);
    launch_chunk_sum((int)p.chunks, nk, nk + out_features, part, dweight, dbias, st);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_linear_status(int32_t *timeouts) {
    if (!timeouts) return NGT_ERR_INVALID_ARGUMENT;
    int n = 0, m = 0;
    int rc = linear_tc_timeouts(&n);
    if (rc == NGT_OK) rc = gemm_bf16_timeouts(&m);
    *timeouts = n + m;
    return rc;
}
