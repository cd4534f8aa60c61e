// Row-wise fp32 operators of the GT / Graphormer layers (sm_100a): LayerNorm forward and backward
// and the column sum that gives a Linear layer's bias gradient.
//
// The models' windows are [rows ~ 10^4, cols 64..1024] fp32.  torch's generic kernels take
// 15-60 us per call at this shape (launch-shaped rather than bandwidth-shaped); these move the
// same bytes in a few microseconds.  Column sums are reduced in a fixed order (per-block partials,
// then one pass over the partials), so results do not depend on scheduling.
//
// Reference: the models' nn.LayerNorm and nn.Linear layers
// (NeutronGT/models/gt_dist_node_level_single_window.py:239-241, 311-325, 360-361, 537, 565;
// graphormer_dist_node_level.py:179, 183, 286).
#include "chunk_sum.cuh"
#include "common.cuh"

namespace ngt {
namespace {

constexpr int kRowThreads = 256;             // 8 warps, one row per warp
constexpr int kColThreads = 256;             // column-sum blocks
constexpr int kRowsPerPartial = 32;          // rows summed by one block of the column-sum kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Lane l of a warp holds columns 4l + 128j (j < VPL) as float4.
template <int VPL>
__global__ void __launch_bounds__(kRowThreads)
    layernorm_fwd_kernel(int64_t rows, int cols, const float *__restrict__ x, const float *__restrict__ gamma,
                         const float *__restrict__ beta, float eps, float *__restrict__ y, float *__restrict__ mean,
                         float *__restrict__ rstd) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *xr = x + row * cols;
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; j++) {
        const int c = 4 * lane + 128 * j;
        v[j] = c < cols ? *reinterpret_cast<const float4 *>(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    const float mu = warp_sum(s) / (float)cols;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; j++) {
        const int c = 4 * lane + 128 * j;
        if (c < cols) {
            const float a = v[j].x - mu, b = v[j].y - mu, cc = v[j].z - mu, d = v[j].w - mu;
            q += (a * a + b * b) + (cc * cc + d * d);
        }
    }
    const float r = rsqrtf(warp_sum(q) / (float)cols + eps);
    float *yr = y + row * cols;
#pragma unroll
    for (int j = 0; j < VPL; j++) {
        const int c = 4 * lane + 128 * j;
        if (c < cols) {
            const float4 g = *reinterpret_cast<const float4 *>(gamma + c);
            const float4 bb = *reinterpret_cast<const float4 *>(beta + c);
            float4 o;
            o.x = (v[j].x - mu) * r * g.x + bb.x;
            o.y = (v[j].y - mu) * r * g.y + bb.y;
            o.z = (v[j].z - mu) * r * g.z + bb.z;
            o.w = (v[j].w - mu) * r * g.w + bb.w;
            *reinterpret_cast<float4 *>(yr + c) = o;
        }
    }
    if (lane == 0) {
        mean[row] = mu;
        rstd[row] = r;
    }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * gamma; per-block partial column sums
// of dy * xhat and dy go to part[blockIdx.x][2][cols] (a block's 8 warps take rows warp, warp + 8,
// ... of its kRowsPerPartial rows).  A warp loads kBatch rows before computing them, so their
// loads overlap; rows are still added to the partials in row order.
template <int VPL>
__global__ void __launch_bounds__(kRowThreads)
    layernorm_bwd_kernel(int64_t rows, int cols, const float *__restrict__ x, const float *__restrict__ dy,
                         const float *__restrict__ gamma, const float *__restrict__ mean,
                         const float *__restrict__ rstd, float *__restrict__ dx, float *__restrict__ part) {
    constexpr int kWarps = kRowThreads / 32;
    constexpr int kBatch = VPL >= 4 ? 1 : 4 / VPL;
    __shared__ float4 red[2][kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float4 ag[VPL], ab[VPL], gm[VPL];
#pragma unroll
    for (int j = 0; j < VPL; j++) {
        const int c = 4 * lane + 128 * j;
        ag[j] = ab[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        gm[j] = c < cols ? __ldg(reinterpret_cast<const float4 *>(gamma + c)) : ag[j];
    }
    const int64_t base = (int64_t)blockIdx.x * kRowsPerPartial + warp;
    for (int k0 = 0; k0 < kRowsPerPartial / kWarps; k0 += kBatch) {
        float mu[kBatch], r[kBatch];
        float4 xv[kBatch][VPL], d[kBatch][VPL];
#pragma unroll
        for (int u = 0; u < kBatch; u++) {          // loads of the batch (zero past the last row)
            const int64_t row = base + (int64_t)(k0 + u) * kWarps;
            const bool ok = row < rows;
            mu[u] = ok ? mean[row] : 0.f;
            r[u] = ok ? rstd[row] : 0.f;
#pragma unroll
            for (int j = 0; j < VPL; j++) {
                const int c = 4 * lane + 128 * j;
                const bool okc = ok && c < cols;
                xv[u][j] = okc ? *reinterpret_cast<const float4 *>(x + row * cols + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                d[u][j] = okc ? *reinterpret_cast<const float4 *>(dy + row * cols + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; u++) {
            const int64_t row = base + (int64_t)(k0 + u) * kWarps;
            float4 xh[VPL], g[VPL];
            float s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int j = 0; j < VPL; j++) {
                const float4 &dv = d[u][j];
                xh[j] = make_float4((xv[u][j].x - mu[u]) * r[u], (xv[u][j].y - mu[u]) * r[u],
                                    (xv[u][j].z - mu[u]) * r[u], (xv[u][j].w - mu[u]) * r[u]);
                g[j] = make_float4(dv.x * gm[j].x, dv.y * gm[j].y, dv.z * gm[j].z, dv.w * gm[j].w);
                s1 += (g[j].x + g[j].y) + (g[j].z + g[j].w);
                s2 += (g[j].x * xh[j].x + g[j].y * xh[j].y) + (g[j].z * xh[j].z + g[j].w * xh[j].w);
                ag[j].x += dv.x * xh[j].x;
                ag[j].y += dv.y * xh[j].y;
                ag[j].z += dv.z * xh[j].z;
                ag[j].w += dv.w * xh[j].w;
                ab[j].x += dv.x;
                ab[j].y += dv.y;
                ab[j].z += dv.z;
                ab[j].w += dv.w;
            }
            const float a = warp_sum(s1) / (float)cols, b = warp_sum(s2) / (float)cols;
            if (row < rows) {
#pragma unroll
                for (int j = 0; j < VPL; j++) {
                    const int c = 4 * lane + 128 * j;
                    if (c < cols) {
                        float4 o;
                        o.x = r[u] * (g[j].x - a - xh[j].x * b);
                        o.y = r[u] * (g[j].y - a - xh[j].y * b);
                        o.z = r[u] * (g[j].z - a - xh[j].z * b);
                        o.w = r[u] * (g[j].w - a - xh[j].w * b);
                        *reinterpret_cast<float4 *>(dx + row * cols + c) = o;
                    }
                }
            }
        }
    }
    // the warps' partials are added in warp order, one column group at a time
#pragma unroll
    for (int j = 0; j < VPL; j++) {
        red[0][warp][lane] = ag[j];
        red[1][warp][lane] = ab[j];
        __syncthreads();
        if (warp == 0) {
            const int c = 4 * lane + 128 * j;
            float4 tg = red[0][0][lane], tb = red[1][0][lane];
            for (int w = 1; w < kWarps; w++) {
                const float4 ug = red[0][w][lane], ub = red[1][w][lane];
                tg.x += ug.x; tg.y += ug.y; tg.z += ug.z; tg.w += ug.w;
                tb.x += ub.x; tb.y += ub.y; tb.z += ub.z; tb.w += ub.w;
            }
            if (c < cols) {
                *reinterpret_cast<float4 *>(part + ((size_t)blockIdx.x * 2) * cols + c) = tg;
                *reinterpret_cast<float4 *>(part + ((size_t)blockIdx.x * 2 + 1) * cols + c) = tb;
            }
        }
        __syncthreads();
    }
}

// part[blockIdx.x][c] = sum of x[r][c] over the block's kRowsPerPartial rows, in row order.
__global__ void __launch_bounds__(kColThreads)
    column_partial_kernel(int64_t rows, int cols, const float *__restrict__ x, float *__restrict__ part) {
    const int c = blockIdx.y * kColThreads + threadIdx.x;
    if (c >= cols) return;
    const int64_t r0 = (int64_t)blockIdx.x * kRowsPerPartial;
    const int64_t r1 = r0 + kRowsPerPartial < rows ? r0 + kRowsPerPartial : rows;
    float s = 0.f;
#pragma unroll 8
    for (int64_t r = r0; r < r1; r++) s += x[r * cols + c];
    part[(size_t)blockIdx.x * cols + c] = s;
}

template <int VPL>
void launch_ln_fwd(int64_t rows, int cols, const float *x, const float *g, const float *b, float eps, float *y,
                   float *mean, float *rstd, cudaStream_t st) {
    const unsigned grid = (unsigned)((rows + kRowThreads / 32 - 1) / (kRowThreads / 32));
    layernorm_fwd_kernel<VPL><<<grid, kRowThreads, 0, st>>>(rows, cols, x, g, b, eps, y, mean, rstd);
}

template <int VPL>
void launch_ln_bwd(int64_t rows, int cols, const float *x, const float *dy, const float *g, const float *mean,
                   const float *rstd, float *dx, float *part, cudaStream_t st) {
    const unsigned grid = (unsigned)((rows + kRowsPerPartial - 1) / kRowsPerPartial);
    layernorm_bwd_kernel<VPL><<<grid, kRowThreads, 0, st>>>(rows, cols, x, dy, g, mean, rstd, dx, part);
}

int vpl_of(int cols) { return (cols + 127) / 128; }

bool shape_ok(int64_t rows, int cols) {
    return rows >= 0 && cols > 0 && cols % 4 == 0 && cols <= 1024 && rows < ((int64_t)1 << 40);
}

}  // namespace
}  // namespace ngt

using namespace ngt;

extern "C" int ngt_rowops_workspace_size(int64_t rows, int cols, size_t *bytes) {
    if (!bytes || rows < 0 || cols <= 0) return NGT_ERR_INVALID_ARGUMENT;
    const int64_t nb = (rows + kRowsPerPartial - 1) / kRowsPerPartial;
    *bytes = sizeof(float) * (size_t)(nb > 0 ? nb : 1) * 2 * (size_t)cols;
    return NGT_OK;
}

extern "C" int ngt_layernorm_forward(int64_t rows, int cols, const float *x, const float *gamma, const float *beta,
                                     float eps, float *y, float *mean, float *rstd, ngt_stream_t stream) {
    if (!shape_ok(rows, cols)) return cols > 1024 || (cols > 0 && cols % 4) ? NGT_ERR_UNSUPPORTED
                                                                            : NGT_ERR_INVALID_ARGUMENT;
    if (rows == 0) return NGT_OK;
    if (!x || !gamma || !beta || !y || !mean || !rstd) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(gamma) || !aligned16(beta) || !aligned16(y)) return NGT_ERR_MISALIGNED;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (vpl_of(cols)) {
    case 1: launch_ln_fwd<1>(rows, cols, x, gamma, beta, eps, y, mean, rstd, st); break;
    case 2: launch_ln_fwd<2>(rows, cols, x, gamma, beta, eps, y, mean, rstd, st); break;
    case 3:
    case 4: launch_ln_fwd<4>(rows, cols, x, gamma, beta, eps, y, mean, rstd, st); break;
    default: launch_ln_fwd<8>(rows, cols, x, gamma, beta, eps, y, mean, rstd, st); break;
    }
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_layernorm_backward(int64_t rows, int cols, const float *x, const float *dy, const float *gamma,
                                      const float *mean, const float *rstd, float *dx, float *dgamma, float *dbeta,
                                      void *workspace, size_t workspace_bytes, ngt_stream_t stream) {
    if (!shape_ok(rows, cols)) return cols > 1024 || (cols > 0 && cols % 4) ? NGT_ERR_UNSUPPORTED
                                                                            : NGT_ERR_INVALID_ARGUMENT;
    if (!dgamma || !dbeta) return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (rows == 0) {
        cudaMemsetAsync(dgamma, 0, sizeof(float) * cols, st);
        cudaMemsetAsync(dbeta, 0, sizeof(float) * cols, st);
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    if (!x || !dy || !gamma || !mean || !rstd || !dx || !workspace) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(x) || !aligned16(dy) || !aligned16(gamma) || !aligned16(dx) || !aligned16(workspace) ||
        !aligned16(dgamma) || !aligned16(dbeta))
        return NGT_ERR_MISALIGNED;
    size_t need = 0;
    ngt_rowops_workspace_size(rows, cols, &need);
    if (workspace_bytes < need) return NGT_ERR_WORKSPACE;
    float *part = static_cast<float *>(workspace);
    switch (vpl_of(cols)) {
    case 1: launch_ln_bwd<1>(rows, cols, x, dy, gamma, mean, rstd, dx, part, st); break;
    case 2: launch_ln_bwd<2>(rows, cols, x, dy, gamma, mean, rstd, dx, part, st); break;
    case 3:
    case 4: launch_ln_bwd<4>(rows, cols, x, dy, gamma, mean, rstd, dx, part, st); break;
    default: launch_ln_bwd<8>(rows, cols, x, dy, gamma, mean, rstd, dx, part, st); break;
    }
    const int nb = (int)((rows + kRowsPerPartial - 1) / kRowsPerPartial);
    launch_chunk_sum(nb, cols, 2 * (int64_t)cols, part, dgamma, dbeta, st);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}

extern "C" int ngt_column_sum(int64_t rows, int cols, const float *x, float *out, void *workspace,
                              size_t workspace_bytes, ngt_stream_t stream) {
    if (rows < 0 || cols <= 0 || !out) return NGT_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (rows == 0) {
        cudaMemsetAsync(out, 0, sizeof(float) * cols, st);
        NGT_CHECK_LAUNCH();
        return NGT_OK;
    }
    if (!x || !workspace) return NGT_ERR_INVALID_ARGUMENT;
    if (!aligned16(out) || !aligned16(workspace)) return NGT_ERR_MISALIGNED;
    size_t need = 0;
    ngt_rowops_workspace_size(rows, cols, &need);
    if (workspace_bytes < need) return NGT_ERR_WORKSPACE;
    const int nb = (int)((rows + kRowsPerPartial - 1) / kRowsPerPartial);
    float *part = static_cast<float *>(workspace);
    column_partial_kernel<<<dim3((unsigned)nb, (unsigned)((cols + kColThreads - 1) / kColThreads)), kColThreads, 0,
                            st>>>(rows, cols, x, part);
    launch_chunk_sum(nb, cols, cols, part, out, nullptr, st);
    NGT_CHECK_LAUNCH();
    return NGT_OK;
}
