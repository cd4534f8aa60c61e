// Fixed-order sum of per-chunk partial vectors (sm_100a): out = sum over c < chunks of part[c],
// part[c] a vector of `total` floats (a multiple of 4, 16-byte aligned).  The first `split`
// floats go to out0, the rest to out1 (out1 may be null to drop them).
//
// A block of 8 warps owns 128 consecutive floats (a float4 per lane).  Warp w adds chunks
// w, w + 8, w + 16, ... in increasing order, 8 loads in flight at a time; warp 0 then adds the 8
// warp sums in warp order.  The order depends only on `chunks`, so results are bitwise
// reproducible run to run.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ngt {
namespace {

__device__ __forceinline__ void add4(float4 &s, const float4 &v) {
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
}

__global__ void __launch_bounds__(256)
    chunk_sum_kernel(int chunks, int64_t split, int64_t total, const float *__restrict__ part,
                     float *__restrict__ out0, float *__restrict__ out1) {
    __shared__ float4 red[8][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t f = ((int64_t)blockIdx.x * 32 + lane) * 4;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (f < total) {
        const float *p = part + f;
        int c = warp;
        for (; c + 56 < chunks; c += 64) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = __ldg(reinterpret_cast<const float4 *>(p + (size_t)(c + 8 * u) * total));
#pragma unroll
            for (int u = 0; u < 8; u++) add4(s, v[u]);
        }
        for (; c < chunks; c += 8) add4(s, __ldg(reinterpret_cast<const float4 *>(p + (size_t)c * total)));
    }
    red[warp][lane] = s;
    __syncthreads();
    if (warp != 0 || f >= total) return;
    float4 o = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; w++) add4(o, red[w][lane]);
    if (f < split) *reinterpret_cast<float4 *>(out0 + f) = o;
    else if (out1) *reinterpret_cast<float4 *>(out1 + (f - split)) = o;
}

inline void launch_chunk_sum(int chunks, int64_t split, int64_t total, const float *part, float *out0, float *out1,
                             cudaStream_t st) {
    const unsigned grid = (unsigned)((total / 4 + 31) / 32);
    chunk_sum_kernel<<<grid, 256, 0, st>>>(chunks, split, total, part, out0, out1);
}

}  // namespace
}  // namespace ngt
