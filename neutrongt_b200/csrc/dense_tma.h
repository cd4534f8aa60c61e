// Warp-specialised, TMA-fed dense attention kernels for head_dim <= 32 (dense_tma.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ngt {

int dense_fwd_tma(int64_t s, int heads, int head_dim, float scale, float score_scale, float drop_p, uint32_t seed,
                  const void *q, const void *k, const void *v, void *out, float *lse, float *ns, int *status,
                  cudaStream_t st);

int dense_bwd_tma(int64_t s, int heads, int head_dim, float scale, float drop_p, uint32_t seed, const void *q,
                  const void *k, const void *v, const void *dout, const float *lse, const float *delta, float *dq_acc,
                  void *dk, void *dv, int *status, cudaStream_t st);

}  // namespace ngt
