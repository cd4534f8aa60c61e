// Split-TF32 tensor-core Linear GEMMs (linear_tc.cu), called by the Linear entry points of linear.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ngt {

// Output columns N <= 256, K and N multiples of 4.
bool linear_tc_supported(int K, int N);

// C[M, N] = A[M, K] B^T (+ bias), with B(n, k) = W[n * K + k] (trans_w false: W is [N, K]) or
// W[k * N + n] (trans_w true: W is [K, N]).  All pointers 16-byte aligned.
int launch_linear_tc(int64_t M, int K, int N, const float *A, const float *W, bool trans_w, const float *bias,
                     float *C, cudaStream_t st);

// Weight grad on the same kernel: part[z] = (dy^T x over rows [z * rows_per_split, ...), the sums
// of dy over those rows) for z < splits, laid out as [out * in] then [out] per split, for a
// fixed-order sum of the splits.  in_features <= 256; rows_per_split a multiple of 16 and
// splits = ceil(rows / rows_per_split).
bool wgrad_tc_supported(int in_features, int out_features);
int launch_wgrad_tc(int64_t rows, int in_features, int out_features, const float *x, const float *dy, float *part,
                    int64_t splits, int64_t rows_per_split, cudaStream_t st);

// Number of CTAs whose bounded waits ran out since the library was loaded (synchronous copy).
int linear_tc_timeouts(int *count);

}  // namespace ngt
