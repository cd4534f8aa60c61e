// bf16 tensor-core Linear GEMMs (gemm_bf16.cu).
#pragma once

namespace ngt {

// Number of bf16 GEMM CTAs whose bounded waits ran out since the library was loaded (synchronous).
int gemm_bf16_timeouts(int *count);

}  // namespace ngt
