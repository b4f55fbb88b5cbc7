// Launchers of the dense-member kernels (iqk_dense.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace iqk {

cudaError_t launch_dense_dequant(int member, const void *const *streams, int n, int64_t row_start,
                                 int64_t rows, void *dst, int out_dtype, cudaStream_t stream,
                                 int num_sms);
cudaError_t launch_dense_gemv(int member, const void *const *streams, int n, int out,
                              const void *x, int tokens, void *y, int y_dtype,
                              cudaStream_t stream);

}  // namespace iqk
