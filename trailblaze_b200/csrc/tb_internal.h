// tb_internal.h — declarations shared between the library's translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tb {

// Launch the matvec d_y[M] = dequant(W) @ d_x[K] on `st`.  Returns 1 when the
// launch was issued, 0 for unsupported arguments or a launch error.
int mv_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_y,
              cudaStream_t st, int *d_err, int num_sms, uint32_t wait_limit);

// Launch the bit-exact dequantisation of M rows of K weights into d_out.
int dq_launch(const void *W, int qtype, int M, int K, float *d_out, int sem, cudaStream_t st);

// Raise a kernel's dynamic shared-memory limit once per device.
bool smem_attr_once(const void *kernel, int bytes);

}  // namespace tb
