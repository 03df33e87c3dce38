// Tensor-parallel helpers (tp.cu) used by the runner.
#pragma once

#include "axb_common.cuh"

namespace axb {
int tp_allreduce(void* comm, void* buf, size_t count, int op, cudaStream_t st);
int tp_residual(__half* x, const float* part, int n, cudaStream_t st);
int tp_argmax(const __half* logits, int ld, int32_t* idx, int rows, int base, unsigned long long* keys, void* comm,
              cudaStream_t st);
}  // namespace axb
