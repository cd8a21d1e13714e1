// In-library access to the device's NCCL communicator (nccl.cu).
#pragma once
#include "common.cuh"

namespace zc {

// World size of the current device's communicator (1 without one); *rank
// receives this process's rank.
int nccl_world(int *rank);
// In-place sum over the communicator on stream `s`.
int nccl_allreduce_sum_f32(float *d, int64_t count, cudaStream_t s);
// In place over world * count floats: rank r ends with the sum of block r.
int nccl_reduce_scatter_sum_f32(float *d, int64_t count, cudaStream_t s);
// In place over world * count floats: block r of rank r goes to every rank.
int nccl_all_gather_f32(float *d, int64_t count, cudaStream_t s);

}  // namespace zc
