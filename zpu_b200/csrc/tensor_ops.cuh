// Element-moving launches the jit-plan lowering uses besides the region
// kernels (tensor_ops.cu).  Every element goes through zpu's f64 conversion
// rules (scalar.toF64 / fromF64, src/zpu/scalar.zig:7-27).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace zc {

// dst <- src over the same dims, both strided views (element strides, any
// sign); the types may differ (converted as zpu converts).
int copy_view(const zpucuda_tensor &src, const zpucuda_tensor &dst, cudaStream_t s);
// n elements of a contiguous `dtype` buffer set to fromF64(v) (ops.pad's fill).
int fill_value(int dtype, void *dst, int64_t n, double v, cudaStream_t s);
// ops.take (src/zpu/ops.zig:1697-1755) on contiguous [outer, sdim, inner] x:
// out[o, t, i] = x[o, idx[t], i], idx[t] = trunc(toF64(indices[t])), a
// negative index counted from the end once; an index out of range sets *err
// (bit 0) and writes 0.
int take_launch(int dtype, const void *x, int idx_dtype, const void *indices, void *out, int64_t outer, int64_t sdim,
                int64_t inner, int64_t k, unsigned int *err, cudaStream_t s);
// ops.scatterAdd (ops.zig:1758-1797): out (contiguous [outer, sdim, inner])
// = 0, then out[o, idx[t], i] += updates[o, t, i] for t ascending, each sum
// in f64 and rounded to the type -- one thread per (o, i) column walks t, so
// repeated indices add in zpu's order.  Bad indices set *err and are skipped.
int scatter_add_launch(int dtype, int idx_dtype, const void *indices, const void *updates, void *out, int64_t outer,
                       int64_t sdim, int64_t inner, int64_t k, unsigned int *err, cudaStream_t s);

}  // namespace zc
