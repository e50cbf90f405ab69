// Averaging of multi-dimensional importance scores (core.py:1019-1031).
//
// The reference turns [..., T] scores into [T] with reshape(-1, T).mean(0) and
// [T, ...] scores with reshape(T, -1).mean(1).  Run on the CPU, Tensor.mean is
// ATen's cascade sum (native/cpu/SumKernel.cpp) followed by one fp32 division,
// and which fp32 additions it makes -- and so the last bit of every mean, and
// with it the top-k / bottom-k boundaries of the selection -- follows from the
// structure restated here:
//  * cascade: values are added one by one into level 0; after every 2^p values
//    (p = max(4, ceil_log2(n) / 4)) level j-1 is folded into level j while the
//    count so far is a multiple of 2^(p*j); leftover values go into level 0, and
//    the result is level 0 + level 1 + level 2 + level 3 (in that order);
//  * row sum: four interleaved cascades over values 4i+k, leftovers added into
//    partial 0, then partial 0 + 1 + 2 + 3;
//  * [R, C] over R: columns are handed out in per-thread blocks whose ends are
//    rounded down to 32 columns; every whole group of 32 columns of a block
//    takes the cascade, the rest of the block the row sum (a block narrower
//    than 8 columns: whole groups of 4 columns cascade).  Every block but the
//    last is whole groups, so only the last block's first column matters;
//  * [T, X] over X: 8-lane vectors, lane l a row sum over elements 8v + l; the
//    X mod 8 leftover elements are added into a scalar from 0, then lanes 0..7;
//    X < 8: one row sum;
//  * the output starts at 0 and receives 0 + sum (so -0 becomes +0).
// One thread per output; the sums are sequential, exactly in that order.
#pragma once

#include "gkv_common.cuh"

namespace gkv {

__device__ __forceinline__ int ceil_log2_sum(int64_t x) {
  return x <= 2 ? 1 : 64 - __clzll((unsigned long long)(x - 1));
}

// cascade over x[0], x[stride], ..., x[(n - 1) * stride]
__device__ float cascade_sum(const float* x, int64_t stride, int64_t n) {
  const int p = max(4, ceil_log2_sum(n) / 4);
  const int64_t step = (int64_t)1 << p;
  const uint64_t mask = (uint64_t)step - 1u;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int64_t i = 0;
  while (i + step <= n) {
    for (int64_t j = 0; j < step; ++j, ++i) a0 = __fadd_rn(a0, x[i * stride]);
    a1 = __fadd_rn(a1, a0);
    a0 = 0.f;
    if (((uint64_t)i & (mask << p)) != 0) continue;
    a2 = __fadd_rn(a2, a1);
    a1 = 0.f;
    if (((uint64_t)i & (mask << (2 * p))) != 0) continue;
    a3 = __fadd_rn(a3, a2);
    a2 = 0.f;
  }
  for (; i < n; ++i) a0 = __fadd_rn(a0, x[i * stride]);
  a0 = __fadd_rn(a0, a1);
  a0 = __fadd_rn(a0, a2);
  return __fadd_rn(a0, a3);
}

__device__ float row_sum(const float* x, int64_t stride, int64_t n) {
  const int64_t n4 = n / 4;
  float part[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) part[k] = cascade_sum(x + k * stride, 4 * stride, n4);
  for (int64_t i = 4 * n4; i < n; ++i) part[0] = __fadd_rn(part[0], x[i * stride]);
  part[0] = __fadd_rn(part[0], part[1]);
  part[0] = __fadd_rn(part[0], part[2]);
  return __fadd_rn(part[0], part[3]);
}

// [rows, cols] fp32 (contiguous) -> mean over rows, one thread per column
__global__ void __launch_bounds__(256) mean_rows_kernel(const float* __restrict__ x, int rows, int cols,
                                                        int last_block, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  bool cascade = true;
  if (c >= last_block) {
    const int n = cols - last_block, j = c - last_block;
    const int a_end = n >= 8 ? n / 32 * 32 : n / 4 * 4;
    cascade = j < a_end;
  }
  const float s = cascade ? cascade_sum(x + c, cols, rows) : row_sum(x + c, cols, rows);
  out[c] = __fdiv_rn(__fadd_rn(0.f, s), __int2float_rn(rows));
}

// [rows, cols] fp32 (contiguous) -> mean over cols, one thread per row
__global__ void __launch_bounds__(256) mean_cols_kernel(const float* __restrict__ x, int rows, int cols,
                                                        float* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float* row = x + (int64_t)r * cols;
  float fin;
  if (cols >= 8) {
    const int nv = cols / 8;
    fin = 0.f;
    for (int c = nv * 8; c < cols; ++c) fin = __fadd_rn(fin, row[c]);
    for (int lane = 0; lane < 8; ++lane) fin = __fadd_rn(fin, row_sum(row + lane, 8, nv));
  } else {
    fin = row_sum(row, 1, cols);
  }
  out[r] = __fdiv_rn(__fadd_rn(0.f, fin), __int2float_rn(cols));
}

cudaError_t launch_mean_scores(const float* x, int rows, int cols, int axis, int last_block, float* out,
                               cudaStream_t st) {
  const int n = axis == 0 ? cols : rows;
  const unsigned blocks = (unsigned)ceil_div(n, 256);
  if (axis == 0) mean_rows_kernel<<<blocks, 256, 0, st>>>(x, rows, cols, last_block, out);
  else mean_cols_kernel<<<blocks, 256, 0, st>>>(x, rows, cols, out);
  return cudaGetLastError();
}

}  // namespace gkv
