// Exact float32 block distances in the reference's CPU evaluation order
// (codec.py:497-499 direct form, codec.py:88-91 expanded form). Shared by the
// CUDA-core assignment kernel and the exact re-scan of the tensor-core one.
#pragma once

#include "common.cuh"

namespace ss {

// NumPy pairwise sum of n <= 16 float32 terms (numpy/_core/src/umath/loops_utils.h).
template <int N>
__device__ __forceinline__ float np_pairwise_sum(const float* r) {
  if constexpr (N < 8) {
    float s = r[0];
#pragma unroll
    for (int i = 1; i < N; ++i) s = __fadd_rn(s, r[i]);
    return s;
  } else {
    float p[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = r[i];
#pragma unroll
    for (int i = 8; i + 8 <= N; i += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) p[j] = __fadd_rn(p[j], r[i + j]);
    }
    float s = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                        __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
#pragma unroll
    for (int i = (N / 8) * 8; i < N; ++i) s = __fadd_rn(s, r[i]);
    return s;
  }
}

template <int BD>
__device__ __forceinline__ float dist_direct(const float* kk, const float* c) {
  float r[BD];
#pragma unroll
  for (int j = 0; j < BD; ++j) {
    float d = __fsub_rn(kk[j], c[j]);
    r[j] = __fmul_rn(d, d);
  }
  return np_pairwise_sum<BD>(r);
}

// ||x||^2 + ||c||^2 - (2x).c as NumPy/BLAS evaluate codec.py:88-90 for one
// centroid: squared norms by pairwise sums, the dot as an FMA chain.
template <int BD>
__device__ __forceinline__ float dist_expanded(const float* kk, const float* c) {
  float r2[BD], c2[BD];
#pragma unroll
  for (int j = 0; j < BD; ++j) {
    r2[j] = __fmul_rn(kk[j], kk[j]);
    c2[j] = __fmul_rn(c[j], c[j]);
  }
  const float xsq = np_pairwise_sum<BD>(r2);
  const float csq = np_pairwise_sum<BD>(c2);
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < BD; ++j) dot = __fmaf_rn(__fmul_rn(2.0f, kk[j]), c[j], dot);
  return __fsub_rn(__fadd_rn(xsq, csq), dot);
}

}  // namespace ss
