// Row-wise RMSNorm with an optional fused residual add.
#pragma once
#include <stdint.h>

#include <cuda_runtime.h>

namespace m3 {

struct NormParams {
  int64_t rows, d;
  const void* x; int64_t sx;         // (rows, d), row stride in elements
  const void* res; int64_t sres;     // optional residual, dtype of x
  const void* w;                     // (d)
  float eps;
  void* out; int64_t sout;           // dtype of x
  void* hout; int64_t shout;         // optional x + res, dtype of x
};

int launch_rmsnorm(const NormParams& p, int xdt, int wdt, cudaStream_t s);

}  // namespace m3
