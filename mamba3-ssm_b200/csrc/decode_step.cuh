// Parameters of the fused decode-step kernels.
#pragma once
#include <stdint.h>

namespace m3 {

struct StepParams {
  int Bn, H, P, D, R, G, S, split, d_inner;
  float A_floor, eps;
  const void* zxbcdt; int64_t s_row;      // (Bn, d_in_proj), row stride in elements
  const float* dt_bias;                   // (H)
  const float* B_bias; const float* C_bias;  // (H, R, D) contiguous
  const float* B_norm_w; const float* C_norm_w;  // (D)
  const float* Dskip;                     // (H)
  const float* mimo_x; const float* mimo_o;  // (H, R, P) contiguous, MIMO only
  const float* angle_in; float* angle_out;   // (Bn, H, S)
  const float* ssm_in; float* ssm_out;       // SISO (Bn,H,P,D), MIMO (Bn,H,D)
  const float* bx_in; float* bx_out;
  void* y; int64_t s_y;                      // (Bn, d_inner), row stride in elements
};

int launch_step(const StepParams& p, int zdt, bool mimo, cudaStream_t s);

}  // namespace m3
