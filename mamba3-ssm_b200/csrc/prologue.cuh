// Parameters of the fused forward prologue and gate kernels (prologue.cu).
#pragma once
#include <stdint.h>

#include <cuda_runtime.h>

#include "siso_scan.cuh"

namespace m3 {

struct PrologueParams {
  int Bn, L, H, P, D, R, G, S, split, d_inner;
  float A_floor, eps;
  const void* zx; int64_t s_zb, s_zl;       // in_proj output (Bn, L, d_in_proj), innermost contiguous
  const float* dt_bias;                     // (H)
  const float* B_bias; const float* C_bias; // (H, R, D) contiguous
  const float* B_norm_w; const float* C_norm_w;  // (D)
  void* Bp; void* Cp;                       // (Bn, L, R, H, D) contiguous, operand dtype
  float* ADT; float* DT; float* trap;       // (Bn, L, H) contiguous
  float* angles;                            // (Bn, L, H, S) contiguous
  const float* angle0;                      // (Bn, H, S) contiguous or null: angles before step 0
};

struct GateParams {
  int64_t rows;  // Bn * L * H
  int L, H, P;
  const void* y; Str3 sy;
  const void* z; Str3 sz;
  void* out; Str3 so;
};

int launch_prologue(const PrologueParams& p, int zdt, int odt, cudaStream_t s);
int launch_gate(const GateParams& p, int ydt, int zdt, int odt, cudaStream_t s);

}  // namespace m3
