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

// Backward of the prologue (prologue_bwd.cu). The fp32 scratch (dtheta, dDT_ang,
// dangle_raw) comes from the caller's workspace (prologue_bwd_workspace_bytes).
struct PrologueBwdParams {
  int Bn, L, H, P, D, R, G, S, split, d_inner;
  float A_floor, eps;
  const void* zx; int64_t s_zb, s_zl;        // forward input: in_proj output (Bn, L, d_in_proj)
  void* dzx; int64_t s_dzb, s_dzl;           // its gradient (same dtype): B, C, dt, A, trap, angle columns
  const float* dt_bias;                      // (H)
  const float* B_bias; const float* C_bias;  // (H, R, D)
  const float* B_norm_w; const float* C_norm_w;  // (D)
  const float* angles;                       // forward angles (Bn, L, H, S)
  const float* DT;                           // forward DT (Bn, L, H)
  const void* dBp; const void* dCp;          // scan gradients (Bn, L, R, H, D), operand dtype
  const float* dADT; const float* dDT; const float* dtrap;  // (Bn, L, H)
  float* dB_bias; float* dC_bias;            // (H, R, D), overwritten
  float* dB_norm_w; float* dC_norm_w;        // (D), overwritten
  float* ddt_bias;                           // (H), overwritten
  float* dtheta; float* dDT_ang; float* dangle_raw;  // scratch
  float* bc_part;  // scratch: the bc kernel's per-CTA partial sums
};

struct GateBwdParams {
  int64_t rows;  // Bn * L * H
  int L, H, P;
  const void* y; Str3 sy;
  const void* z; Str3 sz;
  const void* dout; Str3 sd;
  void* dy; Str3 sdy;
  void* dz; Str3 sdz;
};

int launch_prologue(const PrologueParams& p, int zdt, int odt, cudaStream_t s);
// the word the prologue backward's bulk-copy waits set when they give up
int prologue_error_word(bool reset, int* out);
size_t prologue_bwd_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t S, int64_t R, int64_t D);
int launch_prologue_bwd(const PrologueBwdParams& p, float* ws, int zdt, int odt, cudaStream_t s);
int launch_gate_bwd(const GateBwdParams& p, int ydt, int zdt, int ddt, cudaStream_t s);
int launch_gate(const GateParams& p, int ydt, int zdt, int odt, cudaStream_t s);

}  // namespace m3
