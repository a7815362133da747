// Parameters of the MIMO scan kernels. Element strides; innermost dims contiguous.
#pragma once
#include <stdint.h>

#include "siso_scan.cuh"

namespace m3 {

struct Str4 {
  int64_t b, l, r, h;
};

struct MimoParams {
  int Bn, L, H, P, D, R;
  const void* x;    Str3 sx;
  const void* Bm;   Str4 sB;
  const void* Cm;   Str4 sC;
  const float* adt; Str3 sadt;
  const float* dt;  Str3 sdt;
  const float* trap; Str3 strap;
  const float* Dskip; int64_t sD;
  const float* mimo_x; int64_t smx_h, smx_r;  // (H, R, P) f32
  const float* mimo_o; int64_t smo_h, smo_r;
  const float* h0;   // (B,H,D) contiguous or null
  const float* bx0;
  void* y; Str3 sy;
  float* h_last;
  float* bx_last;
  // backward
  const void* dy; Str3 sdy;
  void* dx; Str3 sdx;
  void* dB; Str4 sdB;
  void* dC; Str4 sdC;
  float* dadt; Str3 sdadt;
  float* ddt; Str3 sddt;
  float* dtrap; Str3 sdtrap;
  float* dD;    // (H) pre-zeroed
  float* dmx;   // (H,R,P) contiguous, pre-zeroed
  float* dmo;
  float* dh0;
  float* dbx0;
  float* work;  // checkpoints
};

size_t mimo_bwd_workspace_floats(int64_t Bn, int64_t L, int64_t H, int64_t P, int64_t D, int64_t R);
int launch_mimo(const MimoParams& p, int xdt, int bcdt, bool bwd, cudaStream_t s);
// Chunk-parallel forward (mimo_chunked.cu): workspace of mimo_fwd_workspace_bytes bytes.
size_t mimo_fwd_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D);
int launch_mimo_fwd_chunked(const MimoParams& p, int xdt, int bcdt, void* ws, cudaStream_t s);
// Single-pass backward (mimo_chunked.cu) from the single-pass forward's workspace (its
// published chunk-end states): M3_ERR_UNSUPPORTED, nothing launched, when the pair does not
// apply (the caller then runs launch_mimo_bwd_chunked).
size_t mimo_bwd_fused_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D);
int launch_mimo_bwd_fused(const MimoParams& p, int xdt, int bcdt, const void* fwd_ws, size_t fwd_bytes, void* ws,
                          size_t ws_bytes, cudaStream_t s);
// the word the single-pass kernels set when a bounded wait gives up
int mimo_error_word(bool reset, int* out);
// Single-pass forward of one layer's scan from its in_proj output (one B / C group): x
// and z from zx, B / C from its group rows normalised, biased per head and rotated by the
// angles inside the kernel, y optionally gated (y * silu(z)). p carries the step scalars,
// D, mimo_x / mimo_o, the optional states and y (x, Bm, Cm unused). Workspace as for
// launch_mimo_fwd_chunked. M3_ERR_UNSUPPORTED, nothing launched, when the layout does not
// allow the tensor maps.
struct MimoGrpParams {
  const void* zx; int64_t s_zb, s_zl;  // (Bn, L, d_proj), innermost contiguous
  int dtype;                           // of zx (and of y)
  const float* angles;                 // (Bn, L, H, S) contiguous
  const float* B_bias; const float* C_bias;      // (H, R, D) contiguous
  const float* B_norm_w; const float* C_norm_w;  // (D)
  float eps;
  int S;     // rotated pairs
  int gate;  // 1: y * silu(z)
};
int launch_mimo_layer_fwd(const MimoParams& p, const MimoGrpParams& q, void* ws, cudaStream_t s);
// Chunk-parallel backward (mimo_chunked.cu), used when its shared-memory layout fits.
bool mimo_bwd_chunked_fits(int P, int R, int D);
size_t mimo_bwd_chunked_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D);
int launch_mimo_bwd_chunked(const MimoParams& p, int xdt, int bcdt, void* ws, cudaStream_t s);

}  // namespace m3
