// Parameters shared by the SISO scan kernels (recurrent fp32 path and the chunked
// tensor-core path). All element strides; the innermost dim of every tensor is
// contiguous.
#pragma once
#include <stdint.h>

namespace m3 {

struct Str3 {
  int64_t b, l, h;
};

struct SisoParams {
  int Bn, L, H, P, D;
  // inputs
  const void* x;    Str3 sx;
  const void* Bm;   Str3 sB;
  const void* Cm;   Str3 sC;
  const float* adt; Str3 sadt;
  const float* dt;  Str3 sdt;
  const float* trap; Str3 strap;
  const float* Dskip; int64_t sD;
  const float* h0;   // (B,H,P,D) contiguous or null
  const float* bx0;  // (B,H,P,D) contiguous or null
  // forward outputs
  void* y; Str3 sy;
  float* h_last;     // (B,H,P,D) or null
  float* bx_last;
  // backward
  const void* dy; Str3 sdy;
  void* dx; Str3 sdx;
  void* dB; Str3 sdB;
  void* dC; Str3 sdC;
  float* dadt; Str3 sdadt;
  float* ddt; Str3 sddt;
  float* dtrap; Str3 sdtrap;
  float* dD;         // (H), pre-zeroed, accumulated with atomics
  float* dh0;        // (B,H,P,D) or null
  float* dbx0;
  float* q;          // workspace (B,H,L): <dy_t, C_t h_t>
  // chunked tensor-core path only: bf16 k_c^T [d][p] of every 128-step chunk, per (b, h)
  // unit in chunk order (written by the forward, read by the backward)
  void* kstates;
};

// Launchers (siso_scan.cu). xdt / bcdt are m3_dtype codes.
int launch_siso_fwd_recurrent(const SisoParams& p, int xdt, int bcdt, cudaStream_t s);
int launch_siso_bwd_recurrent(const SisoParams& p, int xdt, int bcdt, cudaStream_t s);

}  // namespace m3
