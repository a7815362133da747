// Chunked SISO scan backward on the sm_100a tensor cores (tcgen05 + TMA), bf16 I/O,
// headdim P = 64, d_state D = 128 or 64, fp32 accumulators. For d_state 64 the upper halves
// of the C / B tiles stay zero (never loaded), the d-contractions take half the K steps,
// and only the first 64 columns of dC / dB are stored. Gradients of ssm_scan_siso
// (mamba3_ssm/ops.py:145-181, the loop :166-175) for the shapes of the chunked forward.
//
// Forward per chunk of Q = 128 steps (the k-formulation of the chunked forward): k_c is the
// carried matrix at the chunk start (P x D; the forward writes it in bf16), lambda_i the
// in-chunk cumulative log decay (lambda_0 = 0), mu_j = a_{j+1} beta_j + gamma_{j+1},
// E_ij = e^{lambda_i - lambda_{j+1}} (j < i), G = C B^T:
//   Y      = diag(e^lambda) C k_c^T + (M o G) X + D X,  M_ij = E_ij mu_j (j < i), M_ii = beta_i
//   k_next = e^{lambda_Q} k_c + X^T diag(w) B,           w_j = e^{lambda_Q - lambda_{j+1}} mu_j
// Backward, given dY and dk_next (the adjoint carried back from the later chunk), S = dY X^T:
//   dC   = (e^lambda o dY) k_c + (M o S) B
//   dB   = (M o S)^T C + (w o X) dk_next
//   V    = Ghat^T dY + wdec o (B dk_next^T),   Ghat_ij = G_ij E_ij (j < i),
//          wdec_j = e^{lambda_Q - lambda_{j+1}}
//   dX   = mu o V + (beta_i G_ii + D) dY
//   dk_c = e^{lambda_Q} dk_next + dY^T diag(e^lambda) C
// and per step the scalars of the sequential identity (g_t the adjoint of h_t):
//   q_i          = <dy_i, C_i h_i> = e^{lambda_i} dY_i . (C k_c^T)_i + sum_{j<=i} G_ij (M o S)_ij
//   dmu_j        = X_j . V_j                  (= <g_{j+1}, u_j>)
//   dbeta_i      = G_ii S_ii + a_{i+1} dmu_i  (= <g_i, u_i>)
//   dgamma_{j+1} = dmu_j                      (= <g_{j+1}, u_j>)
// A second kernel forms dADT_r = sum_{s>=r} (q_s - beta_s dbeta_s - gamma_s dgamma_s) (the
// identity of the CUDA-core backward), dDT and dtrap. The suffix sum runs inside one chunk
// only and starts from the exact value at the next chunk's first row t0,
//   dADT_{t0} = a_{t0} <g_{t0}, h_{t0-1}> = <dk_c, k_c> - gamma_{t0} dgamma_{t0}
// (k_c = a_{t0} h_{t0-1} + gamma_{t0} u_{t0-1}, dk_c = g_{t0}), which the state warps form
// per chunk: a suffix over the whole sequence would add up the bf16-level errors of every
// later term (at L = 32768 that drifted to several percent of max|dADT|).
//
// Ten MMAs per chunk (M = 128, fp32 accumulators in TMEM):
//   phase 1: G = C B^T, S = dY X^T, Y1 = C k_c^T, T = B dk_next^T, dK^T = C^T (e^lambda o dY)
//   phase 2: U = Ghat^T dY, dC = (e^lambda o dY) k_c + (M o S) B, dB = (M o S)^T C + (w o X) dk_next
// Transposed operands are the same shared-memory tiles read MN-major.
// Roles (one CTA per SM, 16 warps, walking its (b, h) units chunk by chunk from the end):
//   warp 0      lane 0: the TMA loads and the MMA issue, in program order
//   warp 1      per-chunk scalars into two slots; TMEM owner
//   warps 2-3   e^lambda o dY
//   warps 4-11  epilogues, thread = row i; warps 4-7 and 8-11 split the columns
//   warps 12-15 the carried adjoint dk^T (thread = state row d, fp32 registers) and the
//               chunk-start dot product <dk_c, k_c>
// Every wait is bounded; on a timeout the kernel records an error and returns.
#include <cudaTypedefs.h>

#include <cstddef>

#include "m3_common.cuh"
#include "siso_chunk.cuh"
#include "sm100.cuh"

namespace m3 {
namespace {

using namespace sm100;

constexpr int Q = 128;
constexpr int kP = 64;
constexpr int kD = 128;
constexpr int kThreads = 512;
constexpr uint32_t kTile = Q * 64 * 2;  // one SW128 tile: 128 rows x 128 B
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSafeExp2 = 120.f;  // split-exponent factors stay within fp32 below 2^120

// TMEM columns. Phase 1: G, S, Y1, dK, T. Phase 2 writes U, dC, dB over G / S / Y1 (read
// by then); T stays for the phase-2 epilogue; dK is read by the state warps.
constexpr uint32_t kColG = 0, kColS = 128, kColY1 = 256, kColDK = 320, kColT = 448;
constexpr uint32_t kColU = 0, kColDC = 64, kColDB = 192;
// dY rows as packed bf16 pairs (32 columns), copied by the phase-1 epilogue so that the dY
// tile is free for the next chunk once phase 2 has read it
constexpr uint32_t kColDY = 384;

struct __align__(16) BScal {
  float lam2[Q + 4];  // lambda_i log2(e), i = 0..Q
  float lnx[Q];       // lam2[i + 1] (aligned for vector reads by column)
  float colf[Q];      // e^{lambda_{32b+1} - lambda_{j+1}}, b = j / 32 (split decay, column part)
  float colfm[Q];     // colf[j] mu[j]
  float lref[4];      // lam2[32 b + 1]
  float mu[Q];
  float beta[Q];
  float anext[Q];     // a_{i+1}
  float wdec[Q];      // e^{lambda_Q - lambda_{i+1}}
  float el[Q];        // e^{lambda_i}
  float decQ;         // e^{lambda_Q}
  float dskip;
  float a0, g0;       // a and gamma of the chunk's first row (initial-state gradients)
  int n;              // valid rows
  int flags;          // bit b: block b takes the split-exponent path
  int pad[2];
};

struct __align__(1024) BSmem {
  uint8_t c[2][kTile];    // C (d 0-63 | 64-127), rows i
  uint8_t b[2][kTile];    // B
  uint8_t x[kTile];       // X [i][p]; w o X after phase 1
  uint8_t dy[kTile];      // dY [i][p]
  uint8_t edy[kTile];     // e^{lambda_i} dY_i
  uint8_t kc[kTile];      // k_c^T [d][p]
  uint8_t dkn[kTile];     // dk_next^T [d][p], bf16 copy of the carried adjoint
  uint8_t gh[2][kTile];   // Ghat [i][j] (j 0-63 | 64-127)
  uint8_t ms[2][kTile];   // (M o S) [i][j]
  BScal sc[2];
  float qpart[2][Q];
  float gdiag[Q], sdiag[Q];
  float red[4];
  uint64_t ld_full, dy_full, sc_full[2], sc_empty[2], edy_ready, dkn_ready;
  uint64_t p1_done, p1b_done, ep1_done, p2_done, ep2_done, st_sync, xread;
  uint32_t tmem_base;
};

static_assert(sizeof(BSmem) + 1024 <= 232448, "shared memory budget");

// consumers of a scalar slot: e^lambda o dY writers, epilogues, state warps
constexpr uint32_t kScalReaders = 64 + 256 + 128;
// arrivals that complete the phase-1 epilogue: the epilogue threads, the w o X writers and
// the state warps (done reading the k_c tile, which the next chunk's load overwrites)
constexpr uint32_t kEp1Arrivals = 256 + 64 + 128;

__device__ int g_bwd_error;  // set when a bounded wait gives up

struct BwdArgs {
  int Bn, L, H, nch;
  int D;    // d_state: 128, or 64
  int nkd;  // K steps of 16 over d_state
  const float* adt; Str3 sadt;
  const float* dt; Str3 sdt;
  const float* trap; Str3 strap;
  const float* Dskip; int64_t sD;
  const float* h0;
  const float* bx0;
  __nv_bfloat16* dx; Str3 sdx;
  __nv_bfloat16* dB; Str3 sdB;
  __nv_bfloat16* dC; Str3 sdC;
  float* dadt; Str3 sdadt;
  float* ddt; Str3 sddt;
  float* dtrap; Str3 sdtrap;
  float* dD;
  float* dh0;
  float* dbx0;
  float* sq;     // per position [unit][t]: q_t
  float* sbeta;  //                         dbeta_t
  float* sgam;   //                         dgamma_t
  float* skdot;  // per (unit, chunk): <dk_c, k_c> as four per-warp partials
};

struct BPos {
  int u, b, h, c, t0, n;
  bool first, last;
};
// g-th chunk of this CTA: units blockIdx.x + k gridDim.x, chunks from the last to the first
__device__ __forceinline__ BPos bpos(const BwdArgs& a, int g) {
  BPos q;
  const int k = g / a.nch;
  q.c = a.nch - 1 - (g - k * a.nch);
  q.u = blockIdx.x + k * gridDim.x;
  q.b = q.u / a.H;
  q.h = q.u - q.b * a.H;
  q.t0 = q.c * Q;
  q.n = min(Q, a.L - q.t0);
  q.first = q.c == 0;
  q.last = q.c == a.nch - 1;
  return q;
}

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity) {
  if (mbar_wait(bar, parity, 1u << 24)) return true;
  atomicExch(&g_bwd_error, 1);
  return false;
}

// The control thread's waits: polling, so that it resumes as soon as the phase completes
// (a suspended try_wait can resume late); bounded like bwait.
__device__ __forceinline__ bool cwait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_test(bar, parity)) return true;
    if (i > 64) __nanosleep(20);
  }
  atomicExch(&g_bwd_error, 1);
  return false;
}

__device__ __forceinline__ float ld_scal(const float* p, const Str3& s, int b, int t, int h) {
  return p[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h];
}

__device__ __forceinline__ uint32_t lane_addr(uint32_t base, int warp, uint32_t col) {
  return base + ((uint32_t)((warp & 3) * 32) << 16) + col;
}
// byte offset of (row r, element c) in a 128-row SW128 tile with 64 bf16 per row
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)r * 128u + ((((uint32_t)c >> 3) ^ ((uint32_t)r & 7u)) << 4) + (((uint32_t)c & 7u) << 1);
}
__device__ __forceinline__ float2 bf2(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}

// ------------------------------------------------------------------------------------
// warp 1: per-chunk scalars, rows i = lane + 32 k, plus row Q (the next chunk's first)
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void scalar_role(const BwdArgs& a, BSmem& s, int G, int lane) {
  for (int g = 0; g < G; ++g) {
    const int q = g & 1;
    const BPos cp = bpos(a, g);
    float adt[4], av[4], be[4], ga[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = cp.t0 + lane + 32 * k;
      const bool v = t < a.L;
      adt[k] = v ? ld_scal(a.adt, a.sadt, cp.b, t, cp.h) : 0.f;
      const float dt = v ? ld_scal(a.dt, a.sdt, cp.b, t, cp.h) : 0.f;
      const float tr = v ? sigmoidf_(ld_scal(a.trap, a.strap, cp.b, t, cp.h)) : 0.f;
      be[k] = dt * (1.0f - tr) + 0.5f * dt * tr;
      ga[k] = 0.5f * dt * tr;
      av[k] = v ? exp2f(adt[k] * kLog2e) : 0.f;
    }
    float adtQ = 0.f, aQ = 0.f, gQ = 0.f;
    {
      const int t = cp.t0 + Q;
      if (t < a.L) {
        adtQ = ld_scal(a.adt, a.sadt, cp.b, t, cp.h);
        aQ = exp2f(adtQ * kLog2e);
        gQ = 0.5f * ld_scal(a.dt, a.sdt, cp.b, t, cp.h) * sigmoidf_(ld_scal(a.trap, a.strap, cp.b, t, cp.h));
      }
    }
    // lambda: inclusive scan of (i == 0 ? 0 : ADT_i)
    float lam[4];
    float carry = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v = (k == 0 && lane == 0) ? 0.f : adt[k];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      lam[k] = (v + carry) * kLog2e;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    const float lamQ = (carry + adtQ) * kLog2e;
    // next-row values a_{i+1}, gamma_{i+1}, lam2_{i+1}
    float an[4], gn[4], ln[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a1 = __shfl_down_sync(0xffffffffu, av[k], 1);
      const float g1 = __shfl_down_sync(0xffffffffu, ga[k], 1);
      const float l1 = __shfl_down_sync(0xffffffffu, lam[k], 1);
      float aw, gw, lw;
      if (k < 3) {
        aw = __shfl_sync(0xffffffffu, av[k < 3 ? k + 1 : 3], 0);
        gw = __shfl_sync(0xffffffffu, ga[k < 3 ? k + 1 : 3], 0);
        lw = __shfl_sync(0xffffffffu, lam[k < 3 ? k + 1 : 3], 0);
      } else {
        aw = aQ; gw = gQ; lw = lamQ;
      }
      an[k] = lane < 31 ? a1 : aw;
      gn[k] = lane < 31 ? g1 : gw;
      ln[k] = lane < 31 ? l1 : lw;
    }
    // Split decay of the mask, per 32-column block b with reference lam2[32b+1]:
    // E_ij = e^{lambda_i - lambda_{32b+1}} e^{lambda_{32b+1} - lambda_{j+1}}. A block is
    // factorised when its column exponents and the row exponents of rows i >= 32b stay
    // below 2^120; otherwise its elements take one exp2 each.
    float ref[4], lmax[4];
    int flags = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ref[k] = __shfl_sync(0xffffffffu, lam[k], 1);
      float cm = ref[k] - ln[k], lm = lam[k];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
        lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, o));
      }
      lmax[k] = lm;
      if (cm <= kSafeExp2) flags |= 1 << k;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float rm = lmax[k];
#pragma unroll
      for (int k2 = k + 1; k2 < 4; ++k2) rm = fmaxf(rm, lmax[k2]);
      if (!(rm - ref[k] <= kSafeExp2)) flags &= ~(1 << k);
    }
    if (!bwait(&s.sc_empty[q], ((g >> 1) & 1) ^ 1)) return;
    BScal& sl = s.sc[q];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = lane + 32 * k;
      sl.lam2[j] = lam[k];
      sl.lnx[j] = ln[k];
      const float cf = exp2f(ref[k] - ln[k]);
      sl.colf[j] = cf;
      sl.colfm[j] = cf * fmaf(an[k], be[k], gn[k]);
      sl.mu[j] = fmaf(an[k], be[k], gn[k]);
      sl.beta[j] = be[k];
      sl.anext[j] = an[k];
      sl.wdec[j] = exp2f(lamQ - ln[k]);
      sl.el[j] = exp2f(lam[k]);
    }
    if (lane == 0) {
      sl.lam2[Q] = lamQ;
      sl.decQ = exp2f(lamQ);
      sl.dskip = a.Dskip[cp.h * a.sD];
      sl.a0 = av[0];
      sl.g0 = ga[0];
      sl.n = cp.n;
      sl.flags = flags;
#pragma unroll
      for (int k = 0; k < 4; ++k) sl.lref[k] = ref[k];
    }
    mbar_arrive(&s.sc_full[q]);
  }
}

// ------------------------------------------------------------------------------------
// e^{lambda_r} dY_r for the dK^T and dC MMAs, row r (the phase-2 epilogue threads of half 1
// write the next chunk's rows once its dY has landed)
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void write_edy_row(BSmem& s, const BScal& sl, int r) {
  const float f = sl.el[r];
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    const uint4 v = *reinterpret_cast<const uint4*>(s.dy + sw128_off(r, 8 * cc));
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const float2 f2 = bf2(vv[z]);
      o[z] = pack_bf16(f2.x * f, f2.y * f);
    }
    *reinterpret_cast<uint4*>(s.edy + sw128_off(r, 8 * cc)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------------------------
// warps 2-3: w o X in place of X (thread e: rows e and e + 64) for the dB MMA of phase 2,
// once S (phase 1) is complete and the epilogue threads have taken their X rows
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void wx_role(BSmem& s, int G, int e) {
  for (int g = 0; g < G; ++g) {
    const int q = g & 1;
    if (!bwait(&s.sc_full[q], (g >> 1) & 1)) return;
    if (!bwait(&s.xread, g & 1)) return;
    const BScal& sl = s.sc[q];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = e + 64 * rr;
      const float wi = sl.wdec[r] * sl.mu[r];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint4 v = *reinterpret_cast<const uint4*>(s.x + sw128_off(r, 8 * cc));
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          const float2 f = bf2(vv[z]);
          o[z] = pack_bf16(f.x * wi, f.y * wi);
        }
        *reinterpret_cast<uint4*>(s.x + sw128_off(r, 8 * cc)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(&s.ep1_done);
    mbar_arrive(&s.sc_empty[q]);
  }
}

// ------------------------------------------------------------------------------------
// warps 4-11: thread = row i. Half hf takes the 32-column blocks hf and hf + 2.
// Phase-1 epilogue: Ghat and M o S (bf16, shared memory, zero above the diagonal), the
// partial q, the diagonals; half 0 keeps the X row and writes w o X in place, half 1 adds
// the Y1 term of q. Phase-2 epilogue: half 0 dX, dmu and the three per-step scalars,
// half 1 dC and dB.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void zero_block(uint8_t* t, int i, int c0) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) *reinterpret_cast<uint4*>(t + sw128_off(i, c0 + 8 * cc)) = make_uint4(0u, 0u, 0u, 0u);
}

// 32 fp32 values -> bf16 at columns c0 .. c0 + 31 of row i of a SW128 staging tile
__device__ __forceinline__ void stage_row_bf16(uint8_t* tile, int i, int c0, const uint32_t (&r)[32]) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc)
    *reinterpret_cast<uint4*>(tile + sw128_off(i, c0 + 8 * cc)) = make_uint4(pack_bf16(__uint_as_float(r[8 * cc + 0]), __uint_as_float(r[8 * cc + 1])),
                        pack_bf16(__uint_as_float(r[8 * cc + 2]), __uint_as_float(r[8 * cc + 3])),
                        pack_bf16(__uint_as_float(r[8 * cc + 4]), __uint_as_float(r[8 * cc + 5])),
                        pack_bf16(__uint_as_float(r[8 * cc + 6]), __uint_as_float(r[8 * cc + 7])));
}

// One 32-column block of row i of Ghat (pg) and M o S (pm), packed bf16, and the block's
// part of q. kMode 0: below the diagonal, split decay rowf * colf; 1: the diagonal block,
// split decay; 2: any block, one exp2 per element (blocks whose split factors could leave
// the fp32 range). gd / sd receive G_ii / S_ii when the diagonal is in the block.
template <int kMode>
__device__ __forceinline__ void mask_block(const uint32_t (&rg)[32], const uint32_t (&rs)[32], uint32_t (&pg)[16],
                                           uint32_t (&pm)[16], const BScal& sl, int qd, int il, float li,
                                           float rowf, float bi, float& qacc, float& gd, float& sd) {
  const float4* c4 = reinterpret_cast<const float4*>(kMode == 2 ? sl.lnx + 32 * qd : sl.colf + 32 * qd);
  const float4* m4 = reinterpret_cast<const float4*>(kMode == 2 ? sl.mu + 32 * qd : sl.colfm + 32 * qd);
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 cv = c4[e4], mv = m4[e4];
    const float ck[4] = {cv.x, cv.y, cv.z, cv.w}, mk[4] = {mv.x, mv.y, mv.z, mv.w};
    float vg[4], vm[4];
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int jl = 4 * e4 + z;
      const float gij = __uint_as_float(rg[jl]), sij = __uint_as_float(rs[jl]);
      if (kMode == 0) {
        vg[z] = gij * (rowf * ck[z]);
        vm[z] = sij * (rowf * mk[z]);
      } else {
        float e, em;
        if (kMode == 1) {
          e = rowf * ck[z];
          em = rowf * mk[z];
        } else {
          e = exp2f(li - ck[z]);
          em = e * mk[z];
        }
        const bool lo = jl < il, dg = jl == il;
        vg[z] = lo ? gij * e : 0.f;
        vm[z] = lo ? sij * em : (dg ? bi * sij : 0.f);
        gd = dg ? gij : gd;
        sd = dg ? sij : sd;
      }
      qacc = fmaf(gij, vm[z], qacc);
    }
    pg[2 * e4] = pack_bf16(vg[0], vg[1]);
    pg[2 * e4 + 1] = pack_bf16(vg[2], vg[3]);
    pm[2 * e4] = pack_bf16(vm[0], vm[1]);
    pm[2 * e4 + 1] = pack_bf16(vm[2], vm[3]);
  }
}

__device__ __forceinline__ void ep_role(const BwdArgs& a, BSmem& s, uint32_t tbase, int G, int warp, int i, int hf) {
  const int wr = warp & 3;  // this warp's rows are 32 wr .. 32 wr + 31
  const int lane = i & 31;
  uint4 xrow[8];            // X row i (half 0), from the phase-1 to the phase-2 epilogue
  float dd = 0.f;           // sum over the unit of dY_i . X_i (half 0), for dD
  for (int g = 0; g < G; ++g) {
    const int q = g & 1;
    const uint32_t par = g & 1;
    const BPos cp = bpos(a, g);
    if (!bwait(&s.sc_full[q], (g >> 1) & 1)) return;
    if (hf == 1 && g == 0) {
      // e^lambda o dY of the first chunk (later chunks: after the phase-2 epilogue below)
      if (!bwait(&s.dy_full, 0)) return;
      write_edy_row(s, s.sc[0], i);
      fence_proxy_async_smem();
      mbar_arrive(&s.edy_ready);
    }
    if (!bwait(&s.p1_done, par)) return;
    // the X and dY tiles this thread reads arrived by TMA: observe their barriers too
    if (!bwait(&s.ld_full, par) || !bwait(&s.dy_full, par)) return;
    tc_fence_after();
    const BScal& sl = s.sc[q];
    const float li = sl.lam2[i], bi = sl.beta[i];
    float qacc = 0.f;
    if (hf == 0) {
      // X_i for dmu in the phase-2 epilogue; warps 2-3 then overwrite the tile with w o X
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) xrow[cc] = *reinterpret_cast<const uint4*>(s.x + sw128_off(i, 8 * cc));
      mbar_arrive(&s.xread);
    }
#pragma unroll 1
    for (int t2 = 0; t2 < 2; ++t2) {
      const int qd = hf + 2 * t2;
      uint8_t* ght = s.gh[qd >> 1];
      uint8_t* mst = s.ms[qd >> 1];
      const int c0 = (qd & 1) * 32;
      if (qd > wr) {
        zero_block(ght, i, c0);
        zero_block(mst, i, c0);
        continue;
      }
      uint32_t rg[32], rs[32];
      tmem_ld32(lane_addr(tbase, warp, kColG + 32u * qd), rg);
      tmem_ld32(lane_addr(tbase, warp, kColS + 32u * qd), rs);
      tmem_wait_ld();
      const int il = i - 32 * qd;
      uint32_t pg[16], pm[16];
      float gd = 0.f, sd = 0.f;
      if ((sl.flags >> qd) & 1) {
        const float rowf = exp2f(li - sl.lref[qd]);
        if (qd < wr) mask_block<0>(rg, rs, pg, pm, sl, qd, il, li, rowf, bi, qacc, gd, sd);
        else mask_block<1>(rg, rs, pg, pm, sl, qd, il, li, rowf, bi, qacc, gd, sd);
      } else {
        mask_block<2>(rg, rs, pg, pm, sl, qd, il, li, 0.f, bi, qacc, gd, sd);
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        *reinterpret_cast<uint4*>(ght + sw128_off(i, c0 + 8 * cc)) =
            make_uint4(pg[4 * cc], pg[4 * cc + 1], pg[4 * cc + 2], pg[4 * cc + 3]);
        *reinterpret_cast<uint4*>(mst + sw128_off(i, c0 + 8 * cc)) =
            make_uint4(pm[4 * cc], pm[4 * cc + 1], pm[4 * cc + 2], pm[4 * cc + 3]);
      }
      if (il < 32) {
        s.gdiag[i] = gd;
        s.sdiag[i] = sd;
      }
    }
    if (hf == 1) {
      // q_i += e^{lambda_i} dY_i . Y1_i; the dY row also goes to TMEM for the phase-2
      // epilogue (the dY tile is reloaded before then)
      float dot = 0.f;
#pragma unroll 1
      for (int qt = 0; qt < 2; ++qt) {
        uint32_t r[32], w[16];
        tmem_ld32(lane_addr(tbase, warp, kColY1 + 32u * qt), r);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 v = *reinterpret_cast<const uint4*>(s.dy + sw128_off(i, 32 * qt + 8 * cc));
          w[4 * cc] = v.x;
          w[4 * cc + 1] = v.y;
          w[4 * cc + 2] = v.z;
          w[4 * cc + 3] = v.w;
        }
        tmem_st16(lane_addr(tbase, warp, kColDY + 16u * qt), w);
        tmem_wait_ld();
#pragma unroll
        for (int z = 0; z < 16; ++z) {
          const float2 f = bf2(w[z]);
          dot = fmaf(f.x, __uint_as_float(r[2 * z]), dot);
          dot = fmaf(f.y, __uint_as_float(r[2 * z + 1]), dot);
        }
      }
      tmem_wait_st();
      qacc = fmaf(sl.el[i], dot, qacc);
    }
    s.qpart[hf][i] = qacc;
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&s.ep1_done);

    // ---------------- phase-2 epilogue
    if (!bwait(&s.p2_done, par)) return;
    // ep1_done(g) has completed (phase 2 waited for it): the other half's q partial and
    // diagonals are visible after this acquire
    if (!bwait(&s.ep1_done, par)) return;
    tc_fence_after();
    const bool valid = i < cp.n;
    const int t = cp.t0 + (valid ? i : 0);
    if (hf == 0) {
      const float mu_i = sl.mu[i], wd = sl.wdec[i];
      const float gii = s.gdiag[i], sii = s.sdiag[i];
      const float cdiag = fmaf(sl.beta[i], gii, sl.dskip);
      float dmu = 0.f;
      uint4* dst = reinterpret_cast<uint4*>(a.dx + (int64_t)cp.b * a.sdx.b + (int64_t)t * a.sdx.l +
                                            (int64_t)cp.h * a.sdx.h);
#pragma unroll
      for (int qt = 0; qt < 4; ++qt) {
        uint32_t ru[16], rt[16], rd[8];
        tmem_ld16(lane_addr(tbase, warp, kColU + 16u * qt), ru);
        tmem_ld16(lane_addr(tbase, warp, kColT + 16u * qt), rt);
        tmem_ld8(lane_addr(tbase, warp, kColDY + 8u * qt), rd);
        tmem_wait_ld();
        uint32_t out[8];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const uint4 xv = xrow[2 * qt + h2];
          const uint32_t dvv[4] = {rd[4 * h2], rd[4 * h2 + 1], rd[4 * h2 + 2], rd[4 * h2 + 3]};
          const uint32_t xvv[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int z = 0; z < 4; ++z) {
            const int e = 8 * h2 + 2 * z;
            const float2 fd = bf2(dvv[z]), fx = bf2(xvv[z]);
            const float v0 = fmaf(wd, __uint_as_float(rt[e]), __uint_as_float(ru[e]));
            const float v1 = fmaf(wd, __uint_as_float(rt[e + 1]), __uint_as_float(ru[e + 1]));
            dmu = fmaf(fx.x, v0, fmaf(fx.y, v1, dmu));
            out[4 * h2 + z] = pack_bf16(fmaf(mu_i, v0, cdiag * fd.x), fmaf(mu_i, v1, cdiag * fd.y));
          }
        }
        if (valid) {
          dst[2 * qt] = make_uint4(out[0], out[1], out[2], out[3]);
          dst[2 * qt + 1] = make_uint4(out[4], out[5], out[6], out[7]);
        }
      }
      if (valid) {
        const int64_t pos = (int64_t)cp.u * a.L + t;
        a.sq[pos] = s.qpart[0][i] + s.qpart[1][i];
        a.sbeta[pos] = fmaf(sl.anext[i], dmu, gii * sii);
        if (t + 1 < a.L) a.sgam[pos + 1] = dmu;
        dd += sii;
      }
      if (cp.first) {
        // the unit is done: dD[h] += its sum of dY . X
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, o);
        if (lane == 0) atomicAdd(a.dD + cp.h, dd);
        dd = 0.f;
      }
    } else {
      // dC, dB rows -> the Ghat / M o S tiles (read by phase 2 only), stored by TMA
#pragma unroll 1
      for (int qt = 0; qt < 4; ++qt) {
        uint32_t r[32], r2[32];
        tmem_ld32(lane_addr(tbase, warp, kColDC + 32u * qt), r);
        tmem_ld32(lane_addr(tbase, warp, kColDB + 32u * qt), r2);
        tmem_wait_ld();
        stage_row_bf16(s.gh[qt >> 1], i, (qt & 1) * 32, r);
        stage_row_bf16(s.ms[qt >> 1], i, (qt & 1) * 32, r2);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&s.ep2_done);
    if (hf == 1 && g + 1 < G) {
      // e^lambda o dY of the next chunk, whose dY lands during this epilogue (the tile's
      // previous readers, the MMAs of phase 2, are complete)
      const int q1 = (g + 1) & 1;
      if (!bwait(&s.sc_full[q1], ((g + 1) >> 1) & 1)) return;
      if (!bwait(&s.dy_full, (g + 1) & 1)) return;
      write_edy_row(s, s.sc[q1], i);
      fence_proxy_async_smem();
      mbar_arrive(&s.edy_ready);
    }
    mbar_arrive(&s.sc_empty[q]);
  }
}

// ------------------------------------------------------------------------------------
// warps 12-15: the carried adjoint dk^T, thread = state row d (64 fp32 columns p).
// Before phase 1 of chunk c it is dk_next (its bf16 copy feeds T and dB); after phase 1
// it becomes dk_c = e^{lambda_Q} dk_next + dK^T. At a unit's first chunk dk_0 gives
// dh0 = a_0 dk_0, dbx0 = gamma_0 dk_0 and dgamma_0 = <dk_0, bx0>.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void state_role(const BwdArgs& a, BSmem& s, uint32_t tbase, int G, int warp, int d) {
  float dk[kP];
#pragma unroll
  for (int p = 0; p < kP; ++p) dk[p] = 0.f;
  const int lane = d & 31;
  uint32_t nfirst = 0;  // completed phases of st_sync
  for (int g = 0; g < G; ++g) {
    const int q = g & 1;
    const uint32_t par = g & 1;
    const BPos cp = bpos(a, g);
    if (!bwait(&s.sc_full[q], (g >> 1) & 1)) return;
    const BScal& sl = s.sc[q];
    if (cp.last) {
#pragma unroll
      for (int p = 0; p < kP; ++p) dk[p] = 0.f;
    }
    // the previous readers of dkn are T and dB of chunk g-1
    if (g > 0 && !bwait(&s.p2_done, par ^ 1)) return;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
      *reinterpret_cast<uint4*>(s.dkn + sw128_off(d, 8 * cc)) =
          make_uint4(pack_bf16(dk[8 * cc + 0], dk[8 * cc + 1]), pack_bf16(dk[8 * cc + 2], dk[8 * cc + 3]),
                     pack_bf16(dk[8 * cc + 4], dk[8 * cc + 5]), pack_bf16(dk[8 * cc + 6], dk[8 * cc + 7]));
    fence_proxy_async_smem();
    mbar_arrive(&s.dkn_ready);
    if (!bwait(&s.p1b_done, par)) return;
    tc_fence_after();
    const float dec = sl.decQ;
#pragma unroll
    for (int qt = 0; qt < 4; ++qt) {
      uint32_t r[16];
      tmem_ld16(lane_addr(tbase, warp, kColDK + 16u * qt), r);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) dk[16 * qt + e] = fmaf(dec, dk[16 * qt + e], __uint_as_float(r[e]));
    }
    tc_fence_before();
    {
      // <dk_c, k_c>, row d of this warp's part (k_c^T row d: the chunk-start state in bf16)
      float kd = 0.f;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint4 v = *reinterpret_cast<const uint4*>(s.kc + sw128_off(d, 8 * cc));
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv[e]));
          kd = fmaf(dk[8 * cc + 2 * e], f.x, kd);
          kd = fmaf(dk[8 * cc + 2 * e + 1], f.y, kd);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kd += __shfl_xor_sync(0xffffffffu, kd, o);
      if (lane == 0) a.skdot[((int64_t)cp.u * a.nch + cp.c) * 4 + (warp & 3)] = kd;
      mbar_arrive(&s.ep1_done);  // the k_c tile is read
    }
    if (cp.first) {
      const int64_t sb = ((int64_t)cp.b * a.H + cp.h) * kP * a.D + d;
      float gsum = 0.f;
      if (d < a.D) {
#pragma unroll
        for (int p = 0; p < kP; ++p) {
          if (a.dh0) a.dh0[sb + (int64_t)p * a.D] = sl.a0 * dk[p];
          if (a.dbx0) a.dbx0[sb + (int64_t)p * a.D] = sl.g0 * dk[p];
          if (a.bx0) gsum = fmaf(dk[p], a.bx0[sb + (int64_t)p * a.D], gsum);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, o);
      if (lane == 0) s.red[warp & 3] = gsum;
      mbar_arrive(&s.st_sync);
      if (!bwait(&s.st_sync, nfirst & 1)) return;
      ++nfirst;
      if (d == 0) a.sgam[(int64_t)cp.u * a.L] = (s.red[0] + s.red[1]) + (s.red[2] + s.red[3]);
    }
    mbar_arrive(&s.sc_empty[q]);
  }
}

// ------------------------------------------------------------------------------------
// warp 0, lane 0: loads, MMA issue and output stores, in order. Per chunk g:
//   phase 1(g)   once its inputs, e^lambda o dY(g) and dk_next(g) are in shared memory and
//                the phase-2 epilogue of g-1 has read TMEM: G, S, Y1 (commit p1_done; the
//                Ghat / M o S tiles are free once the TMA stores of g-1 have read them),
//                then T and dK^T (commit p1b_done)
//   phase 2(g)   after the phase-1 epilogue: U, dC, dB (commit p2_done)
//   loads(g+1)   C, B, X, k_c, dY as soon as phase 2(g) has read the tiles, so they land
//                during the phase-2 epilogue of g
//   stores(g)    dC, dB by TMA from the Ghat / M o S tiles after the phase-2 epilogue
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void control_role(const CUtensorMap* tm_x, const CUtensorMap* tm_B, const CUtensorMap* tm_C,
                                             const CUtensorMap* tm_dy, const CUtensorMap* tm_k,
                                             const CUtensorMap* tm_dB, const CUtensorMap* tm_dC, const BwdArgs& a,
                                             BSmem& s, uint32_t tbase, int G) {
  constexpr uint32_t I_KK128 = idesc_bf16_f32(128, 128, false, false);  // A, B K-major, N = 128
  constexpr uint32_t I_KM64 = idesc_bf16_f32(128, 64, false, true);     // A K-major, B MN-major, N = 64
  constexpr uint32_t I_MM64 = idesc_bf16_f32(128, 64, true, true);      // both MN-major, N = 64
  constexpr uint32_t I_KM128 = idesc_bf16_f32(128, 128, false, true);   // A K-major, B MN-major, N = 128
  constexpr uint32_t I_MM128 = idesc_bf16_f32(128, 128, true, true);    // both MN-major, N = 128
  const uint32_t c0 = smem_u32(s.c[0]), b0 = smem_u32(s.b[0]), xa = smem_u32(s.x), dya = smem_u32(s.dy),
                 ea = smem_u32(s.edy), ka = smem_u32(s.kc), na = smem_u32(s.dkn), ga = smem_u32(s.gh[0]),
                 ma = smem_u32(s.ms[0]);
  // K-major, K = 128 over two tiles (16 K per step)
  auto k2 = [](uint32_t base, int kk) {
    return sdesc_sw128(base + (uint32_t)(kk >> 2) * kTile + (uint32_t)(kk & 3) * 32u, 16, 1024);
  };
  // K-major, K = 64 in one tile
  auto k1 = [](uint32_t base, int kk) { return sdesc_sw128(base + (uint32_t)kk * 32u, 16, 1024); };
  // MN-major: 16 K rows per step; 64-wide M/N blocks one tile apart
  auto mn = [](uint32_t base, int kk) { return sdesc_sw128(base + (uint32_t)kk * 2048u, kTile, 1024); };
  // last chunk whose loads / MMA phases were issued: on a timeout, wait (bounded) for them
  // before leaving, so no copy or MMA is in flight when the CTA exits
  int lg = -1, p1g = -1, p2g = -1;
  auto drain = [&]() {
    bulk_wait0();
    if (lg >= 0) {
      mbar_wait(&s.ld_full, lg & 1, 1u << 20);
      mbar_wait(&s.dy_full, lg & 1, 1u << 20);
    }
    if (p1g >= 0) mbar_wait(&s.p1b_done, p1g & 1, 1u << 20);
    if (p2g >= 0) mbar_wait(&s.p2_done, p2g & 1, 1u << 20);
  };
  auto load = [&](int gg) {
    const BPos cp = bpos(a, gg);
    // dY first: e^lambda o dY waits for it
    mbar_expect_tx(&s.dy_full, kTile);
    tma_load_4d(s.dy, tm_dy, &s.dy_full, 0, cp.h, cp.t0, cp.b);
    mbar_expect_tx(&s.ld_full, (a.D == kD ? 6 : 4) * kTile);  // C (2 or 1), B (2 or 1), X, k_c
    tma_load_4d(s.c[0], tm_C, &s.ld_full, 0, cp.h, cp.t0, cp.b);
    tma_load_4d(s.b[0], tm_B, &s.ld_full, 0, cp.h, cp.t0, cp.b);
    if (a.D == kD) {
      tma_load_4d(s.c[1], tm_C, &s.ld_full, 64, cp.h, cp.t0, cp.b);
      tma_load_4d(s.b[1], tm_B, &s.ld_full, 64, cp.h, cp.t0, cp.b);
    }
    tma_load_4d(s.x, tm_x, &s.ld_full, 0, cp.h, cp.t0, cp.b);
    tma_load_2d(s.kc, tm_k, &s.ld_full, 0, (cp.u * a.nch + cp.c) * kD);
    lg = gg;
  };
  // dC, dB of chunk gg, staged in the Ghat and M o S tiles
  auto store_outputs = [&](int gg) {
    const BPos op = bpos(a, gg);
    tma_store_4d(tm_dC, s.gh[0], 0, op.h, op.t0, op.b);
    tma_store_4d(tm_dB, s.ms[0], 0, op.h, op.t0, op.b);
    if (a.D == kD) {
      tma_store_4d(tm_dC, s.gh[1], 64, op.h, op.t0, op.b);
      tma_store_4d(tm_dB, s.ms[1], 64, op.h, op.t0, op.b);
    }
    bulk_commit();
  };
  if (G > 0) load(0);
  for (int g = 0; g < G; ++g) {
    const uint32_t par = g & 1;
    if (!cwait(&s.ld_full, par) || !cwait(&s.dy_full, par) || !cwait(&s.edy_ready, par) ||
        !cwait(&s.dkn_ready, par))
      return drain();
    // (the phase-2 epilogue of g-1, which read TMEM, completed before its stores below)
    tc_fence_after();
    // phase 1: what the phase-1 epilogue reads first
#pragma unroll
    for (int kk = 0; kk < a.nkd; ++kk) mma_ss(tbase + kColG, k2(c0, kk), k2(b0, kk), I_KK128, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) mma_ss(tbase + kColS, k1(dya, kk), k1(xa, kk), I_KK128, kk > 0);
#pragma unroll
    for (int kk = 0; kk < a.nkd; ++kk) mma_ss(tbase + kColY1, k2(c0, kk), mn(ka, kk), I_KM64, kk > 0);
    // the epilogue overwrites the staging tiles of g-1: their stores must have read them
    if (g > 0) bulk_wait_read0();
    mma_commit(&s.p1_done);
#pragma unroll
    for (int kk = 0; kk < a.nkd; ++kk) mma_ss(tbase + kColT, k2(b0, kk), mn(na, kk), I_KM64, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) mma_ss(tbase + kColDK, mn(c0, kk), mn(ea, kk), I_MM64, kk > 0);
    mma_commit(&s.p1b_done);
    p1g = g;
    // phase 2
    if (!cwait(&s.ep1_done, par)) return drain();
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) mma_ss(tbase + kColDC, k1(ea, kk), k1(ka, kk), I_KK128, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) mma_ss(tbase + kColDC, k2(ma, kk), mn(b0, kk), I_KM128, 1u);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) mma_ss(tbase + kColDB, mn(ma, kk), mn(c0, kk), I_MM128, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) mma_ss(tbase + kColDB, k1(xa, kk), k1(na, kk), I_KK128, 1u);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) mma_ss(tbase + kColU, mn(ga, kk), mn(dya, kk), I_MM64, kk > 0);
    mma_commit(&s.p2_done);
    p2g = g;
    // the next chunk's tiles, once phase 2 has read these
    if (g + 1 < G) {
      if (!cwait(&s.p2_done, par)) return drain();
      load(g + 1);
    }
    // this chunk's dC, dB once the phase-2 epilogue has staged them
    if (!cwait(&s.ep2_done, par)) return drain();
    store_outputs(g);
  }
  bulk_wait0();
}

// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
siso_chunk_bwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_B,
                      const __grid_constant__ CUtensorMap tm_C, const __grid_constant__ CUtensorMap tm_dy,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_dB,
                      const __grid_constant__ CUtensorMap tm_dC,
                      BwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base, derived from smem_raw so that accesses stay shared-space
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  BSmem& s = *reinterpret_cast<BSmem*>(smem_raw + pad);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int units = a.Bn * a.H;
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int G = my_units * a.nch;

  if (tid == 0) {
    mbar_init(&s.ld_full, 1);
    mbar_init(&s.dy_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.sc_full[i], 32);
      mbar_init(&s.sc_empty[i], kScalReaders);
    }
    mbar_init(&s.edy_ready, 128);
    mbar_init(&s.xread, 128);
    mbar_init(&s.dkn_ready, 128);
    mbar_init(&s.p1_done, 1);
    mbar_init(&s.ep1_done, kEp1Arrivals);
    mbar_init(&s.p2_done, 1);
    mbar_init(&s.ep2_done, 256);
    mbar_init(&s.st_sync, 128);
    mbar_init(&s.p1b_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (a.D < kD) {
    // d_state 64: the upper halves of the C / B tiles are never loaded; they read as zero
    for (int i = tid; i < 2 * (int)(kTile / 16); i += kThreads) {
      uint8_t* t = i < (int)(kTile / 16) ? s.c[1] : s.b[1];
      reinterpret_cast<uint4*>(t)[i % (kTile / 16)] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_B);
      prefetch_tensormap(&tm_C);
      prefetch_tensormap(&tm_dy);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_dB);
      prefetch_tensormap(&tm_dC);
      control_role(&tm_x, &tm_B, &tm_C, &tm_dy, &tm_k, &tm_dB, &tm_dC, a, s, tbase, G);
    }
  } else if (warp == 1) {
    scalar_role(a, s, G, lane);
  } else if (warp < 4) {
    wx_role(s, G, tid - 64);
  } else if (warp < 12) {
    ep_role(a, s, tbase, G, warp, (tid - 128) & 127, (tid - 128) >> 7);
  } else {
    state_role(a, s, tbase, G, warp, tid - 384);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------
// dADT, dDT, dtrap; CTA per (unit, chunk), thread = row. dADT_r is the suffix sum of
// q - beta dbeta - gamma dgamma over the rest of the chunk (fp64) plus the exact value at
// the next chunk's first row t0: <dk, k> of that chunk - gamma_{t0} dgamma_{t0}.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) siso_chunk_bwd_scal_kernel(BwdArgs a) {
  const int u = (int)(blockIdx.x / (unsigned)a.nch), tt = (int)(blockIdx.x - (unsigned)u * a.nch);
  const int b = u / a.H, h = u - b * a.H;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  __shared__ double wsum[4];
  const int t = tt * 128 + tid;
  const bool v = t < a.L;
  double e = 0.0;
  float dbe = 0.f, dga = 0.f, tr = 0.f, dt = 0.f;
  if (v) {
    const int64_t pos = (int64_t)u * a.L + t;
    const float qv = a.sq[pos];
    dbe = a.sbeta[pos];
    dga = a.sgam[pos];
    dt = ld_scal(a.dt, a.sdt, b, t, h);
    tr = sigmoidf_(ld_scal(a.trap, a.strap, b, t, h));
    const float be = dt * (1.0f - tr) + 0.5f * dt * tr;
    const float ga = 0.5f * dt * tr;
    e = (double)qv - (double)be * dbe - (double)ga * dga;
  }
  double sfx = e;  // suffix sum within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_down_sync(0xffffffffu, sfx, o);
    if (lane + o < 32) sfx += y;
  }
  if (lane == 0) wsum[w] = sfx;
  __syncthreads();
  double hi = 0.0;
  for (int w2 = w + 1; w2 < 4; ++w2) hi += wsum[w2];
  double carry = 0.0;  // dADT at the next chunk's first row (none after the last chunk)
  if (tt + 1 < a.nch) {
    const int t1 = (tt + 1) * 128;
    const float* kd = a.skdot + ((int64_t)u * a.nch + tt + 1) * 4;
    const float tr1 = sigmoidf_(ld_scal(a.trap, a.strap, b, t1, h));
    const float ga1 = 0.5f * ld_scal(a.dt, a.sdt, b, t1, h) * tr1;
    carry = ((double)kd[0] + kd[1]) + ((double)kd[2] + kd[3]) - (double)ga1 * a.sgam[(int64_t)u * a.L + t1];
  }
  if (v) {
    a.dadt[(int64_t)b * a.sdadt.b + (int64_t)t * a.sdadt.l + (int64_t)h * a.sdadt.h] = (float)(carry + hi + sfx);
    a.ddt[(int64_t)b * a.sddt.b + (int64_t)t * a.sddt.l + (int64_t)h * a.sddt.h] =
        dbe * (1.0f - 0.5f * tr) + dga * 0.5f * tr;
    a.dtrap[(int64_t)b * a.sdtrap.b + (int64_t)t * a.sdtrap.l + (int64_t)h * a.sdtrap.h] =
        0.5f * dt * (dga - dbe) * tr * (1.0f - tr);
  }
}

// 2-d bf16 map over the chunk states: rows of 64 (p) elements, 128-row boxes
int make_kstate_map(CUtensorMap* m, const void* base, int64_t rows) {
  auto enc = chunk_encode_fn();
  if (!enc) return fail(M3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)kP, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kP * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kD};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M3_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return M3_OK;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool s8(const Str3& s) { return (s.b % 8 == 0) && (s.l % 8 == 0) && (s.h % 8 == 0); }

}  // namespace

size_t siso_chunk_kstate_bytes(int64_t Bn, int64_t L, int64_t H) {
  const int64_t nch = (L + Q - 1) / Q;
  return (size_t)(Bn * H * nch) * kD * kP * sizeof(__nv_bfloat16);
}

size_t siso_chunk_bwd_scratch_bytes(int64_t Bn, int64_t L, int64_t H) {
  const int64_t nch = (L + Q - 1) / Q;
  return 3 * sizeof(float) * (size_t)(Bn * H * L) + 4 * sizeof(float) * (size_t)(Bn * H * nch);
}

bool siso_chunk_bwd_supported(const SisoParams& p, int xdt, int bcdt) {
  if (p.D != kD && p.D != 64) return false;
  SisoParams f = p;
  f.y = nullptr;
  f.sy = Str3{0, 0, 0};
  if (!siso_chunk_supported(f, xdt, bcdt)) return false;
  if (!a16(p.dy) || !a16(p.dx) || !a16(p.dB) || !a16(p.dC)) return false;
  if (!s8(p.sdy) || !s8(p.sdx) || !s8(p.sdB) || !s8(p.sdC)) return false;
  const int64_t nch = (p.L + Q - 1) / Q;
  return (int64_t)p.Bn * p.H * nch * kD < (int64_t)INT32_MAX;
}

int launch_siso_bwd_chunked(const SisoParams& p, float* scratch, cudaStream_t s) {
  CUtensorMap mx, mb, mc, mdy, mk, mdb, mdc;
  const int nch = (p.L + Q - 1) / Q;
  const int units = p.Bn * p.H;
  M3_TRY(chunk_tmap_4d(&mx, p.x, p.P, p.H, p.L, p.Bn, p.sx));
  M3_TRY(chunk_tmap_4d(&mb, p.Bm, p.D, p.H, p.L, p.Bn, p.sB));
  M3_TRY(chunk_tmap_4d(&mc, p.Cm, p.D, p.H, p.L, p.Bn, p.sC));
  M3_TRY(chunk_tmap_4d(&mdy, p.dy, p.P, p.H, p.L, p.Bn, p.sdy));
  M3_TRY(make_kstate_map(&mk, p.kstates, (int64_t)units * nch * kD));
  M3_TRY(chunk_tmap_4d(&mdb, p.dB, p.D, p.H, p.L, p.Bn, p.sdB));
  M3_TRY(chunk_tmap_4d(&mdc, p.dC, p.D, p.H, p.L, p.Bn, p.sdC));
  BwdArgs a{};
  a.Bn = p.Bn; a.L = p.L; a.H = p.H; a.nch = nch;
  a.D = p.D; a.nkd = p.D / 16;
  a.adt = p.adt; a.sadt = p.sadt;
  a.dt = p.dt; a.sdt = p.sdt;
  a.trap = p.trap; a.strap = p.strap;
  a.Dskip = p.Dskip; a.sD = p.sD;
  a.h0 = p.h0; a.bx0 = p.bx0;
  a.dx = reinterpret_cast<__nv_bfloat16*>(p.dx); a.sdx = p.sdx;
  a.dB = reinterpret_cast<__nv_bfloat16*>(p.dB); a.sdB = p.sdB;
  a.dC = reinterpret_cast<__nv_bfloat16*>(p.dC); a.sdC = p.sdC;
  a.dadt = p.dadt; a.sdadt = p.sdadt;
  a.ddt = p.ddt; a.sddt = p.sddt;
  a.dtrap = p.dtrap; a.sdtrap = p.sdtrap;
  a.dD = p.dD; a.dh0 = p.dh0; a.dbx0 = p.dbx0;
  const size_t npos = (size_t)units * p.L;
  a.sq = scratch;
  a.sbeta = scratch + npos;
  a.sgam = scratch + 2 * npos;
  a.skdot = scratch + 3 * npos;
  const size_t smem = sizeof(BSmem) + 1024;
  // the shared-memory opt-in belongs to each device's context: set it once per device
  static std::atomic<bool> smem_set[kMaxDevices];
  M3_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(siso_chunk_bwd_kernel), smem, smem_set));
  int sms = 0;
  M3_TRY(device_sm_count(&sms));
  const int grid = units < sms ? units : sms;
  siso_chunk_bwd_kernel<<<grid, kThreads, smem, s>>>(mx, mb, mc, mdy, mk, mdb, mdc, a);
  M3_TRY(check_launch("siso_chunk_bwd_kernel"));
  const int64_t tiles = (int64_t)units * a.nch;
  if (tiles > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "siso backward: too many (unit, chunk) tiles");
  siso_chunk_bwd_scal_kernel<<<(unsigned)tiles, 128, 0, s>>>(a);
  return check_launch("siso_chunk_bwd_scal_kernel");
}

int chunk_bwd_error_word(bool reset, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_bwd_error, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_bwd_error, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("chunk error word: ") + cudaGetErrorString(e));
  *out = v;
  return M3_OK;
}

}  // namespace m3
