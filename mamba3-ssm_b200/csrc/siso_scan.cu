// SISO exponential-trapezoidal scan on CUDA cores in fp32: the exact path used for fp32
// I/O (parity rel 1e-4) and for shapes outside the chunked tensor-core kernel.
//
// Recurrence (the loop of mamba3_ssm/ops.py:166-175, per (b, h)):
//   u_t = x_t (x) B_t                                   (P x D outer product)
//   h_t = a_t h_{t-1} + beta_t u_t + gamma_t u_{t-1}    a = e^{ADT}, tr = sigmoid(trap),
//                                                       beta = dt(1-tr) + dt tr/2,
//                                                       gamma = dt tr/2
//   y_t = h_t C_t + D x_t
// This is the blend (1-tr) Bx + tr (Bx + Bx_prev)/2 of ops.py:171-173 regrouped.
//
// Forward ("PM" mapping): a CTA owns one (b, h) and a block of p rows; each thread holds
// one p row and DSEG = min(D, 32) state columns in registers, and the y readout reduces
// over D inside the thread plus a shuffle across the TPP = D/DSEG threads of the row.
// Inputs are staged T timesteps at a time into shared memory (converted to fp32).
//
// Backward (three streaming passes, no stored states):
//   A  forward time, "DM" mapping (thread = one d column, PT rows):  dC_t = h_t^T dy_t and
//      q_t = <dy_t, C_t h_t> (workspace);
//   B1 reverse time, PM mapping: adjoint g_t = a_{t+1} g_{t+1} + dy_t C_t^T, giving dx_t,
//      dbeta_t = <g_t, u_t>, dgamma_t = <g_t, u_{t-1}>, then dDT, dtrap and
//      dADT_r = sum_{s>=r} (q_s - beta_s dbeta_s - gamma_s dgamma_s)  (a reverse cumsum:
//      dL/dLambda_s = <dy_s, C_s h_s> - <g_s, w_s> with Lambda the cumulative log decay);
//   B2 reverse time, DM mapping: dB_t = beta_t g_t^T x_t + gamma_{t+1} g_{t+1}^T x_t.
#include "m3_common.cuh"
#include "siso_scan.cuh"

namespace m3 {

namespace {

constexpr int kT = 32;  // timesteps staged per chunk

template <typename T>
__device__ __forceinline__ const T* row_ptr(const void* base, const Str3& s, int b, int t, int h) {
  return reinterpret_cast<const T*>(base) + (int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h;
}
template <typename T>
__device__ __forceinline__ T* row_ptr_w(void* base, const Str3& s, int b, int t, int h) {
  return reinterpret_cast<T*>(base) + (int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h;
}
__device__ __forceinline__ float scal(const float* base, const Str3& s, int b, int t, int h) {
  return base[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h];
}

// dst[r][c] (row pitch W floats) = row (t0 + r), column col0 + c; zero outside [0,L) x [0,ncol)
template <typename T>
__device__ __forceinline__ void stage_rows(float* dst, int W, const void* base, const Str3& s, int b,
                                           int h, int t0, int nrows, int L, int col0, int ncol) {
  for (int i = threadIdx.x; i < nrows * W; i += blockDim.x) {
    const int r = i / W, c = i - r * W;
    const int t = t0 + r, cc = col0 + c;
    float v = 0.f;
    if (t >= 0 && t < L && cc < ncol) v = to_f32(row_ptr<T>(base, s, b, t, h)[cc]);
    dst[i] = v;
  }
}

// per-timestep coefficients for rows t0 + r, r < nrows (zeros outside [0, L))
__device__ __forceinline__ void stage_coeffs(const SisoParams& a, int b, int h, int t0, int nrows,
                                             float* sa, float* sbe, float* sga, float* str_,
                                             float* sdt) {
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
    const int t = t0 + r;
    float av = 0.f, be = 0.f, ga = 0.f, tr = 0.f, dt = 0.f;
    if (t >= 0 && t < a.L) {
      av = expf(scal(a.adt, a.sadt, b, t, h));
      dt = scal(a.dt, a.sdt, b, t, h);
      tr = sigmoidf_(scal(a.trap, a.strap, b, t, h));
      be = dt * (1.0f - tr) + 0.5f * dt * tr;
      ga = 0.5f * dt * tr;
    }
    sa[r] = av;
    sbe[r] = be;
    sga[r] = ga;
    if (str_) str_[r] = tr;
    if (sdt) sdt[r] = dt;
  }
}

template <int TPP>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = TPP / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int DS> struct PMShape {
  static constexpr int DSEG = DS < 32 ? DS : 32;
  static constexpr int TPP = DS / DSEG;
  static constexpr int NV = DSEG / 4;
};

// ------------------------------------------------------------------------------------
// forward, PM mapping
// ------------------------------------------------------------------------------------
template <typename TX, typename TB, int DS>
__global__ void __launch_bounds__(256) siso_fwd_pm_kernel(SisoParams a) {
  using S = PMShape<DS>;
  constexpr int TPP = S::TPP, NV = S::NV, DSEG = S::DSEG;
  const int PB = blockDim.x / TPP;
  const int tid = threadIdx.x, pl = tid / TPP, ds = tid % TPP;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int p0 = blockIdx.y * PB, p = p0 + pl;
  const bool pv = p < a.P;

  extern __shared__ float4 smem4[];
  float* sB = reinterpret_cast<float*>(smem4);
  float* sC = sB + kT * DS;
  float* sX = sC + kT * DS;
  float* sY = sX + kT * PB;
  float* sA = sY + kT * PB;
  float* sBe = sA + kT;
  float* sGa = sBe + kT;

  float hs[DSEG], up[DSEG];
  const int64_t st_off = (((int64_t)b * a.H + h) * a.P + (pv ? p : 0)) * DS;
#pragma unroll
  for (int g = 0; g < NV; ++g)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = 4 * (ds + TPP * g) + k;
      hs[4 * g + k] = (a.h0 && pv) ? a.h0[st_off + d] : 0.f;
      up[4 * g + k] = (a.bx0 && pv) ? a.bx0[st_off + d] : 0.f;
    }
  const float Dk = a.Dskip[h * a.sD];

  for (int t0 = 0; t0 < a.L; t0 += kT) {
    const int nT = min(kT, a.L - t0);
    __syncthreads();
    stage_rows<TB>(sB, DS, a.Bm, a.sB, b, h, t0, nT, a.L, 0, DS);
    stage_rows<TB>(sC, DS, a.Cm, a.sC, b, h, t0, nT, a.L, 0, DS);
    stage_rows<TX>(sX, PB, a.x, a.sx, b, h, t0, nT, a.L, p0, a.P);
    stage_coeffs(a, b, h, t0, nT, sA, sBe, sGa, nullptr, nullptr);
    __syncthreads();
    for (int i = 0; i < nT; ++i) {
      const float xv = sX[i * PB + pl];
      const float av = sA[i], bv = sBe[i], gv = sGa[i];
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const float4* b4 = reinterpret_cast<const float4*>(sB + i * DS);
      const float4* c4 = reinterpret_cast<const float4*>(sC + i * DS);
#pragma unroll
      for (int g = 0; g < NV; ++g) {
        const float4 bb = b4[ds + TPP * g];
        const float4 cc = c4[ds + TPP * g];
        const float bk[4] = {bb.x, bb.y, bb.z, bb.w};
        const float ck[4] = {cc.x, cc.y, cc.z, cc.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * g + k;
          const float u = xv * bk[k];
          const float hn = fmaf(av, hs[j], fmaf(bv, u, gv * up[j]));
          hs[j] = hn;
          up[j] = u;
          acc[k] = fmaf(ck[k], hn, acc[k]);
        }
      }
      float s = group_sum<TPP>((acc[0] + acc[1]) + (acc[2] + acc[3]));
      if (ds == 0) sY[i * PB + pl] = fmaf(Dk, xv, s);
    }
    __syncthreads();
    for (int i = tid; i < nT * PB; i += blockDim.x) {
      const int r = i / PB, c = i - r * PB;
      if (p0 + c < a.P) st(row_ptr_w<TX>(a.y, a.sy, b, t0 + r, h) + p0 + c, sY[i]);
    }
  }
  if (pv) {
#pragma unroll
    for (int g = 0; g < NV; ++g)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = 4 * (ds + TPP * g) + k;
        if (a.h_last) a.h_last[st_off + d] = hs[4 * g + k];
        if (a.bx_last) a.bx_last[st_off + d] = up[4 * g + k];
      }
  }
}

// ------------------------------------------------------------------------------------
// backward pass A: forward time, DM mapping. dC_t[d] = sum_p dy_t[p] h_t[p,d]; q_t.
// thread = (d, psub); rows p = 4*(psub + TPD*g) + k, g < PT/4.
// ------------------------------------------------------------------------------------
template <typename TX, typename TB, int DS, int PT>
__global__ void __launch_bounds__(512) siso_bwd_a_kernel(SisoParams a, int TPD) {
  constexpr int NG = PT / 4;
  const int PM = TPD * PT;  // padded rows held by the CTA (>= P)
  const int tid = threadIdx.x, d = tid / TPD, ps = tid % TPD;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;

  extern __shared__ float4 smem4[];
  float* sB = reinterpret_cast<float*>(smem4);  // [kT][DS]
  float* sC = sB + kT * DS;                       // [kT][DS]
  float* sDC = sC + kT * DS;                      // [kT][DS]
  float* sX = sDC + kT * DS;                      // [kT][PM]
  float* sG = sX + kT * PM;                       // [kT][PM]  dy
  float* sA = sG + kT * PM;
  float* sBe = sA + kT;
  float* sGa = sBe + kT;

  float hs[PT], up[PT];
  const int64_t st_base = ((int64_t)b * a.H + h) * a.P;
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int p = 4 * (ps + TPD * g) + k;
      const bool v = p < a.P;
      hs[4 * g + k] = (a.h0 && v) ? a.h0[(st_base + p) * DS + d] : 0.f;
      up[4 * g + k] = (a.bx0 && v) ? a.bx0[(st_base + p) * DS + d] : 0.f;
    }

  for (int t0 = 0; t0 < a.L; t0 += kT) {
    const int nT = min(kT, a.L - t0);
    __syncthreads();
    stage_rows<TB>(sB, DS, a.Bm, a.sB, b, h, t0, nT, a.L, 0, DS);
    stage_rows<TB>(sC, DS, a.Cm, a.sC, b, h, t0, nT, a.L, 0, DS);
    stage_rows<TX>(sX, PM, a.x, a.sx, b, h, t0, nT, a.L, 0, a.P);
    stage_rows<TX>(sG, PM, a.dy, a.sdy, b, h, t0, nT, a.L, 0, a.P);
    stage_coeffs(a, b, h, t0, nT, sA, sBe, sGa, nullptr, nullptr);
    __syncthreads();
    for (int i = 0; i < nT; ++i) {
      const float bd = sB[i * DS + d];
      const float av = sA[i], bv = sBe[i], gv = sGa[i];
      const float4* x4 = reinterpret_cast<const float4*>(sX + i * PM);
      const float4* g4 = reinterpret_cast<const float4*>(sG + i * PM);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const float4 xx = x4[ps + TPD * g];
        const float4 yy = g4[ps + TPD * g];
        const float xk[4] = {xx.x, xx.y, xx.z, xx.w};
        const float yk[4] = {yy.x, yy.y, yy.z, yy.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * g + k;
          const float u = xk[k] * bd;
          const float hn = fmaf(av, hs[j], fmaf(bv, u, gv * up[j]));
          hs[j] = hn;
          up[j] = u;
          if (k & 1) acc1 = fmaf(yk[k], hn, acc1); else acc0 = fmaf(yk[k], hn, acc0);
        }
      }
      float s = acc0 + acc1;
      for (int o = TPD / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (ps == 0) sDC[i * DS + d] = s;
    }
    __syncthreads();
    for (int i = tid; i < nT * DS; i += blockDim.x) {
      const int r = i / DS, c = i - r * DS;
      st(row_ptr_w<TB>(a.dC, a.sdC, b, t0 + r, h) + c, sDC[i]);
    }
    // q_t = sum_d C_t[d] dC_t[d]: one warp per row
    const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    for (int r = warp; r < nT; r += nw) {
      float s = 0.f;
      for (int c = lane; c < DS; c += 32) s = fmaf(sC[r * DS + c], sDC[r * DS + c], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) a.q[((int64_t)b * a.H + h) * a.L + t0 + r] = s;
    }
  }
}

// ------------------------------------------------------------------------------------
// backward pass B1: reverse time, PM mapping -> dx, dADT, dDT, dtrap, dD, dh0, dbx0.
// Chunk rows are staged with one extra row on each side: row r <-> t = t0 - 1 + r.
// ------------------------------------------------------------------------------------
template <typename TX, typename TB, int DS>
__global__ void __launch_bounds__(512) siso_bwd_b1_kernel(SisoParams a) {
  using S = PMShape<DS>;
  constexpr int TPP = S::TPP, NV = S::NV, DSEG = S::DSEG;
  constexpr int R = kT + 2;
  const int PB = blockDim.x / TPP;
  const int tid = threadIdx.x, pl = tid / TPP, ds = tid % TPP;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int p0 = blockIdx.y * PB, p = p0 + pl;
  const bool pv = p < a.P;

  extern __shared__ float4 smem4[];
  float* sB = reinterpret_cast<float*>(smem4);  // [R][DS]
  float* sC = sB + R * DS;                        // [R][DS]
  float* sX = sC + R * DS;                        // [R][PB]
  float* sG = sX + R * PB;                        // [R][PB] dy
  float* sDX = sG + R * PB;                       // [kT][PB]
  float* sP1 = sDX + kT * PB;                     // [kT][PB]
  float* sP2 = sP1 + kT * PB;                     // [kT][PB]
  float* sA = sP2 + kT * PB;                      // [R]
  float* sBe = sA + R;
  float* sGa = sBe + R;
  float* sTr = sGa + R;
  float* sDt = sTr + R;
  float* sRed = sDt + R;                          // [2][kT]

  float g[DSEG];
#pragma unroll
  for (int j = 0; j < DSEG; ++j) g[j] = 0.f;
  const float Dk = a.Dskip[h * a.sD];
  const int64_t st_off = (((int64_t)b * a.H + h) * a.P + (pv ? p : 0)) * DS;
  float r2_next = 0.f;   // (g_{t+1} B_t)[p] from the previous (later) step
  float ddacc = 0.f;     // sum_t dy_t[p] x_t[p]
  double cum = 0.0;      // reverse cumsum of dL/dLambda
  const int nchunk = (a.L + kT - 1) / kT;

  for (int c = nchunk - 1; c >= 0; --c) {
    const int t0 = c * kT;
    const int nT = min(kT, a.L - t0);
    __syncthreads();
    stage_rows<TB>(sB, DS, a.Bm, a.sB, b, h, t0 - 1, nT + 2, a.L, 0, DS);
    stage_rows<TB>(sC, DS, a.Cm, a.sC, b, h, t0 - 1, nT + 2, a.L, 0, DS);
    stage_rows<TX>(sX, PB, a.x, a.sx, b, h, t0 - 1, nT + 2, a.L, p0, a.P);
    stage_rows<TX>(sG, PB, a.dy, a.sdy, b, h, t0 - 1, nT + 2, a.L, p0, a.P);
    stage_coeffs(a, b, h, t0 - 1, nT + 2, sA, sBe, sGa, sTr, sDt);
    __syncthreads();
    for (int i = nT - 1; i >= 0; --i) {
      const int r = i + 1;  // staged row of t = t0 + i
      const float a_next = sA[r + 1], g_next = sGa[r + 1];
      const float dyv = sG[r * PB + pl];
      const float4* c4 = reinterpret_cast<const float4*>(sC + r * DS);
      const float4* b4 = reinterpret_cast<const float4*>(sB + r * DS);
      const float4* bp4 = reinterpret_cast<const float4*>(sB + (r - 1) * DS);
      float r1 = 0.f, r2 = 0.f;
#pragma unroll
      for (int q = 0; q < NV; ++q) {
        const float4 cc = c4[ds + TPP * q];
        const float4 bb = b4[ds + TPP * q];
        const float4 bp = bp4[ds + TPP * q];
        const float ck[4] = {cc.x, cc.y, cc.z, cc.w};
        const float bk[4] = {bb.x, bb.y, bb.z, bb.w};
        const float pk[4] = {bp.x, bp.y, bp.z, bp.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * q + k;
          const float gn = fmaf(a_next, g[j], dyv * ck[k]);
          g[j] = gn;
          r1 = fmaf(gn, bk[k], r1);
          r2 = fmaf(gn, pk[k], r2);
        }
      }
      r1 = group_sum<TPP>(r1);
      if (c == 0 && i == 0 && a.bx0) {
        // u_{-1} is the carried B*x matrix, not a rank-1 product
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < NV; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (pv) s = fmaf(g[4 * q + k], a.bx0[st_off + 4 * (ds + TPP * q) + k], s);
        r2 = group_sum<TPP>(s);
        if (ds == 0) sP2[i * PB + pl] = r2;
      } else {
        r2 = group_sum<TPP>(r2);
        if (ds == 0) sP2[i * PB + pl] = sX[(r - 1) * PB + pl] * r2;
      }
      const float xv = sX[r * PB + pl];
      if (ds == 0) {
        sDX[i * PB + pl] = fmaf(Dk, dyv, fmaf(sBe[r], r1, g_next * r2_next));
        sP1[i * PB + pl] = xv * r1;
        ddacc = fmaf(dyv, xv, ddacc);
      }
      r2_next = r2;
    }
    __syncthreads();
    for (int i = tid; i < nT * PB; i += blockDim.x) {
      const int r = i / PB, cc = i - r * PB;
      if (p0 + cc < a.P) st(row_ptr_w<TX>(a.dx, a.sdx, b, t0 + r, h) + p0 + cc, sDX[i]);
    }
    // dbeta_t, dgamma_t: reduce the per-row partials of this CTA's p block
    const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    for (int i = warp; i < 2 * nT; i += nw) {
      const float* src = (i < nT) ? (sP1 + i * PB) : (sP2 + (i - nT) * PB);
      float s = 0.f;
      for (int cc = lane; cc < PB; cc += 32) s += src[cc];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sRed[i] = s;
    }
    __syncthreads();
    if (tid == 0) {
      // Only the p block holding row 0 writes the scalars when the head is split over
      // several CTAs (gridDim.y > 1 is not used for the backward; see the launcher).
      for (int i = nT - 1; i >= 0; --i) {
        const int r = i + 1, t = t0 + i;
        const float dbeta = sRed[i], dgam = sRed[nT + i];
        const float qv = a.q[((int64_t)b * a.H + h) * a.L + t];
        cum += (double)qv - (double)sBe[r] * dbeta - (double)sGa[r] * dgam;
        const float tr = sTr[r], dtv = sDt[r];
        a.dadt[(int64_t)b * a.sdadt.b + (int64_t)t * a.sdadt.l + (int64_t)h * a.sdadt.h] = (float)cum;
        a.ddt[(int64_t)b * a.sddt.b + (int64_t)t * a.sddt.l + (int64_t)h * a.sddt.h] =
            dbeta * (1.0f - 0.5f * tr) + dgam * 0.5f * tr;
        a.dtrap[(int64_t)b * a.sdtrap.b + (int64_t)t * a.sdtrap.l + (int64_t)h * a.sdtrap.h] =
            0.5f * dtv * (dgam - dbeta) * tr * (1.0f - tr);
      }
    }
  }
  // gradients of the initial state: h_0 = a_0 h_{-1} + ... + gamma_0 u_{-1}
  if (pv && (a.dh0 || a.dbx0)) {
    const float a0 = expf(scal(a.adt, a.sadt, b, 0, h));
    const float dt0 = scal(a.dt, a.sdt, b, 0, h);
    const float tr0 = sigmoidf_(scal(a.trap, a.strap, b, 0, h));
    const float g0 = 0.5f * dt0 * tr0;
#pragma unroll
    for (int q = 0; q < NV; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = 4 * (ds + TPP * q) + k;
        if (a.dh0) a.dh0[st_off + d] = a0 * g[4 * q + k];
        if (a.dbx0) a.dbx0[st_off + d] = g0 * g[4 * q + k];
      }
  }
  // dD[h] += sum over this CTA's rows
  __shared__ float sdd[32];
  float v = ddacc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((tid & 31) == 0) sdd[tid >> 5] = v;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += sdd[w];
    atomicAdd(a.dD + h, s);
  }
}

// ------------------------------------------------------------------------------------
// backward pass B2: reverse time, DM mapping -> dB_t[d] = beta_t s1_t + gamma_{t+1} s2_{t+1}
//   s1_t = sum_p x_t[p] g_t[p,d],  s2_t = sum_p x_{t-1}[p] g_t[p,d]
// ------------------------------------------------------------------------------------
template <typename TX, typename TB, int DS, int PT>
__global__ void __launch_bounds__(512) siso_bwd_b2_kernel(SisoParams a, int TPD) {
  constexpr int NG = PT / 4;
  constexpr int R = kT + 2;
  const int PM = TPD * PT;
  const int tid = threadIdx.x, d = tid / TPD, ps = tid % TPD;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;

  extern __shared__ float4 smem4[];
  float* sC = reinterpret_cast<float*>(smem4);  // [R][DS]
  float* sDB = sC + R * DS;                       // [kT][DS]
  float* sX = sDB + kT * DS;                      // [R][PM]
  float* sG = sX + R * PM;                        // [R][PM] dy
  float* sA = sG + R * PM;
  float* sBe = sA + R;
  float* sGa = sBe + R;

  float g[PT];
#pragma unroll
  for (int j = 0; j < PT; ++j) g[j] = 0.f;
  float s2_next = 0.f;
  const int nchunk = (a.L + kT - 1) / kT;
  for (int c = nchunk - 1; c >= 0; --c) {
    const int t0 = c * kT;
    const int nT = min(kT, a.L - t0);
    __syncthreads();
    stage_rows<TB>(sC, DS, a.Cm, a.sC, b, h, t0 - 1, nT + 2, a.L, 0, DS);
    stage_rows<TX>(sX, PM, a.x, a.sx, b, h, t0 - 1, nT + 2, a.L, 0, a.P);
    stage_rows<TX>(sG, PM, a.dy, a.sdy, b, h, t0 - 1, nT + 2, a.L, 0, a.P);
    stage_coeffs(a, b, h, t0 - 1, nT + 2, sA, sBe, sGa, nullptr, nullptr);
    __syncthreads();
    for (int i = nT - 1; i >= 0; --i) {
      const int r = i + 1;
      const float a_next = sA[r + 1], gam_next = sGa[r + 1];
      const float cd = sC[r * DS + d];
      const float4* y4 = reinterpret_cast<const float4*>(sG + r * PM);
      const float4* x4 = reinterpret_cast<const float4*>(sX + r * PM);
      const float4* xp4 = reinterpret_cast<const float4*>(sX + (r - 1) * PM);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int q = 0; q < NG; ++q) {
        const float4 yy = y4[ps + TPD * q];
        const float4 xx = x4[ps + TPD * q];
        const float4 xp = xp4[ps + TPD * q];
        const float yk[4] = {yy.x, yy.y, yy.z, yy.w};
        const float xk[4] = {xx.x, xx.y, xx.z, xx.w};
        const float pk[4] = {xp.x, xp.y, xp.z, xp.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * q + k;
          const float gn = fmaf(a_next, g[j], yk[k] * cd);
          g[j] = gn;
          s1 = fmaf(xk[k], gn, s1);
          s2 = fmaf(pk[k], gn, s2);
        }
      }
      for (int o = TPD / 2; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      if (ps == 0) sDB[i * DS + d] = fmaf(sBe[r], s1, gam_next * s2_next);
      s2_next = s2;
    }
    __syncthreads();
    for (int i = tid; i < nT * DS; i += blockDim.x) {
      const int r = i / DS, cc = i - r * DS;
      st(row_ptr_w<TB>(a.dB, a.sdB, b, t0 + r, h) + cc, sDB[i]);
    }
  }
}

// ------------------------------------------------------------------------------------
// launch helpers
// ------------------------------------------------------------------------------------
template <typename K>
int set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  }
  return M3_OK;
}

inline int pm_block_rows(int P, int TPP, int max_threads) {
  const int unit = 32 / TPP;            // rows per warp
  int pb = ((P + unit - 1) / unit) * unit;
  return pb < max_threads / TPP ? pb : max_threads / TPP;
}

// threads per state column in the d-major kernels: enough to cover P rows, and at least
// 32 / DS so that the CTA (DS * TPD threads) is made of whole warps
inline int dm_tpd(int P, int PT, int DS) {
  int t = 1;
  while (t * PT < P || t * DS < 32) t <<= 1;
  return t;
}

template <typename TX, typename TB, int DS>
int fwd_typed(const SisoParams& p, cudaStream_t s) {
  constexpr int TPP = PMShape<DS>::TPP;
  const int PB = pm_block_rows(p.P, TPP, 256);
  const size_t smem = sizeof(float) * ((size_t)kT * (2 * DS + 2 * PB) + 3 * kT);
  auto k = siso_fwd_pm_kernel<TX, TB, DS>;
  M3_TRY(set_smem(k, smem));
  dim3 grid(p.Bn * p.H, (p.P + PB - 1) / PB);
  k<<<grid, PB * TPP, smem, s>>>(p);
  return check_launch("siso_fwd_pm_kernel");
}

template <typename TX, typename TB, int DS, int PT>
int bwd_dm_typed(const SisoParams& p, cudaStream_t s) {
  const int TPD = dm_tpd(p.P, PT, DS);
  const int threads = DS * TPD;
  if (threads > 512 || TPD > 32) return fail(M3_ERR_UNSUPPORTED, "siso backward: headdim too large for d_state");
  const int PM = TPD * PT;
  {
    const size_t smem = sizeof(float) * ((size_t)kT * (3 * DS + 2 * PM) + 3 * kT);
    auto k = siso_bwd_a_kernel<TX, TB, DS, PT>;
    M3_TRY(set_smem(k, smem));
    k<<<p.Bn * p.H, threads, smem, s>>>(p, TPD);
    M3_TRY(check_launch("siso_bwd_a_kernel"));
  }
  {
    constexpr int TPP = PMShape<DS>::TPP;
    const int PB = pm_block_rows(p.P, TPP, 512);
    if (PB < p.P) return fail(M3_ERR_UNSUPPORTED, "siso backward: headdim above 512/(d_state/32)");
    const int R = kT + 2;
    const size_t smem = sizeof(float) * ((size_t)R * (2 * DS + 2 * PB) + (size_t)kT * 3 * PB + 5 * R + 2 * kT);
    auto k = siso_bwd_b1_kernel<TX, TB, DS>;
    M3_TRY(set_smem(k, smem));
    k<<<p.Bn * p.H, PB * TPP, smem, s>>>(p);
    M3_TRY(check_launch("siso_bwd_b1_kernel"));
  }
  {
    const int R = kT + 2;
    const size_t smem = sizeof(float) * ((size_t)R * (DS + 2 * PM) + (size_t)kT * DS + 3 * R);
    auto k = siso_bwd_b2_kernel<TX, TB, DS, PT>;
    M3_TRY(set_smem(k, smem));
    k<<<p.Bn * p.H, threads, smem, s>>>(p, TPD);
    M3_TRY(check_launch("siso_bwd_b2_kernel"));
  }
  return M3_OK;
}

template <typename TX, typename TB>
int fwd_dispatch_d(const SisoParams& p, cudaStream_t s) {
  switch (p.D) {
    case 16: return fwd_typed<TX, TB, 16>(p, s);
    case 32: return fwd_typed<TX, TB, 32>(p, s);
    case 64: return fwd_typed<TX, TB, 64>(p, s);
    case 128: return fwd_typed<TX, TB, 128>(p, s);
    case 256: return fwd_typed<TX, TB, 256>(p, s);
  }
  return fail(M3_ERR_UNSUPPORTED, "siso scan: d_state must be 16, 32, 64, 128 or 256");
}

template <typename TX, typename TB>
int bwd_dispatch_d(const SisoParams& p, cudaStream_t s) {
  // 16 rows per thread while the d-major CTA stays within 512 threads, else 32
  const bool big = dm_tpd(p.P, 16, p.D) * p.D > 512;
  switch (p.D) {
    case 16: return big ? bwd_dm_typed<TX, TB, 16, 32>(p, s) : bwd_dm_typed<TX, TB, 16, 16>(p, s);
    case 32: return big ? bwd_dm_typed<TX, TB, 32, 32>(p, s) : bwd_dm_typed<TX, TB, 32, 16>(p, s);
    case 64: return big ? bwd_dm_typed<TX, TB, 64, 32>(p, s) : bwd_dm_typed<TX, TB, 64, 16>(p, s);
    case 128: return big ? bwd_dm_typed<TX, TB, 128, 32>(p, s) : bwd_dm_typed<TX, TB, 128, 16>(p, s);
  }
  return fail(M3_ERR_UNSUPPORTED, "siso scan backward: d_state must be 16, 32, 64 or 128");
}

}  // namespace

#define M3_DISPATCH_TYPES(fn, xdt, bcdt, ...)                                                \
  do {                                                                                      \
    if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return fn<float, float>(__VA_ARGS__);      \
    if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16)                                          \
      return fn<__nv_bfloat16, __nv_bfloat16>(__VA_ARGS__);                                 \
    if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32) return fn<__nv_bfloat16, float>(__VA_ARGS__); \
    if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16) return fn<float, __nv_bfloat16>(__VA_ARGS__); \
    if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return fn<__half, __half>(__VA_ARGS__);    \
    if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return fn<__half, float>(__VA_ARGS__);     \
    return fail(M3_ERR_UNSUPPORTED, "unsupported dtype combination for x / B,C");            \
  } while (0)

int launch_siso_fwd_recurrent(const SisoParams& p, int xdt, int bcdt, cudaStream_t s) {
  M3_DISPATCH_TYPES(fwd_dispatch_d, xdt, bcdt, p, s);
}

int launch_siso_bwd_recurrent(const SisoParams& p, int xdt, int bcdt, cudaStream_t s) {
  M3_DISPATCH_TYPES(bwd_dispatch_d, xdt, bcdt, p, s);
}

}  // namespace m3
