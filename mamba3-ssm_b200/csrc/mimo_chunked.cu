// Chunk-parallel MIMO scan forward (the loop of mamba3_ssm/ops.py:226-240 with its rank-R
// projections and the D skip), fp32 on CUDA cores.
//
// The MIMO state is one scalar per d, so the recurrence h_t = a_t h_{t-1} + beta_t Bx_t +
// gamma_t Bx_{t-1} (Bx_t = sum_r xr_t[r] B_t[r, :], xr_t = mimo_x x_t) is D independent
// first-order scans. Time is cut into chunks (64 steps forward, 32 backward) and every
// (b, h, chunk) gets its own CTA:
//   1. local:  the chunk's end state from a zero start, S_c, and its decay product A_c
//   2. carry:  per (b, h, d), in chunk order, carry_c = A_{c-1} carry_{c-1} + S_{c-1}
//              (carry_0 = h0), written over S; the last one is h_last
//   3. output: each chunk again from its carry, the readouts yr_t = C_t h_t + D xr_t and
//              y_t = mimo_o^T yr_t
// Bx_{t0-1}, which the first step of a chunk needs for its gamma term, is recomputed from
// x_{t0-1} and B_{t0-1} (bx0 for the first chunk). The kernels read x and B twice and C
// once; the per-chunk work is a few hundred steps of independent FMAs instead of one
// serial walk of the whole sequence per (b, h).
#include <algorithm>

#include "m3_common.cuh"
#include "mimo_scan.cuh"
#include "siso_chunk.cuh"
#include "sm100.cuh"

namespace m3 {
namespace {

constexpr int kTcF = 64;  // time steps per chunk, forward
constexpr int kTcB = 32;  // time steps per chunk, backward (four per-step state arrays in smem)
constexpr int kCT = 128;  // threads per CTA

template <typename T>
__device__ __forceinline__ float ldxc(const void* base, const Str3& s, int b, int t, int h, int p) {
  return to_f32(reinterpret_cast<const T*>(base)[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h + p]);
}
template <typename T>
__device__ __forceinline__ float ldbcc(const void* base, const Str4& s, int b, int t, int r, int h, int d) {
  return to_f32(reinterpret_cast<const T*>(base)[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)r * s.r +
                                                  (int64_t)h * s.h + d]);
}
__device__ __forceinline__ float scalc(const float* base, const Str3& s, int b, int t, int h) {
  return base[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h];
}

// Shared memory of one chunk: x rows t0-1 .. t0+n-1 (row 0 is t0-1), their rank
// projections xr, the step coefficients, mimo_x / mimo_o, and (output kernel) the states
// H and readouts yr of the chunk.
struct CSmem {
  float *x, *xr, *a, *be, *ga, *mx, *mo, *H, *yr;
};

template <int TC>
__host__ __device__ inline size_t csmem_floats(int P, int R, int D, bool out) {
  size_t n = (size_t)(TC + 1) * P + (size_t)(TC + 1) * R + 3 * (size_t)TC + 2 * (size_t)R * P;
  if (out) n += (size_t)TC * D + (size_t)TC * R;
  return n;
}

template <int TC>
__device__ inline CSmem ccarve(float* p, int P, int R, int D, bool out) {
  CSmem s;
  s.x = p; p += (TC + 1) * P;
  s.xr = p; p += (TC + 1) * R;
  s.a = p; p += TC;
  s.be = p; p += TC;
  s.ga = p; p += TC;
  s.mx = p; p += R * P;
  s.mo = p; p += R * P;
  s.H = out ? p : nullptr; p += out ? TC * D : 0;
  s.yr = out ? p : nullptr;
  return s;
}

template <typename TX>
__device__ void stage(const MimoParams& a, const CSmem& s, int b, int h, int t0, int n, bool out) {
  const int P = a.P, R = a.R, tid = threadIdx.x;
  for (int i = tid; i < R * P; i += kCT) {
    const int r = i / P, p = i - r * P;
    s.mx[i] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + p];
    if (out) s.mo[i] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + p];
  }
  for (int i = tid; i < (n + 1) * P; i += kCT) {
    const int r = i / P, p = i - r * P, t = t0 - 1 + r;
    s.x[i] = t >= 0 ? ldxc<TX>(a.x, a.sx, b, t, h, p) : 0.f;
  }
  for (int r = tid; r < n; r += kCT) {
    const int t = t0 + r;
    const float dt = scalc(a.dt, a.sdt, b, t, h);
    const float tr = sigmoidf_(scalc(a.trap, a.strap, b, t, h));
    s.a[r] = expf(scalc(a.adt, a.sadt, b, t, h));
    s.be[r] = dt * (1.0f - tr) + 0.5f * dt * tr;
    s.ga[r] = 0.5f * dt * tr;
  }
  __syncthreads();
  for (int i = tid; i < (n + 1) * R; i += kCT) {
    const int r = i / R, k = i - r * R;
    float acc = 0.f;
    for (int p = 0; p < P; ++p) acc = fmaf(s.x[r * P + p], s.mx[k * P + p], acc);
    s.xr[i] = acc;
  }
  __syncthreads();
}

// Bx_t[d] from the staged rank projections of row `row` (time t)
template <typename TB>
__device__ __forceinline__ float bx_at(const MimoParams& a, const float* xr_row, int b, int t, int h, int d) {
  float acc = 0.f;
  for (int r = 0; r < a.R; ++r) acc = fmaf(xr_row[r], ldbcc<TB>(a.Bm, a.sB, b, t, r, h, d), acc);
  return acc;
}

template <typename TB>
__device__ __forceinline__ float bx_before(const MimoParams& a, const CSmem& s, int b, int h, int t0, int d) {
  if (t0 > 0) return bx_at<TB>(a, s.xr, b, t0 - 1, h, d);
  return a.bx0 ? a.bx0[((int64_t)b * a.H + h) * a.D + d] : 0.f;
}

template <typename TX, typename TB, int TC>
__global__ void __launch_bounds__(kCT) mimo_local_kernel(MimoParams a, float* S, float* Adec, int nch) {
  extern __shared__ float4 csm4[];
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * TC, n = min(TC, a.L - t0);
  const CSmem s = ccarve<TC>(reinterpret_cast<float*>(csm4), a.P, a.R, a.D, false);
  stage<TX>(a, s, b, h, t0, n, false);
  for (int d = threadIdx.x; d < a.D; d += kCT) {
    float bxp = bx_before<TB>(a, s, b, h, t0, d);
    float hv = 0.f;
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      const float bx = bx_at<TB>(a, s.xr + (t + 1) * a.R, b, t0 + t, h, d);
      hv = fmaf(s.a[t], hv, fmaf(s.be[t], bx, s.ga[t] * bxp));
      bxp = bx;
    }
    S[((int64_t)u * nch + c) * a.D + d] = hv;
  }
  if (threadIdx.x == 0) {
    float prod = 1.f;
    for (int t = 0; t < n; ++t) prod *= s.a[t];
    Adec[(int64_t)u * nch + c] = prod;
  }
}

__global__ void __launch_bounds__(kCT) mimo_carry_kernel(MimoParams a, float* S, const float* Adec, int nch,
                                                          bool write_last) {
  const int u = blockIdx.x;
  for (int d = threadIdx.x; d < a.D; d += kCT) {
    float run = a.h0 ? a.h0[(int64_t)u * a.D + d] : 0.f;
    for (int c = 0; c < nch; ++c) {
      const int64_t i = ((int64_t)u * nch + c) * a.D + d;
      const float loc = S[i];
      S[i] = run;
      run = fmaf(Adec[(int64_t)u * nch + c], run, loc);
    }
    if (write_last && a.h_last) a.h_last[(int64_t)u * a.D + d] = run;
  }
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kCT) mimo_out_kernel(MimoParams a, const float* S, int nch) {
  extern __shared__ float4 csm4[];
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * kTcF, n = min(kTcF, a.L - t0);
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x;
  const CSmem s = ccarve<kTcF>(reinterpret_cast<float*>(csm4), P, R, D, true);
  stage<TX>(a, s, b, h, t0, n, true);
  // states of the chunk from its carry
  for (int d = tid; d < D; d += kCT) {
    float bxp = bx_before<TB>(a, s, b, h, t0, d);
    float hv = S[((int64_t)u * nch + c) * D + d];
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      const float bx = bx_at<TB>(a, s.xr + (t + 1) * R, b, t0 + t, h, d);
      hv = fmaf(s.a[t], hv, fmaf(s.be[t], bx, s.ga[t] * bxp));
      s.H[t * D + d] = hv;
      bxp = bx;
    }
    if (c == nch - 1 && a.bx_last) a.bx_last[(int64_t)u * D + d] = bxp;
  }
  __syncthreads();
  // yr_t[r] = C_t[r, :] . h_t + D xr_t[r]: a warp takes four (t, r) items at a time, lanes
  // over d, so four items' loads of C are in flight together
  const float Dk = a.Dskip[h * a.sD];
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kIt = 4;
  for (int pr0 = warp * kIt; pr0 < n * R; pr0 += (kCT / 32) * kIt) {
    float acc[kIt];
#pragma unroll
    for (int j = 0; j < kIt; ++j) {
      const int pr = pr0 + j;
      acc[j] = 0.f;
      if (pr < n * R) {
        const int t = pr / R, r = pr - t * R;
        for (int d = lane; d < D; d += 32) acc[j] = fmaf(ldbcc<TB>(a.Cm, a.sC, b, t0 + t, r, h, d), s.H[t * D + d], acc[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < kIt; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    if (lane < kIt && pr0 + lane < n * R) {
      float v = acc[0];
#pragma unroll
      for (int j = 1; j < kIt; ++j) v = lane == j ? acc[j] : v;
      const int pr = pr0 + lane, t = pr / R, r = pr - t * R;
      s.yr[pr] = fmaf(Dk, s.xr[(t + 1) * R + r], v);
    }
  }
  __syncthreads();
  // y_t = mimo_o^T yr_t
  for (int i = tid; i < n * P; i += kCT) {
    const int t = i / P, p = i - t * P;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(s.yr[t * R + r], s.mo[r * P + p], acc);
    st(reinterpret_cast<TX*>(a.y) + (int64_t)b * a.sy.b + (int64_t)(t0 + t) * a.sy.l + (int64_t)h * a.sy.h + p, acc);
  }
}

// ------------------------------------------------------------------------------------
// Backward. The adjoint of the state obeys the reverse recurrence
//   g_t = a_{t+1} g_{t+1} + E_t,   E_t = sum_r dyr_t[r] C_t[r, :],   dyr_t = mimo_o dy_t
// (D independent scans again), so it is chunked the same way in reverse:
//   B1 local:  g at each chunk start from a zero adjoint after the chunk, and the decay
//              product a_{t0+1} .. a_{t0+n} that carries the adjoint across the chunk
//   B2 carry:  in reverse chunk order, the adjoint entering each chunk from the right
//              (written over the local values); g_0 gives dh0 = a_0 g_0, dbx0 = gamma_0 g_0
//   B3 full:   each chunk recomputes its forward states (from the forward carries) and
//              its adjoints (from the backward carries) and emits dx, dB, dC, dDT, dtrap,
//              the per-step terms of dADT with their chunk total, and partial sums of dD,
//              dmimo_x, dmimo_o (atomics)
//   B4:        dADT_r = sum_{s >= r} (q_s - beta_s dbeta_s - gamma_s dgamma_s), the
//              suffix sums of B3's per-step terms across chunks (offsets in fp64)
// ------------------------------------------------------------------------------------
struct BSmem {
  float *dy, *dyr, *an;  // dy rows t0..t0+n-1, their mimo_o projections, a_{t0+1}..a_{t0+n}
};

template <typename TX>
__device__ void stage_dy(const MimoParams& a, const BSmem& s, const float* mo, int b, int h, int t0, int n) {
  const int P = a.P, R = a.R, tid = threadIdx.x;
  for (int i = tid; i < n * P; i += kCT) {
    const int r = i / P, p = i - r * P;
    s.dy[i] = ldxc<TX>(a.dy, a.sdy, b, t0 + r, h, p);
  }
  for (int r = tid; r < n; r += kCT) {
    const int t = t0 + 1 + r;
    s.an[r] = t < a.L ? expf(scalc(a.adt, a.sadt, b, t, h)) : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < n * R; i += kCT) {
    const int r = i / R, k = i - r * R;
    float acc = 0.f;
    for (int p = 0; p < P; ++p) acc = fmaf(s.dy[r * P + p], mo[k * P + p], acc);
    s.dyr[i] = acc;
  }
  __syncthreads();
}

template <typename TB>
__device__ __forceinline__ float e_at(const MimoParams& a, const float* dyr_row, int b, int t, int h, int d) {
  float acc = 0.f;
  for (int r = 0; r < a.R; ++r) acc = fmaf(dyr_row[r], ldbcc<TB>(a.Cm, a.sC, b, t, r, h, d), acc);
  return acc;
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kCT) mimo_bwd_local_kernel(MimoParams a, float* Gl, float* Ab, int nch) {
  extern __shared__ float4 csm4[];
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * kTcB, n = min(kTcB, a.L - t0);
  const int P = a.P, R = a.R, tid = threadIdx.x;
  float* p = reinterpret_cast<float*>(csm4);
  float* mo = p; p += R * P;
  BSmem s;
  s.dy = p; p += kTcB * P;
  s.dyr = p; p += kTcB * R;
  s.an = p;
  for (int i = tid; i < R * P; i += kCT) {
    const int r = i / P, q = i - r * P;
    mo[i] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + q];
  }
  __syncthreads();
  stage_dy<TX>(a, s, mo, b, h, t0, n);
  for (int d = tid; d < a.D; d += kCT) {
    float gv = 0.f;
#pragma unroll 4
    for (int t = n - 1; t >= 0; --t) gv = fmaf(s.an[t], gv, e_at<TB>(a, s.dyr + t * R, b, t0 + t, h, d));
    Gl[((int64_t)u * nch + c) * a.D + d] = gv;
  }
  if (tid == 0) {
    float prod = 1.f;
    for (int t = 0; t < n; ++t) prod *= s.an[t];
    Ab[(int64_t)u * nch + c] = prod;
  }
}

__global__ void __launch_bounds__(kCT) mimo_bwd_carry_kernel(MimoParams a, float* Gl, const float* Ab, int nch) {
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  for (int d = threadIdx.x; d < a.D; d += kCT) {
    float run = 0.f;
    for (int c = nch - 1; c >= 0; --c) {
      const int64_t i = ((int64_t)u * nch + c) * a.D + d;
      const float loc = Gl[i];
      Gl[i] = run;
      run = fmaf(Ab[(int64_t)u * nch + c], run, loc);
    }
    if (a.dh0 || a.dbx0) {
      const float a0 = expf(scalc(a.adt, a.sadt, b, 0, h));
      const float dt0 = scalc(a.dt, a.sdt, b, 0, h);
      const float tr0 = sigmoidf_(scalc(a.trap, a.strap, b, 0, h));
      if (a.dh0) a.dh0[(int64_t)u * a.D + d] = a0 * run;
      if (a.dbx0) a.dbx0[(int64_t)u * a.D + d] = 0.5f * dt0 * tr0 * run;
    }
  }
}

// B3 shared memory (floats), chunk of kTcB steps; row r of x / xr / scalars is t0 - 1 + r
// for x, xr, and t0 + r for a, be, ga (row n = t0 + n); BX row r is Bx_{t0-1+r}; G row n is
// the adjoint entering from the next chunk.
__host__ __device__ inline size_t bsmem_floats(int P, int R, int D) {
  constexpr int T = kTcB;
  return 2 * (size_t)R * P + (size_t)(T + 1) * P + (size_t)(T + 1) * R + (size_t)T * P + 3 * (size_t)T * R +
         3 * (size_t)(T + 1) + 2 * (size_t)T + (size_t)T * D + 2 * (size_t)(T + 1) * D + (size_t)T * D + 4 * (size_t)T;
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kCT) mimo_bwd_full_kernel(MimoParams a, const float* Hc, const float* Gc,
                                                            double* tot, int nch) {
  extern __shared__ float4 csm4[];
  constexpr int T = kTcB;
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * T, n = min(T, a.L - t0);
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* p = reinterpret_cast<float*>(csm4);
  float* mx = p; p += R * P;
  float* mo = p; p += R * P;
  float* xs = p; p += (T + 1) * P;
  float* xr = p; p += (T + 1) * R;
  float* dyv = p; p += T * P;
  float* dyr = p; p += T * R;
  float* dxr = p; p += T * R;
  float* yr = p; p += T * R;
  float* av = p; p += T + 1;
  float* be = p; p += T + 1;
  float* ga = p; p += T + 1;
  float* trv = p; p += T;
  float* dtv = p; p += T;
  float* Hs = p; p += T * D;
  float* BX = p; p += (T + 1) * D;
  float* Gs = p; p += (T + 1) * D;
  float* Es = p; p += T * D;
  float* red = p;  // dbeta, dgamma, q, z per step
  // ---- staging
  for (int i = tid; i < R * P; i += kCT) {
    const int r = i / P, q = i - r * P;
    mx[i] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + q];
    mo[i] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + q];
  }
  for (int i = tid; i < (n + 1) * P; i += kCT) {
    const int r = i / P, q = i - r * P, t = t0 - 1 + r;
    xs[i] = t >= 0 ? ldxc<TX>(a.x, a.sx, b, t, h, q) : 0.f;
  }
  for (int i = tid; i < n * P; i += kCT) {
    const int r = i / P, q = i - r * P;
    dyv[i] = ldxc<TX>(a.dy, a.sdy, b, t0 + r, h, q);
  }
  for (int r = tid; r <= n; r += kCT) {
    const int t = t0 + r;
    float A = 0.f, bb = 0.f, gg = 0.f, tr = 0.f, dt = 0.f;
    if (t < a.L) {
      dt = scalc(a.dt, a.sdt, b, t, h);
      tr = sigmoidf_(scalc(a.trap, a.strap, b, t, h));
      A = expf(scalc(a.adt, a.sadt, b, t, h));
      bb = dt * (1.0f - tr) + 0.5f * dt * tr;
      gg = 0.5f * dt * tr;
    }
    av[r] = A; be[r] = bb; ga[r] = gg;
    if (r < n) { trv[r] = tr; dtv[r] = dt; }
  }
  __syncthreads();
  for (int i = tid; i < (n + 1) * R; i += kCT) {
    const int r = i / R, k = i - r * R;
    float acc = 0.f;
    for (int q = 0; q < P; ++q) acc = fmaf(xs[r * P + q], mx[k * P + q], acc);
    xr[i] = acc;
  }
  for (int i = tid; i < n * R; i += kCT) {
    const int r = i / R, k = i - r * R;
    float acc = 0.f;
    for (int q = 0; q < P; ++q) acc = fmaf(dyv[r * P + q], mo[k * P + q], acc);
    dyr[i] = acc;
  }
  __syncthreads();
  // ---- forward states from the carry, adjoints from the backward carry (thread = d)
  for (int d = tid; d < D; d += kCT) {
    float bxp = t0 > 0 ? bx_at<TB>(a, xr, b, t0 - 1, h, d)
                       : (a.bx0 ? a.bx0[(int64_t)u * D + d] : 0.f);
    float hv = Hc[((int64_t)u * nch + c) * D + d];
    BX[d] = bxp;
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      const float bx = bx_at<TB>(a, xr + (t + 1) * R, b, t0 + t, h, d);
      hv = fmaf(av[t], hv, fmaf(be[t], bx, ga[t] * bxp));
      Hs[t * D + d] = hv;
      BX[(t + 1) * D + d] = bx;
      bxp = bx;
    }
    float gv = Gc[((int64_t)u * nch + c) * D + d];
    Gs[n * D + d] = gv;
#pragma unroll 4
    for (int t = n - 1; t >= 0; --t) {
      const float e = e_at<TB>(a, dyr + t * R, b, t0 + t, h, d);
      Es[t * D + d] = e;
      gv = fmaf(av[t + 1], gv, e);
      Gs[t * D + d] = gv;
    }
  }
  __syncthreads();
  // ---- per (t, r): readout yr and dC; dB and dxr (one warp per pair, lanes over d)
  const float Dk = a.Dskip[h * a.sD];
  for (int pr = warp; pr < n * R; pr += kCT / 32) {
    const int t = pr / R, r = pr - t * R, tt = t0 + t;
    const float dyv_r = dyr[pr], xr_r = xr[(t + 1) * R + r];
    float acc = 0.f, accb = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float hd = Hs[t * D + d];
      acc = fmaf(ldbcc<TB>(a.Cm, a.sC, b, tt, r, h, d), hd, acc);
      const float v = fmaf(be[t], Gs[t * D + d], ga[t + 1] * Gs[(t + 1) * D + d]);
      accb = fmaf(ldbcc<TB>(a.Bm, a.sB, b, tt, r, h, d), v, accb);
      st(reinterpret_cast<TB*>(a.dC) + (int64_t)b * a.sdC.b + (int64_t)tt * a.sdC.l + (int64_t)r * a.sdC.r +
             (int64_t)h * a.sdC.h + d, dyv_r * hd);
      st(reinterpret_cast<TB*>(a.dB) + (int64_t)b * a.sdB.b + (int64_t)tt * a.sdB.l + (int64_t)r * a.sdB.r +
             (int64_t)h * a.sdB.h + d, xr_r * v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc += __shfl_xor_sync(0xffffffffu, acc, o);
      accb += __shfl_xor_sync(0xffffffffu, accb, o);
    }
    if (lane == 0) {
      yr[pr] = fmaf(Dk, xr_r, acc);
      dxr[pr] = fmaf(Dk, dyv_r, accb);
    }
  }
  // ---- per t: dbeta, dgamma, q (one warp per step)
  for (int t = warp; t < n; t += kCT / 32) {
    float db = 0.f, dg = 0.f, q = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float g = Gs[t * D + d];
      db = fmaf(g, BX[(t + 1) * D + d], db);
      dg = fmaf(g, BX[t * D + d], dg);
      q = fmaf(Es[t * D + d], Hs[t * D + d], q);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      db += __shfl_xor_sync(0xffffffffu, db, o);
      dg += __shfl_xor_sync(0xffffffffu, dg, o);
      q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    if (lane == 0) {
      const int tt = t0 + t;
      const float tr = trv[t], dt = dtv[t];
      red[t] = q - be[t] * db - ga[t] * dg;
      a.ddt[(int64_t)b * a.sddt.b + (int64_t)tt * a.sddt.l + (int64_t)h * a.sddt.h] =
          db * (1.0f - 0.5f * tr) + dg * 0.5f * tr;
      a.dtrap[(int64_t)b * a.sdtrap.b + (int64_t)tt * a.sdtrap.l + (int64_t)h * a.sdtrap.h] =
          0.5f * dt * (dg - db) * tr * (1.0f - tr);
    }
  }
  __syncthreads();
  // ---- within-chunk suffix sums of the dADT terms (fp64); the chunk total for B4
  if (tid == 0) {
    double cum = 0.0;
    for (int t = n - 1; t >= 0; --t) {
      cum += (double)red[t];
      a.dadt[(int64_t)b * a.sdadt.b + (int64_t)(t0 + t) * a.sdadt.l + (int64_t)h * a.sdadt.h] = (float)cum;
    }
    tot[(int64_t)u * nch + c] = cum;
  }
  // ---- dx = mimo_x^T dxr
  for (int i = tid; i < n * P; i += kCT) {
    const int t = i / P, q = i - t * P;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(dxr[t * R + r], mx[r * P + q], acc);
    st(reinterpret_cast<TX*>(a.dx) + (int64_t)b * a.sdx.b + (int64_t)(t0 + t) * a.sdx.l + (int64_t)h * a.sdx.h + q, acc);
  }
  // ---- dmimo_x += dxr x^T, dmimo_o += yr dy^T, dD += <dyr, xr>
  for (int i = tid; i < R * P; i += kCT) {
    const int r = i / P, q = i - r * P;
    float ax = 0.f, ao = 0.f;
    for (int t = 0; t < n; ++t) {
      ax = fmaf(dxr[t * R + r], xs[(t + 1) * P + q], ax);
      ao = fmaf(yr[t * R + r], dyv[t * P + q], ao);
    }
    atomicAdd(a.dmx + (int64_t)h * R * P + i, ax);
    atomicAdd(a.dmo + (int64_t)h * R * P + i, ao);
  }
  if (warp == 0) {
    float v = 0.f;
    for (int i = lane; i < n * R; i += 32) v = fmaf(dyr[i], xr[(i / R + 1) * R + i % R], v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) atomicAdd(a.dD + h, v);
  }
}

// B4: add to every step's dADT the terms of all later chunks
__global__ void __launch_bounds__(kCT) mimo_bwd_dadt_kernel(MimoParams a, const double* tot, int nch, int T) {
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  double off = 0.0;
  for (int c = nch - 1; c >= 0; --c) {
    const int t0 = c * T, n = min(T, a.L - t0);
    if (c < nch - 1)
      for (int t = threadIdx.x; t < n; t += kCT) {
        float* q = a.dadt + (int64_t)b * a.sdadt.b + (int64_t)(t0 + t) * a.sdadt.l + (int64_t)h * a.sdadt.h;
        *q = (float)((double)*q + off);
      }
    off += tot[(int64_t)u * nch + c];
  }
}

// ------------------------------------------------------------------------------------
// Single-pass forward. One CTA per (b, h, chunk) takes its chunk from a ticket counter
// (chunk-major, so every chunk it waits for belongs to a CTA that started earlier) and
// pulls the chunk's B and C tiles into shared memory with one TMA box each. Each state
// column d is then one thread's: it scans the chunk from a zero state, publishes that
// local end state S_c[d] (and, once per chunk, the decay product A_c), finds its carry
// (the state entering the chunk) by looking back over the chunks before it, publishes its
// inclusive state I_c[d] = S_c[d] + A_c carry[d], and adds (a_t0 ... a_t) carry[d] to the
// chunk's states. A chunk whose I_j[d] is published ends the walk; one with only S_j[d]
// is folded in and the walk goes on,
//   carry_c = S_{c-1} + A_{c-1} (S_{c-2} + A_{c-2} ( ... + I_j)).
// Every published value shares a 64-bit word with its status (1: S, 2: I), written and
// read with single-copy-atomic 64-bit accesses, so no fence is needed between a value and
// its flag. B, C and x are read once. Every wait (TMA boxes, predecessors' words) is
// bounded; a wait that gives up sets the error word and the kernel finishes with its
// outputs invalid.
// ------------------------------------------------------------------------------------
constexpr int kFT = 256;                   // threads per CTA
constexpr uint32_t kSpinLimit = 1u << 22;  // polls of a predecessor's word before giving up

__device__ int g_mimo_error;  // set when a bounded wait gives up

// x / d for 0 <= x < 2^31 by a multiply-high and a shift (Granlund and Montgomery,
// "Division by invariant integers using multiplication", 1994: the round-up multiplier
// m = floor(2^32 (2^s - d) / d) + 1 with s = ceil(log2 d), q = (mulhi(x, m) + x) >> s).
struct FastDiv {
  uint32_t m, s;
};
inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  f.s = s;
  f.m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  return f;
}
__device__ __forceinline__ int fdiv(int x, FastDiv f) {
  return (int)((__umulhi((uint32_t)x, f.m) + (uint32_t)x) >> f.s);
}

// Workspace of the single-pass forward: the ticket counter, then the value words and the
// decay words, all cleared before every launch.
inline int64_t fused_ws_bytes(int64_t cells, int64_t D) { return 16 + 8 * cells * (D + 1); }

// Shared-memory layout (byte offsets from a 128-byte aligned base): two mbarriers and the
// ticket, the B box (rows t0-1 .. t0+Q-1, [row][r][d], row 0 = t0-1), the C box (rows
// t0 .. t0+Q-1), the x box (rows t0-1 .. t0+Q-1, [row][p]), the chunk's bx and then states
// (fp32 [t][d]), the rank projections of x, the step coefficients (a, beta, gamma, -) and
// the running decay products, mimo_x and mimo_o (rows padded to P + 4 floats), the
// readouts and the carries. The group-row form (grp) has no C box: its B box holds the raw
// group rows of B and C ([row][2R][d], rows t0-1 .. t0+Q-1), and it adds the z box (rows
// t0 .. t0+Q, when the gate is fused), the RMS factors of those rows ([row][2R]) and the
// (cos, sin) table of the rotated pairs ([row][S]).
struct FusedSmem {
  uint32_t bs, cs, xs, zs, hs, xr, coef, cum, mx, mo, yr, carry, rs, tab, total;
};
__host__ __device__ inline uint32_t aup(uint32_t v, uint32_t k) { return (v + k - 1) / k * k; }
__host__ __device__ inline FusedSmem fused_smem(int Q, int P, int R, int D, int eb, int ex, bool grp = false,
                                                int S = 0, bool gate = false) {
  FusedSmem L;
  uint32_t o = 128;
  L.bs = o; o = aup(o + (uint32_t)((Q + 1) * (grp ? 2 * R : R) * D * eb), 128);
  L.cs = o; o = aup(o + (uint32_t)(grp ? 0 : Q * R * D * eb), 128);
  L.xs = o; o = aup(o + (uint32_t)((Q + 1) * P * ex), 128);
  L.zs = o; o = aup(o + (uint32_t)(grp && gate ? (Q + 1) * P * ex : 0), 128);
  L.hs = o; o = aup(o + (uint32_t)(Q * D * 4), 16);
  L.xr = o; o = aup(o + (uint32_t)((Q + 1) * R * 4), 16);
  L.coef = o; o = aup(o + (uint32_t)(Q * 16), 16);
  L.cum = o; o = aup(o + (uint32_t)(Q * 4), 16);
  L.mx = o; o = aup(o + (uint32_t)(R * (P + 4) * 4), 16);
  L.mo = o; o = aup(o + (uint32_t)(R * (P + 4) * 4), 16);
  L.yr = o; o = aup(o + (uint32_t)(Q * R * 4), 16);
  L.carry = o; o = aup(o + (uint32_t)(D * 4), 16);
  L.rs = o; o = aup(o + (uint32_t)(grp ? (Q + 1) * 2 * R * 4 : 0), 16);
  L.tab = o; o = aup(o + (uint32_t)(grp ? (Q + 1) * S * 8 : 0), 16);
  L.total = o + 128;  // slack for aligning the dynamic shared-memory base
  return L;
}

// Operands of the group-row form: B_t[r] and C_t[r] of head h are
//   rot_{t,h}(RMSNorm(raw_t[r]) * w + bias[h, r]),
// raw the group rows of the in_proj output, rot the rotation of pairs (2k, 2k+1), k < S,
// by angles[b, t, h, k]. The rotation is the same for every rank of a (t, h), so
//   Bx_t = rot(w o sum_r xr_t[r] rs_t[r] raw_t[r] + sum_r xr_t[r] bias[h, r]) and
//   C_t[r] . h_t = rs_t[r] (raw_t[r] o w) . rot^T(h_t) + bias[h, r] . rot^T(h_t),
// one rotation per (t, pair) for B and one for the states.
struct GrpArgs {
  const float* angles;                            // (Bn, L, H, S) contiguous
  const float* B_bias; const float* C_bias;       // (H, R, D) contiguous, 16-byte aligned
  const float* B_norm_w; const float* C_norm_w;   // (D), 16-byte aligned
  float eps;                                      // RMSNorm epsilon
  int S;                                          // rotated pairs
  int gate;                                       // y * silu(z), z from the z box
  FastDiv fS;                                     // divisor S (S > 0)
};

struct FusedArgs {
  FastDiv fP4, fD4, fR, fU, fH;  // divisors headdim / 4, d_state / 4, rank, units, heads
  int nch, units;
  int ahead;  // CTAs resident on the device: a CTA prefetches the chunk of ticket + ahead into L2
  int yvec;   // y rows start on 16-byte boundaries: four outputs per store
  FusedSmem L;  // shared-memory layout (computed on the host)
  unsigned* ticket;
  unsigned long long* rec;   // [unit][chunk][d]: S or I value | status << 32
  unsigned long long* arec;  // [unit][chunk]: A value | 1 << 32
};

__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, float v, uint32_t status) {
  const unsigned long long w = ((unsigned long long)status << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// four consecutive elements (16-byte aligned for fp32, 8-byte for 16-bit types) as floats
__device__ __forceinline__ float4 ld4f(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4f(const __nv_bfloat16* p) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float4 ld4f(const __half* p) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&lo);
  w.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = w;
}
__device__ __forceinline__ void st4(__half* p, float4 v) {
  const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&lo);
  w.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = w;
}
__device__ __forceinline__ void fma4(float4& acc, float s, float4 v) {
  acc.x = fmaf(s, v.x, acc.x);
  acc.y = fmaf(s, v.y, acc.y);
  acc.z = fmaf(s, v.z, acc.z);
  acc.w = fmaf(s, v.w, acc.w);
}
__device__ __forceinline__ void fma4(float4& acc, float4 u, float4 v) {
  acc.x = fmaf(u.x, v.x, acc.x);
  acc.y = fmaf(u.y, v.y, acc.y);
  acc.z = fmaf(u.z, v.z, acc.z);
  acc.w = fmaf(u.w, v.w, acc.w);
}

// Bounded wait for a TMA box; on giving up, set the error word and wait once more (also
// bounded) so that no copy is still writing shared memory when the CTA ends.
__device__ __forceinline__ void wait_copies(uint64_t* bar) {
  if (sm100::mbar_wait(bar, 0, 1u << 24)) return;
  atomicExch(&g_mimo_error, 1);
  sm100::mbar_wait(bar, 0, 1u << 24);
}

// The carry of column d of chunk c of unit u from the words of the chunks before it.
__device__ __forceinline__ float look_back(const FusedArgs& f, int u, int c, int d, int D, bool& ok) {
  const int64_t base = (int64_t)u * f.nch;
  float acc = 0.f, accA = 1.f;
  int j = c - 1;
  for (uint32_t spins = 0; spins < kSpinLimit; ++spins) {
    const unsigned long long w = ld_relaxed64(f.rec + (base + j) * D + d);
    const unsigned long long av = ld_relaxed64(f.arec + base + j);
    const uint32_t st = (uint32_t)(w >> 32);
    if (st == 2) return fmaf(accA, __uint_as_float((uint32_t)w), acc);
    if (st == 1 && (av >> 32) != 0) {
      acc = fmaf(accA, __uint_as_float((uint32_t)w), acc);
      accA *= __uint_as_float((uint32_t)av);
      if (--j < 0) break;  // chunk 0 publishes its inclusive state only: unreachable
      continue;
    }
    __nanosleep(32);
  }
  ok = false;
  return 0.f;
}

// rotation of the pair (u, v) by (cos, sin) = cs, and by its transpose
__device__ __forceinline__ void rot2(float& u, float& v, float2 cs) {
  const float t = u * cs.x - v * cs.y;
  v = u * cs.y + v * cs.x;
  u = t;
}
__device__ __forceinline__ void rot2t(float& u, float& v, float2 cs) {
  const float t = u * cs.x + v * cs.y;
  v = v * cs.x - u * cs.y;
  u = t;
}
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// GRP: the group-row form (GrpArgs): mapB covers the group rows of B and C of the in_proj
// output, mapX its z and x columns as 2H heads (z heads first), mapC is unused.
template <typename TX, typename TB, int Q, bool GRP>
__global__ void __launch_bounds__(kFT)
    mimo_fused_fwd_kernel(const __grid_constant__ CUtensorMap mapB, const __grid_constant__ CUtensorMap mapC,
                          const __grid_constant__ CUtensorMap mapX, MimoParams a, FusedArgs f, GrpArgs g) {
  static_assert(Q <= kFT, "a thread per step of the chunk");
  extern __shared__ __align__(128) unsigned char fsm_raw[];
  unsigned char* fsm = fsm_raw + ((128u - (sm100::smem_u32(fsm_raw) & 127u)) & 127u);
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x, lane = tid & 31;
  const int P4 = P >> 2, D4 = D >> 2, MS = P + 4, R2 = 2 * R;
  const int S = GRP ? g.S : 0;
  const FusedSmem& L = f.L;
  uint64_t* barB = reinterpret_cast<uint64_t*>(fsm);
  uint64_t* barC = barB + 1;
  int* tk_s = reinterpret_cast<int*>(fsm + 16);
  const TB* Bs = reinterpret_cast<const TB*>(fsm + L.bs);
  const TB* Cs = reinterpret_cast<const TB*>(fsm + L.cs);
  const TX* xs = reinterpret_cast<const TX*>(fsm + L.xs);
  const TX* zs = reinterpret_cast<const TX*>(fsm + L.zs);
  float* hs = reinterpret_cast<float*>(fsm + L.hs);
  float* xr = reinterpret_cast<float*>(fsm + L.xr);
  float4* coef = reinterpret_cast<float4*>(fsm + L.coef);
  float* cum = reinterpret_cast<float*>(fsm + L.cum);
  float* mx = reinterpret_cast<float*>(fsm + L.mx);
  float* mo = reinterpret_cast<float*>(fsm + L.mo);
  float* yr = reinterpret_cast<float*>(fsm + L.yr);
  float* carry_s = reinterpret_cast<float*>(fsm + L.carry);
  float* rs = reinterpret_cast<float*>(fsm + L.rs);
  float2* tab = reinterpret_cast<float2*>(fsm + L.tab);

  if (tid == 0) {
    *tk_s = (int)atomicAdd(f.ticket, 1u);
    sm100::mbar_init(barB, 1);
    sm100::mbar_init(barC, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const int tk = *tk_s;
  const int c = fdiv(tk, f.fU), u = tk - c * f.units, b = fdiv(u, f.fH), h = u - b * a.H;
  const int t0 = c * Q, n = min(Q, a.L - t0);
  // the step scalars first: their loads are in flight while the boxes are requested
  float s_adt = 0.f, s_dt = 0.f, s_tr = 0.f;
  if (tid < n) {
    s_adt = scalc(a.adt, a.sadt, b, t0 + tid, h);
    s_dt = scalc(a.dt, a.sdt, b, t0 + tid, h);
    s_tr = scalc(a.trap, a.strap, b, t0 + tid, h);
  }
  if (tid == 0) {
    // whole boxes: rows outside the sequence (t0-1 of the first chunk, the tail of the
    // last) arrive as zeros and still count toward the transaction bytes
    if constexpr (GRP) {
      sm100::mbar_expect_tx(barB, (uint32_t)((Q + 1) * (R2 * D * sizeof(TB) + P * sizeof(TX))));
      sm100::tma_load_4d(fsm + L.bs, &mapB, barB, 0, 0, t0 - 1, b);
      sm100::tma_load_4d(fsm + L.xs, &mapX, barB, 0, a.H + h, t0 - 1, b);
      if (g.gate) {
        // the x map's box: Q + 1 rows from t0, the last one unused
        sm100::mbar_expect_tx(barC, (uint32_t)((Q + 1) * P * sizeof(TX)));
        sm100::tma_load_4d(fsm + L.zs, &mapX, barC, 0, h, t0, b);
      }
    } else {
      sm100::mbar_expect_tx(barB, (uint32_t)((Q + 1) * (R * D * sizeof(TB) + P * sizeof(TX))));
      sm100::tma_load_5d(fsm + L.bs, &mapB, barB, 0, h, 0, t0 - 1, b);
      sm100::tma_load_4d(fsm + L.xs, &mapX, barB, 0, h, t0 - 1, b);
      sm100::mbar_expect_tx(barC, (uint32_t)(Q * R * D * sizeof(TB)));
      sm100::tma_load_5d(fsm + L.cs, &mapC, barC, 0, h, 0, t0, b);
    }
  }
  // the inputs of the chunk that the CTA `ahead` tickets later will take, into L2
  const int tf = tk + f.ahead;
  if (tf < f.units * f.nch && tid < 32) {
    const int cf = fdiv(tf, f.fU), uf = tf - cf * f.units, bf = fdiv(uf, f.fH), hf = uf - bf * a.H;
    const int tf0 = cf * Q;
    if (tid == 0) {  // rows from max(t0 - 1, 0): no prefetch starts outside the tensor
      if constexpr (GRP) {
        sm100::tma_prefetch_l2_4d(&mapB, 0, 0, max(tf0 - 1, 0), bf);
        sm100::tma_prefetch_l2_4d(&mapX, 0, a.H + hf, max(tf0 - 1, 0), bf);
        if (g.gate) sm100::tma_prefetch_l2_4d(&mapX, 0, hf, tf0, bf);
      } else {
        sm100::tma_prefetch_l2_5d(&mapB, 0, hf, 0, max(tf0 - 1, 0), bf);
        sm100::tma_prefetch_l2_5d(&mapC, 0, hf, 0, tf0, bf);
        sm100::tma_prefetch_l2_4d(&mapX, 0, hf, max(tf0 - 1, 0), bf);
      }
    }
    for (int t = tf0 + tid; t < min(tf0 + Q, a.L); t += 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.adt + (int64_t)bf * a.sadt.b + (int64_t)t * a.sadt.l + (int64_t)hf * a.sadt.h));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.dt + (int64_t)bf * a.sdt.b + (int64_t)t * a.sdt.l + (int64_t)hf * a.sdt.h));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.trap + (int64_t)bf * a.strap.b + (int64_t)t * a.strap.l + (int64_t)hf * a.strap.h));
      if (GRP && S > 0) {  // the angle row of step t and of step t - 1 (the first's row t0 - 1)
        const float* ar = g.angles + (((int64_t)bf * a.L + t) * a.H + hf) * S;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(ar));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(ar + S - 1));
        if (t == tf0 && t > 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(ar - (int64_t)a.H * S));
      }
    }
  }
  for (int i = tid; i < R * P; i += kFT) {
    const int r = fdiv(i >> 2, f.fP4), p = i - r * P;
    mx[r * MS + p] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + p];
    mo[r * MS + p] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + p];
  }
  if (tid < n) {
    const float tr = sigmoidf_(s_tr);
    coef[tid] = make_float4(expf(s_adt), s_dt * (1.0f - tr) + 0.5f * s_dt * tr, 0.5f * s_dt * tr, 0.f);
  }
  if constexpr (GRP) {
    // (cos, sin) of the rotated pairs of rows t0-1 .. t0+n-1 (identity before the sequence)
    const float* ab = g.angles + ((int64_t)b * a.L * a.H + h) * S;
    for (int i = tid; i < (n + 1) * S; i += kFT) {
      const int row = fdiv(i, g.fS), k = i - row * S, t = t0 - 1 + row;
      float sn = 0.f, cs = 1.f;
      if (t >= 0) sincos_reduced(ab[(int64_t)t * a.H * S + k], &sn, &cs);
      tab[i] = make_float2(cs, sn);
    }
  }
  __syncthreads();
  wait_copies(barB);
  // xr_t[k] = mimo_x[k, :] . x_t, four p per step, each row starting at its own p block;
  // GRP: also the RMS factors of the group rows, 1 / sqrt(mean(raw^2) + eps)
  const int nxr = (n + 1) * R;
  for (int i = tid; i < (GRP ? 3 * nxr : nxr); i += kFT) {
    if (!GRP || i < nxr) {
      const int row = fdiv(i, f.fR), k = i - row * R;
      const TX* xrow = xs + row * P;
      const float* mrow = mx + k * MS;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int pb = row - fdiv(row, f.fP4) * P4;
      for (int e = 0; e < P4; ++e) {
        fma4(acc, ld4f(xrow + 4 * pb), ld4f(mrow + 4 * pb));
        pb = pb + 1 == P4 ? 0 : pb + 1;
      }
      xr[i] = (acc.x + acc.y) + (acc.z + acc.w);
    } else {
      const int j = i - nxr;  // row * 2R + k
      const TB* grow = Bs + (size_t)j * D;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int kb = j - fdiv(j, f.fD4) * D4;
      for (int e = 0; e < D4; ++e) {
        const float4 v = ld4f(grow + 4 * kb);
        fma4(acc, v, v);
        kb = kb + 1 == D4 ? 0 : kb + 1;
      }
      rs[j] = 1.0f / sqrtf(((acc.x + acc.y) + (acc.z + acc.w)) / (float)D + g.eps);
    }
  }
  __syncthreads();
  if constexpr (GRP) {
    // bx of rows t0-1 (only after the first chunk; into the carry array) .. t0+n-1 (into
    // the state array): w o sum_r xr rs raw_r + sum_r xr bias_r, then the rotation
    for (int i = tid + (c > 0 ? 0 : D4); i < (n + 1) * D4; i += kFT) {
      const int row = fdiv(i, f.fD4), d = 4 * (i - row * D4);
      const float* xrow = xr + row * R;
      const float* rrow = rs + row * R2;
      const TB* brow = Bs + (size_t)row * R2 * D + d;
      const float* bb = g.B_bias + (size_t)h * R * D + d;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f), accb = acc;
      for (int r = 0; r < R; ++r) {
        fma4(acc, xrow[r] * rrow[r], ld4f(brow + (size_t)r * D));
        fma4(accb, xrow[r], ldg4(bb + (size_t)r * D));
      }
      fma4(accb, acc, ldg4(g.B_norm_w + d));
      const int j0 = d >> 1;
      if (j0 < S) rot2(accb.x, accb.y, tab[row * S + j0]);
      if (j0 + 1 < S) rot2(accb.z, accb.w, tab[row * S + j0 + 1]);
      *reinterpret_cast<float4*>(row == 0 ? carry_s + d : hs + (row - 1) * D + d) = accb;
    }
  } else {
    // bx_t[d] = sum_r xr_t[r] B_t[r, d] for t0 .. t0+n-1 (four columns a thread), into the
    // state array
    for (int i = tid; i < n * D4; i += kFT) {
      const int t = fdiv(i, f.fD4), d = 4 * (i - t * D4);
      const float* xrow = xr + (t + 1) * R;
      const TB* brow = Bs + (size_t)(t + 1) * R * D + d;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < R; ++r) fma4(acc, xrow[r], ld4f(brow + (size_t)r * D));
      *reinterpret_cast<float4*>(hs + t * D + d) = acc;
    }
  }
  __syncthreads();
  const int64_t cell = (int64_t)u * f.nch + c;
  bool ok = true;
  for (int d = tid; d < D; d += kFT) {
    float bxp = 0.f;
    if (c > 0) {
      if constexpr (GRP) {
        bxp = carry_s[d];  // this thread's own column: read here, overwritten below
      } else {
        for (int r = 0; r < R; ++r) bxp = fmaf(xr[r], to_f32(Bs[(size_t)r * D + d]), bxp);
      }
    } else if (a.bx0) {
      bxp = a.bx0[(int64_t)u * D + d];
    }
    // the chunk from a zero state, eight steps per batch of shared-memory reads; column 0
    // also records the running decay products
    float hv = 0.f, pr = 1.f;
    for (int tb = 0; tb < n; tb += 8) {
      float bxv[8];
      float4 cf[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool in = tb + j < n;
        bxv[j] = in ? hs[(tb + j) * D + d] : 0.f;
        cf[j] = in ? coef[tb + j] : make_float4(1.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        hv = fmaf(cf[j].x, hv, fmaf(cf[j].y, bxv[j], cf[j].z * bxp));
        pr *= cf[j].x;
        if (tb + j < n) {
          bxp = bxv[j];
          hs[(tb + j) * D + d] = hv;
          if (d == 0) cum[tb + j] = pr;
        }
      }
    }
    if (c == f.nch - 1 && a.bx_last) a.bx_last[(int64_t)u * D + d] = bxp;
    float carry;
    if (c == 0) {
      carry = a.h0 ? a.h0[(int64_t)u * D + d] : 0.f;
    } else {
      st_relaxed64(f.rec + cell * D + d, hv, 1);
      if (d == 0) st_relaxed64(f.arec + cell, pr, 1);
      carry = look_back(f, u, c, d, D, ok);
    }
    const float incl = fmaf(pr, carry, hv);
    st_relaxed64(f.rec + cell * D + d, incl, 2);
    if (c == f.nch - 1 && a.h_last) a.h_last[(int64_t)u * D + d] = incl;
    carry_s[d] = carry;
  }
  if (!ok) atomicExch(&g_mimo_error, 1);
  __syncthreads();
  // the chunk's states from the carries: h_t = hloc_t + (a_t0 ... a_t) carry (GRP: stored
  // rotated back, rot^T h_t, for the readouts against the unrotated C rows)
  for (int i = tid; i < n * D4; i += kFT) {
    const int t = fdiv(i, f.fD4), d = 4 * (i - t * D4);
    float4 hv = *reinterpret_cast<const float4*>(hs + t * D + d);
    fma4(hv, cum[t], *reinterpret_cast<const float4*>(carry_s + d));
    if constexpr (GRP) {
      const int j0 = d >> 1;
      if (j0 < S) rot2t(hv.x, hv.y, tab[(t + 1) * S + j0]);
      if (j0 + 1 < S) rot2t(hv.z, hv.w, tab[(t + 1) * S + j0 + 1]);
    }
    *reinterpret_cast<float4*>(hs + t * D + d) = hv;
  }
  if (!GRP || g.gate) wait_copies(barC);
  __syncthreads();
  // yr_t[r] = C_t[r, :] . h_t + D xr_t[r]: a thread per (t, r), four columns per step, each
  // lane starting at its own column block so that a warp's reads fall in distinct banks
  const float Dk = a.Dskip[h * a.sD];
  for (int it = tid; it < n * R; it += kFT) {
    const int t = fdiv(it, f.fR), r = it - t * R;
    const float* hrow = hs + (size_t)t * D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int k = lane - fdiv(lane, f.fD4) * D4;
    if constexpr (GRP) {
      // rs (raw o w) . h' + bias . h', h' = rot^T h
      const TB* crow = Bs + ((size_t)(t + 1) * R2 + R + r) * D;
      const float* cb = g.C_bias + ((size_t)h * R + r) * D;
      float4 accb = acc;
#pragma unroll 4
      for (int e = 0; e < D4; ++e) {
        const float4 hv = ld4f(hrow + 4 * k), wv = ldg4(g.C_norm_w + 4 * k);
        fma4(acc, ld4f(crow + 4 * k), make_float4(wv.x * hv.x, wv.y * hv.y, wv.z * hv.z, wv.w * hv.w));
        fma4(accb, ldg4(cb + 4 * k), hv);
        k = k + 1 == D4 ? 0 : k + 1;
      }
      const float dot = fmaf(rs[(t + 1) * R2 + R + r], (acc.x + acc.y) + (acc.z + acc.w),
                             (accb.x + accb.y) + (accb.z + accb.w));
      yr[it] = fmaf(Dk, xr[(t + 1) * R + r], dot);
    } else {
      const TB* crow = Cs + (size_t)it * D;
#pragma unroll 4
      for (int e = 0; e < D4; ++e) {
        fma4(acc, ld4f(crow + 4 * k), ld4f(hrow + 4 * k));
        k = k + 1 == D4 ? 0 : k + 1;
      }
      yr[it] = fmaf(Dk, xr[(t + 1) * R + r], (acc.x + acc.y) + (acc.z + acc.w));
    }
  }
  __syncthreads();
  // y_t = mimo_o^T yr_t, four outputs a thread (GRP with the gate: times silu(z_t))
  TX* yb = reinterpret_cast<TX*>(a.y) + (int64_t)b * a.sy.b + (int64_t)h * a.sy.h;
  for (int i = tid; i < n * P4; i += kFT) {
    const int t = fdiv(i, f.fP4), p = 4 * (i - t * P4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < R; ++r) fma4(acc, yr[t * R + r], ld4f(mo + r * MS + p));
    if (GRP && g.gate) {
      const float4 zv = ld4f(zs + t * P + p);
      acc.x *= zv.x * fast_sigmoid(zv.x);
      acc.y *= zv.y * fast_sigmoid(zv.y);
      acc.z *= zv.z * fast_sigmoid(zv.z);
      acc.w *= zv.w * fast_sigmoid(zv.w);
    }
    TX* yp = yb + (int64_t)(t0 + t) * a.sy.l + p;
    if (f.yvec) {
      st4(yp, acc);
    } else {
      st(yp, acc.x);
      st(yp + 1, acc.y);
      st(yp + 2, acc.z);
      st(yp + 3, acc.w);
    }
  }
}

// ------------------------------------------------------------------------------------
// Single-pass backward (the gradients of the single-pass forward, same chunks). The
// adjoint of the state runs backwards in time,
//   g_t = a_{t+1} g_{t+1} + E_t,   E_t[d] = sum_r dyr_t[r] C_t[r, d],   dyr_t = mimo_o dy_t,
// so CTAs take chunks from the end (ticket order last chunk first) and look forward for
// the adjoint entering their chunk from the right: a chunk publishes its local adjoint at
// its first step, S_c = g_t0 from a zero adjoint after the chunk, and the decay product
// A_c = a_{t0+1} .. a_{t0+n}; the carry of chunk c is g_{t0+n} = S_{c+1} + A_{c+1}(S_{c+2}
// + ...). The forward states come from the forward's published chunk-end states (I_{c-1}
// is the state entering chunk c), so nothing of the forward is recomputed but the chunk's
// own steps. Per chunk one CTA then emits dx, dB, dC, dDT, dtrap, the per-step terms of
// dADT with their chunk total (the cross-chunk suffix sums are mimo_bwd_dadt_kernel's),
// and partial sums of dD, dmimo_x, dmimo_o (atomics). x, B, C and dy arrive as TMA boxes.
// ------------------------------------------------------------------------------------
struct FusedBwdSmem {
  uint32_t bs, cs, xs, dys, bx, hs, gs, xr, dyr, dxr, yr, coef, trdt, dbg, red, mx, mo, rq, carry, total;
};
__host__ __device__ inline FusedBwdSmem fused_bwd_smem(int Q, int P, int R, int D, int eb, int ex) {
  FusedBwdSmem L;
  uint32_t o = 128;
  L.bs = o; o = aup(o + (uint32_t)((Q + 1) * R * D * eb), 128);   // rows t0-1 .. t0+Q-1
  L.cs = o; o = aup(o + (uint32_t)(Q * R * D * eb), 128);         // rows t0 .. t0+Q-1
  L.xs = o; o = aup(o + (uint32_t)((Q + 1) * P * ex), 128);       // rows t0-1 .. t0+Q-1
  L.dys = o; o = aup(o + (uint32_t)(Q * P * ex), 128);            // rows t0 .. t0+Q-1
  L.bx = o; o = aup(o + (uint32_t)((Q + 1) * D * 4), 16);         // bx rows t0-1 .. t0+Q-1
  L.hs = o; o = aup(o + (uint32_t)(Q * D * 4), 16);               // states t0 .. t0+Q-1
  L.gs = o; o = aup(o + (uint32_t)((Q + 1) * D * 4), 16);         // E, then adjoints t0 .. t0+Q
  L.xr = o; o = aup(o + (uint32_t)((Q + 1) * R * 4), 16);
  L.dyr = o; o = aup(o + (uint32_t)(Q * R * 4), 16);
  L.dxr = o; o = aup(o + (uint32_t)(Q * R * 4), 16);
  L.yr = o; o = aup(o + (uint32_t)(Q * R * 4), 16);
  L.coef = o; o = aup(o + (uint32_t)((Q + 1) * 16), 16);          // (a, beta, gamma, -) t0 .. t0+Q
  L.trdt = o; o = aup(o + (uint32_t)(Q * 8), 16);                 // (sigmoid(trap), dt)
  L.dbg = o; o = aup(o + (uint32_t)(Q * 8), 16);                  // (dbeta, dgamma)
  L.red = o; o = aup(o + (uint32_t)(Q * 4), 16);                  // per-step dADT terms
  L.mx = o; o = aup(o + (uint32_t)(R * (P + 4) * 4), 16);
  L.mo = o; o = aup(o + (uint32_t)(R * (P + 4) * 4), 16);
  L.rq = o; o = aup(o + (uint32_t)(Q * 4), 16);                   // a_{t+1} .. a_{t0+n} per step
  L.carry = o; o = aup(o + (uint32_t)(D * 4), 16);                // adjoint entering from the right
  L.total = o + 128;
  return L;
}

struct FusedBwdArgs {
  FastDiv fP4, fD4, fR, fU, fH;
  int nch, units, ahead;
  int bvec;  // dB / dC rows start on 16-byte boundaries (four gradients per store)
  int xvec;  // dx rows likewise
  FusedBwdSmem L;
  const unsigned long long* fwd_rec;  // the forward's words: I_c = the state after chunk c
  unsigned* ticket;
  unsigned long long* rec;   // [unit][chunk][d]: adjoint S or I | status << 32
  unsigned long long* arec;  // [unit][chunk]: A | 1 << 32
  double* tot;               // [unit][chunk]: the chunk's dADT total
};

// The adjoint entering chunk c of unit u from the right (column d), from the words of the
// chunks after it.
__device__ __forceinline__ float look_ahead(const FusedBwdArgs& f, int u, int c, int d, int D, bool& ok) {
  const int64_t base = (int64_t)u * f.nch;
  float acc = 0.f, accA = 1.f;
  int j = c + 1;
  for (uint32_t spins = 0; spins < kSpinLimit; ++spins) {
    const unsigned long long w = ld_relaxed64(f.rec + (base + j) * D + d);
    const unsigned long long av = ld_relaxed64(f.arec + base + j);
    const uint32_t st = (uint32_t)(w >> 32);
    if (st == 2) return fmaf(accA, __uint_as_float((uint32_t)w), acc);
    if (st == 1 && (av >> 32) != 0) {
      acc = fmaf(accA, __uint_as_float((uint32_t)w), acc);
      accA *= __uint_as_float((uint32_t)av);
      if (++j >= f.nch) break;  // the last chunk publishes its inclusive adjoint only: unreachable
      continue;
    }
    __nanosleep(32);
  }
  ok = false;
  return 0.f;
}

template <typename T>
__device__ __forceinline__ void st4v(T* p, float4 v, bool vec) {
  if (vec) {
    st4(p, v);
  } else {
    st(p, v.x);
    st(p + 1, v.y);
    st(p + 2, v.z);
    st(p + 3, v.w);
  }
}

template <typename TX, typename TB, int Q>
__global__ void __launch_bounds__(kFT)
    mimo_fused_bwd_kernel(const __grid_constant__ CUtensorMap mapB, const __grid_constant__ CUtensorMap mapC,
                          const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapDY,
                          MimoParams a, FusedBwdArgs f) {
  static_assert(Q < kFT, "a thread per step of the chunk and the one after it");
  extern __shared__ __align__(128) unsigned char fsm_raw[];
  unsigned char* fsm = fsm_raw + ((128u - (sm100::smem_u32(fsm_raw) & 127u)) & 127u);
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P4 = P >> 2, D4 = D >> 2, MS = P + 4;
  const FusedBwdSmem& L = f.L;
  uint64_t* bar = reinterpret_cast<uint64_t*>(fsm);
  int* tk_s = reinterpret_cast<int*>(fsm + 16);
  const TB* Bs = reinterpret_cast<const TB*>(fsm + L.bs);
  const TB* Cs = reinterpret_cast<const TB*>(fsm + L.cs);
  const TX* xs = reinterpret_cast<const TX*>(fsm + L.xs);
  const TX* dys = reinterpret_cast<const TX*>(fsm + L.dys);
  float* bxs = reinterpret_cast<float*>(fsm + L.bx);
  float* hs = reinterpret_cast<float*>(fsm + L.hs);
  float* gs = reinterpret_cast<float*>(fsm + L.gs);
  float* xr = reinterpret_cast<float*>(fsm + L.xr);
  float* dyr = reinterpret_cast<float*>(fsm + L.dyr);
  float* dxr = reinterpret_cast<float*>(fsm + L.dxr);
  float* yr = reinterpret_cast<float*>(fsm + L.yr);
  float4* coef = reinterpret_cast<float4*>(fsm + L.coef);
  float2* trdt = reinterpret_cast<float2*>(fsm + L.trdt);
  float2* dbg = reinterpret_cast<float2*>(fsm + L.dbg);
  float* red = reinterpret_cast<float*>(fsm + L.red);
  float* mx = reinterpret_cast<float*>(fsm + L.mx);
  float* mo = reinterpret_cast<float*>(fsm + L.mo);
  float* rq = reinterpret_cast<float*>(fsm + L.rq);
  float* carry_s = reinterpret_cast<float*>(fsm + L.carry);

  if (tid == 0) {
    *tk_s = (int)atomicAdd(f.ticket, 1u);
    sm100::mbar_init(bar, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const int tk = *tk_s;
  const int ci = fdiv(tk, f.fU), u = tk - ci * f.units, c = f.nch - 1 - ci;
  const int b = fdiv(u, f.fH), h = u - b * a.H;
  const int t0 = c * Q, n = min(Q, a.L - t0);
  // the step scalars of t0 .. t0+n (the one after the chunk for the adjoint; zero past the
  // end) and the state entering the chunk, first: their loads are in flight meanwhile
  float s_adt = 0.f, s_dt = 0.f, s_tr = 0.f;
  const bool sv = tid <= n && t0 + tid < a.L;
  if (sv) {
    s_adt = scalc(a.adt, a.sadt, b, t0 + tid, h);
    s_dt = scalc(a.dt, a.sdt, b, t0 + tid, h);
    s_tr = scalc(a.trap, a.strap, b, t0 + tid, h);
  }
  float hin = 0.f;
  if (tid < D) {
    if (c > 0)
      hin = __uint_as_float((uint32_t)f.fwd_rec[((int64_t)u * f.nch + c - 1) * D + tid]);
    else if (a.h0)
      hin = a.h0[(int64_t)u * D + tid];
  }
  if (tid == 0) {
    sm100::mbar_expect_tx(bar, (uint32_t)((Q + 1) * (R * D * sizeof(TB) + P * sizeof(TX)) +
                                          Q * (R * D * sizeof(TB) + P * sizeof(TX))));
    sm100::tma_load_5d(fsm + L.bs, &mapB, bar, 0, h, 0, t0 - 1, b);
    sm100::tma_load_5d(fsm + L.cs, &mapC, bar, 0, h, 0, t0, b);
    sm100::tma_load_4d(fsm + L.xs, &mapX, bar, 0, h, t0 - 1, b);
    sm100::tma_load_4d(fsm + L.dys, &mapDY, bar, 0, h, t0, b);
  }
  const int tf = tk + f.ahead;
  if (tf < f.units * f.nch && tid < 32) {
    const int cif = fdiv(tf, f.fU), uf = tf - cif * f.units, bf = fdiv(uf, f.fH), hf = uf - bf * a.H;
    const int tf0 = (f.nch - 1 - cif) * Q;
    if (tid == 0) {  // rows from max(t0 - 1, 0): no prefetch starts outside the tensor
      sm100::tma_prefetch_l2_5d(&mapB, 0, hf, 0, max(tf0 - 1, 0), bf);
      sm100::tma_prefetch_l2_5d(&mapC, 0, hf, 0, tf0, bf);
      sm100::tma_prefetch_l2_4d(&mapX, 0, hf, max(tf0 - 1, 0), bf);
      sm100::tma_prefetch_l2_4d(&mapDY, 0, hf, tf0, bf);
    }
    for (int t = tf0 + tid; t < min(tf0 + Q + 1, a.L); t += 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.adt + (int64_t)bf * a.sadt.b + (int64_t)t * a.sadt.l + (int64_t)hf * a.sadt.h));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.dt + (int64_t)bf * a.sdt.b + (int64_t)t * a.sdt.l + (int64_t)hf * a.sdt.h));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.trap + (int64_t)bf * a.strap.b + (int64_t)t * a.strap.l + (int64_t)hf * a.strap.h));
    }
  }
  for (int i = tid; i < R * P; i += kFT) {
    const int r = fdiv(i >> 2, f.fP4), p = i - r * P;
    mx[r * MS + p] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + p];
    mo[r * MS + p] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + p];
  }
  if (tid <= n) {
    const float tr = sv ? sigmoidf_(s_tr) : 0.f;
    coef[tid] = sv ? make_float4(expf(s_adt), s_dt * (1.0f - tr) + 0.5f * s_dt * tr, 0.5f * s_dt * tr, 0.f)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < n) trdt[tid] = make_float2(tr, s_dt);
  }
  __syncthreads();
  wait_copies(bar);
  // xr for x rows t0-1 .. t0+n-1 and dyr for dy rows t0 .. t0+n-1, four p per step
  for (int i = tid; i < (2 * n + 1) * R; i += kFT) {
    const bool isx = i < (n + 1) * R;
    const int j = isx ? i : i - (n + 1) * R;
    const int row = fdiv(j, f.fR), k = j - row * R;
    const TX* vrow = (isx ? xs : dys) + row * P;
    const float* mrow = (isx ? mx : mo) + k * MS;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int pb = row - fdiv(row, f.fP4) * P4;
    for (int e = 0; e < P4; ++e) {
      fma4(acc, ld4f(vrow + 4 * pb), ld4f(mrow + 4 * pb));
      pb = pb + 1 == P4 ? 0 : pb + 1;
    }
    (isx ? xr : dyr)[j] = (acc.x + acc.y) + (acc.z + acc.w);
  }
  __syncthreads();
  // bx for rows t0-1 .. t0+n-1 and E for t0 .. t0+n-1, four columns a thread
  for (int i = tid; i < (2 * n + 1) * D4; i += kFT) {
    const bool isb = i < (n + 1) * D4;
    const int j = isb ? i : i - (n + 1) * D4;
    const int row = fdiv(j, f.fD4), d = 4 * (j - row * D4);
    const float* wrow = (isb ? xr : dyr) + row * R;
    const TB* mrow = (isb ? Bs : Cs) + (size_t)row * R * D + d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < R; ++r) fma4(acc, wrow[r], ld4f(mrow + (size_t)r * D));
    *reinterpret_cast<float4*>((isb ? bxs : gs) + row * D + d) = acc;
  }
  __syncthreads();
  // per column: the chunk's states from the entering state, its local adjoint from a zero
  // adjoint after it, the adjoint carry from the chunks after it, the true adjoints
  const int64_t cell = (int64_t)u * f.nch + c;
  bool ok = true;
  if (tid < D) {
    const int d = tid;
    if (c == 0) bxs[d] = a.bx0 ? a.bx0[(int64_t)u * D + d] : 0.f;
    float hv = hin, bxp = bxs[d];
    for (int tb = 0; tb < n; tb += 8) {
      float bxv[8];
      float4 cf[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool in = tb + j < n;
        bxv[j] = in ? bxs[(tb + j + 1) * D + d] : 0.f;
        cf[j] = in ? coef[tb + j] : make_float4(1.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        hv = fmaf(cf[j].x, hv, fmaf(cf[j].y, bxv[j], cf[j].z * bxp));
        if (tb + j < n) {
          bxp = bxv[j];
          hs[(tb + j) * D + d] = hv;
        }
      }
    }
    // the local adjoint from a zero adjoint after the chunk, eight steps per batch of
    // shared-memory reads; column 0 records the decay from each step to the chunk's end
    float gl = 0.f, pr = 1.f;
    for (int te = n; te > 0; te -= 8) {
      float ev[8], an[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = te - 1 - j;
        ev[j] = t >= 0 ? gs[t * D + d] : 0.f;
        an[j] = t >= 0 ? coef[t + 1].x : 1.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = te - 1 - j;
        gl = fmaf(an[j], gl, ev[j]);
        pr *= an[j];
        if (t >= 0) {
          gs[t * D + d] = gl;
          if (d == 0) rq[t] = pr;
        }
      }
    }
    float carry = 0.f;
    if (c < f.nch - 1) {
      st_relaxed64(f.rec + cell * D + d, gl, 1);
      if (d == 0) st_relaxed64(f.arec + cell, pr, 1);
      carry = look_ahead(f, u, c, d, D, ok);
    }
    const float g0 = fmaf(pr, carry, gl);  // the true adjoint at the chunk's first step
    st_relaxed64(f.rec + cell * D + d, g0, 2);
    carry_s[d] = carry;
    gs[n * D + d] = carry;
    if (c == 0) {
      if (a.dh0) a.dh0[(int64_t)u * D + d] = coef[0].x * g0;
      if (a.dbx0) a.dbx0[(int64_t)u * D + d] = coef[0].z * g0;
    }
  }
  if (!ok) atomicExch(&g_mimo_error, 1);
  __syncthreads();
  // the true adjoints g_t = gl_t + (a_{t+1} .. a_{t0+n}) carry, four columns a thread
  for (int i = tid; i < n * D4; i += kFT) {
    const int t = fdiv(i, f.fD4), d = 4 * (i - t * D4);
    float4 g4 = *reinterpret_cast<const float4*>(gs + t * D + d);
    fma4(g4, rq[t], *reinterpret_cast<const float4*>(carry_s + d));
    *reinterpret_cast<float4*>(gs + t * D + d) = g4;
  }
  __syncthreads();
  if (!ok) atomicExch(&g_mimo_error, 1);
  __syncthreads();
  // per (t, four-column block): v = beta_t g_t + gamma_{t+1} g_{t+1} once, then for each
  // rank dC = dyr h, dB = xr v and the partial dots dxr = B . v, yr = C . h, and the step's
  // dbeta = g_t . bx_t, dgamma = g_t . bx_{t-1}; lpr lanes per step, ranks four at a time
  const float Dk = a.Dskip[h * a.sD];
  int lpr = 1;
  while (lpr * 2 <= 32 && lpr * 2 <= D4) lpr *= 2;
  const int rpw = 32 / lpr, part = lane & (lpr - 1);
  TB* dBb = reinterpret_cast<TB*>(a.dB) + (int64_t)b * a.sdB.b + (int64_t)h * a.sdB.h;
  TB* dCb = reinterpret_cast<TB*>(a.dC) + (int64_t)b * a.sdC.b + (int64_t)h * a.sdC.h;
  for (int tw = warp * rpw; tw < n; tw += (kFT / 32) * rpw) {
    const int t = tw + lane / lpr;
    const bool tv = t < n;
    const int tc = tv ? t : 0;
    const float be = coef[tc].y, gan = coef[tc + 1].z;
    TB* dBt = dBb + (int64_t)(t0 + tc) * a.sdB.l;
    TB* dCt = dCb + (int64_t)(t0 + tc) * a.sdC.l;
    float sb = 0.f, sg = 0.f;
    for (int r0 = 0; r0 < R; r0 += 4) {
      float sx[4] = {0.f, 0.f, 0.f, 0.f}, sy[4] = {0.f, 0.f, 0.f, 0.f};
      if (tv)
        for (int blk = part; blk < D4; blk += lpr) {
          const int d = 4 * blk;
          const float4 h4 = *reinterpret_cast<const float4*>(hs + tc * D + d);
          const float4 g4 = *reinterpret_cast<const float4*>(gs + tc * D + d);
          const float4 g4n = *reinterpret_cast<const float4*>(gs + (tc + 1) * D + d);
          const float4 v4 = make_float4(fmaf(be, g4.x, gan * g4n.x), fmaf(be, g4.y, gan * g4n.y),
                                        fmaf(be, g4.z, gan * g4n.z), fmaf(be, g4.w, gan * g4n.w));
          if (r0 == 0) {
            const float4 b1 = *reinterpret_cast<const float4*>(bxs + (tc + 1) * D + d);
            const float4 b0 = *reinterpret_cast<const float4*>(bxs + tc * D + d);
            sb = fmaf(g4.x, b1.x, fmaf(g4.y, b1.y, fmaf(g4.z, b1.z, fmaf(g4.w, b1.w, sb))));
            sg = fmaf(g4.x, b0.x, fmaf(g4.y, b0.y, fmaf(g4.z, b0.z, fmaf(g4.w, b0.w, sg))));
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int r = r0 + q;
            if (r < R) {
              const float4 b4 = ld4f(Bs + ((size_t)(tc + 1) * R + r) * D + d);
              const float4 c4 = ld4f(Cs + ((size_t)tc * R + r) * D + d);
              sx[q] = fmaf(b4.x, v4.x, fmaf(b4.y, v4.y, fmaf(b4.z, v4.z, fmaf(b4.w, v4.w, sx[q]))));
              sy[q] = fmaf(c4.x, h4.x, fmaf(c4.y, h4.y, fmaf(c4.z, h4.z, fmaf(c4.w, h4.w, sy[q]))));
              const float dv = dyr[tc * R + r], xv = xr[(tc + 1) * R + r];
              st4v(dCt + (int64_t)r * a.sdC.r + d, make_float4(dv * h4.x, dv * h4.y, dv * h4.z, dv * h4.w), f.bvec);
              st4v(dBt + (int64_t)r * a.sdB.r + d, make_float4(xv * v4.x, xv * v4.y, xv * v4.z, xv * v4.w), f.bvec);
            }
          }
        }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        for (int o = lpr >> 1; o > 0; o >>= 1) {
          sx[q] += __shfl_xor_sync(0xffffffffu, sx[q], o);
          sy[q] += __shfl_xor_sync(0xffffffffu, sy[q], o);
        }
      if (tv && part == 0)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = r0 + q;
          if (r < R) {
            dxr[tc * R + r] = fmaf(Dk, dyr[tc * R + r], sx[q]);
            yr[tc * R + r] = fmaf(Dk, xr[(tc + 1) * R + r], sy[q]);
          }
        }
    }
    for (int o = lpr >> 1; o > 0; o >>= 1) {
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
      sg += __shfl_xor_sync(0xffffffffu, sg, o);
    }
    if (tv && part == 0) dbg[tc] = make_float2(sb, sg);
  }
  __syncthreads();
  // per t: q = sum_r dyr (yr - D xr) = E_t . h_t, the dADT term, dDT and dtrap
  if (tid < n) {
    const int t = tid;
    float qv = 0.f;
    for (int r = 0; r < R; ++r) qv = fmaf(dyr[t * R + r], fmaf(-Dk, xr[(t + 1) * R + r], yr[t * R + r]), qv);
    const float2 bg = dbg[t], td = trdt[t];
    const float4 cf = coef[t];
    red[t] = qv - cf.y * bg.x - cf.z * bg.y;
    const int64_t tt = t0 + t;
    a.ddt[(int64_t)b * a.sddt.b + tt * a.sddt.l + (int64_t)h * a.sddt.h] = bg.x * (1.0f - 0.5f * td.x) + bg.y * 0.5f * td.x;
    a.dtrap[(int64_t)b * a.sdtrap.b + tt * a.sdtrap.l + (int64_t)h * a.sdtrap.h] =
        0.5f * td.y * (bg.y - bg.x) * td.x * (1.0f - td.x);
  }
  // dx = mimo_x^T dxr, four p a thread
  TX* dxb = reinterpret_cast<TX*>(a.dx) + (int64_t)b * a.sdx.b + (int64_t)h * a.sdx.h;
  for (int i = tid; i < n * P4; i += kFT) {
    const int t = fdiv(i, f.fP4), p = 4 * (i - t * P4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < R; ++r) fma4(acc, dxr[t * R + r], ld4f(mx + r * MS + p));
    st4v(dxb + (int64_t)(t0 + t) * a.sdx.l + p, acc, f.xvec);
  }
  // dmimo_x += dxr x^T, dmimo_o += yr dy^T, dD += <dyr, xr>
  for (int i = tid; i < R * P; i += kFT) {
    const int r = fdiv(i >> 2, f.fP4), p = i - r * P;
    float ax = 0.f, ao = 0.f;
    for (int t = 0; t < n; ++t) {
      ax = fmaf(dxr[t * R + r], to_f32(xs[(t + 1) * P + p]), ax);
      ao = fmaf(yr[t * R + r], to_f32(dys[t * P + p]), ao);
    }
    atomicAdd(a.dmx + (int64_t)h * R * P + i, ax);
    atomicAdd(a.dmo + (int64_t)h * R * P + i, ao);
  }
  if (warp == kFT / 32 - 1) {
    float v = 0.f;
    for (int i = lane; i < n * R; i += 32) {
      const int t = fdiv(i, f.fR), r = i - t * R;
      v = fmaf(dyr[i], xr[(t + 1) * R + r], v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) atomicAdd(a.dD + h, v);
  }
  __syncthreads();
  // within-chunk suffix sums of the dADT terms (fp64); the chunk total for the cross-chunk sums
  if (tid == 0) {
    double cum = 0.0;
    for (int t = n - 1; t >= 0; --t) {
      cum += (double)red[t];
      a.dadt[(int64_t)b * a.sdadt.b + (int64_t)(t0 + t) * a.sdadt.l + (int64_t)h * a.sdadt.h] = (float)cum;
    }
    f.tot[cell] = cum;
  }
}

template <typename K>
int opt_in(K k, size_t smem) {
  if (smem <= 48 * 1024) return M3_OK;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  return M3_OK;
}

// The single-pass forward applies when its TMA boxes can be described: x, B and C 16-byte
// aligned with strides of whole 16-byte units, rows of whole 16-byte units, headdim and
// d_state at most 256 (one box dimension), d_state a multiple of 4, rank at most 8.
template <typename TX, typename TB>
bool fused_applies(const MimoParams& p) {
  const int64_t eb = sizeof(TB), ex = sizeof(TX);
  auto al = [&](const void* ptr, const Str4& st) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (st.b * eb) % 16 == 0 && (st.l * eb) % 16 == 0 &&
           (st.r * eb) % 16 == 0 && (st.h * eb) % 16 == 0 && st.b > 0 && st.l > 0 && st.r > 0 && st.h > 0;
  };
  const bool xal = reinterpret_cast<uintptr_t>(p.x) % 16 == 0 && (p.sx.b * ex) % 16 == 0 && (p.sx.l * ex) % 16 == 0 &&
                   (p.sx.h * ex) % 16 == 0 && p.sx.b > 0 && p.sx.l > 0 && p.sx.h > 0 && (p.P * ex) % 16 == 0 &&
                   p.P <= 256;
  return p.D % 4 == 0 && p.D <= 256 && p.R <= 8 && (p.D * eb) % 16 == 0 && al(p.Bm, p.sB) && al(p.Cm, p.sC) &&
         xal && chunk_encode_fn() != nullptr;
}

// Chunk length of the single-pass forward: the longest of 64 / 32 / 16 steps whose shared
// memory lets four CTAs share an SM, else the shortest that fits at all.
template <typename TX, typename TB>
int fused_chunk(const MimoParams& p) {
  for (int q : {64, 32, 16})
    if (fused_smem(q, p.P, p.R, p.D, (int)sizeof(TB), (int)sizeof(TX)).total <= 55u * 1024u) return q;
  return fused_smem(16, p.P, p.R, p.D, (int)sizeof(TB), (int)sizeof(TX)).total <= 200u * 1024u ? 16 : 0;
}

template <typename TB> constexpr CUtensorMapDataType tmap_type();
template <> constexpr CUtensorMapDataType tmap_type<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <> constexpr CUtensorMapDataType tmap_type<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <> constexpr CUtensorMapDataType tmap_type<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

// 5-d map over (d, h, r, t, b) of a (B, L, R, H, D) tensor with a (D, 1, R, rows, 1) box,
// no swizzle: the box lands in shared memory as [t][r][d].
template <typename TB>
bool make_bc_map(CUtensorMap* m, const void* base, const MimoParams& p, const Str4& st, int rows) {
  auto enc = chunk_encode_fn();
  if (!enc) return false;
  const cuuint64_t eb = sizeof(TB);
  cuuint64_t dims[5] = {(cuuint64_t)p.D, (cuuint64_t)p.H, (cuuint64_t)p.R, (cuuint64_t)p.L, (cuuint64_t)p.Bn};
  cuuint64_t strides[4] = {(cuuint64_t)st.h * eb, (cuuint64_t)st.r * eb, (cuuint64_t)st.l * eb, (cuuint64_t)st.b * eb};
  cuuint32_t box[5] = {(cuuint32_t)p.D, 1, (cuuint32_t)p.R, (cuuint32_t)rows, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(m, tmap_type<TB>(), 5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-d map over (p, h, t, b) of a (B, L, H, P) tensor with a (P, 1, rows, 1) box: [t][p].
template <typename TX>
bool make_row_map(CUtensorMap* m, const void* base, const Str3& st, const MimoParams& p, int rows) {
  auto enc = chunk_encode_fn();
  if (!enc) return false;
  const cuuint64_t ex = sizeof(TX);
  cuuint64_t dims[4] = {(cuuint64_t)p.P, (cuuint64_t)p.H, (cuuint64_t)p.L, (cuuint64_t)p.Bn};
  cuuint64_t strides[3] = {(cuuint64_t)st.h * ex, (cuuint64_t)st.l * ex, (cuuint64_t)st.b * ex};
  cuuint32_t box[4] = {(cuuint32_t)p.P, 1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, tmap_type<TX>(), 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
template <typename TX>
bool make_x_map(CUtensorMap* m, const MimoParams& p, int rows) { return make_row_map<TX>(m, p.x, p.sx, p, rows); }

// rows of 4 elements starting on 16-byte boundaries at every (b, t, h[, r]) and column 4k
template <typename T>
bool vec4_rows(const void* ptr, const Str3& st) {
  const int64_t e = sizeof(T);
  return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (st.b * e) % 16 == 0 && (st.l * e) % 16 == 0 &&
         (st.h * e) % 16 == 0;
}
template <typename T>
bool vec4_rows(const void* ptr, const Str4& st) {
  const int64_t e = sizeof(T);
  return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (st.b * e) % 16 == 0 && (st.l * e) % 16 == 0 &&
         (st.r * e) % 16 == 0 && (st.h * e) % 16 == 0;
}

// Returns M3_ERR_UNSUPPORTED (nothing launched) when a tensor map cannot be made.
template <typename TX, typename TB, int Q>
int run_fused(const MimoParams& p, void* ws, cudaStream_t s) {
  const int64_t nch = (p.L + Q - 1) / Q, units = (int64_t)p.Bn * p.H, cells = units * nch;
  if (cells >= INT32_MAX) return M3_ERR_UNSUPPORTED;
  CUtensorMap mB, mC, mX;
  if (!make_bc_map<TB>(&mB, p.Bm, p, p.sB, Q + 1) || !make_bc_map<TB>(&mC, p.Cm, p, p.sC, Q) ||
      !make_x_map<TX>(&mX, p, Q + 1))
    return M3_ERR_UNSUPPORTED;
  FusedArgs f;
  f.fP4 = make_fastdiv((uint32_t)(p.P / 4));
  f.fD4 = make_fastdiv((uint32_t)(p.D / 4));
  f.fR = make_fastdiv((uint32_t)p.R);
  f.fU = make_fastdiv((uint32_t)units);
  f.fH = make_fastdiv((uint32_t)p.H);
  f.nch = (int)nch;
  f.units = (int)units;
  {
    const int64_t ey = sizeof(TX);
    f.yvec = reinterpret_cast<uintptr_t>(p.y) % 16 == 0 && (p.sy.b * ey) % 16 == 0 && (p.sy.l * ey) % 16 == 0 &&
             (p.sy.h * ey) % 16 == 0;
  }
  char* w = static_cast<char*>(ws);
  f.ticket = reinterpret_cast<unsigned*>(w);
  f.rec = reinterpret_cast<unsigned long long*>(w + 16);
  f.arec = f.rec + cells * p.D;
  f.L = fused_smem(Q, p.P, p.R, p.D, (int)sizeof(TB), (int)sizeof(TX));
  const size_t smem = f.L.total;
  static LaunchCache lc;
  M3_TRY(kernel_residency(reinterpret_cast<const void*>(mimo_fused_fwd_kernel<TX, TB, Q, false>), kFT, smem, &lc,
                          &f.ahead));
  cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)fused_ws_bytes(cells, p.D), s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  mimo_fused_fwd_kernel<TX, TB, Q, false><<<(unsigned)cells, kFT, smem, s>>>(mB, mC, mX, p, f, GrpArgs{});
  return check_launch("mimo_fused_fwd_kernel");
}

// 4-d map with a (box0, box1, rows, 1) box over dims (n0, n1, L, Bn), element strides
// (s1, s_l, s_b) for dims 1..3, no swizzle: the box lands as [row][i1][i0].
template <typename T>
bool make_map4(CUtensorMap* m, const void* base, int64_t n0, int64_t n1, int64_t L, int64_t Bn, int64_t s1,
               int64_t s_l, int64_t s_b, int box0, int box1, int rows) {
  auto enc = chunk_encode_fn();
  if (!enc) return false;
  const cuuint64_t e = sizeof(T);
  cuuint64_t dims[4] = {(cuuint64_t)n0, (cuuint64_t)n1, (cuuint64_t)L, (cuuint64_t)Bn};
  cuuint64_t strides[3] = {(cuuint64_t)s1 * e, (cuuint64_t)s_l * e, (cuuint64_t)s_b * e};
  cuuint32_t box[4] = {(cuuint32_t)box0, (cuuint32_t)box1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, tmap_type<T>(), 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Chunk length of the group-row form: the longest of 64 / 32 / 16 steps whose shared memory
// lets four CTAs share an SM, else 16 when it fits at all, else 0.
inline int grp_chunk(const MimoParams& p, int e, int S, bool gate) {
  for (int q : {64, 32, 16})
    if (fused_smem(q, p.P, p.R, p.D, e, e, true, S, gate).total <= 55u * 1024u) return q;
  return fused_smem(16, p.P, p.R, p.D, e, e, true, S, gate).total <= 200u * 1024u ? 16 : 0;
}

// Group-row form of the single-pass forward from the in_proj output zx (Bn, L, d_proj):
// z at columns [0, H P), x at [H P, 2 H P), the B group rows at [2 H P, 2 H P + R D) and the
// C rows right after. Returns M3_ERR_UNSUPPORTED (nothing launched) when a map cannot be
// made.
template <typename T, int Q>
int run_fused_grp(const MimoParams& p, const GrpArgs& g0, const T* zx, int64_t s_zb, int64_t s_zl, void* ws,
                  cudaStream_t s) {
  const int64_t nch = (p.L + Q - 1) / Q, units = (int64_t)p.Bn * p.H, cells = units * nch;
  if (cells >= INT32_MAX) return M3_ERR_UNSUPPORTED;
  const int64_t di = (int64_t)p.H * p.P;
  CUtensorMap mB, mX;
  if (!make_map4<T>(&mB, zx + 2 * di, p.D, 2 * p.R, p.L, p.Bn, p.D, s_zl, s_zb, p.D, 2 * p.R, Q + 1) ||
      !make_map4<T>(&mX, zx, p.P, 2 * p.H, p.L, p.Bn, p.P, s_zl, s_zb, p.P, 1, Q + 1))
    return M3_ERR_UNSUPPORTED;
  GrpArgs g = g0;
  if (g.S > 0) g.fS = make_fastdiv((uint32_t)g.S);
  FusedArgs f;
  f.fP4 = make_fastdiv((uint32_t)(p.P / 4));
  f.fD4 = make_fastdiv((uint32_t)(p.D / 4));
  f.fR = make_fastdiv((uint32_t)p.R);
  f.fU = make_fastdiv((uint32_t)units);
  f.fH = make_fastdiv((uint32_t)p.H);
  f.nch = (int)nch;
  f.units = (int)units;
  {
    const int64_t ey = sizeof(T);
    f.yvec = reinterpret_cast<uintptr_t>(p.y) % 16 == 0 && (p.sy.b * ey) % 16 == 0 && (p.sy.l * ey) % 16 == 0 &&
             (p.sy.h * ey) % 16 == 0;
  }
  char* w = static_cast<char*>(ws);
  f.ticket = reinterpret_cast<unsigned*>(w);
  f.rec = reinterpret_cast<unsigned long long*>(w + 16);
  f.arec = f.rec + cells * p.D;
  f.L = fused_smem(Q, p.P, p.R, p.D, (int)sizeof(T), (int)sizeof(T), true, g.S, g.gate != 0);
  const size_t smem = f.L.total;
  static LaunchCache lc;
  M3_TRY(kernel_residency(reinterpret_cast<const void*>(mimo_fused_fwd_kernel<T, T, Q, true>), kFT, smem, &lc,
                          &f.ahead));
  cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)fused_ws_bytes(cells, p.D), s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  // mapC is not read by the group-row form; mB stands in for it
  mimo_fused_fwd_kernel<T, T, Q, true><<<(unsigned)cells, kFT, smem, s>>>(mB, mB, mX, p, f, g);
  return check_launch("mimo_fused_fwd_kernel");
}

// Workspace of the single-pass backward: ticket, adjoint words and decay words (cleared
// before each launch), then the per-chunk dADT totals.
inline int64_t fused_bwd_ws_bytes(int64_t cells, int64_t D) { return fused_ws_bytes(cells, D) + 8 * cells + 16; }

// Returns M3_ERR_UNSUPPORTED (nothing launched) when the single-pass pair does not apply.
template <typename TX, typename TB, int Q>
int run_fused_bwd(const MimoParams& p, const void* fwd_ws, size_t fwd_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s) {
  const int64_t nch = (p.L + Q - 1) / Q, units = (int64_t)p.Bn * p.H, cells = units * nch;
  if (cells >= INT32_MAX || fwd_bytes < (size_t)fused_ws_bytes(cells, p.D) ||
      ws_bytes < (size_t)fused_bwd_ws_bytes(cells, p.D))
    return M3_ERR_UNSUPPORTED;
  if (!vec4_rows<TX>(p.dy, p.sdy) || (p.P * (int64_t)sizeof(TX)) % 16 != 0) return M3_ERR_UNSUPPORTED;
  const FusedBwdSmem L = fused_bwd_smem(Q, p.P, p.R, p.D, (int)sizeof(TB), (int)sizeof(TX));
  if (L.total > 200u * 1024u) return M3_ERR_UNSUPPORTED;
  CUtensorMap mB, mC, mX, mDY;
  if (!make_bc_map<TB>(&mB, p.Bm, p, p.sB, Q + 1) || !make_bc_map<TB>(&mC, p.Cm, p, p.sC, Q) ||
      !make_row_map<TX>(&mX, p.x, p.sx, p, Q + 1) || !make_row_map<TX>(&mDY, p.dy, p.sdy, p, Q))
    return M3_ERR_UNSUPPORTED;
  FusedBwdArgs f;
  f.fP4 = make_fastdiv((uint32_t)(p.P / 4));
  f.fD4 = make_fastdiv((uint32_t)(p.D / 4));
  f.fR = make_fastdiv((uint32_t)p.R);
  f.fU = make_fastdiv((uint32_t)units);
  f.fH = make_fastdiv((uint32_t)p.H);
  f.nch = (int)nch;
  f.units = (int)units;
  f.bvec = vec4_rows<TB>(p.dB, p.sdB) && vec4_rows<TB>(p.dC, p.sdC);
  f.xvec = vec4_rows<TX>(p.dx, p.sdx);
  f.L = L;
  f.fwd_rec = reinterpret_cast<const unsigned long long*>(static_cast<const char*>(fwd_ws) + 16);
  char* w = static_cast<char*>(ws);
  f.ticket = reinterpret_cast<unsigned*>(w);
  f.rec = reinterpret_cast<unsigned long long*>(w + 16);
  f.arec = f.rec + cells * p.D;
  f.tot = reinterpret_cast<double*>(w + ((fused_ws_bytes(cells, p.D) + 15) & ~int64_t(15)));
  static LaunchCache lc;
  M3_TRY(kernel_residency(reinterpret_cast<const void*>(mimo_fused_bwd_kernel<TX, TB, Q>), kFT, L.total, &lc,
                          &f.ahead));
  cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)fused_ws_bytes(cells, p.D), s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  mimo_fused_bwd_kernel<TX, TB, Q><<<(unsigned)cells, kFT, L.total, s>>>(mB, mC, mX, mDY, p, f);
  M3_TRY(check_launch("mimo_fused_bwd_kernel"));
  mimo_bwd_dadt_kernel<<<(unsigned)units, kCT, 0, s>>>(p, f.tot, (int)nch, Q);
  return check_launch("mimo_bwd_dadt_kernel");
}

template <typename TX, typename TB>
int run_bwd_fused(const MimoParams& p, const void* fwd_ws, size_t fwd_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s) {
  if (!fused_applies<TX, TB>(p)) return M3_ERR_UNSUPPORTED;
  switch (fused_chunk<TX, TB>(p)) {
    case 64: return run_fused_bwd<TX, TB, 64>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
    case 32: return run_fused_bwd<TX, TB, 32>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
    case 16: return run_fused_bwd<TX, TB, 16>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
    default: return M3_ERR_UNSUPPORTED;
  }
}

template <typename TX, typename TB>
int run_chunked(const MimoParams& p, void* ws_raw, cudaStream_t s) {
  if (fused_applies<TX, TB>(p)) {
    int rc = M3_ERR_UNSUPPORTED;
    switch (fused_chunk<TX, TB>(p)) {
      case 64: rc = run_fused<TX, TB, 64>(p, ws_raw, s); break;
      case 32: rc = run_fused<TX, TB, 32>(p, ws_raw, s); break;
      case 16: rc = run_fused<TX, TB, 16>(p, ws_raw, s); break;
      default: break;
    }
    if (rc != M3_ERR_UNSUPPORTED) return rc;
  }
  float* ws = static_cast<float*>(ws_raw);
  const int nch = (p.L + kTcF - 1) / kTcF;
  const int units = p.Bn * p.H;
  float* S = ws;
  float* Adec = ws + (size_t)units * nch * p.D;
  const size_t sm_loc = csmem_floats<kTcF>(p.P, p.R, p.D, false) * sizeof(float);
  const size_t sm_out = csmem_floats<kTcF>(p.P, p.R, p.D, true) * sizeof(float);
  if (sm_out > 200 * 1024) return fail(M3_ERR_UNSUPPORTED, "mimo scan: shapes too large for shared memory");
  M3_TRY(opt_in(mimo_local_kernel<TX, TB, kTcF>, sm_loc));
  M3_TRY(opt_in(mimo_out_kernel<TX, TB>, sm_out));
  const dim3 grid(nch, units);
  mimo_local_kernel<TX, TB, kTcF><<<grid, kCT, sm_loc, s>>>(p, S, Adec, nch);
  M3_TRY(check_launch("mimo_local_kernel"));
  mimo_carry_kernel<<<units, kCT, 0, s>>>(p, S, Adec, nch, true);
  M3_TRY(check_launch("mimo_carry_kernel"));
  mimo_out_kernel<TX, TB><<<grid, kCT, sm_out, s>>>(p, S, nch);
  return check_launch("mimo_out_kernel");
}

template <typename TX, typename TB>
int run_bwd_chunked(const MimoParams& p0, void* ws, cudaStream_t s) {
  MimoParams p = p0;
  const int nch = (p.L + kTcB - 1) / kTcB;
  const int units = p.Bn * p.H;
  double* tot = reinterpret_cast<double*>(ws);
  float* Hc = reinterpret_cast<float*>(tot + (size_t)units * nch);
  float* Af = Hc + (size_t)units * nch * p.D;
  float* Gc = Af + (size_t)units * nch;
  float* Ab = Gc + (size_t)units * nch * p.D;
  const size_t sm_loc = csmem_floats<kTcB>(p.P, p.R, p.D, false) * sizeof(float);
  const size_t sm_bl = ((size_t)p.R * p.P + (size_t)kTcB * p.P + (size_t)kTcB * p.R + kTcB) * sizeof(float);
  const size_t sm_full = bsmem_floats(p.P, p.R, p.D) * sizeof(float);
  M3_TRY(opt_in(mimo_local_kernel<TX, TB, kTcB>, sm_loc));
  M3_TRY(opt_in(mimo_bwd_local_kernel<TX, TB>, sm_bl));
  M3_TRY(opt_in(mimo_bwd_full_kernel<TX, TB>, sm_full));
  const dim3 grid(nch, units);
  // forward states at the chunk starts
  mimo_local_kernel<TX, TB, kTcB><<<grid, kCT, sm_loc, s>>>(p, Hc, Af, nch);
  M3_TRY(check_launch("mimo_local_kernel"));
  mimo_carry_kernel<<<units, kCT, 0, s>>>(p, Hc, Af, nch, false);
  M3_TRY(check_launch("mimo_carry_kernel"));
  // adjoints entering each chunk from the right
  mimo_bwd_local_kernel<TX, TB><<<grid, kCT, sm_bl, s>>>(p, Gc, Ab, nch);
  M3_TRY(check_launch("mimo_bwd_local_kernel"));
  mimo_bwd_carry_kernel<<<units, kCT, 0, s>>>(p, Gc, Ab, nch);
  M3_TRY(check_launch("mimo_bwd_carry_kernel"));
  mimo_bwd_full_kernel<TX, TB><<<grid, kCT, sm_full, s>>>(p, Hc, Gc, tot, nch);
  M3_TRY(check_launch("mimo_bwd_full_kernel"));
  mimo_bwd_dadt_kernel<<<units, kCT, 0, s>>>(p, tot, nch, kTcB);
  return check_launch("mimo_bwd_dadt_kernel");
}

}  // namespace

bool mimo_bwd_chunked_fits(int P, int R, int D) { return bsmem_floats(P, R, D) * sizeof(float) <= 200 * 1024; }

size_t mimo_bwd_chunked_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D) {
  const int64_t nch = (L + kTcB - 1) / kTcB, cells = Bn * H * nch;
  return (size_t)cells * sizeof(double) + sizeof(float) * (size_t)cells * (2 * D + 2);
}

int launch_mimo_bwd_chunked(const MimoParams& p, int xdt, int bcdt, void* ws, cudaStream_t s) {
  if (p.L >= (int64_t)65535 * kTcB) return fail(M3_ERR_UNSUPPORTED, "mimo scan: sequence too long for the chunk grid");
  if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return run_bwd_chunked<float, float>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16) return run_bwd_chunked<__nv_bfloat16, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32) return run_bwd_chunked<__nv_bfloat16, float>(p, ws, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16) return run_bwd_chunked<float, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return run_bwd_chunked<__half, __half>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return run_bwd_chunked<__half, float>(p, ws, s);
  return fail(M3_ERR_UNSUPPORTED, "unsupported dtype combination for x / B,C");
}

size_t mimo_fwd_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D) {
  // the larger of the three-pass layout (64-step chunks: a state and a decay each) and the
  // single-pass one at its shortest chunk (16 steps)
  const int64_t three = 4 * Bn * H * ((L + kTcF - 1) / kTcF) * (D + 1);
  const int64_t single = fused_ws_bytes(Bn * H * ((L + 15) / 16), D);
  return (size_t)std::max(three, single);
}

size_t mimo_bwd_fused_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t D) {
  return (size_t)fused_bwd_ws_bytes(Bn * H * ((L + 15) / 16), D);
}

int launch_mimo_bwd_fused(const MimoParams& p, int xdt, int bcdt, const void* fwd_ws, size_t fwd_bytes, void* ws,
                          size_t ws_bytes, cudaStream_t s) {
  if (!fwd_ws || !ws) return M3_ERR_UNSUPPORTED;
  if (p.L >= (int64_t)65535 * 16 * 1024) return M3_ERR_UNSUPPORTED;
  if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return run_bwd_fused<float, float>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16)
    return run_bwd_fused<__nv_bfloat16, __nv_bfloat16>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32)
    return run_bwd_fused<__nv_bfloat16, float>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16)
    return run_bwd_fused<float, __nv_bfloat16>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return run_bwd_fused<__half, __half>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return run_bwd_fused<__half, float>(p, fwd_ws, fwd_bytes, ws, ws_bytes, s);
  return M3_ERR_UNSUPPORTED;
}

int mimo_error_word(bool reset, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_mimo_error, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_mimo_error, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("mimo error word: ") + cudaGetErrorString(e));
  *out = v;
  return M3_OK;
}

int launch_mimo_fwd_chunked(const MimoParams& p, int xdt, int bcdt, void* ws, cudaStream_t s) {
  if (p.L >= (int64_t)65535 * kTcF) return fail(M3_ERR_UNSUPPORTED, "mimo scan: sequence too long for the chunk grid");
  if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return run_chunked<float, float>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16) return run_chunked<__nv_bfloat16, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32) return run_chunked<__nv_bfloat16, float>(p, ws, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16) return run_chunked<float, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return run_chunked<__half, __half>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return run_chunked<__half, float>(p, ws, s);
  return fail(M3_ERR_UNSUPPORTED, "unsupported dtype combination for x / B,C");
}

template <typename T>
static int grp_dispatch(const MimoParams& p, const GrpArgs& g, const MimoGrpParams& q, void* ws, cudaStream_t s) {
  const T* zx = static_cast<const T*>(q.zx);
  int rc = M3_ERR_UNSUPPORTED;
  switch (grp_chunk(p, (int)sizeof(T), q.S, q.gate != 0)) {
    case 64: rc = run_fused_grp<T, 64>(p, g, zx, q.s_zb, q.s_zl, ws, s); break;
    case 32: rc = run_fused_grp<T, 32>(p, g, zx, q.s_zb, q.s_zl, ws, s); break;
    case 16: rc = run_fused_grp<T, 16>(p, g, zx, q.s_zb, q.s_zl, ws, s); break;
    default: break;
  }
  if (rc == M3_ERR_UNSUPPORTED)
    return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: too many chunks, or a tensor map could not be made");
  return rc;
}

int launch_mimo_layer_fwd(const MimoParams& p, const MimoGrpParams& q, void* ws, cudaStream_t s) {
  const int64_t e = q.dtype == M3_FLOAT32 ? 4 : 2;
  auto a16 = [](const void* v) { return reinterpret_cast<uintptr_t>(v) % 16 == 0; };
  const int64_t di = (int64_t)p.H * p.P;
  if (!(a16(q.zx) && (2 * di * e) % 16 == 0 && q.s_zb > 0 && q.s_zl > 0 && (q.s_zb * e) % 16 == 0 &&
        (q.s_zl * e) % 16 == 0 && (p.P * e) % 16 == 0 && p.P <= 256 && (p.D * e) % 16 == 0 && p.D % 4 == 0 &&
        p.D <= 256 && p.R <= 8 && 2 * q.S <= p.D && a16(q.B_bias) && a16(q.C_bias) && a16(q.B_norm_w) &&
        a16(q.C_norm_w)))
    return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: the in_proj output or the parameters are not laid out on "
                                    "16-byte units (or d_state / headdim / rank out of range)");
  if (grp_chunk(p, (int)e, q.S, q.gate != 0) == 0)
    return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: shapes too large for shared memory");
  if (!chunk_encode_fn()) return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: tensor-map encoder unavailable");
  GrpArgs g{};
  g.angles = q.angles;
  g.B_bias = q.B_bias; g.C_bias = q.C_bias;
  g.B_norm_w = q.B_norm_w; g.C_norm_w = q.C_norm_w;
  g.eps = q.eps;
  g.S = q.S;
  g.gate = q.gate;
  if (q.dtype == M3_FLOAT32) return grp_dispatch<float>(p, g, q, ws, s);
  if (q.dtype == M3_BFLOAT16) return grp_dispatch<__nv_bfloat16>(p, g, q, ws, s);
  if (q.dtype == M3_FLOAT16) return grp_dispatch<__half>(p, g, q, ws, s);
  return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: unsupported dtype");
}

}  // namespace m3
