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
__global__ void __launch_bounds__(kCT) mimo_bwd_dadt_kernel(MimoParams a, const double* tot, int nch) {
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  double off = 0.0;
  for (int c = nch - 1; c >= 0; --c) {
    const int t0 = c * kTcB, n = min(kTcB, a.L - t0);
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
// (chunk-major, so every chunk it waits for belongs to a CTA that started earlier), pulls
// the chunk's rows of B and C into shared memory with bulk copies, scans the chunk from a
// zero state, publishes that local end state S_c and the chunk's decay product A_c, and
// then finds its carry (the state entering the chunk) by looking back over the chunks
// before it: a chunk whose inclusive state I_j (the true state at its end) is published
// ends the walk; one with only (A_j, S_j) is folded in and the walk goes on,
//   carry_c = S_{c-1} + A_{c-1} (S_{c-2} + A_{c-2} ( ... + I_j)).
// Its own I_c = S_c + A_c carry_c is published as soon as the carry is known, and the
// states of the chunk are h_t = hloc_t + (a_t0 ... a_t) carry_c. B, C and x are read once.
// Every wait (bulk copies, predecessors' flags) is bounded; a wait that gives up sets the
// error word and the kernel finishes with its outputs invalid.
// ------------------------------------------------------------------------------------
constexpr int kFT = 128;                 // threads per CTA
constexpr int kLkMax = 8;                // state columns per lane in the look-back (d_state <= 256)
constexpr uint32_t kSpinLimit = 1u << 22;  // flag polls (about 64 ns apart) before giving up

__device__ int g_mimo_error;  // set when a bounded wait gives up

// Workspace of the single-pass forward: ticket counter, chunk flags (0 none, 1 local
// aggregate, 2 inclusive state), then per chunk A_c, S_c[D], I_c[D]. The counter and the
// flags are cleared before every launch.
struct FusedWs {
  unsigned* ticket;
  int* flag;
  float *A, *S, *I;
};
inline int64_t align16(int64_t v) { return (v + 15) & ~int64_t(15); }
inline int64_t fused_flag_bytes(int64_t cells) { return 16 + align16(4 * cells); }
inline int64_t fused_ws_bytes(int64_t cells, int64_t D) { return fused_flag_bytes(cells) + align16(4 * cells) + 8 * cells * D; }
inline FusedWs fused_ws(void* base, int64_t cells, int64_t D) {
  char* p = static_cast<char*>(base);
  FusedWs w;
  w.ticket = reinterpret_cast<unsigned*>(p);
  w.flag = reinterpret_cast<int*>(p + 16);
  w.A = reinterpret_cast<float*>(p + fused_flag_bytes(cells));
  w.S = reinterpret_cast<float*>(p + fused_flag_bytes(cells) + align16(4 * cells));
  w.I = w.S + cells * D;
  return w;
}

// Shared-memory layout (byte offsets, each 16-byte aligned): two mbarriers and the ticket,
// B rows t0-1 .. t0+n-1 ([row][r][d], row 0 = t0-1), C rows t0 .. t0+n-1, the chunk's
// states (fp32 [t][d]), x rows t0-1 .. t0+n-1 (fp32), their rank projections, the step
// coefficients and their running product, mimo_x, mimo_o, the readouts yr and the carry.
struct FusedSmem {
  uint32_t bs, cs, hs, xs, xr, a, be, ga, cum, mx, mo, yr, carry, total;
};
__host__ __device__ inline uint32_t a16(uint32_t v) { return (v + 15u) & ~15u; }
__host__ __device__ inline FusedSmem fused_smem(int Q, int P, int R, int D, int eb) {
  FusedSmem L;
  uint32_t o = 32;
  L.bs = o; o = a16(o + (uint32_t)((Q + 1) * R * D * eb));
  L.cs = o; o = a16(o + (uint32_t)(Q * R * D * eb));
  L.hs = o; o = a16(o + (uint32_t)(Q * D * 4));
  L.xs = o; o = a16(o + (uint32_t)((Q + 1) * P * 4));
  L.xr = o; o = a16(o + (uint32_t)((Q + 1) * R * 4));
  L.a = o; o = a16(o + (uint32_t)(Q * 4));
  L.be = o; o = a16(o + (uint32_t)(Q * 4));
  L.ga = o; o = a16(o + (uint32_t)(Q * 4));
  L.cum = o; o = a16(o + (uint32_t)(Q * 4));
  L.mx = o; o = a16(o + (uint32_t)(R * P * 4));
  L.mo = o; o = a16(o + (uint32_t)(R * P * 4));
  L.yr = o; o = a16(o + (uint32_t)(Q * R * 4));
  L.carry = o; o = a16(o + (uint32_t)(D * 4));
  L.total = o;
  return L;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float2 ld2f(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 ld2f(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 ld2f(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }

// Bounded wait for this CTA's bulk copies; on giving up, set the error word and wait once
// more (also bounded) so that no copy is still writing shared memory when the CTA ends.
__device__ __forceinline__ void wait_copies(uint64_t* bar) {
  if (sm100::mbar_wait(bar, 0, 1u << 24)) return;
  atomicExch(&g_mimo_error, 1);
  sm100::mbar_wait(bar, 0, 1u << 24);
}

template <typename TX, typename TB, int Q>
__global__ void __launch_bounds__(kFT) mimo_fused_fwd_kernel(MimoParams a, FusedWs w, int nch, int units) {
  extern __shared__ __align__(128) unsigned char fsm[];
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const FusedSmem L = fused_smem(Q, P, R, D, (int)sizeof(TB));
  uint64_t* barB = reinterpret_cast<uint64_t*>(fsm);
  uint64_t* barC = barB + 1;
  int* tk_s = reinterpret_cast<int*>(fsm + 16);
  TB* Bs = reinterpret_cast<TB*>(fsm + L.bs);
  TB* Cs = reinterpret_cast<TB*>(fsm + L.cs);
  float* hs = reinterpret_cast<float*>(fsm + L.hs);
  float* cum = reinterpret_cast<float*>(fsm + L.cum);
  float* carry = reinterpret_cast<float*>(fsm + L.carry);
  CSmem s;
  s.x = reinterpret_cast<float*>(fsm + L.xs);
  s.xr = reinterpret_cast<float*>(fsm + L.xr);
  s.a = reinterpret_cast<float*>(fsm + L.a);
  s.be = reinterpret_cast<float*>(fsm + L.be);
  s.ga = reinterpret_cast<float*>(fsm + L.ga);
  s.mx = reinterpret_cast<float*>(fsm + L.mx);
  s.mo = reinterpret_cast<float*>(fsm + L.mo);
  s.H = hs;
  s.yr = reinterpret_cast<float*>(fsm + L.yr);

  if (tid == 0) {
    *tk_s = (int)atomicAdd(w.ticket, 1u);
    sm100::mbar_init(barB, 1);
    sm100::mbar_init(barC, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const int tk = *tk_s;
  const int c = tk / units, u = tk - c * units, b = u / a.H, h = u - b * a.H;
  const int t0 = c * Q, n = min(Q, a.L - t0);
  const int hb = c > 0 ? 1 : 0;  // the row t0-1 of B, for the first step's gamma term
  const uint32_t rowb = (uint32_t)(D * sizeof(TB));
  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_expect_tx(barB, (uint32_t)((n + hb) * R) * rowb);
      sm100::mbar_expect_tx(barC, (uint32_t)(n * R) * rowb);
    }
    __syncwarp();
    const TB* gB = reinterpret_cast<const TB*>(a.Bm) + (int64_t)b * a.sB.b + (int64_t)h * a.sB.h;
    for (int i = lane; i < (n + hb) * R; i += 32) {
      const int tt = i / R, r = i - tt * R;
      sm100::bulk_load(Bs + ((size_t)(tt + 1 - hb) * R + r) * D, gB + (int64_t)(t0 - hb + tt) * a.sB.l + (int64_t)r * a.sB.r,
                       rowb, barB);
    }
    const TB* gC = reinterpret_cast<const TB*>(a.Cm) + (int64_t)b * a.sC.b + (int64_t)h * a.sC.h;
    for (int i = lane; i < n * R; i += 32) {
      const int tt = i / R, r = i - tt * R;
      sm100::bulk_load(Cs + (size_t)i * D, gC + (int64_t)(t0 + tt) * a.sC.l + (int64_t)r * a.sC.r, rowb, barC);
    }
  }
  stage<TX>(a, s, b, h, t0, n, true);
  if (tid == kFT - 1) {
    float pr = 1.f;
    for (int t = 0; t < n; ++t) cum[t] = pr *= s.a[t];
  }
  // local scan from a zero state
  wait_copies(barB);
  for (int d = tid; d < D; d += kFT) {
    float bxp = 0.f;
    if (hb) {
      for (int r = 0; r < R; ++r) bxp = fmaf(s.xr[r], to_f32(Bs[(size_t)r * D + d]), bxp);
    } else if (a.bx0) {
      bxp = a.bx0[(int64_t)u * D + d];
    }
    float hv = 0.f;
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      const float* xr = s.xr + (t + 1) * R;
      const TB* brow = Bs + (size_t)(t + 1) * R * D + d;
      float bx = 0.f;
      for (int r = 0; r < R; ++r) bx = fmaf(xr[r], to_f32(brow[(size_t)r * D]), bx);
      hv = fmaf(s.a[t], hv, fmaf(s.be[t], bx, s.ga[t] * bxp));
      hs[t * D + d] = hv;
      bxp = bx;
    }
    if (c == nch - 1 && a.bx_last) a.bx_last[(int64_t)u * D + d] = bxp;
  }
  __syncthreads();
  // publish, then the carry
  const int64_t cell = (int64_t)u * nch + c;
  const float Ac = cum[n - 1];
  if (c == 0) {
    for (int d = tid; d < D; d += kFT) {
      const float cv = a.h0 ? a.h0[(int64_t)u * D + d] : 0.f;
      carry[d] = cv;
      w.I[cell * D + d] = fmaf(Ac, cv, hs[(n - 1) * D + d]);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release(w.flag + cell, 2);
  } else {
    for (int d = tid; d < D; d += kFT) w.S[cell * D + d] = hs[(n - 1) * D + d];
    if (tid == 0) w.A[cell] = Ac;
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release(w.flag + cell, 1);
    if (warp == 0) {
      float accA = 1.f, acc[kLkMax];
#pragma unroll
      for (int k = 0; k < kLkMax; ++k) acc[k] = 0.f;
      bool ok = true;
      for (int j = c - 1;; --j) {
        const int64_t cj = (int64_t)u * nch + j;
        int f = 0;
        if (lane == 0) {
          for (uint32_t i = 0; i < kSpinLimit; ++i) {
            f = ld_acquire(w.flag + cj);
            if (f != 0) break;
            __nanosleep(64);
          }
        }
        f = __shfl_sync(0xffffffffu, f, 0);
        __syncwarp();
        if (f == 0) {
          ok = false;
          break;
        }
        if (f == 2) {
#pragma unroll
          for (int k = 0; k < kLkMax; ++k) {
            const int d = lane + 32 * k;
            if (d < D) acc[k] = fmaf(accA, __ldcg(w.I + cj * D + d), acc[k]);
          }
          break;
        }
#pragma unroll
        for (int k = 0; k < kLkMax; ++k) {
          const int d = lane + 32 * k;
          if (d < D) acc[k] = fmaf(accA, __ldcg(w.S + cj * D + d), acc[k]);
        }
        accA *= __ldcg(w.A + cj);
        if (j == 0) {  // chunk 0 always publishes its inclusive state: unreachable
          ok = false;
          break;
        }
      }
      if (!ok && lane == 0) atomicExch(&g_mimo_error, 1);
#pragma unroll
      for (int k = 0; k < kLkMax; ++k) {
        const int d = lane + 32 * k;
        if (d < D) {
          const float cv = ok ? acc[k] : 0.f;
          carry[d] = cv;
          w.I[cell * D + d] = fmaf(Ac, cv, hs[(n - 1) * D + d]);
        }
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) st_release(w.flag + cell, 2);
    }
    __syncthreads();
  }
  // the chunk's states from its carry
  for (int i = tid; i < n * D; i += kFT) {
    const int t = i / D, d = i - t * D;
    hs[i] = fmaf(cum[t], carry[d], hs[i]);
  }
  wait_copies(barC);
  __syncthreads();
  if (c == nch - 1 && a.h_last)
    for (int d = tid; d < D; d += kFT) a.h_last[(int64_t)u * D + d] = hs[(n - 1) * D + d];
  // yr_t[r] = C_t[r, :] . h_t + D xr_t[r]: a thread per (t, r), two columns per step, each
  // lane starting at its own column pair so that a warp's reads fall in distinct banks
  const float Dk = a.Dskip[h * a.sD];
  const int D2 = D >> 1;
  for (int it = tid; it < n * R; it += kFT) {
    const int t = it / R, r = it - t * R;
    const TB* crow = Cs + (size_t)it * D;
    const float* hrow = hs + (size_t)t * D;
    float acc0 = 0.f, acc1 = 0.f;
    int k = lane % D2;
    for (int e = 0; e < D2; ++e) {
      const float2 cv = ld2f(crow + 2 * k), hv = ld2f(hrow + 2 * k);
      acc0 = fmaf(cv.x, hv.x, acc0);
      acc1 = fmaf(cv.y, hv.y, acc1);
      k = k + 1 == D2 ? 0 : k + 1;
    }
    s.yr[it] = fmaf(Dk, s.xr[(t + 1) * R + r], acc0 + acc1);
  }
  __syncthreads();
  // y_t = mimo_o^T yr_t
  for (int i = tid; i < n * P; i += kFT) {
    const int t = i / P, p = i - t * P;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(s.yr[t * R + r], s.mo[r * P + p], acc);
    st(reinterpret_cast<TX*>(a.y) + (int64_t)b * a.sy.b + (int64_t)(t0 + t) * a.sy.l + (int64_t)h * a.sy.h + p, acc);
  }
}

template <typename K>
int opt_in(K k, size_t smem) {
  if (smem <= 48 * 1024) return M3_OK;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  return M3_OK;
}

// The single-pass forward applies when every row of B and C that it copies starts on a
// 16-byte boundary and is a whole number of 16-byte units, and d_state <= 256.
template <typename TB>
bool fused_applies(const MimoParams& p) {
  const int64_t eb = sizeof(TB);
  auto al = [&](const void* ptr, const Str4& st) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (st.b * eb) % 16 == 0 && (st.l * eb) % 16 == 0 &&
           (st.r * eb) % 16 == 0 && (st.h * eb) % 16 == 0;
  };
  return p.D % 2 == 0 && p.D <= 32 * kLkMax && (p.D * eb) % 16 == 0 && al(p.Bm, p.sB) && al(p.Cm, p.sC);
}

// Chunk length of the single-pass forward: the longest of 64 / 32 / 16 steps whose shared
// memory lets four CTAs share an SM, else the shortest that fits at all.
template <typename TB>
int fused_chunk(const MimoParams& p) {
  for (int q : {64, 32, 16})
    if (fused_smem(q, p.P, p.R, p.D, (int)sizeof(TB)).total <= 55u * 1024u) return q;
  return fused_smem(16, p.P, p.R, p.D, (int)sizeof(TB)).total <= 200u * 1024u ? 16 : 0;
}

template <typename TX, typename TB, int Q>
int run_fused(const MimoParams& p, void* ws, cudaStream_t s) {
  const int64_t nch = (p.L + Q - 1) / Q, units = (int64_t)p.Bn * p.H, cells = units * nch;
  if (cells >= INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "mimo scan: too many chunks for the grid");
  const FusedWs w = fused_ws(ws, cells, p.D);
  const size_t smem = fused_smem(Q, p.P, p.R, p.D, (int)sizeof(TB)).total;
  M3_TRY(opt_in(mimo_fused_fwd_kernel<TX, TB, Q>, smem));
  cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)fused_flag_bytes(cells), s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  mimo_fused_fwd_kernel<TX, TB, Q><<<(unsigned)cells, kFT, smem, s>>>(p, w, (int)nch, (int)units);
  return check_launch("mimo_fused_fwd_kernel");
}

template <typename TX, typename TB>
int run_chunked(const MimoParams& p, void* ws_raw, cudaStream_t s) {
  if (fused_applies<TB>(p)) {
    switch (fused_chunk<TB>(p)) {
      case 64: return run_fused<TX, TB, 64>(p, ws_raw, s);
      case 32: return run_fused<TX, TB, 32>(p, ws_raw, s);
      case 16: return run_fused<TX, TB, 16>(p, ws_raw, s);
      default: break;
    }
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
  mimo_bwd_dadt_kernel<<<units, kCT, 0, s>>>(p, tot, nch);
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

}  // namespace m3
