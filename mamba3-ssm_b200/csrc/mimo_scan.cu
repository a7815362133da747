// MIMO exponential-trapezoidal scan (the loop of mamba3_ssm/ops.py:226-240), fused with
// its rank-R projections and the D skip, on CUDA cores in fp32.
//
// Per (b, h) the state is one scalar per d:
//   xr_t  = mimo_x x_t                    (R values; mimo_x is (R, P) for this head)
//   Bx_t  = sum_r xr_t[r] B_t[r, :]       (D values)
//   h_t   = a_t h_{t-1} + beta_t Bx_t + gamma_t Bx_{t-1}
//   yr_t  = C_t h_t + D xr_t              (R values)
//   y_t   = mimo_o^T yr_t                 (P values)
// A CTA owns one (b, h) and walks the sequence in chunks of T timesteps. Everything but
// the h recurrence is data-parallel inside a chunk (projections, Bx, readouts); the
// recurrence itself is one FMA per (t, d), run by one thread per d. The reference splits
// this into einsum -> state kernel -> einsum with three HBM round trips
// (cuda_backend.py:442-463); here x is read once and y written once.
//
// The backward kernel runs two sweeps per (b, h): a forward sweep that stores the state
// and Bx at every chunk start (workspace, 2*D floats per chunk), then a reverse sweep that
// recomputes each chunk from its checkpoint and applies the adjoint
//   g_t = a_{t+1} g_{t+1} + C_t^T dyr_t,   v_t = beta_t g_t + gamma_{t+1} g_{t+1}
// with dADT from the reverse cumsum of <dyr_t, C_t h_t> - beta_t dbeta_t - gamma_t dgamma_t.
#include "m3_common.cuh"
#include "mimo_scan.cuh"

namespace m3 {
namespace {

constexpr int kThreads = 128;

template <typename T>
__device__ __forceinline__ float ldx(const void* base, const Str3& s, int b, int t, int h, int p) {
  return to_f32(reinterpret_cast<const T*>(base)[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h + p]);
}
template <typename T>
__device__ __forceinline__ float ldbc(const void* base, const Str4& s, int b, int t, int r, int h, int d) {
  return to_f32(reinterpret_cast<const T*>(base)[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)r * s.r +
                                                  (int64_t)h * s.h + d]);
}
__device__ __forceinline__ float scal(const float* base, const Str3& s, int b, int t, int h) {
  return base[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h];
}

struct Smem {
  float *x, *dy, *Bm, *Cm, *xr, *yr, *dyr, *dxr, *bx, *H, *G, *E, *a, *be, *ga, *tr, *dt, *mx, *mo, *red;
};

// Layout of the dynamic shared memory for chunk length T (rows of per-t arrays carry one
// extra row where noted: bx row 0 is the previous chunk's last Bx; G/a/be/ga/tr/dt have a
// trailing row for t0 + T).
__host__ __device__ inline size_t smem_floats(int T, int P, int R, int D, bool bwd) {
  size_t n = 0;
  n += (size_t)T * P;              // x
  n += bwd ? (size_t)T * P : 0;    // dy
  n += 2 * (size_t)T * R * D;      // B, C
  n += 2 * (size_t)T * R;          // xr, yr
  n += bwd ? 2 * (size_t)T * R : 0;  // dyr, dxr
  n += (size_t)(T + 1) * D;        // bx
  n += (size_t)T * D;              // H
  n += bwd ? (size_t)(T + 1) * D + (size_t)T * D : 0;  // G, E
  n += 5 * (size_t)(T + 1);        // a, be, ga, tr, dt
  n += 2 * (size_t)R * P;          // mx, mo
  n += 3 * (size_t)T + 32;         // red (dbeta, dgamma, q per row)
  return n;
}

__device__ inline Smem carve(float* base, int T, int P, int R, int D, bool bwd) {
  Smem s;
  float* p = base;
  s.x = p; p += T * P;
  s.dy = p; p += bwd ? T * P : 0;
  s.Bm = p; p += T * R * D;
  s.Cm = p; p += T * R * D;
  s.xr = p; p += T * R;
  s.yr = p; p += T * R;
  s.dyr = p; p += bwd ? T * R : 0;
  s.dxr = p; p += bwd ? T * R : 0;
  s.bx = p; p += (T + 1) * D;
  s.H = p; p += T * D;
  s.G = p; p += bwd ? (T + 1) * D : 0;
  s.E = p; p += bwd ? T * D : 0;
  s.a = p; p += T + 1;
  s.be = p; p += T + 1;
  s.ga = p; p += T + 1;
  s.tr = p; p += T + 1;
  s.dt = p; p += T + 1;
  s.mx = p; p += R * P;
  s.mo = p; p += R * P;
  s.red = p;
  return s;
}

// Stage x (and dy), B, C and coefficients of rows t0 .. t0+T-1; coefficients of t0+T too.
template <typename TX, typename TB>
__device__ void stage_chunk(const MimoParams& a, const Smem& s, int b, int h, int t0, int T, bool bwd) {
  const int P = a.P, R = a.R, D = a.D, L = a.L, tid = threadIdx.x;
  for (int i = tid; i < T * P; i += blockDim.x) {
    const int r = i / P, c = i - r * P, t = t0 + r;
    s.x[i] = t < L ? ldx<TX>(a.x, a.sx, b, t, h, c) : 0.f;
    if (bwd) s.dy[i] = t < L ? ldx<TX>(a.dy, a.sdy, b, t, h, c) : 0.f;
  }
  for (int i = tid; i < T * R * D; i += blockDim.x) {
    const int r = i / (R * D), rem = i - r * R * D, k = rem / D, d = rem - k * D, t = t0 + r;
    s.Bm[i] = t < L ? ldbc<TB>(a.Bm, a.sB, b, t, k, h, d) : 0.f;
    s.Cm[i] = t < L ? ldbc<TB>(a.Cm, a.sC, b, t, k, h, d) : 0.f;
  }
  for (int r = tid; r <= T; r += blockDim.x) {
    const int t = t0 + r;
    float av = 0.f, be = 0.f, ga = 0.f, tr = 0.f, dt = 0.f;
    if (t < L) {
      av = expf(scal(a.adt, a.sadt, b, t, h));
      dt = scal(a.dt, a.sdt, b, t, h);
      tr = sigmoidf_(scal(a.trap, a.strap, b, t, h));
      be = dt * (1.0f - tr) + 0.5f * dt * tr;
      ga = 0.5f * dt * tr;
    }
    s.a[r] = av; s.be[r] = be; s.ga[r] = ga; s.tr[r] = tr; s.dt[r] = dt;
  }
}

// xr = mimo_x x (rows < T), Bx rows 1..T, then the recurrence into H (thread d carries hd).
__device__ void chunk_forward(const MimoParams& a, const Smem& s, int T, float* hreg) {
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x;
  for (int i = tid; i < T * R; i += blockDim.x) {
    const int t = i / R, r = i - t * R;
    float acc = 0.f;
    for (int p = 0; p < P; ++p) acc = fmaf(s.x[t * P + p], s.mx[r * P + p], acc);
    s.xr[i] = acc;
  }
  __syncthreads();
  for (int i = tid; i < T * D; i += blockDim.x) {
    const int t = i / D, d = i - t * D;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(s.xr[t * R + r], s.Bm[(t * R + r) * D + d], acc);
    s.bx[(t + 1) * D + d] = acc;
  }
  __syncthreads();
  for (int d = tid, j = 0; d < D; d += blockDim.x, ++j) {
    float hv = hreg[j];
    for (int t = 0; t < T; ++t) {
      hv = fmaf(s.a[t], hv, fmaf(s.be[t], s.bx[(t + 1) * D + d], s.ga[t] * s.bx[t * D + d]));
      s.H[t * D + d] = hv;
    }
    hreg[j] = hv;
  }
  __syncthreads();
}

// yr = C H + D xr  (rows < T)
__device__ void chunk_readout(const MimoParams& a, const Smem& s, int T, float Dk) {
  const int R = a.R, D = a.D, tid = threadIdx.x;
  for (int i = tid; i < T * R; i += blockDim.x) {
    const int t = i / R;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(s.Cm[i * D + d], s.H[t * D + d], acc);
    s.yr[i] = fmaf(Dk, s.xr[i], acc);
  }
  __syncthreads();
}

constexpr int kMaxDPerThread = 2;  // D <= 256 with 128 threads

template <typename TX, typename TB>
__global__ void __launch_bounds__(kThreads) mimo_fwd_kernel(MimoParams a, int T) {
  extern __shared__ float4 smem4[];
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  Smem s = carve(reinterpret_cast<float*>(smem4), T, P, R, D, false);
  for (int i = tid; i < R * P; i += blockDim.x) {
    const int r = i / P, p = i - r * P;
    s.mx[i] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + p];
    s.mo[i] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + p];
  }
  float hreg[kMaxDPerThread];
  const int64_t sto = ((int64_t)b * a.H + h) * D;
  for (int d = tid, j = 0; j < kMaxDPerThread; d += blockDim.x, ++j) {
    hreg[j] = (d < D && a.h0) ? a.h0[sto + d] : 0.f;
    if (d < D) s.bx[d] = a.bx0 ? a.bx0[sto + d] : 0.f;
  }
  const float Dk = a.Dskip[h * a.sD];
  for (int t0 = 0; t0 < a.L; t0 += T) {
    const int nT = min(T, a.L - t0);
    __syncthreads();
    stage_chunk<TX, TB>(a, s, b, h, t0, nT, false);
    __syncthreads();
    chunk_forward(a, s, nT, hreg);
    chunk_readout(a, s, nT, Dk);
    for (int i = tid; i < nT * P; i += blockDim.x) {
      const int t = i / P, p = i - t * P;
      float acc = 0.f;
      for (int r = 0; r < R; ++r) acc = fmaf(s.yr[t * R + r], s.mo[r * P + p], acc);
      st(reinterpret_cast<TX*>(a.y) + (int64_t)b * a.sy.b + (int64_t)(t0 + t) * a.sy.l + (int64_t)h * a.sy.h + p, acc);
    }
    __syncthreads();
    for (int d = tid; d < D; d += blockDim.x) s.bx[d] = s.bx[nT * D + d];
  }
  for (int d = tid, j = 0; j < kMaxDPerThread; d += blockDim.x, ++j) {
    if (d < D) {
      if (a.h_last) a.h_last[sto + d] = hreg[j];
      if (a.bx_last) a.bx_last[sto + d] = s.bx[d];
    }
  }
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kThreads) mimo_bwd_kernel(MimoParams a, int T) {
  extern __shared__ float4 smem4[];
  const int P = a.P, R = a.R, D = a.D, L = a.L, tid = threadIdx.x;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  Smem s = carve(reinterpret_cast<float*>(smem4), T, P, R, D, true);
  for (int i = tid; i < R * P; i += blockDim.x) {
    const int r = i / P, p = i - r * P;
    s.mx[i] = a.mimo_x[(int64_t)h * a.smx_h + (int64_t)r * a.smx_r + p];
    s.mo[i] = a.mimo_o[(int64_t)h * a.smo_h + (int64_t)r * a.smo_r + p];
  }
  const int nchunk = (L + T - 1) / T;
  const int64_t sto = ((int64_t)b * a.H + h) * D;
  float* ck = a.work + ((int64_t)b * a.H + h) * (int64_t)nchunk * 2 * D;  // [chunk][h | bx][D]
  float hreg[kMaxDPerThread];
  for (int d = tid, j = 0; j < kMaxDPerThread; d += blockDim.x, ++j) {
    hreg[j] = (d < D && a.h0) ? a.h0[sto + d] : 0.f;
    if (d < D) s.bx[d] = a.bx0 ? a.bx0[sto + d] : 0.f;
  }
  const float Dk = a.Dskip[h * a.sD];
  // ---- sweep 1: checkpoints at chunk starts
  for (int c = 0; c < nchunk; ++c) {
    const int t0 = c * T, nT = min(T, L - t0);
    __syncthreads();
    for (int d = tid, j = 0; j < kMaxDPerThread; d += blockDim.x, ++j)
      if (d < D) {
        ck[(int64_t)c * 2 * D + d] = hreg[j];
        ck[(int64_t)c * 2 * D + D + d] = s.bx[d];
      }
    stage_chunk<TX, TB>(a, s, b, h, t0, nT, false);
    __syncthreads();
    chunk_forward(a, s, nT, hreg);
    for (int d = tid; d < D; d += blockDim.x) s.bx[d] = s.bx[nT * D + d];
  }
  // ---- sweep 2: reverse
  float greg[kMaxDPerThread] = {0.f, 0.f};
  float gnext_row[kMaxDPerThread] = {0.f, 0.f};  // g_{t0+T} for the chunk being processed
  // per-thread accumulators of dmimo_x / dmimo_o for (r,p) pairs i = tid + k*blockDim
  constexpr int kMaxRP = 16;  // R*P <= 2048
  float dmx_acc[kMaxRP], dmo_acc[kMaxRP];
#pragma unroll
  for (int k = 0; k < kMaxRP; ++k) { dmx_acc[k] = 0.f; dmo_acc[k] = 0.f; }
  float dd_acc = 0.f;
  double cum = 0.0;
  for (int c = nchunk - 1; c >= 0; --c) {
    const int t0 = c * T, nT = min(T, L - t0);
    __syncthreads();
    for (int d = tid, j = 0; j < kMaxDPerThread; d += blockDim.x, ++j)
      if (d < D) {
        hreg[j] = ck[(int64_t)c * 2 * D + d];
        s.bx[d] = ck[(int64_t)c * 2 * D + D + d];
      }
    stage_chunk<TX, TB>(a, s, b, h, t0, nT, true);
    __syncthreads();
    chunk_forward(a, s, nT, hreg);   // H, bx rows, xr
    chunk_readout(a, s, nT, Dk);     // yr (with skip)
    // dyr = mo dy
    for (int i = tid; i < nT * R; i += blockDim.x) {
      const int t = i / R, r = i - t * R;
      float acc = 0.f;
      for (int p = 0; p < P; ++p) acc = fmaf(s.dy[t * P + p], s.mo[r * P + p], acc);
      s.dyr[i] = acc;
    }
    __syncthreads();
    // E[t][d] = sum_r dyr C ; dC = dyr H
    for (int i = tid; i < nT * D; i += blockDim.x) {
      const int t = i / D, d = i - t * D;
      float acc = 0.f;
      for (int r = 0; r < R; ++r) {
        const float dyr = s.dyr[t * R + r];
        acc = fmaf(dyr, s.Cm[(t * R + r) * D + d], acc);
        st(reinterpret_cast<TB*>(a.dC) + (int64_t)b * a.sdC.b + (int64_t)(t0 + t) * a.sdC.l +
               (int64_t)r * a.sdC.r + (int64_t)h * a.sdC.h + d,
           dyr * s.H[t * D + d]);
      }
      s.E[i] = acc;
    }
    __syncthreads();
    // reverse recurrence for g; G row T holds g_{t0+T}
    for (int d = tid, j = 0; d < D; d += blockDim.x, ++j) {
      s.G[nT * D + d] = gnext_row[j];
      float gv = greg[j];
      for (int t = nT - 1; t >= 0; --t) {
        gv = fmaf(s.a[t + 1], gv, s.E[t * D + d]);
        s.G[t * D + d] = gv;
      }
      greg[j] = gv;
      gnext_row[j] = gv;
    }
    __syncthreads();
    // dB = xr v ; dxr = D dyr + B v   (v = beta G_t + gamma_{t+1} G_{t+1})
    for (int i = tid; i < nT * R * D; i += blockDim.x) {
      const int t = i / (R * D), rem = i - t * R * D, r = rem / D, d = rem - r * D;
      const float v = s.be[t] * s.G[t * D + d] + s.ga[t + 1] * s.G[(t + 1) * D + d];
      st(reinterpret_cast<TB*>(a.dB) + (int64_t)b * a.sdB.b + (int64_t)(t0 + t) * a.sdB.l +
             (int64_t)r * a.sdB.r + (int64_t)h * a.sdB.h + d,
         s.xr[t * R + r] * v);
    }
    for (int i = tid; i < nT * R; i += blockDim.x) {
      const int t = i / R, r = i - t * R;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) {
        const float v = s.be[t] * s.G[t * D + d] + s.ga[t + 1] * s.G[(t + 1) * D + d];
        acc = fmaf(v, s.Bm[(t * R + r) * D + d], acc);
      }
      s.dxr[i] = fmaf(Dk, s.dyr[i], acc);
      dd_acc = fmaf(s.dyr[i], s.xr[i], dd_acc);
    }
    // per-t scalars: dbeta, dgamma, q into red[0..3T)
    const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    for (int t = warp; t < nT; t += nw) {
      float db = 0.f, dg = 0.f, q = 0.f;
      for (int d = lane; d < D; d += 32) {
        const float g = s.G[t * D + d];
        db = fmaf(g, s.bx[(t + 1) * D + d], db);
        dg = fmaf(g, s.bx[t * D + d], dg);
        q = fmaf(s.E[t * D + d], s.H[t * D + d], q);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        db += __shfl_xor_sync(0xffffffffu, db, o);
        dg += __shfl_xor_sync(0xffffffffu, dg, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
      }
      if (lane == 0) {
        s.red[t] = db;
        s.red[T + t] = dg;
        s.red[2 * T + t] = q;
      }
    }
    __syncthreads();
    if (tid == 0) {
      for (int t = nT - 1; t >= 0; --t) {
        const float db = s.red[t], dg = s.red[T + t], q = s.red[2 * T + t];
        cum += (double)q - (double)s.be[t] * db - (double)s.ga[t] * dg;
        const float tr = s.tr[t], dt = s.dt[t];
        const int tt = t0 + t;
        a.dadt[(int64_t)b * a.sdadt.b + (int64_t)tt * a.sdadt.l + (int64_t)h * a.sdadt.h] = (float)cum;
        a.ddt[(int64_t)b * a.sddt.b + (int64_t)tt * a.sddt.l + (int64_t)h * a.sddt.h] =
            db * (1.0f - 0.5f * tr) + dg * 0.5f * tr;
        a.dtrap[(int64_t)b * a.sdtrap.b + (int64_t)tt * a.sdtrap.l + (int64_t)h * a.sdtrap.h] =
            0.5f * dt * (dg - db) * tr * (1.0f - tr);
      }
    }
    // dx = mx^T dxr ; dmimo_x += dxr x^T ; dmimo_o += yr dy^T
    for (int i = tid; i < nT * P; i += blockDim.x) {
      const int t = i / P, p = i - t * P;
      float acc = 0.f;
      for (int r = 0; r < R; ++r) acc = fmaf(s.dxr[t * R + r], s.mx[r * P + p], acc);
      st(reinterpret_cast<TX*>(a.dx) + (int64_t)b * a.sdx.b + (int64_t)(t0 + t) * a.sdx.l + (int64_t)h * a.sdx.h + p, acc);
    }
#pragma unroll
    for (int k = 0; k < kMaxRP; ++k) {
      const int i = tid + k * kThreads;
      if (i < R * P) {
        const int r = i / P, p = i - r * P;
        float ax = 0.f, ao = 0.f;
        for (int t = 0; t < nT; ++t) {
          ax = fmaf(s.dxr[t * R + r], s.x[t * P + p], ax);
          ao = fmaf(s.yr[t * R + r], s.dy[t * P + p], ao);
        }
        dmx_acc[k] += ax;
        dmo_acc[k] += ao;
      }
    }
  }
  __syncthreads();
  // initial-state gradients
  if (a.dh0 || a.dbx0) {
    const float a0 = expf(scal(a.adt, a.sadt, b, 0, h));
    const float dt0 = scal(a.dt, a.sdt, b, 0, h);
    const float tr0 = sigmoidf_(scal(a.trap, a.strap, b, 0, h));
    for (int d = tid, j = 0; d < D; d += blockDim.x, ++j) {
      if (a.dh0) a.dh0[sto + d] = a0 * greg[j];
      if (a.dbx0) a.dbx0[sto + d] = 0.5f * dt0 * tr0 * greg[j];
    }
  }
#pragma unroll
  for (int k = 0; k < kMaxRP; ++k) {
    const int i = tid + k * kThreads;
    if (i < R * P) {
      atomicAdd(a.dmx + (int64_t)h * R * P + i, dmx_acc[k]);
      atomicAdd(a.dmo + (int64_t)h * R * P + i, dmo_acc[k]);
    }
  }
  float v = dd_acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((tid & 31) == 0) atomicAdd(a.dD + h, v);
}

int choose_T(int P, int R, int D, bool bwd) {
  for (int T = 32; T >= 2; T /= 2)
    if (smem_floats(T, P, R, D, bwd) * sizeof(float) <= 200 * 1024) return T;
  return 0;
}

template <typename TX, typename TB>
int run(const MimoParams& p, bool bwd, cudaStream_t s) {
  if (p.D > kThreads * kMaxDPerThread) return fail(M3_ERR_UNSUPPORTED, "mimo scan: d_state above 256");
  if (bwd && p.R * p.P > 16 * kThreads) return fail(M3_ERR_UNSUPPORTED, "mimo scan backward: mimo_rank*headdim above 2048");
  const int T = choose_T(p.P, p.R, p.D, bwd);
  if (T == 0) return fail(M3_ERR_UNSUPPORTED, "mimo scan: shapes too large for shared memory");
  const size_t smem = smem_floats(T, p.P, p.R, p.D, bwd) * sizeof(float);
  if (!bwd) {
    auto k = mimo_fwd_kernel<TX, TB>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    }
    k<<<p.Bn * p.H, kThreads, smem, s>>>(p, T);
    return check_launch("mimo_fwd_kernel");
  }
  auto k = mimo_bwd_kernel<TX, TB>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  }
  k<<<p.Bn * p.H, kThreads, smem, s>>>(p, T);
  return check_launch("mimo_bwd_kernel");
}

}  // namespace

size_t mimo_bwd_workspace_floats(int64_t Bn, int64_t L, int64_t H, int64_t P, int64_t D, int64_t R) {
  if (mimo_bwd_chunked_fits((int)P, (int)R, (int)D))
    return (mimo_bwd_chunked_workspace_bytes(Bn, L, H, D) + sizeof(float) - 1) / sizeof(float);
  const int T = choose_T((int)P, (int)R, (int)D, true);
  if (T == 0) return 0;
  const int64_t nchunk = (L + T - 1) / T;
  return (size_t)(Bn * H * nchunk * 2 * D);
}

int launch_mimo(const MimoParams& p, int xdt, int bcdt, bool bwd, cudaStream_t s) {
  // the chunk-parallel backward where its shared-memory layout fits; the per-(b, h) sweep
  // kernel otherwise
  if (bwd && mimo_bwd_chunked_fits(p.P, p.R, p.D)) return launch_mimo_bwd_chunked(p, xdt, bcdt, p.work, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return run<float, float>(p, bwd, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16) return run<__nv_bfloat16, __nv_bfloat16>(p, bwd, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32) return run<__nv_bfloat16, float>(p, bwd, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16) return run<float, __nv_bfloat16>(p, bwd, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return run<__half, __half>(p, bwd, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return run<__half, float>(p, bwd, s);
  return fail(M3_ERR_UNSUPPORTED, "unsupported dtype combination for x / B,C");
}

}  // namespace m3
