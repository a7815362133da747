// Chunk-parallel MIMO scan forward (the loop of mamba3_ssm/ops.py:226-240 with its rank-R
// projections and the D skip), fp32 on CUDA cores.
//
// The MIMO state is one scalar per d, so the recurrence h_t = a_t h_{t-1} + beta_t Bx_t +
// gamma_t Bx_{t-1} (Bx_t = sum_r xr_t[r] B_t[r, :], xr_t = mimo_x x_t) is D independent
// first-order scans. Time is cut into chunks of kTc steps and every (b, h, chunk) gets its
// own CTA:
//   1. local:  the chunk's end state from a zero start, S_c, and its decay product A_c
//   2. carry:  per (b, h, d), in chunk order, carry_c = A_{c-1} carry_{c-1} + S_{c-1}
//              (carry_0 = h0), written over S; the last one is h_last
//   3. output: each chunk again from its carry, the readouts yr_t = C_t h_t + D xr_t and
//              y_t = mimo_o^T yr_t
// Bx_{t0-1}, which the first step of a chunk needs for its gamma term, is recomputed from
// x_{t0-1} and B_{t0-1} (bx0 for the first chunk). The kernels read x and B twice and C
// once; the per-chunk work is a few hundred steps of independent FMAs instead of one
// serial walk of the whole sequence per (b, h).
#include "m3_common.cuh"
#include "mimo_scan.cuh"

namespace m3 {
namespace {

constexpr int kTc = 64;   // time steps per chunk
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

__host__ __device__ inline size_t csmem_floats(int P, int R, int D, bool out) {
  size_t n = (size_t)(kTc + 1) * P + (size_t)(kTc + 1) * R + 3 * (size_t)kTc + 2 * (size_t)R * P;
  if (out) n += (size_t)kTc * D + (size_t)kTc * R;
  return n;
}

__device__ inline CSmem ccarve(float* p, int P, int R, int D, bool out) {
  CSmem s;
  s.x = p; p += (kTc + 1) * P;
  s.xr = p; p += (kTc + 1) * R;
  s.a = p; p += kTc;
  s.be = p; p += kTc;
  s.ga = p; p += kTc;
  s.mx = p; p += R * P;
  s.mo = p; p += R * P;
  s.H = out ? p : nullptr; p += out ? kTc * D : 0;
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

template <typename TX, typename TB>
__global__ void __launch_bounds__(kCT) mimo_local_kernel(MimoParams a, float* S, float* Adec, int nch) {
  extern __shared__ float4 csm4[];
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * kTc, n = min(kTc, a.L - t0);
  const CSmem s = ccarve(reinterpret_cast<float*>(csm4), a.P, a.R, a.D, false);
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

__global__ void __launch_bounds__(kCT) mimo_carry_kernel(MimoParams a, float* S, const float* Adec, int nch) {
  const int u = blockIdx.x;
  for (int d = threadIdx.x; d < a.D; d += kCT) {
    float run = a.h0 ? a.h0[(int64_t)u * a.D + d] : 0.f;
    for (int c = 0; c < nch; ++c) {
      const int64_t i = ((int64_t)u * nch + c) * a.D + d;
      const float loc = S[i];
      S[i] = run;
      run = fmaf(Adec[(int64_t)u * nch + c], run, loc);
    }
    if (a.h_last) a.h_last[(int64_t)u * a.D + d] = run;
  }
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kCT) mimo_out_kernel(MimoParams a, const float* S, int nch) {
  extern __shared__ float4 csm4[];
  const int c = blockIdx.x, u = blockIdx.y, b = u / a.H, h = u - b * a.H;
  const int t0 = c * kTc, n = min(kTc, a.L - t0);
  const int P = a.P, R = a.R, D = a.D, tid = threadIdx.x;
  const CSmem s = ccarve(reinterpret_cast<float*>(csm4), P, R, D, true);
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
  // yr_t[r] = C_t[r, :] . h_t + D xr_t[r]: one warp per (t, r), lanes over d
  const float Dk = a.Dskip[h * a.sD];
  const int warp = tid >> 5, lane = tid & 31;
  for (int pr = warp; pr < n * R; pr += kCT / 32) {
    const int t = pr / R, r = pr - t * R;
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) acc = fmaf(ldbcc<TB>(a.Cm, a.sC, b, t0 + t, r, h, d), s.H[t * D + d], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s.yr[pr] = fmaf(Dk, s.xr[(t + 1) * R + r], acc);
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

template <typename K>
int opt_in(K k, size_t smem) {
  if (smem <= 48 * 1024) return M3_OK;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  return M3_OK;
}

template <typename TX, typename TB>
int run_chunked(const MimoParams& p, float* ws, cudaStream_t s) {
  const int nch = (p.L + kTc - 1) / kTc;
  const int units = p.Bn * p.H;
  float* S = ws;
  float* Adec = ws + (size_t)units * nch * p.D;
  const size_t sm_loc = csmem_floats(p.P, p.R, p.D, false) * sizeof(float);
  const size_t sm_out = csmem_floats(p.P, p.R, p.D, true) * sizeof(float);
  if (sm_out > 200 * 1024) return fail(M3_ERR_UNSUPPORTED, "mimo scan: shapes too large for shared memory");
  M3_TRY(opt_in(mimo_local_kernel<TX, TB>, sm_loc));
  M3_TRY(opt_in(mimo_out_kernel<TX, TB>, sm_out));
  const dim3 grid(nch, units);
  mimo_local_kernel<TX, TB><<<grid, kCT, sm_loc, s>>>(p, S, Adec, nch);
  M3_TRY(check_launch("mimo_local_kernel"));
  mimo_carry_kernel<<<units, kCT, 0, s>>>(p, S, Adec, nch);
  M3_TRY(check_launch("mimo_carry_kernel"));
  mimo_out_kernel<TX, TB><<<grid, kCT, sm_out, s>>>(p, S, nch);
  return check_launch("mimo_out_kernel");
}

}  // namespace

size_t mimo_fwd_workspace_floats(int64_t Bn, int64_t L, int64_t H, int64_t D) {
  const int64_t nch = (L + kTc - 1) / kTc;
  return (size_t)(Bn * H * nch * (D + 1));
}

int launch_mimo_fwd_chunked(const MimoParams& p, int xdt, int bcdt, float* ws, cudaStream_t s) {
  if (p.L >= (int64_t)65535 * kTc) return fail(M3_ERR_UNSUPPORTED, "mimo scan: sequence too long for the chunk grid");
  if (xdt == M3_FLOAT32 && bcdt == M3_FLOAT32) return run_chunked<float, float>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_BFLOAT16) return run_chunked<__nv_bfloat16, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_BFLOAT16 && bcdt == M3_FLOAT32) return run_chunked<__nv_bfloat16, float>(p, ws, s);
  if (xdt == M3_FLOAT32 && bcdt == M3_BFLOAT16) return run_chunked<float, __nv_bfloat16>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT16) return run_chunked<__half, __half>(p, ws, s);
  if (xdt == M3_FLOAT16 && bcdt == M3_FLOAT32) return run_chunked<__half, float>(p, ws, s);
  return fail(M3_ERR_UNSUPPORTED, "unsupported dtype combination for x / B,C");
}

}  // namespace m3
