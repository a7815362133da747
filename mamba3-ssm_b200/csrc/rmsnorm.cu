// RMSNorm of the reference (mamba3_ssm/ops.py:94-102: x.float() / sqrt(mean(x^2) + eps)
// * weight, returned in x.dtype), with the block's residual add (block.py:20-29:
// x + mixer(norm(x))) optionally fused in front: h = x + res is rounded to x.dtype exactly
// as the eager add would, written out, and normalised.
// Where every operand is 16-byte aligned (base, row stride, d) the row moves in 16-byte
// vectors and stays in registers between the two passes: up to kCtaRowsMax rows (a decode
// batch) one CTA per row, one vector per thread, the sum of squares reduced across the CTA,
// so a few hundred rows still spread over every SM; beyond that one warp per row.
// Otherwise one warp per row, element-wise.
#include "m3_common.cuh"
#include "rmsnorm.cuh"

namespace m3 {
namespace {

constexpr int kRowsPerCta = 8;

template <typename T>
struct alignas(16) Vec {
  static constexpr int N = 16 / sizeof(T);
  T e[N];
};

constexpr int kVecPerThread = 4;
constexpr int kMaxRowThreads = 512;
// up to this many rows (a decode batch) one CTA per row; beyond, one warp per row
constexpr int64_t kCtaRowsMax = 2048;

// N weights from element i0 (16-byte aligned): one vector when the weight has x's width,
// else as float4s
template <typename TX, typename TW>
__device__ __forceinline__ void load_w(const TW* w, int64_t i0, float (&out)[16 / sizeof(TX)]) {
  constexpr int N = 16 / sizeof(TX);
  if constexpr (sizeof(TW) == sizeof(TX)) {
    const Vec<TW> v = *reinterpret_cast<const Vec<TW>*>(w + i0);
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = to_f32(v.e[k]);
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = to_f32(w[i0 + k]);
  }
}

template <typename TX, typename TW>
__global__ void __launch_bounds__(kMaxRowThreads) rmsnorm_vec_kernel(NormParams p) {
  using V = Vec<TX>;
  constexpr int N = V::N;
  __shared__ float red[32];
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = blockIdx.x;
  const int nv = (int)(p.d / N);
  const V* x = reinterpret_cast<const V*>(reinterpret_cast<const TX*>(p.x) + r * p.sx);
  const V* res = p.res ? reinterpret_cast<const V*>(reinterpret_cast<const TX*>(p.res) + r * p.sres) : nullptr;
  V* hout = p.hout ? reinterpret_cast<V*>(reinterpret_cast<TX*>(p.hout) + r * p.shout) : nullptr;
  V* out = reinterpret_cast<V*>(reinterpret_cast<TX*>(p.out) + r * p.sout);
  const TW* w = reinterpret_cast<const TW*>(p.w);
  V hv[kVecPerThread];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int i = tid + nt * j;
    if (i < nv) {
      hv[j] = x[i];
      if (res) {
        const V rv = res[i];
#pragma unroll
        for (int k = 0; k < N; ++k) hv[j].e[k] = from_f32<TX>(to_f32(hv[j].e[k]) + to_f32(rv.e[k]));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int i = tid + nt * j;
    if (i < nv) {
      if (hout) hout[i] = hv[j];
#pragma unroll
      for (int k = 0; k < N; ++k) ss = fmaf(to_f32(hv[j].e[k]), to_f32(hv[j].e[k]), ss);
    }
  }
  for (int i = tid + nt * kVecPerThread; i < nv; i += nt) {  // rows longer than the register cache
    V v = x[i];
    if (res) {
      const V rv = res[i];
#pragma unroll
      for (int k = 0; k < N; ++k) v.e[k] = from_f32<TX>(to_f32(v.e[k]) + to_f32(rv.e[k]));
      if (hout) hout[i] = v;
    }
#pragma unroll
    for (int k = 0; k < N; ++k) ss = fmaf(to_f32(v.e[k]), to_f32(v.e[k]), ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (nt >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / (float)p.d + p.eps);
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int i = tid + nt * j;
    if (i < nv) {
      float wk[N];
      load_w<TX, TW>(w, (int64_t)i * N, wk);
      V o;
#pragma unroll
      for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(hv[j].e[k]) / rms * wk[k]);
      out[i] = o;
    }
  }
  for (int i = tid + nt * kVecPerThread; i < nv; i += nt) {
    V v;
    if (hout) v = hout[i];  // written above by this thread (hout may alias x)
    else {
      v = x[i];
      if (res) {
        const V rv = res[i];
#pragma unroll
        for (int k = 0; k < N; ++k) v.e[k] = from_f32<TX>(to_f32(v.e[k]) + to_f32(rv.e[k]));
      }
    }
    float wk[N];
    load_w<TX, TW>(w, (int64_t)i * N, wk);
    V o;
#pragma unroll
    for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(v.e[k]) / rms * wk[k]);
    out[i] = o;
  }
}

// One warp per row (many rows: a CTA per row would leave too few rows per SM in flight
// for the register budget); the row cached in registers up to 32 * kWarpVec vectors.
constexpr int kWarpVec = 8;

template <typename TX, typename TW>
__global__ void __launch_bounds__(32 * kRowsPerCta) rmsnorm_vec_warp_kernel(NormParams p) {
  using V = Vec<TX>;
  constexpr int N = V::N;
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (r >= p.rows) return;
  const int nv = (int)(p.d / N);
  const V* x = reinterpret_cast<const V*>(reinterpret_cast<const TX*>(p.x) + r * p.sx);
  const V* res = p.res ? reinterpret_cast<const V*>(reinterpret_cast<const TX*>(p.res) + r * p.sres) : nullptr;
  V* hout = p.hout ? reinterpret_cast<V*>(reinterpret_cast<TX*>(p.hout) + r * p.shout) : nullptr;
  V* out = reinterpret_cast<V*>(reinterpret_cast<TX*>(p.out) + r * p.sout);
  const TW* w = reinterpret_cast<const TW*>(p.w);
  V hv[kWarpVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kWarpVec; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      hv[j] = x[i];
      if (res) {
        const V rv = res[i];
#pragma unroll
        for (int k = 0; k < N; ++k) hv[j].e[k] = from_f32<TX>(to_f32(hv[j].e[k]) + to_f32(rv.e[k]));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kWarpVec; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      if (hout) hout[i] = hv[j];
#pragma unroll
      for (int k = 0; k < N; ++k) ss = fmaf(to_f32(hv[j].e[k]), to_f32(hv[j].e[k]), ss);
    }
  }
  for (int i = lane + 32 * kWarpVec; i < nv; i += 32) {  // rows longer than the register cache
    V v = x[i];
    if (res) {
      const V rv = res[i];
#pragma unroll
      for (int k = 0; k < N; ++k) v.e[k] = from_f32<TX>(to_f32(v.e[k]) + to_f32(rv.e[k]));
      if (hout) hout[i] = v;
    }
#pragma unroll
    for (int k = 0; k < N; ++k) ss = fmaf(to_f32(v.e[k]), to_f32(v.e[k]), ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = sqrtf(ss / (float)p.d + p.eps);
#pragma unroll
  for (int j = 0; j < kWarpVec; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      float wk[N];
      load_w<TX, TW>(w, (int64_t)i * N, wk);
      V o;
#pragma unroll
      for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(hv[j].e[k]) / rms * wk[k]);
      out[i] = o;
    }
  }
  for (int i = lane + 32 * kWarpVec; i < nv; i += 32) {
    V v;
    if (hout) v = hout[i];  // written above by this lane (hout may alias x)
    else {
      v = x[i];
      if (res) {
        const V rv = res[i];
#pragma unroll
        for (int k = 0; k < N; ++k) v.e[k] = from_f32<TX>(to_f32(v.e[k]) + to_f32(rv.e[k]));
      }
    }
    float wk[N];
    load_w<TX, TW>(w, (int64_t)i * N, wk);
    V o;
#pragma unroll
    for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(v.e[k]) / rms * wk[k]);
    out[i] = o;
  }
}

template <typename TX, typename TW>
__global__ void __launch_bounds__(32 * kRowsPerCta) rmsnorm_kernel(NormParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (r >= p.rows) return;
  const TX* x = reinterpret_cast<const TX*>(p.x) + r * p.sx;
  const TX* res = p.res ? reinterpret_cast<const TX*>(p.res) + r * p.sres : nullptr;
  TX* hout = p.hout ? reinterpret_cast<TX*>(p.hout) + r * p.shout : nullptr;
  const TW* w = reinterpret_cast<const TW*>(p.w);
  TX* out = reinterpret_cast<TX*>(p.out) + r * p.sout;
  float ss = 0.f;
  for (int64_t i = lane; i < p.d; i += 32) {
    float v = to_f32(x[i]);
    if (res) {
      const TX h = from_f32<TX>(v + to_f32(res[i]));  // the eager add, rounded to x.dtype
      if (hout) hout[i] = h;
      v = to_f32(h);
    }
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = sqrtf(ss / (float)p.d + p.eps);
  for (int64_t i = lane; i < p.d; i += 32) {
    // h as written in the first pass (hout may alias x); out may alias x or res
    float v;
    if (hout) v = to_f32(hout[i]);
    else if (res) v = to_f32(from_f32<TX>(to_f32(x[i]) + to_f32(res[i])));
    else v = to_f32(x[i]);
    out[i] = from_f32<TX>(v / rms * to_f32(w[i]));
  }
}

bool al16(const void* ptr, int64_t stride_elems, int esize) {
  return ptr == nullptr || ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (stride_elems * esize) % 16 == 0);
}

template <typename TX, typename TW>
void launch_t(const NormParams& p, unsigned grid, cudaStream_t s) {
  const int es = (int)sizeof(TX);
  const bool vec = (p.d * es) % 16 == 0 && al16(p.x, p.sx, es) && al16(p.res, p.sres, es) &&
                   al16(p.out, p.sout, es) && al16(p.hout, p.shout, es) && al16(p.w, 0, es) &&
                   p.rows <= INT32_MAX;
  if (vec && p.rows > kCtaRowsMax) {
    rmsnorm_vec_warp_kernel<TX, TW><<<grid, 32 * kRowsPerCta, 0, s>>>(p);
  } else if (vec) {
    // one thread per 16-byte vector, whole warps, at most kMaxRowThreads
    const int64_t nv = p.d / (16 / es);
    int nt = (int)((nv + 31) / 32 * 32);
    if (nt > kMaxRowThreads) nt = kMaxRowThreads;
    if (nt < 32) nt = 32;
    rmsnorm_vec_kernel<TX, TW><<<(unsigned)p.rows, nt, 0, s>>>(p);
  } else {
    rmsnorm_kernel<TX, TW><<<grid, 32 * kRowsPerCta, 0, s>>>(p);
  }
}

}  // namespace

int launch_rmsnorm(const NormParams& p, int xdt, int wdt, cudaStream_t s) {
  if (p.rows == 0 || p.d == 0) return M3_OK;
  const unsigned grid = (unsigned)((p.rows + kRowsPerCta - 1) / kRowsPerCta);
  if (xdt == M3_FLOAT32 && wdt == M3_FLOAT32) launch_t<float, float>(p, grid, s);
  else if (xdt == M3_BFLOAT16 && wdt == M3_BFLOAT16) launch_t<__nv_bfloat16, __nv_bfloat16>(p, grid, s);
  else if (xdt == M3_BFLOAT16 && wdt == M3_FLOAT32) launch_t<__nv_bfloat16, float>(p, grid, s);
  else if (xdt == M3_FLOAT16 && wdt == M3_FLOAT16) launch_t<__half, __half>(p, grid, s);
  else if (xdt == M3_FLOAT16 && wdt == M3_FLOAT32) launch_t<__half, float>(p, grid, s);
  else if (xdt == M3_FLOAT32 && wdt == M3_BFLOAT16) launch_t<float, __nv_bfloat16>(p, grid, s);
  else if (xdt == M3_FLOAT32 && wdt == M3_FLOAT16) launch_t<float, __half>(p, grid, s);
  else return fail(M3_ERR_UNSUPPORTED, "rmsnorm: unsupported dtype pair");
  return check_launch("rmsnorm_kernel");
}

}  // namespace m3
