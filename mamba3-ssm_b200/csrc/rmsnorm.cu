// RMSNorm of the reference (mamba3_ssm/ops.py:94-102: x.float() / sqrt(mean(x^2) + eps)
// * weight, returned in x.dtype), with the block's residual add (block.py:20-29:
// x + mixer(norm(x))) optionally fused in front: h = x + res is rounded to x.dtype exactly
// as the eager add would, written out, and normalised.
// One warp per row. Where every operand is 16-byte aligned (base, row stride, d) the row
// moves in 16-byte vectors, all of a lane's loads issued together and the row kept in
// registers between the two passes (up to 32 * kMaxVec vectors); otherwise element-wise.
#include "m3_common.cuh"
#include "rmsnorm.cuh"

namespace m3 {
namespace {

constexpr int kRowsPerCta = 8;
constexpr int kMaxVec = 8;

template <typename T>
struct alignas(16) Vec {
  static constexpr int N = 16 / sizeof(T);
  T e[N];
};

template <typename TX, typename TW>
__global__ void __launch_bounds__(32 * kRowsPerCta) rmsnorm_vec_kernel(NormParams p) {
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
  V hv[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
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
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      if (hout) hout[i] = hv[j];
#pragma unroll
      for (int k = 0; k < N; ++k) ss = fmaf(to_f32(hv[j].e[k]), to_f32(hv[j].e[k]), ss);
    }
  }
  for (int i = lane + 32 * kMaxVec; i < nv; i += 32) {  // rows longer than the register cache
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
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      V o;
#pragma unroll
      for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(hv[j].e[k]) / rms * to_f32(w[i * N + k]));
      out[i] = o;
    }
  }
  for (int i = lane + 32 * kMaxVec; i < nv; i += 32) {
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
    V o;
#pragma unroll
    for (int k = 0; k < N; ++k) o.e[k] = from_f32<TX>(to_f32(v.e[k]) / rms * to_f32(w[i * N + k]));
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
                   al16(p.out, p.sout, es) && al16(p.hout, p.shout, es);
  if (vec) rmsnorm_vec_kernel<TX, TW><<<grid, 32 * kRowsPerCta, 0, s>>>(p);
  else rmsnorm_kernel<TX, TW><<<grid, 32 * kRowsPerCta, 0, s>>>(p);
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
