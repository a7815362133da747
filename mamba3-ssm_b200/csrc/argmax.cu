// Row-wise argmax of the decode step's logits (the greedy token choice of
// MambaLMHeadModel decoding: logits.argmax(-1)), written as int64 token ids. Same result as
// torch.argmax: the first index of the maximum, NaN counting as the maximum (its first
// occurrence). One CTA per row; 16-byte vector loads where the row allows.
#include "m3_common.cuh"
#include "argmax.cuh"

namespace m3 {
namespace {

constexpr int kThreads = 512;

// (v, i) beats (bv, bi): larger value, NaN above every number, ties to the lower index
__device__ __forceinline__ bool beats(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) argmax_rows_kernel(const T* __restrict__ x, int64_t n, int64_t sx,
                                                             int64_t* __restrict__ out, bool vec) {
  __shared__ float sv[kThreads / 32];
  __shared__ int64_t si[kThreads / 32];
  const int64_t r = blockIdx.x;
  const T* row = x + r * sx;
  float best = -INFINITY;
  int64_t bi = n;  // beyond every index: any element beats it
  if (vec) {
    // four independent running maxima per thread, so four vector loads are in flight
    constexpr int N = 16 / sizeof(T), kCh = 4;
    const int64_t nv = n / N;
    float cb[kCh];
    int64_t ci[kCh];
#pragma unroll
    for (int c = 0; c < kCh; ++c) { cb[c] = -INFINITY; ci[c] = n; }
    for (int64_t j0 = threadIdx.x; j0 < nv; j0 += (int64_t)kThreads * kCh) {
      uint4 u[kCh];
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int64_t j = j0 + (int64_t)c * kThreads;
        u[c] = j < nv ? reinterpret_cast<const uint4*>(row)[j] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int64_t j = j0 + (int64_t)c * kThreads;
        if (j < nv) {
          const T* e = reinterpret_cast<const T*>(&u[c]);
#pragma unroll
          for (int k = 0; k < N; ++k) {
            const float v = to_f32(e[k]);
            if (beats(v, j * N + k, cb[c], ci[c])) { cb[c] = v; ci[c] = j * N + k; }
          }
        }
      }
    }
#pragma unroll
    for (int c = 0; c < kCh; ++c)
      if (beats(cb[c], ci[c], best, bi)) { best = cb[c]; bi = ci[c]; }
  } else {
    for (int64_t j = threadIdx.x; j < n; j += kThreads) {
      const float v = to_f32(row[j]);
      if (beats(v, j, best, bi)) { best = v; bi = j; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (beats(ov, oi, best, bi)) { best = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < kThreads / 32 ? sv[lane] : -INFINITY;
    bi = lane < kThreads / 32 ? si[lane] : n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (beats(ov, oi, best, bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) out[r] = bi < n ? bi : 0;
  }
}

}  // namespace

int launch_argmax_rows(const void* x, int dtype, int64_t rows, int64_t n, int64_t sx, int64_t* out,
                       cudaStream_t s) {
  if (rows == 0) return M3_OK;
  if (rows > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "argmax: too many rows");
  const int es = dtype == M3_FLOAT32 ? 4 : 2;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (n * es) % 16 == 0 && (sx * es) % 16 == 0;
  const unsigned grid = (unsigned)rows;
  if (dtype == M3_FLOAT32)
    argmax_rows_kernel<float><<<grid, kThreads, 0, s>>>(static_cast<const float*>(x), n, sx, out, vec);
  else if (dtype == M3_BFLOAT16)
    argmax_rows_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, sx, out, vec);
  else if (dtype == M3_FLOAT16)
    argmax_rows_kernel<__half><<<grid, kThreads, 0, s>>>(static_cast<const __half*>(x), n, sx, out, vec);
  else
    return fail(M3_ERR_UNSUPPORTED, "argmax: unsupported dtype");
  return check_launch("argmax_rows_kernel");
}

}  // namespace m3
