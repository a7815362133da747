// Shared device/host helpers of libmamba3_b200: element loads/stores for the three I/O
// dtypes, the thread-local error string, and argument checks for m3_tensor views.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "mamba3_b200.h"

namespace m3 {

// CUDA devices one process may drive (per-device launch settings are tracked up to this)
constexpr int kMaxDevices = 64;

// ------------------------------------------------------------------------------------
// element conversion
// ------------------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

template <typename T> __device__ __forceinline__ float ld(const T* p) { return to_f32(*p); }
template <typename T> __device__ __forceinline__ void st(T* p, float v) { *p = from_f32<T>(v); }

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }
// torch.nn.functional.softplus, beta = 1, threshold = 20
__device__ __forceinline__ float softplusf_(float v) { return v > 20.0f ? v : log1pf(expf(v)); }

// Logistic function from the hardware exp / divide approximations (relative error a few
// 1e-7), for gates and the trapezoid weight of the inference paths.
__device__ __forceinline__ float fast_sigmoid(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }

// sin and cos of an angle of any size: Cody-Waite reduction by 2 pi with a two-part
// constant (k = rint(x / 2pi), r = (x - k C1) - k C2, C1 = 2 pi rounded to fp32,
// C2 = 2 pi - C1), then the hardware approximations on |r| <= pi (absolute error ~1e-6).
__device__ __forceinline__ void sincos_reduced(float x, float* sn, float* cs) {
  const float k = rintf(x * 0.159154943091895336f);
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.74845553146951715e-07f, r);
  __sincosf(r, sn, cs);
}

template <typename T> struct DT_;
template <> struct DT_<float> { static constexpr int id = M3_FLOAT32; };
template <> struct DT_<__nv_bfloat16> { static constexpr int id = M3_BFLOAT16; };
template <> struct DT_<__half> { static constexpr int id = M3_FLOAT16; };

// ------------------------------------------------------------------------------------
// host-side error handling
// ------------------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);
// The current device's ordinal (M3_ERR_UNSUPPORTED beyond kMaxDevices).
int current_device(int* dev);
// SM count of the current device, cached per device; safe from several host threads.
int device_sm_count(int* sms);
// Sets a kernel's dynamic shared-memory opt-in once per device (done[] has kMaxDevices
// entries, one per device context); safe from several host threads.
int ensure_dynamic_smem(const void* kernel, size_t bytes, std::atomic<bool>* done);
// Per kernel (one static LaunchCache each) and device: the dynamic shared-memory opt-in
// (raised to the largest size asked so far), the preferred carveout, and the number of CTAs
// of `threads` threads that fit on the whole device at `smem` bytes, recomputed only when
// the size changes. Safe from several host threads.
struct LaunchCache {
  std::atomic<long long> word[kMaxDevices];      // (smem << 32) | resident CTAs, 0 = not yet
  std::atomic<long long> smem_max[kMaxDevices];  // the opt-in set so far
};
int kernel_residency(const void* kernel, int threads, size_t smem, LaunchCache* c, int* resident);

inline size_t dtype_size(int dt) { return dt == M3_FLOAT32 ? 4 : 2; }

// Strided view passed by value to kernels (inner dimension contiguous).
struct View4 {
  const void* p;
  int64_t s0, s1, s2;  // strides of dims 0..2 in elements (dim 3 is contiguous)
};

}  // namespace m3

#define M3_TRY(expr)                  \
  do {                                \
    int _rc = (expr);                 \
    if (_rc != M3_OK) return _rc;     \
  } while (0)
