// extern "C" entry points of libmamba3_b200: argument validation, dispatch to the
// kernels, and the thread-local error string. Nothing here allocates device memory.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "argmax.cuh"
#include "decode_step.cuh"
#include "m3_common.cuh"
#include "mimo_scan.cuh"
#include "prologue.cuh"
#include "rmsnorm.cuh"
#include "siso_chunk.cuh"
#include "siso_scan.cuh"

namespace m3 {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return M3_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(M3_ERR_UNSUPPORTED, "device ordinal beyond the supported range");
  return M3_OK;
}

int device_sm_count(int* sms) {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  M3_TRY(current_device(&dev));
  int n = cache[dev].load(std::memory_order_acquire);
  if (n <= 0) {
    cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || n <= 0)
      return fail(M3_ERR_CUDA, std::string("multiprocessor count: ") + cudaGetErrorString(e));
    cache[dev].store(n, std::memory_order_release);  // concurrent first callers store the same value
  }
  *sms = n;
  return M3_OK;
}

int ensure_dynamic_smem(const void* kernel, size_t bytes, std::atomic<bool>* done) {
  int dev = 0;
  M3_TRY(current_device(&dev));
  if (done[dev].load(std::memory_order_acquire)) return M3_OK;
  // idempotent: two threads that both get here set the same attribute twice
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  done[dev].store(true, std::memory_order_release);
  return M3_OK;
}

int kernel_residency(const void* kernel, int threads, size_t smem, LaunchCache* c, int* resident) {
  int dev = 0;
  M3_TRY(current_device(&dev));
  const long long want = (long long)smem;
  const long long w = c->word[dev].load(std::memory_order_acquire);
  if (w > 0 && (w >> 32) == want) {
    *resident = (int)(w & 0xffffffffLL);
    return M3_OK;
  }
  // the opt-in only ever grows, so a launch of a larger size on another host thread never
  // finds it lowered under it
  long long cur = c->smem_max[dev].load(std::memory_order_acquire);
  while (want > cur) {
    if (c->smem_max[dev].compare_exchange_weak(cur, want)) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
      if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      break;
    }
  }
  // all of the unified L1 / shared array as shared memory: the CTAs that fit are then set by
  // registers and shared memory, not by the carveout (a hint; its failure is not an error)
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    cudaGetLastError();
  int per_sm = 0, sms = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(e));
  M3_TRY(device_sm_count(&sms));
  const int n = std::max(1, per_sm * sms);
  c->word[dev].store((want << 32) | (long long)n, std::memory_order_release);
  *resident = n;
  return M3_OK;
}

// Fixed scratch of the allocation-free SISO backward (m3_siso_scan_bwd_noalloc): room for
// the per-position workspace of up to M3_NOALLOC_MAX_POSITIONS (batch * heads * seqlen)
// positions, 4 bytes each (8 MiB). Lives in every GPU that loads the library, for the
// lifetime of the process, and is shared by all calls on that GPU.
static __device__ __align__(256) float g_noalloc_scratch[M3_NOALLOC_MAX_POSITIONS];

namespace {

constexpr unsigned kAnyFloat = (1u << M3_FLOAT32) | (1u << M3_BFLOAT16) | (1u << M3_FLOAT16);
constexpr unsigned kF32 = 1u << M3_FLOAT32;

std::string shape_str(const m3_tensor* t) {
  std::string s = "(";
  for (int i = 0; i < t->ndim; ++i) s += std::to_string(t->shape[i]) + (i + 1 < t->ndim ? "," : "");
  return s + ")";
}

bool present(const m3_tensor* t) { return t != nullptr && t->data != nullptr; }

int check_device_ptr(const void* p, const char* name) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": not a CUDA pointer (" + cudaGetErrorString(e) + ")");
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": host memory is not accepted (no CPU path)");
  return M3_OK;
}

// shape must match `shape` (entries < 0 are free); dtype in `mask`; innermost stride 1
// unless the dim has extent 1; `contig` requires the full row-major layout.
int check(const m3_tensor* t, const char* name, int ndim, const int64_t* shape, unsigned mask,
          bool contig, bool optional, bool devcheck) {
  if (!present(t)) {
    if (optional) return M3_OK;
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": missing");
  }
  if (t->ndim != ndim)
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": expected " + std::to_string(ndim) +
                                             " dims, got " + std::to_string(t->ndim));
  for (int i = 0; i < ndim; ++i)
    if (shape[i] >= 0 && t->shape[i] != shape[i]) {
      std::string want = "(";
      for (int j = 0; j < ndim; ++j) want += (shape[j] >= 0 ? std::to_string(shape[j]) : std::string("*")) + (j + 1 < ndim ? "," : "");
      return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": shape " + shape_str(t) + " != " + want + ")");
    }
  if (t->dtype < 0 || t->dtype > 2 || !(mask & (1u << t->dtype)))
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": unsupported dtype " + std::to_string(t->dtype));
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= t->shape[i];
  if (n == 0) return M3_OK;  // empty views carry arbitrary strides and are never dereferenced
  if (ndim > 0 && t->shape[ndim - 1] > 1 && t->stride[ndim - 1] != 1)
    return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": innermost dimension must be contiguous");
  if (contig) {
    int64_t st = 1;
    for (int i = ndim - 1; i >= 0; --i) {
      if (t->shape[i] > 1 && t->stride[i] != st)
        return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": must be contiguous");
      st *= t->shape[i];
    }
  }
  for (int i = 0; i < ndim; ++i)
    if (t->stride[i] < 0) return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": negative stride");
  if (devcheck) return check_device_ptr(t->data, name);
  return M3_OK;
}

// strides of dims (0,1,2) of a 4-d view
Str3 s3(const m3_tensor* t) { return Str3{t->stride[0], t->stride[1], t->stride[2]}; }
Str3 s3_scal(const m3_tensor* t) { return Str3{t->stride[0], t->stride[1], t->stride[2]}; }
Str4 s4(const m3_tensor* t) { return Str4{t->stride[0], t->stride[1], t->stride[2], t->stride[3]}; }

template <typename T>
T* fptr(const m3_tensor* t) { return present(t) ? reinterpret_cast<T*>(t->data) : nullptr; }

int memset_async(void* p, size_t bytes, cudaStream_t s, const char* what) {
  if (!p || bytes == 0) return M3_OK;
  cudaError_t e = cudaMemsetAsync(p, 0, bytes, s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return M3_OK;
}

int copy_or_zero(void* dst, const void* src, size_t bytes, cudaStream_t s, const char* what) {
  if (!dst || bytes == 0) return M3_OK;
  cudaError_t e = src ? cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s) : cudaMemsetAsync(dst, 0, bytes, s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return M3_OK;
}

// Shared checks of the scan operands. bc_ndim 4 (SISO) or 5 (MIMO).
int check_scan_inputs(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                      const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, int bc_ndim,
                      int64_t* Bn, int64_t* L, int64_t* H, int64_t* P, int64_t* Ds, int64_t* R) {
  if (!present(x)) return fail(M3_ERR_INVALID_ARGUMENT, "x: missing");
  if (x->ndim != 4) return fail(M3_ERR_INVALID_ARGUMENT, "x: expected (B, L, H, P)");
  *Bn = x->shape[0]; *L = x->shape[1]; *H = x->shape[2]; *P = x->shape[3];
  if (!present(B) || B->ndim != bc_ndim) return fail(M3_ERR_INVALID_ARGUMENT, bc_ndim == 4 ? "B: expected (B, L, H, D)" : "B: expected (B, L, R, H, D)");
  *Ds = B->shape[bc_ndim - 1];
  *R = bc_ndim == 5 ? B->shape[2] : 1;
  const bool empty = (*Bn) * (*L) * (*H) * (*P) == 0;
  const int64_t xs[4] = {*Bn, *L, *H, *P};
  M3_TRY(check(x, "x", 4, xs, kAnyFloat, false, false, !empty));
  if (bc_ndim == 4) {
    const int64_t bs[4] = {*Bn, *L, *H, *Ds};
    M3_TRY(check(B, "B", 4, bs, kAnyFloat, false, false, !empty));
    M3_TRY(check(C, "C", 4, bs, 1u << B->dtype, false, false, !empty));
  } else {
    const int64_t bs[5] = {*Bn, *L, *R, *H, *Ds};
    M3_TRY(check(B, "B", 5, bs, kAnyFloat, false, false, !empty));
    M3_TRY(check(C, "C", 5, bs, 1u << B->dtype, false, false, !empty));
  }
  const int64_t ss[3] = {*Bn, *L, *H};
  M3_TRY(check(ADT, "ADT", 3, ss, kF32, false, false, false));
  M3_TRY(check(DT, "DT", 3, ss, kF32, false, false, false));
  M3_TRY(check(trap, "trap", 3, ss, kF32, false, false, false));
  const int64_t hs[1] = {*H};
  if (!present(D) || D->ndim != 1 || D->shape[0] != *H || D->dtype != M3_FLOAT32)
    return fail(M3_ERR_INVALID_ARGUMENT, "D: expected (H) float32");
  (void)hs;
  if (*Ds <= 0 && !empty) return fail(M3_ERR_INVALID_ARGUMENT, "B: d_state must be positive");
  return M3_OK;
}

}  // namespace
}  // namespace m3

using namespace m3;

extern "C" {

int m3_abi_version(void) { return M3_ABI_VERSION; }

const char* m3_last_error_string(void) { return g_last_error.c_str(); }

int m3_siso_scan_fwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                     const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                     const m3_tensor* bx0, m3_tensor* y, m3_tensor* h_last, m3_tensor* bx_last, void* stream) {
  int64_t Bn, L, H, P, Ds, R;
  M3_TRY(check_scan_inputs(x, B, C, ADT, DT, trap, D, 4, &Bn, &L, &H, &P, &Ds, &R));
  const int64_t xs[4] = {Bn, L, H, P}, st[4] = {Bn, H, P, Ds};
  const bool empty = Bn * L * H * P == 0;
  M3_TRY(check(y, "y", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(h0, "h0", 4, st, kF32, true, true, false));
  M3_TRY(check(bx0, "bx0", 4, st, kF32, true, true, false));
  M3_TRY(check(h_last, "h_last", 4, st, kF32, true, true, false));
  M3_TRY(check(bx_last, "bx_last", 4, st, kF32, true, true, false));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (Bn * H * P * Ds == 0) return M3_OK;
  if (L == 0) {
    const size_t bytes = sizeof(float) * Bn * H * P * Ds;
    M3_TRY(copy_or_zero(fptr<void>(h_last), fptr<void>(h0), bytes, s, "h_last"));
    return copy_or_zero(fptr<void>(bx_last), fptr<void>(bx0), bytes, s, "bx_last");
  }
  if (Bn > INT32_MAX || L > INT32_MAX || H > INT32_MAX || P > 65535)
    return fail(M3_ERR_UNSUPPORTED, "siso scan: dimension too large");
  SisoParams p{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds;
  p.x = x->data; p.sx = s3(x);
  p.Bm = B->data; p.sB = s3(B);
  p.Cm = C->data; p.sC = s3(C);
  p.adt = fptr<const float>(ADT); p.sadt = s3_scal(ADT);
  p.dt = fptr<const float>(DT); p.sdt = s3_scal(DT);
  p.trap = fptr<const float>(trap); p.strap = s3_scal(trap);
  p.Dskip = fptr<const float>(D); p.sD = D->stride[0];
  p.h0 = fptr<const float>(h0); p.bx0 = fptr<const float>(bx0);
  p.y = y->data; p.sy = s3(y);
  p.h_last = fptr<float>(h_last); p.bx_last = fptr<float>(bx_last);
  if (siso_chunk_supported(p, x->dtype, B->dtype)) return launch_siso_fwd_chunked(p, x->dtype, B->dtype, s);
  return launch_siso_fwd_recurrent(p, x->dtype, B->dtype, s);
}

// Bytes of the workspace the chunked tensor-core backward needs: the forward's chunk states
// (recomputed inside m3_siso_scan_bwd) followed by three per-position scratch arrays.
static size_t chunked_bwd_ws_bytes(int64_t Bn, int64_t L, int64_t H) {
  const size_t ks = (siso_chunk_kstate_bytes(Bn, L, H) + 255) & ~size_t(255);
  return ks + siso_chunk_bwd_scratch_bytes(Bn, L, H);
}

size_t m3_siso_scan_bwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                                       int64_t dstate) {
  const size_t rec = sizeof(float) * (size_t)(batch * nheads * seqlen);
  // headdim 64 / d_state 128 or 64 may take the chunked path (bf16); size for it
  if (headdim == 64 && (dstate == 128 || dstate == 64)) {
    const size_t ch = chunked_bwd_ws_bytes(batch, seqlen, nheads);
    return ch > rec ? ch : rec;
  }
  return rec;
}

size_t m3_siso_scan_kstates_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                                 int64_t dstate, int x_dtype, int bc_dtype) {
  if (headdim != 64 || (dstate != 128 && dstate != 64) || x_dtype != M3_BFLOAT16 || bc_dtype != M3_BFLOAT16 || seqlen <= 0 ||
      batch * nheads <= 0)
    return 0;
  return siso_chunk_kstate_bytes(batch, seqlen, nheads);
}

size_t m3_siso_scan_bwd_kstates_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads) {
  return siso_chunk_bwd_scratch_bytes(batch, seqlen, nheads);
}

namespace m3 {
namespace {
// Shared argument checks and parameter fill of the SISO backward entries. Returns M3_OK
// with *done set when nothing is left to launch (empty shapes).
int prep_siso_bwd(SisoParams& p, const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                  const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                  const m3_tensor* bx0, const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB, m3_tensor* dC,
                  m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dh0,
                  m3_tensor* dbx0, cudaStream_t s, bool* done) {
  *done = false;
  int64_t Bn, L, H, P, Ds, R;
  M3_TRY(check_scan_inputs(x, B, C, ADT, DT, trap, D, 4, &Bn, &L, &H, &P, &Ds, &R));
  const bool empty = Bn * L * H * P == 0;
  const int64_t xs[4] = {Bn, L, H, P}, bs[4] = {Bn, L, H, Ds}, st[4] = {Bn, H, P, Ds}, ss[3] = {Bn, L, H}, hs[1] = {H};
  M3_TRY(check(h0, "h0", 4, st, kF32, true, true, false));
  M3_TRY(check(bx0, "bx0", 4, st, kF32, true, true, false));
  M3_TRY(check(dy, "dy", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(dx, "dx", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(dB, "dB", 4, bs, 1u << B->dtype, false, false, !empty));
  M3_TRY(check(dC, "dC", 4, bs, 1u << B->dtype, false, false, !empty));
  M3_TRY(check(dADT, "dADT", 3, ss, kF32, false, false, false));
  M3_TRY(check(dDT, "dDT", 3, ss, kF32, false, false, false));
  M3_TRY(check(dtrap, "dtrap", 3, ss, kF32, false, false, false));
  M3_TRY(check(dD, "dD", 1, hs, kF32, true, false, false));
  M3_TRY(check(dh0, "dh0", 4, st, kF32, true, true, false));
  M3_TRY(check(dbx0, "dbx0", 4, st, kF32, true, true, false));
  M3_TRY(memset_async(dD->data, sizeof(float) * H, s, "dD"));
  if (Bn * H * P * Ds == 0) {
    *done = true;
    return M3_OK;
  }
  if (L == 0) {
    const size_t bytes = sizeof(float) * Bn * H * P * Ds;
    M3_TRY(copy_or_zero(fptr<void>(dh0), nullptr, bytes, s, "dh0"));
    M3_TRY(copy_or_zero(fptr<void>(dbx0), nullptr, bytes, s, "dbx0"));
    *done = true;
    return M3_OK;
  }
  if (Bn > INT32_MAX || L > INT32_MAX || H > INT32_MAX || P > 65535)
    return fail(M3_ERR_UNSUPPORTED, "siso scan: dimension too large");
  p = SisoParams{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds;
  p.x = x->data; p.sx = s3(x);
  p.Bm = B->data; p.sB = s3(B);
  p.Cm = C->data; p.sC = s3(C);
  p.adt = fptr<const float>(ADT); p.sadt = s3_scal(ADT);
  p.dt = fptr<const float>(DT); p.sdt = s3_scal(DT);
  p.trap = fptr<const float>(trap); p.strap = s3_scal(trap);
  p.Dskip = fptr<const float>(D); p.sD = D->stride[0];
  p.h0 = fptr<const float>(h0); p.bx0 = fptr<const float>(bx0);
  p.dy = dy->data; p.sdy = s3(dy);
  p.dx = dx->data; p.sdx = s3(dx);
  p.dB = dB->data; p.sdB = s3(dB);
  p.dC = dC->data; p.sdC = s3(dC);
  p.dadt = fptr<float>(dADT); p.sdadt = s3_scal(dADT);
  p.ddt = fptr<float>(dDT); p.sddt = s3_scal(dDT);
  p.dtrap = fptr<float>(dtrap); p.sdtrap = s3_scal(dtrap);
  p.dD = fptr<float>(dD);
  p.dh0 = fptr<float>(dh0); p.dbx0 = fptr<float>(dbx0);
  return M3_OK;
}
}  // namespace
}  // namespace m3

int m3_siso_scan_bwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                     const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                     const m3_tensor* bx0, const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB, m3_tensor* dC,
                     m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dh0,
                     m3_tensor* dbx0, void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SisoParams p;
  bool done = false;
  M3_TRY(prep_siso_bwd(p, x, B, C, ADT, DT, trap, D, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0, s,
                       &done));
  if (done) return M3_OK;
  const size_t need = sizeof(float) * (size_t)p.Bn * p.H * p.L;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(M3_ERR_WORKSPACE, "siso backward: workspace of " + std::to_string(need) + " bytes required");
  // chunked tensor-core path: recompute the forward's chunk states into the workspace, then
  // the reverse-chunk kernel (taken when the workspace has room for both)
  if (siso_chunk_bwd_supported(p, x->dtype, B->dtype) && workspace_bytes >= chunked_bwd_ws_bytes(p.Bn, p.L, p.H) &&
      (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
    const size_t ks = (siso_chunk_kstate_bytes(p.Bn, p.L, p.H) + 255) & ~size_t(255);
    SisoParams f = p;
    f.y = nullptr; f.sy = Str3{0, 0, 0};
    f.h_last = nullptr; f.bx_last = nullptr;
    f.kstates = workspace;
    M3_TRY(launch_siso_fwd_chunked(f, x->dtype, B->dtype, s));
    p.kstates = workspace;
    return launch_siso_bwd_chunked(p, reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ks), s);
  }
  p.q = reinterpret_cast<float*>(workspace);
  return launch_siso_bwd_recurrent(p, x->dtype, B->dtype, s);
}

int m3_siso_scan_fwd_kstates(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                             const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                             const m3_tensor* bx0, m3_tensor* y, m3_tensor* h_last, m3_tensor* bx_last,
                             void* kstates, size_t kstates_bytes, void* stream) {
  int64_t Bn, L, H, P, Ds, R;
  M3_TRY(check_scan_inputs(x, B, C, ADT, DT, trap, D, 4, &Bn, &L, &H, &P, &Ds, &R));
  const size_t need = m3_siso_scan_kstates_size(Bn, L, H, P, Ds, x->dtype, B->dtype);
  if (need == 0) return fail(M3_ERR_UNSUPPORTED, "siso scan: no chunk states for this shape / dtype");
  if (kstates == nullptr || kstates_bytes < need || (reinterpret_cast<uintptr_t>(kstates) & 255) != 0)
    return fail(M3_ERR_WORKSPACE, "siso scan: kstates of " + std::to_string(need) + " bytes (256-byte aligned) required");
  const int64_t xs[4] = {Bn, L, H, P}, st[4] = {Bn, H, P, Ds};
  M3_TRY(check(y, "y", 4, xs, 1u << x->dtype, false, false, true));
  M3_TRY(check(h0, "h0", 4, st, kF32, true, true, false));
  M3_TRY(check(bx0, "bx0", 4, st, kF32, true, true, false));
  M3_TRY(check(h_last, "h_last", 4, st, kF32, true, true, false));
  M3_TRY(check(bx_last, "bx_last", 4, st, kF32, true, true, false));
  if (Bn > INT32_MAX || L > INT32_MAX || H > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "siso scan: dimension too large");
  SisoParams p{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds;
  p.x = x->data; p.sx = s3(x);
  p.Bm = B->data; p.sB = s3(B);
  p.Cm = C->data; p.sC = s3(C);
  p.adt = fptr<const float>(ADT); p.sadt = s3_scal(ADT);
  p.dt = fptr<const float>(DT); p.sdt = s3_scal(DT);
  p.trap = fptr<const float>(trap); p.strap = s3_scal(trap);
  p.Dskip = fptr<const float>(D); p.sD = D->stride[0];
  p.h0 = fptr<const float>(h0); p.bx0 = fptr<const float>(bx0);
  p.y = y->data; p.sy = s3(y);
  p.h_last = fptr<float>(h_last); p.bx_last = fptr<float>(bx_last);
  p.kstates = kstates;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!siso_chunk_supported(p, x->dtype, B->dtype))
    return fail(M3_ERR_UNSUPPORTED, "siso scan: inputs not eligible for the chunked kernel (alignment / strides)");
  return launch_siso_fwd_chunked(p, x->dtype, B->dtype, s);
}

int m3_siso_scan_bwd_kstates(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                             const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                             const m3_tensor* bx0, const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB,
                             m3_tensor* dC, m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD,
                             m3_tensor* dh0, m3_tensor* dbx0, const void* kstates, size_t kstates_bytes,
                             void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SisoParams p;
  bool done = false;
  M3_TRY(prep_siso_bwd(p, x, B, C, ADT, DT, trap, D, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0, s,
                       &done));
  if (done) return M3_OK;
  const size_t kneed = m3_siso_scan_kstates_size(p.Bn, p.L, p.H, p.P, p.D, x->dtype, B->dtype);
  if (kneed == 0 || !siso_chunk_bwd_supported(p, x->dtype, B->dtype))
    return fail(M3_ERR_UNSUPPORTED, "siso backward: inputs not eligible for the chunked kernel");
  if (kstates == nullptr || kstates_bytes < kneed || (reinterpret_cast<uintptr_t>(kstates) & 255) != 0)
    return fail(M3_ERR_INVALID_ARGUMENT, "siso backward: kstates of " + std::to_string(kneed) + " bytes required");
  const size_t need = siso_chunk_bwd_scratch_bytes(p.Bn, p.L, p.H);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15) != 0)
    return fail(M3_ERR_WORKSPACE, "siso backward: workspace of " + std::to_string(need) + " bytes required");
  p.kstates = const_cast<void*>(kstates);
  return launch_siso_bwd_chunked(p, reinterpret_cast<float*>(workspace), s);
}

// Device address of g_noalloc_scratch, looked up once per device with that device
// current (host code cannot use the symbol itself as a device pointer).
static float* noalloc_scratch_for_current_device() {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      fail(M3_ERR_CUDA, std::string("cudaGetSymbolAddress(noalloc scratch): ") + cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  return addr[dev];
}

int m3_siso_scan_bwd_noalloc(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                             const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* h0,
                             const m3_tensor* bx0, const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB,
                             m3_tensor* dC, m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD,
                             m3_tensor* dh0, m3_tensor* dbx0, void* stream) {
  if (!present(x) || x->ndim != 4) return fail(M3_ERR_INVALID_ARGUMENT, "x: expected (B, L, H, P)");
  const int64_t positions = x->shape[0] * x->shape[1] * x->shape[2];
  if (positions > (int64_t)M3_NOALLOC_MAX_POSITIONS)
    return fail(M3_ERR_WORKSPACE, "siso backward (no-alloc): batch*heads*seqlen = " + std::to_string(positions) +
                                      " exceeds the fixed scratch of " + std::to_string(M3_NOALLOC_MAX_POSITIONS) +
                                      " positions; use m3_siso_scan_bwd with a caller workspace");
  float* scratch = nullptr;
  if (positions > 0) {
    scratch = noalloc_scratch_for_current_device();
    if (!scratch) return M3_ERR_CUDA;
  }
  // every position of the scratch that the kernels read is written first in the same call,
  // so nothing needs clearing between calls
  return m3_siso_scan_bwd(x, B, C, ADT, DT, trap, D, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0,
                          scratch, sizeof(float) * (size_t)M3_NOALLOC_MAX_POSITIONS, stream);
}

static int fill_mimo(MimoParams& p, const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                     const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D,
                     const m3_tensor* mimo_x, const m3_tensor* mimo_o, const m3_tensor* h0,
                     const m3_tensor* bx0, int64_t* dims) {
  int64_t Bn, L, H, P, Ds, R;
  M3_TRY(check_scan_inputs(x, B, C, ADT, DT, trap, D, 5, &Bn, &L, &H, &P, &Ds, &R));
  const int64_t ms[3] = {H, R, P}, st[3] = {Bn, H, Ds};
  M3_TRY(check(mimo_x, "mimo_x", 3, ms, kF32, false, false, false));
  M3_TRY(check(mimo_o, "mimo_o", 3, ms, kF32, false, false, false));
  M3_TRY(check(h0, "h0", 3, st, kF32, true, true, false));
  M3_TRY(check(bx0, "bx0", 3, st, kF32, true, true, false));
  if (Bn > INT32_MAX || L > INT32_MAX || H > INT32_MAX || P > 65535 || R > 8)
    return fail(M3_ERR_UNSUPPORTED, "mimo scan: dimension too large (rank must be <= 8)");
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds; p.R = (int)R;
  p.x = x->data; p.sx = s3(x);
  p.Bm = B->data; p.sB = s4(B);
  p.Cm = C->data; p.sC = s4(C);
  p.adt = fptr<const float>(ADT); p.sadt = s3_scal(ADT);
  p.dt = fptr<const float>(DT); p.sdt = s3_scal(DT);
  p.trap = fptr<const float>(trap); p.strap = s3_scal(trap);
  p.Dskip = fptr<const float>(D); p.sD = D->stride[0];
  p.mimo_x = fptr<const float>(mimo_x); p.smx_h = mimo_x->stride[0]; p.smx_r = mimo_x->stride[1];
  p.mimo_o = fptr<const float>(mimo_o); p.smo_h = mimo_o->stride[0]; p.smo_r = mimo_o->stride[1];
  p.h0 = fptr<const float>(h0); p.bx0 = fptr<const float>(bx0);
  dims[0] = Bn; dims[1] = L; dims[2] = H; dims[3] = P; dims[4] = Ds; dims[5] = R;
  return M3_OK;
}

int m3_mimo_scan_fwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                     const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* mimo_x,
                     const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, m3_tensor* y,
                     m3_tensor* h_last, m3_tensor* bx_last, void* stream) {
  MimoParams p{};
  int64_t d[6];
  M3_TRY(fill_mimo(p, x, B, C, ADT, DT, trap, D, mimo_x, mimo_o, h0, bx0, d));
  const int64_t xs[4] = {d[0], d[1], d[2], d[3]}, st[3] = {d[0], d[2], d[4]};
  const bool empty = d[0] * d[1] * d[2] * d[3] == 0;
  M3_TRY(check(y, "y", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(h_last, "h_last", 3, st, kF32, true, true, false));
  M3_TRY(check(bx_last, "bx_last", 3, st, kF32, true, true, false));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d[0] * d[2] * d[4] == 0) return M3_OK;
  if (d[1] == 0 || d[3] == 0) {
    const size_t bytes = sizeof(float) * d[0] * d[2] * d[4];
    if (d[1] == 0) {
      M3_TRY(copy_or_zero(fptr<void>(h_last), fptr<void>(h0), bytes, s, "h_last"));
      return copy_or_zero(fptr<void>(bx_last), fptr<void>(bx0), bytes, s, "bx_last");
    }
  }
  p.y = y->data; p.sy = s3(y);
  p.h_last = fptr<float>(h_last); p.bx_last = fptr<float>(bx_last);
  return launch_mimo(p, x->dtype, B->dtype, false, s);
}

size_t m3_mimo_scan_fwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t dstate) {
  if (batch < 0 || seqlen < 0 || nheads < 0 || dstate < 0) return 0;
  return mimo_fwd_workspace_bytes(batch, seqlen, nheads, dstate);
}

int m3_mimo_scan_fwd_ws(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                        const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* mimo_x,
                        const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, m3_tensor* y,
                        m3_tensor* h_last, m3_tensor* bx_last, void* workspace, size_t workspace_bytes,
                        void* stream) {
  MimoParams p{};
  int64_t d[6];
  M3_TRY(fill_mimo(p, x, B, C, ADT, DT, trap, D, mimo_x, mimo_o, h0, bx0, d));
  const int64_t xs[4] = {d[0], d[1], d[2], d[3]}, st[3] = {d[0], d[2], d[4]};
  const bool empty = d[0] * d[1] * d[2] * d[3] == 0;
  M3_TRY(check(y, "y", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(h_last, "h_last", 3, st, kF32, true, true, false));
  M3_TRY(check(bx_last, "bx_last", 3, st, kF32, true, true, false));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d[0] * d[2] * d[4] == 0) return M3_OK;
  if (d[1] == 0 || d[3] == 0) {
    const size_t bytes = sizeof(float) * d[0] * d[2] * d[4];
    if (d[1] == 0) {
      M3_TRY(copy_or_zero(fptr<void>(h_last), fptr<void>(h0), bytes, s, "h_last"));
      return copy_or_zero(fptr<void>(bx_last), fptr<void>(bx0), bytes, s, "bx_last");
    }
  }
  const size_t need = mimo_fwd_workspace_bytes(d[0], d[1], d[2], d[4]);
  if (!workspace || workspace_bytes < need)
    return fail(M3_ERR_WORKSPACE, "workspace: need " + std::to_string(need) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0) return fail(M3_ERR_INVALID_ARGUMENT, "workspace: not 16-byte aligned");
  M3_TRY(check_device_ptr(workspace, "workspace"));
  p.y = y->data; p.sy = s3(y);
  p.h_last = fptr<float>(h_last); p.bx_last = fptr<float>(bx_last);
  return launch_mimo_fwd_chunked(p, x->dtype, B->dtype, workspace, s);
}

size_t m3_mimo_scan_bwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                                       int64_t dstate, int64_t rank) {
  return sizeof(float) * mimo_bwd_workspace_floats(batch, seqlen, nheads, headdim, dstate, rank);
}

static int mimo_bwd_common(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                           const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* mimo_x,
                           const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, const m3_tensor* dy,
                           m3_tensor* dx, m3_tensor* dB, m3_tensor* dC, m3_tensor* dADT, m3_tensor* dDT,
                           m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dmimo_x, m3_tensor* dmimo_o, m3_tensor* dh0,
                           m3_tensor* dbx0, const void* fwd_workspace, size_t fwd_workspace_bytes, void* workspace,
                           size_t workspace_bytes, void* stream) {
  MimoParams p{};
  int64_t d[6];
  M3_TRY(fill_mimo(p, x, B, C, ADT, DT, trap, D, mimo_x, mimo_o, h0, bx0, d));
  const int64_t Bn = d[0], L = d[1], H = d[2], P = d[3], Ds = d[4], R = d[5];
  const bool empty = Bn * L * H * P == 0;
  const int64_t xs[4] = {Bn, L, H, P}, bs[5] = {Bn, L, R, H, Ds}, ss[3] = {Bn, L, H}, hs[1] = {H},
                ms[3] = {H, R, P}, st[3] = {Bn, H, Ds};
  M3_TRY(check(dy, "dy", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(dx, "dx", 4, xs, 1u << x->dtype, false, false, !empty));
  M3_TRY(check(dB, "dB", 5, bs, 1u << B->dtype, false, false, !empty));
  M3_TRY(check(dC, "dC", 5, bs, 1u << B->dtype, false, false, !empty));
  M3_TRY(check(dADT, "dADT", 3, ss, kF32, false, false, false));
  M3_TRY(check(dDT, "dDT", 3, ss, kF32, false, false, false));
  M3_TRY(check(dtrap, "dtrap", 3, ss, kF32, false, false, false));
  M3_TRY(check(dD, "dD", 1, hs, kF32, true, false, false));
  M3_TRY(check(dmimo_x, "dmimo_x", 3, ms, kF32, true, false, false));
  M3_TRY(check(dmimo_o, "dmimo_o", 3, ms, kF32, true, false, false));
  M3_TRY(check(dh0, "dh0", 3, st, kF32, true, true, false));
  M3_TRY(check(dbx0, "dbx0", 3, st, kF32, true, true, false));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  M3_TRY(memset_async(dD->data, sizeof(float) * H, s, "dD"));
  M3_TRY(memset_async(dmimo_x->data, sizeof(float) * H * R * P, s, "dmimo_x"));
  M3_TRY(memset_async(dmimo_o->data, sizeof(float) * H * R * P, s, "dmimo_o"));
  if (Bn * H * Ds == 0) return M3_OK;
  if (L == 0) {
    const size_t bytes = sizeof(float) * Bn * H * Ds;
    M3_TRY(copy_or_zero(fptr<void>(dh0), nullptr, bytes, s, "dh0"));
    return copy_or_zero(fptr<void>(dbx0), nullptr, bytes, s, "dbx0");
  }
  if (workspace && reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
    return fail(M3_ERR_INVALID_ARGUMENT, "mimo backward: workspace not 16-byte aligned");
  if (fwd_workspace && reinterpret_cast<uintptr_t>(fwd_workspace) % 16 != 0)
    return fail(M3_ERR_INVALID_ARGUMENT, "mimo backward: forward workspace not 16-byte aligned");
  p.dy = dy->data; p.sdy = s3(dy);
  p.dx = dx->data; p.sdx = s3(dx);
  p.dB = dB->data; p.sdB = s4(dB);
  p.dC = dC->data; p.sdC = s4(dC);
  p.dadt = fptr<float>(dADT); p.sdadt = s3_scal(dADT);
  p.ddt = fptr<float>(dDT); p.sddt = s3_scal(dDT);
  p.dtrap = fptr<float>(dtrap); p.sdtrap = s3_scal(dtrap);
  p.dD = fptr<float>(dD);
  p.dmx = fptr<float>(dmimo_x); p.dmo = fptr<float>(dmimo_o);
  p.dh0 = fptr<float>(dh0); p.dbx0 = fptr<float>(dbx0);
  if (fwd_workspace) {
    M3_TRY(check_device_ptr(fwd_workspace, "fwd_workspace"));
    const int rc = launch_mimo_bwd_fused(p, x->dtype, B->dtype, fwd_workspace, fwd_workspace_bytes, workspace,
                                         workspace_bytes, s);
    if (rc != M3_ERR_UNSUPPORTED) return rc;
  }
  const size_t need = m3_mimo_scan_bwd_workspace_size(Bn, L, H, P, Ds, R);
  if (need == 0) return fail(M3_ERR_UNSUPPORTED, "mimo backward: shapes too large for shared memory");
  if (workspace == nullptr || workspace_bytes < need)
    return fail(M3_ERR_WORKSPACE, "mimo backward: workspace of " + std::to_string(need) + " bytes required");
  p.work = reinterpret_cast<float*>(workspace);
  return launch_mimo(p, x->dtype, B->dtype, true, s);
}

int m3_mimo_scan_bwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                     const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* mimo_x,
                     const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, const m3_tensor* dy,
                     m3_tensor* dx, m3_tensor* dB, m3_tensor* dC, m3_tensor* dADT, m3_tensor* dDT,
                     m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dmimo_x, m3_tensor* dmimo_o, m3_tensor* dh0,
                     m3_tensor* dbx0, void* workspace, size_t workspace_bytes, void* stream) {
  return mimo_bwd_common(x, B, C, ADT, DT, trap, D, mimo_x, mimo_o, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD,
                         dmimo_x, dmimo_o, dh0, dbx0, nullptr, 0, workspace, workspace_bytes, stream);
}

size_t m3_mimo_scan_bwd_ws_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                                          int64_t dstate, int64_t rank) {
  if (batch < 0 || seqlen < 0 || nheads < 0 || headdim < 0 || dstate < 0 || rank < 0) return 0;
  return std::max(m3_mimo_scan_bwd_workspace_size(batch, seqlen, nheads, headdim, dstate, rank),
                  mimo_bwd_fused_workspace_bytes(batch, seqlen, nheads, dstate));
}

int m3_mimo_scan_bwd_ws(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                        const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D, const m3_tensor* mimo_x,
                        const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, const m3_tensor* dy,
                        m3_tensor* dx, m3_tensor* dB, m3_tensor* dC, m3_tensor* dADT, m3_tensor* dDT,
                        m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dmimo_x, m3_tensor* dmimo_o, m3_tensor* dh0,
                        m3_tensor* dbx0, const void* fwd_workspace, size_t fwd_workspace_bytes, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return mimo_bwd_common(x, B, C, ADT, DT, trap, D, mimo_x, mimo_o, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD,
                         dmimo_x, dmimo_o, dh0, dbx0, fwd_workspace, fwd_workspace_bytes, workspace, workspace_bytes,
                         stream);
}

static int step_common(bool mimo, const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                       const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                       const m3_tensor* C_norm_w, const m3_tensor* Dskip, const m3_tensor* mimo_x,
                       const m3_tensor* mimo_o, const m3_tensor* angle_in, const m3_tensor* ssm_in,
                       const m3_tensor* bx_in, m3_tensor* angle_out, m3_tensor* ssm_out, m3_tensor* bx_out,
                       m3_tensor* y_gated, void* stream) {
  if (!dims) return fail(M3_ERR_INVALID_ARGUMENT, "dims: missing");
  const int64_t H = dims->nheads, P = dims->headdim, Ds = dims->d_state, G = dims->ngroups,
                R = mimo ? dims->mimo_rank : 1, S = dims->num_rope_angles, di = dims->d_inner;
  if (H <= 0 || P <= 0 || Ds <= 0 || G <= 0 || R <= 0 || S < 0 || di != H * P || dims->rope_split != 2 * S ||
      dims->rope_split > Ds || (G != 1 && G != H))
    return fail(M3_ERR_INVALID_ARGUMENT, "dims: inconsistent layer dimensions");
  if (!mimo && dims->mimo_rank != 1) return fail(M3_ERR_INVALID_ARGUMENT, "dims: SISO step needs mimo_rank 1");
  if (!present(zxbcdt) || zxbcdt->ndim != 2) return fail(M3_ERR_INVALID_ARGUMENT, "zxbcdt: expected (batch, d_in_proj)");
  const int64_t Bn = zxbcdt->shape[0];
  const int64_t dproj = 2 * di + 2 * Ds * G * R + 3 * H + S;
  const int64_t zs[2] = {Bn, dproj}, ys[2] = {Bn, di}, h1[1] = {H}, hrd[3] = {H, R, Ds}, d1[1] = {Ds},
                hrp[3] = {H, R, P}, as[3] = {Bn, H, S};
  M3_TRY(check(zxbcdt, "zxbcdt", 2, zs, kAnyFloat, false, false, Bn > 0));
  M3_TRY(check(y_gated, "y_gated", 2, ys, 1u << zxbcdt->dtype, false, false, false));
  M3_TRY(check(dt_bias, "dt_bias", 1, h1, kF32, true, false, false));
  M3_TRY(check(B_bias, "B_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(C_bias, "C_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(B_norm_w, "B_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(C_norm_w, "C_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(Dskip, "D", 1, h1, kF32, true, false, false));
  if (mimo) {
    M3_TRY(check(mimo_x, "mimo_x", 3, hrp, kF32, true, false, false));
    M3_TRY(check(mimo_o, "mimo_o", 3, hrp, kF32, true, false, false));
  }
  if (S > 0) {
    M3_TRY(check(angle_in, "angle_in", 3, as, kF32, true, false, false));
    M3_TRY(check(angle_out, "angle_out", 3, as, kF32, true, false, false));
  }
  if (mimo) {
    const int64_t st[3] = {Bn, H, Ds};
    M3_TRY(check(ssm_in, "ssm_in", 3, st, kF32, true, false, false));
    M3_TRY(check(bx_in, "bx_in", 3, st, kF32, true, false, false));
    M3_TRY(check(ssm_out, "ssm_out", 3, st, kF32, true, false, false));
    M3_TRY(check(bx_out, "bx_out", 3, st, kF32, true, false, false));
  } else {
    const int64_t st[4] = {Bn, H, P, Ds};
    M3_TRY(check(ssm_in, "ssm_in", 4, st, kF32, true, false, false));
    M3_TRY(check(bx_in, "bx_in", 4, st, kF32, true, false, false));
    M3_TRY(check(ssm_out, "ssm_out", 4, st, kF32, true, false, false));
    M3_TRY(check(bx_out, "bx_out", 4, st, kF32, true, false, false));
  }
  if (Bn == 0) return M3_OK;
  if (!mimo) {
    for (const m3_tensor* t : {ssm_in, bx_in, (const m3_tensor*)ssm_out, (const m3_tensor*)bx_out})
      if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0)
        return fail(M3_ERR_INVALID_ARGUMENT, "siso step: state buffers must be 16-byte aligned");
  }
  StepParams p{};
  p.Bn = (int)Bn; p.H = (int)H; p.P = (int)P; p.D = (int)Ds; p.R = (int)R; p.G = (int)G; p.S = (int)S;
  p.split = dims->rope_split; p.d_inner = (int)di; p.A_floor = dims->A_floor; p.eps = dims->norm_eps;
  p.zxbcdt = zxbcdt->data; p.s_row = zxbcdt->stride[0];
  p.dt_bias = fptr<const float>(dt_bias);
  p.B_bias = fptr<const float>(B_bias); p.C_bias = fptr<const float>(C_bias);
  p.B_norm_w = fptr<const float>(B_norm_w); p.C_norm_w = fptr<const float>(C_norm_w);
  p.Dskip = fptr<const float>(Dskip);
  p.mimo_x = mimo ? fptr<const float>(mimo_x) : nullptr;
  p.mimo_o = mimo ? fptr<const float>(mimo_o) : nullptr;
  p.angle_in = S > 0 ? fptr<const float>(angle_in) : nullptr;
  p.angle_out = S > 0 ? fptr<float>(angle_out) : nullptr;
  p.ssm_in = fptr<const float>(ssm_in); p.ssm_out = fptr<float>(ssm_out);
  p.bx_in = fptr<const float>(bx_in); p.bx_out = fptr<float>(bx_out);
  p.y = y_gated->data; p.s_y = y_gated->stride[0];
  return launch_step(p, zxbcdt->dtype, mimo, reinterpret_cast<cudaStream_t>(stream));
}

int m3_siso_step(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias, const m3_tensor* B_bias,
                 const m3_tensor* C_bias, const m3_tensor* B_norm_w, const m3_tensor* C_norm_w, const m3_tensor* Dskip,
                 const m3_tensor* angle_in, const m3_tensor* ssm_in, const m3_tensor* bx_in, m3_tensor* angle_out,
                 m3_tensor* ssm_out, m3_tensor* bx_out, m3_tensor* y_gated, void* stream) {
  return step_common(false, dims, zxbcdt, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, Dskip, nullptr, nullptr,
                     angle_in, ssm_in, bx_in, angle_out, ssm_out, bx_out, y_gated, stream);
}

int m3_mimo_step(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias, const m3_tensor* B_bias,
                 const m3_tensor* C_bias, const m3_tensor* B_norm_w, const m3_tensor* C_norm_w, const m3_tensor* Dskip,
                 const m3_tensor* mimo_x, const m3_tensor* mimo_o, const m3_tensor* angle_in, const m3_tensor* ssm_in,
                 const m3_tensor* bx_in, m3_tensor* angle_out, m3_tensor* ssm_out, m3_tensor* bx_out,
                 m3_tensor* y_gated, void* stream) {
  return step_common(true, dims, zxbcdt, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, Dskip, mimo_x, mimo_o,
                     angle_in, ssm_in, bx_in, angle_out, ssm_out, bx_out, y_gated, stream);
}


int m3_rmsnorm(const m3_tensor* x, const m3_tensor* residual, const m3_tensor* weight, float eps,
               m3_tensor* out, m3_tensor* residual_out, void* stream) {
  if (!present(x) || x->ndim < 1) return fail(M3_ERR_INVALID_ARGUMENT, "x: missing or 0-d");
  const int nd = x->ndim;
  const int64_t d = x->shape[nd - 1];
  int64_t rows = 1;
  for (int i = 0; i < nd - 1; ++i) rows *= x->shape[i];
  const bool empty = rows * d == 0;
  // every operand: (..., d) whose leading dims collapse into rows of one stride
  auto rows_of = [&](const m3_tensor* t, const char* name, bool optional, unsigned mask, int64_t* srow) -> int {
    if (!present(t)) {
      if (optional) return M3_OK;
      return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": missing");
    }
    M3_TRY(check(t, name, nd, x->shape, mask, false, false, !empty));
    if (empty) return M3_OK;
    for (int i = 0; i + 2 < nd; ++i)
      if (t->shape[i] > 1 && t->stride[i] != t->stride[i + 1] * t->shape[i + 1])
        return fail(M3_ERR_INVALID_ARGUMENT, std::string(name) + ": leading dims must collapse into rows");
    *srow = nd >= 2 ? t->stride[nd - 2] : d;
    return M3_OK;
  };
  NormParams p{};
  p.rows = rows; p.d = d; p.eps = eps;
  M3_TRY(rows_of(x, "x", false, kAnyFloat, &p.sx));
  M3_TRY(rows_of(residual, "residual", true, 1u << x->dtype, &p.sres));
  M3_TRY(rows_of(out, "out", false, 1u << x->dtype, &p.sout));
  M3_TRY(rows_of(residual_out, "residual_out", true, 1u << x->dtype, &p.shout));
  const int64_t ws[1] = {d};
  M3_TRY(check(weight, "weight", 1, ws, kAnyFloat, true, false, !empty));
  if (present(residual_out) && !present(residual))
    return fail(M3_ERR_INVALID_ARGUMENT, "residual_out: given without residual");
  if (present(residual_out) && present(out) && residual_out->data == out->data && !empty)
    return fail(M3_ERR_INVALID_ARGUMENT, "out: must not alias residual_out");
  p.x = x->data; p.res = present(residual) ? residual->data : nullptr;
  p.w = weight->data; p.out = out->data; p.hout = present(residual_out) ? residual_out->data : nullptr;
  return launch_rmsnorm(p, x->dtype, weight->dtype, reinterpret_cast<cudaStream_t>(stream));
}


int m3_argmax_rows(const m3_tensor* logits, m3_tensor* out, void* stream) {
  if (!present(logits) || logits->ndim < 1) return fail(M3_ERR_INVALID_ARGUMENT, "logits: missing or 0-d");
  if (!present(out)) return fail(M3_ERR_INVALID_ARGUMENT, "out: missing");
  const int nd = logits->ndim;
  const int64_t n = logits->shape[nd - 1];
  int64_t rows = 1;
  for (int i = 0; i < nd - 1; ++i) rows *= logits->shape[i];
  M3_TRY(check(logits, "logits", nd, logits->shape, kAnyFloat, false, false, rows * n > 0));
  if (n <= 0 && rows > 0) return fail(M3_ERR_INVALID_ARGUMENT, "logits: empty last dimension");
  for (int i = 0; i + 2 < nd; ++i)
    if (logits->shape[i] > 1 && logits->stride[i] != logits->stride[i + 1] * logits->shape[i + 1])
      return fail(M3_ERR_INVALID_ARGUMENT, "logits: leading dims must collapse into rows");
  if (out->dtype != M3_INT64) return fail(M3_ERR_INVALID_ARGUMENT, "out: expected int64");
  int64_t on = 1, expect = 1;
  for (int i = out->ndim - 1; i >= 0; --i) {
    if (out->shape[i] > 1 && out->stride[i] != expect)
      return fail(M3_ERR_INVALID_ARGUMENT, "out: must be contiguous");
    expect *= out->shape[i];
    on *= out->shape[i];
  }
  if (on != rows) return fail(M3_ERR_INVALID_ARGUMENT, "out: one element per logits row expected");
  if (rows == 0) return M3_OK;
  M3_TRY(check_device_ptr(out->data, "out"));
  const int64_t sx = nd >= 2 ? logits->stride[nd - 2] : n;
  return launch_argmax_rows(logits->data, logits->dtype, rows, n, sx, static_cast<int64_t*>(out->data),
                            reinterpret_cast<cudaStream_t>(stream));
}

int m3_device_timeouts(int reset, int* flag_out) {
  if (!flag_out) return fail(M3_ERR_INVALID_ARGUMENT, "flag_out: missing");
  int f = 0, b = 0, m = 0, q = 0;
  M3_TRY(chunk_error_word(reset != 0, &f));
  M3_TRY(chunk_bwd_error_word(reset != 0, &b));
  M3_TRY(mimo_error_word(reset != 0, &m));
  M3_TRY(prologue_error_word(reset != 0, &q));
  *flag_out = f | b | m | q;
  return M3_OK;
}


int m3_layer_prologue(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                      const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                      const m3_tensor* C_norm_w, const m3_tensor* angle0, m3_tensor* B_proj, m3_tensor* C_proj,
                      m3_tensor* ADT, m3_tensor* DT, m3_tensor* trap, m3_tensor* angles, void* stream) {
  if (!dims) return fail(M3_ERR_INVALID_ARGUMENT, "dims: missing");
  const int64_t H = dims->nheads, P = dims->headdim, Ds = dims->d_state, G = dims->ngroups,
                R = dims->mimo_rank, S = dims->num_rope_angles, di = dims->d_inner;
  if (H <= 0 || P <= 0 || Ds <= 0 || G <= 0 || R <= 0 || S < 0 || di != H * P || dims->rope_split != 2 * S ||
      dims->rope_split > Ds || (G != 1 && G != H))
    return fail(M3_ERR_INVALID_ARGUMENT, "dims: inconsistent layer dimensions");
  if (!present(zxbcdt) || zxbcdt->ndim != 3) return fail(M3_ERR_INVALID_ARGUMENT, "zxbcdt: expected (batch, seqlen, d_in_proj)");
  const int64_t Bn = zxbcdt->shape[0], L = zxbcdt->shape[1];
  const int64_t dproj = 2 * di + 2 * Ds * G * R + 3 * H + S;
  const bool empty = Bn * L == 0;
  const int64_t zs[3] = {Bn, L, dproj}, bs[5] = {Bn, L, R, H, Ds}, ss[3] = {Bn, L, H}, as[4] = {Bn, L, H, S},
                h1[1] = {H}, hrd[3] = {H, R, Ds}, d1[1] = {Ds};
  M3_TRY(check(zxbcdt, "zxbcdt", 3, zs, kAnyFloat, false, false, !empty));
  // B_proj and C_proj: both present, or both absent (angles and step scalars only)
  const bool with_bc = present(B_proj) || present(C_proj);
  if (with_bc) {
    M3_TRY(check(B_proj, "B_proj", 5, bs, kAnyFloat, true, false, !empty));
    M3_TRY(check(C_proj, "C_proj", 5, bs, 1u << B_proj->dtype, true, false, !empty));
  }
  M3_TRY(check(ADT, "ADT", 3, ss, kF32, true, false, false));
  M3_TRY(check(DT, "DT", 3, ss, kF32, true, false, false));
  M3_TRY(check(trap, "trap", 3, ss, kF32, true, false, false));
  M3_TRY(check(angles, "angles", 4, as, kF32, true, S == 0, false));
  M3_TRY(check(dt_bias, "dt_bias", 1, h1, kF32, true, false, false));
  M3_TRY(check(B_bias, "B_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(C_bias, "C_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(B_norm_w, "B_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(C_norm_w, "C_norm_w", 1, d1, kF32, true, false, false));
  const int64_t a0s[3] = {Bn, H, S};
  M3_TRY(check(angle0, "angle0", 3, a0s, kF32, true, true, false));
  if (empty) return M3_OK;
  if (Bn > INT32_MAX || L > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "prologue: dimension too large");
  PrologueParams p{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds; p.R = (int)R; p.G = (int)G;
  p.S = (int)S; p.split = dims->rope_split; p.d_inner = (int)di; p.A_floor = dims->A_floor; p.eps = dims->norm_eps;
  p.zx = zxbcdt->data; p.s_zb = zxbcdt->stride[0]; p.s_zl = zxbcdt->stride[1];
  p.dt_bias = fptr<const float>(dt_bias);
  p.B_bias = fptr<const float>(B_bias); p.C_bias = fptr<const float>(C_bias);
  p.B_norm_w = fptr<const float>(B_norm_w); p.C_norm_w = fptr<const float>(C_norm_w);
  p.Bp = with_bc ? B_proj->data : nullptr;
  p.Cp = with_bc ? C_proj->data : nullptr;
  p.ADT = fptr<float>(ADT); p.DT = fptr<float>(DT); p.trap = fptr<float>(trap); p.angles = fptr<float>(angles);
  p.angle0 = S > 0 ? fptr<const float>(angle0) : nullptr;
  return launch_prologue(p, zxbcdt->dtype, with_bc ? B_proj->dtype : zxbcdt->dtype,
                         reinterpret_cast<cudaStream_t>(stream));
}

int m3_mimo_layer_scan_fwd(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* ADT,
                           const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* angles,
                           const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                           const m3_tensor* C_norm_w, const m3_tensor* D, const m3_tensor* mimo_x,
                           const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, int32_t gate,
                           m3_tensor* out, m3_tensor* h_last, m3_tensor* bx_last, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!dims) return fail(M3_ERR_INVALID_ARGUMENT, "dims: missing");
  const int64_t H = dims->nheads, P = dims->headdim, Ds = dims->d_state, G = dims->ngroups,
                R = dims->mimo_rank, S = dims->num_rope_angles, di = dims->d_inner;
  if (H <= 0 || P <= 0 || Ds <= 0 || G <= 0 || R <= 0 || S < 0 || di != H * P || dims->rope_split != 2 * S ||
      dims->rope_split > Ds || (G != 1 && G != H))
    return fail(M3_ERR_INVALID_ARGUMENT, "dims: inconsistent layer dimensions");
  if (gate != 0 && gate != 1) return fail(M3_ERR_INVALID_ARGUMENT, "gate: must be 0 or 1");
  if (!present(zxbcdt) || zxbcdt->ndim != 3) return fail(M3_ERR_INVALID_ARGUMENT, "zxbcdt: expected (batch, seqlen, d_in_proj)");
  const int64_t Bn = zxbcdt->shape[0], L = zxbcdt->shape[1];
  const int64_t dproj = 2 * di + 2 * Ds * G * R + 3 * H + S;
  const bool empty = Bn * L == 0;
  const int64_t zs[3] = {Bn, L, dproj}, ss[3] = {Bn, L, H}, as[4] = {Bn, L, H, S}, h1[1] = {H},
                hrd[3] = {H, R, Ds}, d1[1] = {Ds}, ms[3] = {H, R, P}, st[3] = {Bn, H, Ds}, ys[4] = {Bn, L, H, P};
  M3_TRY(check(zxbcdt, "zxbcdt", 3, zs, kAnyFloat, false, false, !empty));
  M3_TRY(check(ADT, "ADT", 3, ss, kF32, false, false, false));
  M3_TRY(check(DT, "DT", 3, ss, kF32, false, false, false));
  M3_TRY(check(trap, "trap", 3, ss, kF32, false, false, false));
  M3_TRY(check(angles, "angles", 4, as, kF32, true, S == 0, false));
  M3_TRY(check(B_bias, "B_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(C_bias, "C_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(B_norm_w, "B_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(C_norm_w, "C_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(D, "D", 1, h1, kF32, false, false, false));
  M3_TRY(check(mimo_x, "mimo_x", 3, ms, kF32, false, false, false));
  M3_TRY(check(mimo_o, "mimo_o", 3, ms, kF32, false, false, false));
  M3_TRY(check(h0, "h0", 3, st, kF32, true, true, false));
  M3_TRY(check(bx0, "bx0", 3, st, kF32, true, true, false));
  M3_TRY(check(out, "out", 4, ys, 1u << zxbcdt->dtype, false, false, !empty));
  M3_TRY(check(h_last, "h_last", 3, st, kF32, true, true, false));
  M3_TRY(check(bx_last, "bx_last", 3, st, kF32, true, true, false));
  if (G != 1) return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: one B / C group only");
  if (Bn > INT32_MAX || L > INT32_MAX || H > INT32_MAX || P > 65535 || R > 8)
    return fail(M3_ERR_UNSUPPORTED, "mimo layer scan: dimension too large (rank must be <= 8)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (Bn * H * Ds == 0) return M3_OK;
  if (L == 0) {
    const size_t bytes = sizeof(float) * Bn * H * Ds;
    M3_TRY(copy_or_zero(fptr<void>(h_last), fptr<void>(h0), bytes, s, "h_last"));
    return copy_or_zero(fptr<void>(bx_last), fptr<void>(bx0), bytes, s, "bx_last");
  }
  const size_t need = mimo_fwd_workspace_bytes(Bn, L, H, Ds);
  if (!workspace || workspace_bytes < need)
    return fail(M3_ERR_WORKSPACE, "workspace: need " + std::to_string(need) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0) return fail(M3_ERR_INVALID_ARGUMENT, "workspace: not 16-byte aligned");
  M3_TRY(check_device_ptr(workspace, "workspace"));
  MimoParams p{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds; p.R = (int)R;
  p.adt = fptr<const float>(ADT); p.sadt = s3_scal(ADT);
  p.dt = fptr<const float>(DT); p.sdt = s3_scal(DT);
  p.trap = fptr<const float>(trap); p.strap = s3_scal(trap);
  p.Dskip = fptr<const float>(D); p.sD = D->stride[0];
  p.mimo_x = fptr<const float>(mimo_x); p.smx_h = mimo_x->stride[0]; p.smx_r = mimo_x->stride[1];
  p.mimo_o = fptr<const float>(mimo_o); p.smo_h = mimo_o->stride[0]; p.smo_r = mimo_o->stride[1];
  p.h0 = fptr<const float>(h0); p.bx0 = fptr<const float>(bx0);
  p.y = out->data; p.sy = s3(out);
  p.h_last = fptr<float>(h_last); p.bx_last = fptr<float>(bx_last);
  MimoGrpParams q{};
  q.zx = zxbcdt->data; q.s_zb = zxbcdt->stride[0]; q.s_zl = zxbcdt->stride[1];
  q.dtype = zxbcdt->dtype;
  q.angles = S > 0 ? fptr<const float>(angles) : nullptr;
  q.B_bias = fptr<const float>(B_bias); q.C_bias = fptr<const float>(C_bias);
  q.B_norm_w = fptr<const float>(B_norm_w); q.C_norm_w = fptr<const float>(C_norm_w);
  q.eps = dims->norm_eps;
  q.S = (int)S;
  q.gate = gate;
  return launch_mimo_layer_fwd(p, q, workspace, s);
}

size_t m3_layer_prologue_bwd_workspace_size(const m3_layer_dims* dims, int64_t batch, int64_t seqlen) {
  if (!dims || batch < 0 || seqlen < 0) return 0;
  return prologue_bwd_workspace_bytes(batch, seqlen, dims->nheads, dims->num_rope_angles, dims->mimo_rank,
                                      dims->d_state);
}

int m3_layer_prologue_bwd(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                          const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                          const m3_tensor* C_norm_w, const m3_tensor* DT, const m3_tensor* angles,
                          const m3_tensor* dB_proj, const m3_tensor* dC_proj, const m3_tensor* dADT,
                          const m3_tensor* dDT, const m3_tensor* dtrap, m3_tensor* d_zxbcdt, m3_tensor* d_dt_bias,
                          m3_tensor* d_B_bias, m3_tensor* d_C_bias, m3_tensor* d_B_norm_w, m3_tensor* d_C_norm_w,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!dims) return fail(M3_ERR_INVALID_ARGUMENT, "dims: missing");
  const int64_t H = dims->nheads, P = dims->headdim, Ds = dims->d_state, G = dims->ngroups,
                R = dims->mimo_rank, S = dims->num_rope_angles, di = dims->d_inner;
  if (H <= 0 || P <= 0 || Ds <= 0 || G <= 0 || R <= 0 || S < 0 || di != H * P || dims->rope_split != 2 * S ||
      dims->rope_split > Ds || (G != 1 && G != H))
    return fail(M3_ERR_INVALID_ARGUMENT, "dims: inconsistent layer dimensions");
  if (!present(zxbcdt) || zxbcdt->ndim != 3) return fail(M3_ERR_INVALID_ARGUMENT, "zxbcdt: expected (batch, seqlen, d_in_proj)");
  const int64_t Bn = zxbcdt->shape[0], L = zxbcdt->shape[1];
  const int64_t dproj = 2 * di + 2 * Ds * G * R + 3 * H + S;
  const bool empty = Bn * L == 0;
  const int64_t zs[3] = {Bn, L, dproj}, bs[5] = {Bn, L, R, H, Ds}, ss[3] = {Bn, L, H}, as[4] = {Bn, L, H, S},
                h1[1] = {H}, hrd[3] = {H, R, Ds}, d1[1] = {Ds};
  M3_TRY(check(zxbcdt, "zxbcdt", 3, zs, kAnyFloat, false, false, !empty));
  M3_TRY(check(d_zxbcdt, "d_zxbcdt", 3, zs, 1u << zxbcdt->dtype, false, false, !empty));
  M3_TRY(check(dB_proj, "dB_proj", 5, bs, kAnyFloat, true, false, !empty));
  M3_TRY(check(dC_proj, "dC_proj", 5, bs, 1u << dB_proj->dtype, true, false, !empty));
  M3_TRY(check(DT, "DT", 3, ss, kF32, true, false, false));
  M3_TRY(check(dADT, "dADT", 3, ss, kF32, true, false, false));
  M3_TRY(check(dDT, "dDT", 3, ss, kF32, true, false, false));
  M3_TRY(check(dtrap, "dtrap", 3, ss, kF32, true, false, false));
  M3_TRY(check(angles, "angles", 4, as, kF32, true, S == 0, false));
  M3_TRY(check(dt_bias, "dt_bias", 1, h1, kF32, true, false, false));
  M3_TRY(check(B_bias, "B_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(C_bias, "C_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(B_norm_w, "B_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(C_norm_w, "C_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(d_dt_bias, "d_dt_bias", 1, h1, kF32, true, false, false));
  M3_TRY(check(d_B_bias, "d_B_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(d_C_bias, "d_C_bias", 3, hrd, kF32, true, false, false));
  M3_TRY(check(d_B_norm_w, "d_B_norm_w", 1, d1, kF32, true, false, false));
  M3_TRY(check(d_C_norm_w, "d_C_norm_w", 1, d1, kF32, true, false, false));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (empty) {
    // no positions: every parameter gradient is zero
    M3_TRY(memset_async(d_dt_bias->data, sizeof(float) * H, s, "d_dt_bias"));
    M3_TRY(memset_async(d_B_bias->data, sizeof(float) * H * R * Ds, s, "d_B_bias"));
    M3_TRY(memset_async(d_C_bias->data, sizeof(float) * H * R * Ds, s, "d_C_bias"));
    M3_TRY(memset_async(d_B_norm_w->data, sizeof(float) * Ds, s, "d_B_norm_w"));
    return memset_async(d_C_norm_w->data, sizeof(float) * Ds, s, "d_C_norm_w");
  }
  if (Bn > INT32_MAX || L > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "prologue backward: dimension too large");
  const size_t need = prologue_bwd_workspace_bytes(Bn, L, H, S, R, Ds);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15) != 0)
    return fail(M3_ERR_WORKSPACE, "prologue backward: workspace of " + std::to_string(need) + " bytes required");
  PrologueBwdParams p{};
  p.Bn = (int)Bn; p.L = (int)L; p.H = (int)H; p.P = (int)P; p.D = (int)Ds; p.R = (int)R; p.G = (int)G;
  p.S = (int)S; p.split = dims->rope_split; p.d_inner = (int)di; p.A_floor = dims->A_floor; p.eps = dims->norm_eps;
  p.zx = zxbcdt->data; p.s_zb = zxbcdt->stride[0]; p.s_zl = zxbcdt->stride[1];
  p.dzx = d_zxbcdt->data; p.s_dzb = d_zxbcdt->stride[0]; p.s_dzl = d_zxbcdt->stride[1];
  p.dt_bias = fptr<const float>(dt_bias);
  p.B_bias = fptr<const float>(B_bias); p.C_bias = fptr<const float>(C_bias);
  p.B_norm_w = fptr<const float>(B_norm_w); p.C_norm_w = fptr<const float>(C_norm_w);
  p.angles = fptr<const float>(angles); p.DT = fptr<const float>(DT);
  p.dBp = dB_proj->data; p.dCp = dC_proj->data;
  p.dADT = fptr<const float>(dADT); p.dDT = fptr<const float>(dDT); p.dtrap = fptr<const float>(dtrap);
  p.dB_bias = fptr<float>(d_B_bias); p.dC_bias = fptr<float>(d_C_bias);
  p.dB_norm_w = fptr<float>(d_B_norm_w); p.dC_norm_w = fptr<float>(d_C_norm_w);
  p.ddt_bias = fptr<float>(d_dt_bias);
  return launch_prologue_bwd(p, reinterpret_cast<float*>(workspace), zxbcdt->dtype, dB_proj->dtype, s);
}

int m3_silu_gate_bwd(const m3_tensor* y, const m3_tensor* z, const m3_tensor* dout, m3_tensor* dy, m3_tensor* dz,
                     void* stream) {
  if (!present(y) || y->ndim != 4) return fail(M3_ERR_INVALID_ARGUMENT, "y: expected (B, L, H, P)");
  const int64_t* sh = y->shape;
  const bool empty = sh[0] * sh[1] * sh[2] * sh[3] == 0;
  M3_TRY(check(y, "y", 4, sh, kAnyFloat, false, false, !empty));
  M3_TRY(check(z, "z", 4, sh, 1u << y->dtype, false, false, !empty));
  M3_TRY(check(dout, "dout", 4, sh, 1u << y->dtype, false, false, !empty));
  M3_TRY(check(dy, "dy", 4, sh, 1u << y->dtype, false, false, !empty));
  M3_TRY(check(dz, "dz", 4, sh, 1u << y->dtype, false, false, !empty));
  if (empty) return M3_OK;
  if (sh[1] > INT32_MAX || sh[2] > INT32_MAX || sh[3] > INT32_MAX)
    return fail(M3_ERR_UNSUPPORTED, "gate backward: dimension too large");
  GateBwdParams p{};
  p.rows = sh[0] * sh[1] * sh[2];
  p.L = (int)sh[1]; p.H = (int)sh[2]; p.P = (int)sh[3];
  p.y = y->data; p.sy = s3(y);
  p.z = z->data; p.sz = s3(z);
  p.dout = dout->data; p.sd = s3(dout);
  p.dy = dy->data; p.sdy = s3(dy);
  p.dz = dz->data; p.sdz = s3(dz);
  return launch_gate_bwd(p, y->dtype, z->dtype, dout->dtype, reinterpret_cast<cudaStream_t>(stream));
}

int m3_silu_gate(const m3_tensor* y, const m3_tensor* z, m3_tensor* out, void* stream) {
  if (!present(y) || y->ndim != 4) return fail(M3_ERR_INVALID_ARGUMENT, "y: expected (B, L, H, P)");
  const int64_t* sh = y->shape;
  const bool empty = sh[0] * sh[1] * sh[2] * sh[3] == 0;
  M3_TRY(check(y, "y", 4, sh, kAnyFloat, false, false, !empty));
  M3_TRY(check(z, "z", 4, sh, kAnyFloat, false, false, !empty));
  M3_TRY(check(out, "out", 4, sh, kAnyFloat, false, false, !empty));
  if (empty) return M3_OK;
  if (sh[1] > INT32_MAX || sh[2] > INT32_MAX || sh[3] > INT32_MAX) return fail(M3_ERR_UNSUPPORTED, "gate: dimension too large");
  GateParams p{};
  p.rows = sh[0] * sh[1] * sh[2]; p.L = (int)sh[1]; p.H = (int)sh[2]; p.P = (int)sh[3];
  p.y = y->data; p.sy = s3(y); p.z = z->data; p.sz = s3(z); p.out = out->data; p.so = s3(out);
  return launch_gate(p, y->dtype, z->dtype, out->dtype, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
