// Chunked SISO scan forward on the sm_100a tensor cores (tcgen05 + TMA), bf16 I/O,
// headdim P = 64, d_state D = 128. fp32 state and accumulators.
//
// Math. With u_t = x_t (x) B_t and the per-step coefficients of the reference loop
// (mamba3_ssm/ops.py:166-175: a = e^{ADT}, tr = sigmoid(trap), beta = dt(1-tr) + dt tr/2,
// gamma = dt tr/2), define the carried matrix k_t = a_t h_{t-1} + gamma_t u_{t-1}
// (so h_t = k_t + beta_t u_t). For a chunk of Q = 128 steps starting at t0, with
// lambda_i = sum_{r=1..i} ADT_{t0+r} (lambda_0 = 0) and mu_j = a_{j+1} beta_j + gamma_{j+1}:
//   y_i     = e^{lambda_i} C_i k_c + sum_{j<i} e^{lambda_i - lambda_{j+1}} mu_j (C_i.B_j) x_j
//             + (beta_i C_i.B_i + D) x_i
//   k_{c+1} = e^{lambda_Q} k_c + sum_j e^{lambda_Q - lambda_{j+1}} mu_j x_j B_j^T
// Four tcgen05 MMAs per chunk (M = 128, accumulators in TMEM):
//   G   = C B^T                  (128 x 128, K = D)        A, B: K-major smem (TMA, SW128)
//   Y1  = C k_c^T                (128 x 64,  K = D)        B: k_c^T in smem, MN-major
//   Y2  = G' X                   (128 x 64,  K = Q)        A: G' in TMEM (bf16), B: X MN-major
//   dK^T = B^T (w o X)           (128 x 64,  K = Q)        A: B tile read MN-major
// where G' = G masked and scaled on the CUDA cores (exp2 of lambda differences), then
// y = e^{lambda} Y1 + Y2 + D x and k^T = e^{lambda_Q} k^T + dK^T (fp32, in registers).
//
// One CTA (4 warps, 128 threads) owns one (b, h) and walks its chunks in order; thread i
// owns TMEM lane i (row i of G, Y1, Y2; state row d = i of k^T). Shared memory holds one
// 80 KB stage (C, B, X) plus a 16 KB buffer that carries k_c^T, then w o X, then k_{c+1}^T;
// two CTAs fit on one SM (TMEM 2 x 256 columns), so one CTA's math overlaps the other's
// loads. The next chunk's TMA is issued as soon as the last MMA reading the stage is done.
#include <cudaTypedefs.h>

#include "m3_common.cuh"
#include "siso_chunk.cuh"
#include "sm100.cuh"

namespace m3 {
namespace {

using namespace sm100;

constexpr int Q = 128;
constexpr int kP = 64;
constexpr int kD = 128;
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t COL_G = 0, COL_DK = 64, COL_Y1 = 128, COL_Y2 = 192;
constexpr uint32_t kTileBytes = Q * 64 * 2;           // one SW128 tile: 128 rows x 128 B
constexpr uint32_t kStageBytes = 5 * kTileBytes;      // C(2) + B(2) + X
constexpr float kLog2e = 1.4426950408889634f;

struct __align__(1024) Smem {
  uint8_t C[2][kTileBytes];   // C[t][d], d halves 0-63 / 64-127, K-major SW128
  uint8_t Bt[2][kTileBytes];  // B[t][d], same layout
  uint8_t X[kTileBytes];      // x[t][p], SW128
  uint8_t S[kTileBytes];      // k_c^T[d][p] -> (w o x)[t][p] -> k_{c+1}^T[d][p]
  float lam2[Q + 1];          // lambda_i * log2(e)
  float mu[Q];
  float beta[Q];
  float wgt[Q];               // state-update weights
  float av[Q + 1];            // a_t of rows t0 .. t0+Q
  float gv[Q + 1];            // gamma_t of rows t0 .. t0+Q
  float warp_sum[4];
  float adt_next;
  float decay_end;
  uint32_t tmem_base;
  uint64_t bar_tma;
  uint64_t bar_mma;
};

__device__ int g_chunk_error;  // set when a bounded wait gives up (diagnostics)

struct ChunkArgs {
  int Bn, L, H;
  const float* adt; Str3 sadt;
  const float* dt; Str3 sdt;
  const float* trap; Str3 strap;
  const float* Dskip; int64_t sD;
  const float* h0;
  const float* bx0;
  __nv_bfloat16* y; Str3 sy;
  float* h_last;
  float* bx_last;
};

__device__ __forceinline__ uint32_t tmem_lane_addr(uint32_t base, int warp, uint32_t col) {
  return base + ((uint32_t)(warp * 32) << 16) + col;
}

// element (row r, column c) of a 128-row SW128 tile of 64 bf16 per row
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)r * 128u + ((((uint32_t)c >> 3) ^ ((uint32_t)r & 7u)) << 4) + (((uint32_t)c & 7u) << 1);
}

__global__ void __launch_bounds__(kThreads, 2)
siso_chunk_fwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_B,
                      const __grid_constant__ CUtensorMap tm_C, ChunkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int L = a.L;
  const int nchunk = (L + Q - 1) / Q;

  if (tid == 0) {
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_B);
    prefetch_tensormap(&tm_C);
    mbar_init(&s.bar_tma, 1);
    mbar_init(&s.bar_mma, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  // initial carried state k_0^T[d][p] = a_0 h0[p][d] + gamma_0 bx0[p][d]   (thread = d)
  float kst[kP];
  {
    const int d = tid;
    float a0 = 0.f, g0 = 0.f;
    if (a.h0 || a.bx0) {
      a0 = expf(a.adt[(int64_t)b * a.sadt.b + (int64_t)h * a.sadt.h]);
      const float dt0 = a.dt[(int64_t)b * a.sdt.b + (int64_t)h * a.sdt.h];
      const float tr0 = sigmoidf_(a.trap[(int64_t)b * a.strap.b + (int64_t)h * a.strap.h]);
      g0 = 0.5f * dt0 * tr0;
    }
    const int64_t sb = ((int64_t)b * a.H + h) * kP * kD;
#pragma unroll
    for (int p = 0; p < kP; ++p) {
      float v = 0.f;
      if (a.h0) v = a0 * a.h0[sb + (int64_t)p * kD + d];
      if (a.bx0) v = fmaf(g0, a.bx0[sb + (int64_t)p * kD + d], v);
      kst[p] = v;
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 v;
      v.x = pack_bf16(kst[8 * c + 0], kst[8 * c + 1]);
      v.y = pack_bf16(kst[8 * c + 2], kst[8 * c + 3]);
      v.z = pack_bf16(kst[8 * c + 4], kst[8 * c + 5]);
      v.w = pack_bf16(kst[8 * c + 6], kst[8 * c + 7]);
      *reinterpret_cast<uint4*>(s.S + sw128_off(d, 8 * c)) = v;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;
  const float Dk = a.Dskip[h * a.sD];

  if (tid == 0) {
    mbar_expect_tx(&s.bar_tma, kStageBytes);
    tma_load_4d(s.C[0], &tm_C, &s.bar_tma, 0, h, 0, b);
    tma_load_4d(s.C[1], &tm_C, &s.bar_tma, 64, h, 0, b);
    tma_load_4d(s.Bt[0], &tm_B, &s.bar_tma, 0, h, 0, b);
    tma_load_4d(s.Bt[1], &tm_B, &s.bar_tma, 64, h, 0, b);
    tma_load_4d(s.X, &tm_x, &s.bar_tma, 0, h, 0, b);
  }
  constexpr uint32_t I_G = idesc_bf16_f32(128, 128, false, false);
  constexpr uint32_t I_Y1 = idesc_bf16_f32(128, 64, false, true);
  constexpr uint32_t I_Y2 = idesc_bf16_f32(128, 64, false, true);
  constexpr uint32_t I_DK = idesc_bf16_f32(128, 64, true, true);
  const uint32_t aC = smem_u32(s.C[0]), aB = smem_u32(s.Bt[0]), aX = smem_u32(s.X), aS = smem_u32(s.S);
  uint32_t tma_phase = 0, mma_phase = 0;
  bool ok = true;
  bool tma_pending = true;

  for (int c = 0; c < nchunk; ++c) {
    const int t0 = c * Q;
    const int n = min(Q, L - t0);
    const bool last = (c == nchunk - 1);
    // ---- per-row coefficients (overlap the TMA in flight)
    const int t = t0 + tid;
    float adt = 0.f, be = 0.f, ga = 0.f, av = 0.f;
    if (t < L) {
      adt = a.adt[(int64_t)b * a.sadt.b + (int64_t)t * a.sadt.l + (int64_t)h * a.sadt.h];
      const float dt = a.dt[(int64_t)b * a.sdt.b + (int64_t)t * a.sdt.l + (int64_t)h * a.sdt.h];
      const float tr = sigmoidf_(a.trap[(int64_t)b * a.strap.b + (int64_t)t * a.strap.l + (int64_t)h * a.strap.h]);
      be = dt * (1.0f - tr) + 0.5f * dt * tr;
      ga = 0.5f * dt * tr;
      av = expf(adt);
    }
    s.av[tid] = av;
    s.gv[tid] = ga;
    s.beta[tid] = be;
    float adt_next = 0.f;
    if (tid == 0) {
      const int tn = t0 + Q;
      float an = 0.f, gn = 0.f;
      if (tn < L) {
        adt_next = a.adt[(int64_t)b * a.sadt.b + (int64_t)tn * a.sadt.l + (int64_t)h * a.sadt.h];
        const float dt = a.dt[(int64_t)b * a.sdt.b + (int64_t)tn * a.sdt.l + (int64_t)h * a.sdt.h];
        const float tr = sigmoidf_(a.trap[(int64_t)b * a.strap.b + (int64_t)tn * a.strap.l + (int64_t)h * a.strap.h]);
        an = expf(adt_next);
        gn = 0.5f * dt * tr;
      }
      s.av[Q] = an;
      s.gv[Q] = gn;
      s.adt_next = adt_next;
    }
    // inclusive scan of v_i = (i == 0 ? 0 : ADT_{t0+i})
    float v = (tid == 0) ? 0.f : adt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) s.warp_sum[warp] = v;
    __syncthreads();
    float off = 0.f;
    for (int w = 0; w < warp; ++w) off += s.warp_sum[w];
    const float lam = v + off;
    s.lam2[tid] = lam * kLog2e;
    if (tid == Q - 1) s.lam2[Q] = (lam + s.adt_next) * kLog2e;
    __syncthreads();
    // mu_j and the state-update weights w_j (the last chunk produces h_{L-1} instead of k)
    {
      const int j = tid;
      const float muj = s.av[j + 1] * be + s.gv[j + 1];
      s.mu[j] = muj;
      float w;
      if (!last) {
        w = exp2f(s.lam2[Q] - s.lam2[j + 1]) * muj;
      } else {
        const int e = n - 1;
        w = (j < e) ? exp2f(s.lam2[e] - s.lam2[j + 1]) * muj : (j == e ? be : 0.f);
      }
      s.wgt[j] = w;
      if (tid == 0) s.decay_end = exp2f(last ? s.lam2[n - 1] : s.lam2[Q]);
    }
    // ---- wait for the stage, issue G and Y1
    ok = __syncthreads_and(ok && mbar_wait(&s.bar_tma, tma_phase));
    tma_phase ^= 1;
    tma_pending = false;
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t koff = (uint32_t)(kk >> 2) * kTileBytes + (uint32_t)(kk & 3) * 32u;
        const uint64_t dc = sdesc_sw128(aC + koff, 16, 1024);
        const uint64_t db = sdesc_sw128(aB + koff, 16, 1024);
        mma_ss(tbase + COL_G, dc, db, I_G, kk > 0);
        const uint64_t dk = sdesc_sw128(aS + (uint32_t)kk * 2048u, kTileBytes, 1024);
        mma_ss(tbase + COL_Y1, dc, dk, I_Y1, kk > 0);
      }
      mma_commit(&s.bar_mma);
    }
    __syncthreads();
    // my x row (kept for the epilogue) -- read before the stage is refilled
    uint32_t xr[32];
    {
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint4 q = *reinterpret_cast<const uint4*>(s.X + sw128_off(tid, 8 * cc));
        xr[4 * cc + 0] = q.x; xr[4 * cc + 1] = q.y; xr[4 * cc + 2] = q.z; xr[4 * cc + 3] = q.w;
      }
    }
    ok = __syncthreads_and(mbar_wait(&s.bar_mma, mma_phase));
    mma_phase ^= 1;
    if (!ok) break;
    tc_fence_after();
    // ---- w o X into S (k_c^T no longer needed: Y1 is done), mask G -> G' (bf16) in TMEM
    {
      const float wj = s.wgt[tid];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 q;
        uint32_t* qq = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 p2 = *reinterpret_cast<const __nv_bfloat162*>(&xr[4 * cc + e]);
          const float2 f = __bfloat1622float2(p2);
          qq[e] = pack_bf16(f.x * wj, f.y * wj);
        }
        *reinterpret_cast<uint4*>(s.S + sw128_off(tid, 8 * cc)) = q;
      }
    }
    {
      const int i = tid;
      const float li = s.lam2[i];
      const float bi = s.beta[i];
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t g[32];
        tmem_ld32(tmem_lane_addr(tbase, warp, COL_G + 32 * qd), g);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float vv[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            const int j = 32 * qd + 2 * e + z;
            const float gij = __uint_as_float(g[2 * e + z]);
            float r = 0.f;
            if (j < i) r = gij * exp2f(li - s.lam2[j + 1]) * s.mu[j];
            else if (j == i) r = gij * bi;
            vv[z] = r;
          }
          pk[e] = pack_bf16(vv[0], vv[1]);
        }
        tmem_st16(tmem_lane_addr(tbase, warp, COL_G + 16 * qd), pk);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- Y2 = G' X ; dK^T = B^T (w o X)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t dx = sdesc_sw128(aX + (uint32_t)kk * 2048u, kTileBytes, 1024);
        mma_ts(tbase + COL_Y2, tbase + COL_G + 8u * kk, dx, I_Y2, kk > 0);
        const uint64_t dbt = sdesc_sw128(aB + (uint32_t)kk * 2048u, kTileBytes, 1024);
        const uint64_t dxs = sdesc_sw128(aS + (uint32_t)kk * 2048u, kTileBytes, 1024);
        mma_ss(tbase + COL_DK, dbt, dxs, I_DK, kk > 0);
      }
      mma_commit(&s.bar_mma);
    }
    ok = __syncthreads_and(mbar_wait(&s.bar_mma, mma_phase));
    mma_phase ^= 1;
    if (!ok) break;
    tc_fence_after();
    // final B*x (last chunk only): bx_last[p][d] = x_{L-1}[p] * B_{L-1}[d], thread = d
    if (last && a.bx_last) {
      const int d = tid, e = n - 1;
      const float bd = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(
          s.Bt[d >> 6] + sw128_off(e, d & 63)));
      const int64_t sb = ((int64_t)b * a.H + h) * kP * kD;
      for (int p = 0; p < kP; ++p) {
        const float xv = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(s.X + sw128_off(e, p)));
        a.bx_last[sb + (int64_t)p * kD + d] = xv * bd;
      }
    }
    __syncthreads();
    // ---- stage free: prefetch the next chunk
    if (c + 1 < nchunk) tma_pending = true;
    if (tid == 0 && c + 1 < nchunk) {
      const int tn = t0 + Q;
      mbar_expect_tx(&s.bar_tma, kStageBytes);
      tma_load_4d(s.C[0], &tm_C, &s.bar_tma, 0, h, tn, b);
      tma_load_4d(s.C[1], &tm_C, &s.bar_tma, 64, h, tn, b);
      tma_load_4d(s.Bt[0], &tm_B, &s.bar_tma, 0, h, tn, b);
      tma_load_4d(s.Bt[1], &tm_B, &s.bar_tma, 64, h, tn, b);
      tma_load_4d(s.X, &tm_x, &s.bar_tma, 0, h, tn, b);
    }
    // ---- state update: k^T = decay * k^T + dK^T  (thread = d), bf16 copy into S
    {
      const float dec = s.decay_end;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
        tmem_ld32(tmem_lane_addr(tbase, warp, COL_DK + 32 * half), r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) kst[32 * half + e] = fmaf(dec, kst[32 * half + e], __uint_as_float(r[e]));
      }
      if (!last) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint4 q;
          q.x = pack_bf16(kst[8 * cc + 0], kst[8 * cc + 1]);
          q.y = pack_bf16(kst[8 * cc + 2], kst[8 * cc + 3]);
          q.z = pack_bf16(kst[8 * cc + 4], kst[8 * cc + 5]);
          q.w = pack_bf16(kst[8 * cc + 6], kst[8 * cc + 7]);
          *reinterpret_cast<uint4*>(s.S + sw128_off(tid, 8 * cc)) = q;
        }
      } else if (a.h_last) {
        const int64_t sb = ((int64_t)b * a.H + h) * kP * kD;
        for (int p = 0; p < kP; ++p) a.h_last[sb + (int64_t)p * kD + tid] = kst[p];
      }
    }
    // ---- y = e^{lambda} Y1 + Y2 + D x   (thread = row i)
    {
      const int i = tid;
      const float sc = exp2f(s.lam2[i]);
      const bool valid = (t0 + i) < L;
      __nv_bfloat16* yrow = a.y + (int64_t)b * a.sy.b + (int64_t)(t0 + i) * a.sy.l + (int64_t)h * a.sy.h;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t y1[32], y2[32];
        tmem_ld32(tmem_lane_addr(tbase, warp, COL_Y1 + 32 * half), y1);
        tmem_ld32(tmem_lane_addr(tbase, warp, COL_Y2 + 32 * half), y2);
        tmem_wait_ld();
        uint32_t outp[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 xf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xr[16 * half + e]));
          const float o0 = fmaf(sc, __uint_as_float(y1[2 * e]), __uint_as_float(y2[2 * e])) + Dk * xf.x;
          const float o1 = fmaf(sc, __uint_as_float(y1[2 * e + 1]), __uint_as_float(y2[2 * e + 1])) + Dk * xf.y;
          outp[e] = pack_bf16(o0, o1);
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(yrow + 32 * half);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(outp[4 * q4], outp[4 * q4 + 1], outp[4 * q4 + 2], outp[4 * q4 + 3]);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
  }
  if (!ok) {
    // a wait gave up: record it, let an in-flight stage load land (bounded), then release TMEM
    if (tid == 0) atomicExch(&g_chunk_error, 1);
    if (tma_pending) mbar_wait(&s.bar_tma, tma_phase, 1u << 20);
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 4-d bf16 map over (inner, H, L, B) with a (64, 1, 128, 1) box, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, int64_t inner, int64_t H, int64_t L, int64_t Bn, const Str3& st) {
  auto enc = get_encode();
  if (!enc) return fail(M3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)Bn};
  cuuint64_t strides[3] = {(cuuint64_t)st.h * 2, (cuuint64_t)st.l * 2, (cuuint64_t)st.b * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)Q, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M3_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return M3_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool strides_ok(const Str3& s) { return (s.b % 8 == 0) && (s.l % 8 == 0) && (s.h % 8 == 0); }

}  // namespace

bool siso_chunk_supported(const SisoParams& p, int xdt, int bcdt) {
  if (xdt != M3_BFLOAT16 || bcdt != M3_BFLOAT16) return false;
  if (p.P != kP || p.D != kD) return false;
  if (!aligned16(p.x) || !aligned16(p.Bm) || !aligned16(p.Cm) || !aligned16(p.y)) return false;
  if (!strides_ok(p.sx) || !strides_ok(p.sB) || !strides_ok(p.sC) || !strides_ok(p.sy)) return false;
  if (!get_encode()) return false;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

int launch_siso_fwd_chunked(const SisoParams& p, int xdt, int bcdt, cudaStream_t s) {
  (void)xdt; (void)bcdt;
  CUtensorMap mx, mb, mc;
  M3_TRY(make_map(&mx, p.x, p.P, p.H, p.L, p.Bn, p.sx));
  M3_TRY(make_map(&mb, p.Bm, p.D, p.H, p.L, p.Bn, p.sB));
  M3_TRY(make_map(&mc, p.Cm, p.D, p.H, p.L, p.Bn, p.sC));
  ChunkArgs a{};
  a.Bn = p.Bn; a.L = p.L; a.H = p.H;
  a.adt = p.adt; a.sadt = p.sadt;
  a.dt = p.dt; a.sdt = p.sdt;
  a.trap = p.trap; a.strap = p.strap;
  a.Dskip = p.Dskip; a.sD = p.sD;
  a.h0 = p.h0; a.bx0 = p.bx0;
  a.y = reinterpret_cast<__nv_bfloat16*>(p.y); a.sy = p.sy;
  a.h_last = p.h_last; a.bx_last = p.bx_last;
  const size_t smem = sizeof(Smem) + 1024;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(siso_chunk_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    attr_set = true;
  }
  siso_chunk_fwd_kernel<<<p.Bn * p.H, kThreads, smem, s>>>(mx, mb, mc, a);
  return check_launch("siso_chunk_fwd_kernel");
}

}  // namespace m3
