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
// Four tcgen05 MMAs per chunk (M = 128, fp32 accumulators in TMEM):
//   G    = C B^T        (128 x 128, K = D)   A, B: K-major smem tiles (TMA, 128B swizzle)
//   Y1   = C k_c^T      (128 x 64,  K = D)   B: k_c^T (bf16) in smem, MN-major
//   Y2   = G' X         (128 x 64,  K = Q)   A: G' (bf16) in TMEM, B: X tile MN-major
//   dK^T = B^T (w o X)  (128 x 64,  K = Q)   A: the B tile read MN-major
// G' is G masked to j <= i and scaled: G'_ij = G_ij e^{lambda_i - lambda_{j+1}} mu_j for
// j < i, G'_ii = beta_i G_ii + D (the D skip rides on the diagonal). The decay factor is
// split per 32-column block b as e^{lambda_i - lambda_{32b+1}} * e^{lambda_{32b+1} -
// lambda_{j+1}}; a block whose exponents could leave the fp32 range falls back to one exp2
// per element. Then y = e^{lambda} Y1 + Y2 and k^T = e^{lambda_Q} k^T + dK^T.
//
// Warp-specialised, persistent CTA (one per SM, 16 warps), walking its (b, h) units
// chunk by chunk. Shared-memory buffers are split by lifetime so that the large C / B
// tiles are released as soon as the early MMAs have read them:
//   C, B (64 KB)  2-stage ring; read by G, Y1 and dK, freed after Y1
//   X    (16 KB)  per chunk parity; read by the mask warpgroup (w o X) and by Y2
//   w o X (16 KB) per chunk parity;  k_c^T (16 KB) one buffer
// Roles (warp w issues from SM sub-partition w % 4, and TMEM lanes 32 (w % 4) .. +31 are
// the only ones it can reach):
//   warp 3      TMA producer (one thread polling the C/B ring and the X ring)
//   warp 1      tcgen05 MMA issuer (one thread polling three streams: G fed by the loads;
//               dK and Y1 fed by the mask and state warps; Y2 gated by the mask) and TMEM
//               owner (512 columns: per chunk parity G (128, G' packed in place) and Y2
//               (64); one Y1 (64) and one dK (64))
//   warps 4-7   even chunks, thread = row: the chunk's scalars (decay cumsum across the
//               four warps, mu, block factors, state weights) into a 4-slot ring, the
//               w o X rows for dK, G -> G' in TMEM (in place, packed bf16), then the
//               epilogue y = e^{lambda} Y1 + Y2 -> global (bf16)
//   warps 12-15 odd chunks: the same
//   warps 8-11  state: k^T (fp32, registers) <- decay k^T + dK^T and its bf16 copy for
//               the next Y1
//   warps 0, 2  idle
// All hand-offs are mbarriers; every wait is bounded (blocking waits by a poll count, the
// polling producer and issuer by an idle count), and on a timeout the kernel records an
// error and drains.
#include <cudaTypedefs.h>

#include <cstddef>

#include "m3_common.cuh"
#include "siso_chunk.cuh"
#include "sm100.cuh"

namespace m3 {
namespace {

using namespace sm100;

constexpr int Q = 128;
constexpr int kP = 64;
constexpr int kD = 128;
constexpr int kThreads = 512;
constexpr int NS = 2;    // C/B stages
constexpr int NSC = 4;   // scalar slots
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTileBytes = Q * 64 * 2;       // one SW128 tile: 128 rows x 128 B
constexpr uint32_t kCBBytes = 4 * kTileBytes;     // C(2) + B(2)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSafeExp2 = 120.f;
constexpr uint32_t kIdleLimit = 1u << 22;  // idle polls (~32 ns apart) before the producers give up

// TMEM columns: per chunk parity p G (128; G' packed into its first 64) and Y2 (64); one
// Y1 (64) and one dK (64), each consumed before the next chunk's is written.
__device__ __forceinline__ uint32_t col_g(int p) { return 128u * p; }
__device__ __forceinline__ uint32_t col_y2(int p) { return 256u + 64u * p; }
constexpr uint32_t kColY1 = 384u;
constexpr uint32_t kColDK = 448u;

struct __align__(16) ScalSlot {
  float colf[Q];      // e^{lambda_{32b+1} - lambda_{j+1}} mu_j (read as float4)
  float mu[Q];
  float lam2[Q + 1];  // lambda_i * log2(e)
  float decay_end;
  float dskip;        // D of the unit's head (added on the diagonal of G')
  float a0, g0;       // a, gamma of the unit's first row (initial state)
  int n;              // valid rows in the chunk
  int flags;          // bit0 first chunk of unit, bit1 last, bits 4..7 block b factorisable
};

// Values one warp of a mask warpgroup hands to the other three while the chunk's scalars
// are formed (index 4: the row after the chunk, t0 + Q).
struct WgXch {
  float tot[4];                          // warp sums of the decay exponents
  float a0[5], g0[5], adt0[5];           // a, gamma and ADT of each warp's first row
  float amax[5], pmax[5];                // max |ADT| and max ADT per warp
  float m[4], gmax[4], rm[4], ref[4];    // split-exponent bounds per 32-row block
};

struct __align__(1024) Smem {
  uint8_t cb[NS][4][kTileBytes];     // C(d 0-63), C(d 64-127), B(0-63), B(64-127)
  uint8_t xr[2][kTileBytes];         // x[t][p], per chunk parity
  uint8_t xs[2][kTileBytes];         // (w o x)[t][p], per chunk parity
  uint8_t kbuf[kTileBytes];          // k_c^T[d][p]
  ScalSlot sc[NSC];
  WgXch xch[2];                      // per mask warpgroup: cross-warp scalar exchange
  uint64_t wg_bar[2];                // per mask warpgroup: 128-thread barrier (bounded waits)
  uint64_t cb_full[NS], cb_empty[NS], x_full[2], x_empty[2];
  uint64_t xs_full[2], xs_empty[2], k_ready;
  uint64_t g_full[2], gp_ready[2], y_full[2], y2_free[2];
  uint64_t y1_full[2], y1_free, dk_full, dk_free;  // y1_full per parity: its two waiters
                                                   // are a chunk apart
                                                   // are a chunk apart
  uint64_t scal_full[NSC], scal_empty[NSC];
  uint32_t tmem_base;
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory budget");
static_assert(offsetof(ScalSlot, colf) % 16 == 0 && sizeof(ScalSlot) % 16 == 0 && offsetof(Smem, sc) % 16 == 0,
              "float4 reads of the column factors need 16-byte alignment");

__device__ int g_chunk_error;  // set when a bounded wait gives up

struct ChunkArgs {
  int Bn, L, H;
  int D;     // d_state: 128, or 64 (the second halves of the C / B tiles then stay zero)
  const float* adt; Str3 sadt;
  const float* dt; Str3 sdt;
  const float* trap; Str3 strap;
  const float* Dskip; int64_t sD;
  const float* h0;
  const float* bx0;
  __nv_bfloat16* y; Str3 sy;
  float* h_last;
  __nv_bfloat16* kst;  // optional: bf16 k_c^T of every chunk, [unit][chunk][d][p]
};

__device__ __forceinline__ uint32_t lane_addr(uint32_t base, int warp, uint32_t col) {
  return base + ((uint32_t)((warp & 3) * 32) << 16) + col;
}
// byte offset of (row r, element c) in a 128-row SW128 tile with 64 bf16 per row
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)r * 128u + ((((uint32_t)c >> 3) ^ ((uint32_t)r & 7u)) << 4) + (((uint32_t)c & 7u) << 1);
}

struct ChunkPos {
  int b, h, c, t0, n;
  bool first, last;
};
__device__ __forceinline__ ChunkPos chunk_pos(const ChunkArgs& a, int g, int nch) {
  ChunkPos q;
  const int k = g / nch;
  q.c = g - k * nch;
  const int u = blockIdx.x + k * gridDim.x;
  q.b = u / a.H;
  q.h = u - q.b * a.H;
  q.t0 = q.c * Q;
  q.n = min(Q, a.L - q.t0);
  q.first = q.c == 0;
  q.last = q.c == nch - 1;
  return q;
}

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity) {
  if (mbar_wait(bar, parity, 1u << 24)) return true;
  atomicExch(&g_chunk_error, 1);
  return false;
}

__device__ __forceinline__ float ld_scal(const float* p, const Str3& s, int b, int t, int h) {
  return p[(int64_t)b * s.b + (int64_t)t * s.l + (int64_t)h * s.h];
}


// xs[i][:] = w_i x[i][:] for row i; the row's eight 16-byte chunks are loaded before any
// store, so the loads are not held behind possibly aliasing stores
__device__ __forceinline__ void write_xs_row(const uint8_t* __restrict__ xt, uint8_t* __restrict__ xs, float wt,
                                             int i) {
  uint4 row[8];
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) row[cc] = *reinterpret_cast<const uint4*>(xt + sw128_off(i, 8 * cc));
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    const uint4 v = row[cc];
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv[e]));
      o[e] = pack_bf16(f.x * wt, f.y * wt);
    }
    *reinterpret_cast<uint4*>(xs + sw128_off(i, 8 * cc)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// bx_last[b][h][p][d] = x[b][L-1][h][p] B[b][L-1][h][d]: the carried B x of the last step,
// a function of the inputs alone, so it is written by this small kernel after the scan
// (block = (b, h) unit, thread = d) and the scan kernel does not carry it
__global__ void __launch_bounds__(128) bx_last_kernel(const __nv_bfloat16* __restrict__ x, Str3 sx,
                                                      const __nv_bfloat16* __restrict__ Bm, Str3 sB, int H, int L,
                                                      int D, float* __restrict__ bx_last) {
  const int u = blockIdx.x, b = u / H, h = u - b * H, d = threadIdx.x;
  if (d >= D) return;
  const int64_t t = L - 1;
  const float bd = __bfloat162float(Bm[(int64_t)b * sB.b + t * sB.l + (int64_t)h * sB.h + d]);
  const __nv_bfloat16* xr = x + (int64_t)b * sx.b + t * sx.l + (int64_t)h * sx.h;
  float* out = bx_last + (int64_t)u * kP * D + d;
#pragma unroll 4
  for (int pp = 0; pp < kP; ++pp) out[(int64_t)pp * D] = __bfloat162float(xr[pp]) * bd;
}

// ------------------------------------------------------------------------------------
// Per-chunk scalars, formed by the chunk's mask warpgroup: thread i owns row i. The raw
// ADT / DT / trap of a row are loaded two chunks ahead (the warpgroup's next chunk);
// thread Q-1 also loads row t0 + Q, whose a, gamma and ADT close the chunk.
// ------------------------------------------------------------------------------------
struct RawRow {
  float adt, dt, tr;     // row t0 + i
  float adtQ, dtQ, trQ;  // row t0 + Q (thread Q-1 only)
};

__device__ __forceinline__ void load_raw_row(const ChunkArgs& a, const ChunkPos& cp, int i, RawRow& r) {
  const int t = cp.t0 + i;
  const bool v = t < a.L;
  r.adt = v ? ld_scal(a.adt, a.sadt, cp.b, t, cp.h) : 0.f;
  r.dt = v ? ld_scal(a.dt, a.sdt, cp.b, t, cp.h) : 0.f;
  r.tr = v ? ld_scal(a.trap, a.strap, cp.b, t, cp.h) : 0.f;
  r.adtQ = r.dtQ = r.trQ = 0.f;
  if (i == Q - 1 && cp.t0 + Q < a.L) {
    r.adtQ = ld_scal(a.adt, a.sadt, cp.b, cp.t0 + Q, cp.h);
    r.dtQ = ld_scal(a.dt, a.sdt, cp.b, cp.t0 + Q, cp.h);
    r.trQ = ld_scal(a.trap, a.strap, cp.b, cp.t0 + Q, cp.h);
  }
}

// 128-thread barrier of one mask warpgroup on an mbarrier, with a bounded wait (a thread
// that gave up elsewhere cannot leave the others blocked for good).
__device__ __forceinline__ bool wg_sync(uint64_t* bar, uint32_t& phase) {
  mbar_arrive(bar);
  const bool ok = wait_or_flag(bar, phase);
  phase ^= 1u;
  return ok;
}

// Row i's values for the chunk: lambda_i (log2 units), beta_i and the state weight w_i in
// registers; colf, mu and lambda of every row in the scalar slot; the chunk's decay, the
// first row's a / gamma, and the split-exponent flags in the slot (thread 0). Returns false
// after a timed-out wait.
__device__ __forceinline__ bool scal_phase(const ChunkArgs& a, Smem& s, int g, int nch, int i, const RawRow& raw,
                                           uint32_t& wg_phase, float& li, float& bi, float& wk) {
  const int p = g & 1, q = g % NSC, lane = i & 31, wq = i >> 5;
  const ChunkPos cp = chunk_pos(a, g, nch);
  WgXch& X = s.xch[p];
  const bool v = cp.t0 + i < a.L;
  const float adt = raw.adt;
  const float tr = v ? sigmoidf_(raw.tr) : 0.f;
  const float be = raw.dt * (1.0f - tr) + 0.5f * raw.dt * tr;
  const float ga = 0.5f * raw.dt * tr;
  const float av = v ? exp2f(adt * kLog2e) : 0.f;
  // lambda: inclusive scan of (row 0 ? 0 : ADT_r), per warp here and across warps below
  float incl = (i == 0) ? 0.f : adt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  float amax = fabsf(adt), pmax = adt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, o));
  }
  if (lane == 31) X.tot[wq] = incl;
  if (lane == 0) {
    X.a0[wq] = av;
    X.g0[wq] = ga;
    X.adt0[wq] = adt;
    X.amax[wq] = amax;
    X.pmax[wq] = pmax;
  }
  if (i == Q - 1) {
    const bool vq = cp.t0 + Q < a.L;
    const float trq = vq ? sigmoidf_(raw.trQ) : 0.f;
    X.a0[4] = vq ? exp2f(raw.adtQ * kLog2e) : 0.f;
    X.g0[4] = 0.5f * raw.dtQ * trq;
    X.adt0[4] = raw.adtQ;
    X.amax[4] = fabsf(raw.adtQ);
    X.pmax[4] = raw.adtQ;
  }
  if (!wg_sync(&s.wg_bar[p], wg_phase)) return false;
  float pre = 0.f, total = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float tw = X.tot[w];
    if (w < wq) pre += tw;
    total += tw;
  }
  const float lam = (incl + pre) * kLog2e;
  const float lamQ = (total + X.adt0[4]) * kLog2e;
  // next-row values a_{i+1}, gamma_{i+1}, lambda_{i+1}
  float l1 = __shfl_down_sync(0xffffffffu, lam, 1);
  float a1 = __shfl_down_sync(0xffffffffu, av, 1);
  float g1 = __shfl_down_sync(0xffffffffu, ga, 1);
  if (lane == 31) {
    l1 = (pre + X.tot[wq] + X.adt0[wq + 1]) * kLog2e;  // row 32 (wq + 1), or t0 + Q
    a1 = X.a0[wq + 1];
    g1 = X.g0[wq + 1];
  }
  const float mu = a1 * be + g1;
  const float ref = __shfl_sync(0xffffffffu, lam, 1);  // lambda_{32 wq + 1}: block wq's reference
  float am = X.amax[4], pm = X.pmax[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    am = fmaxf(am, X.amax[w]);
    pm = fmaxf(pm, X.pmax[w]);
  }
  // Split-exponent safety. Column factors span at most 32 steps, row factors at most 128:
  // with |ADT| <= 2.5 and ADT <= 0.6 everywhere in the chunk every block is safe.
  const bool all_safe = am <= 2.5f && pm <= 0.6f;
  if (!wait_or_flag(&s.scal_empty[q], ((g / NSC) & 1) ^ 1)) return false;
  ScalSlot& sl = s.sc[q];
  sl.lam2[i] = lam;
  sl.mu[i] = mu;
  sl.colf[i] = exp2f(ref - l1) * mu;
  if (i == Q - 1) sl.lam2[Q] = lamQ;
  const int e = cp.n - 1;  // last valid row
  float lam_end = lamQ;
  if (cp.last) {  // uniform over the warpgroup
    if (!wg_sync(&s.wg_bar[p], wg_phase)) return false;
    lam_end = sl.lam2[e];
  }
  wk = !cp.last ? exp2f(lamQ - l1) * mu : (i < e ? exp2f(lam_end - l1) * mu : (i == e ? be : 0.f));
  int flags = (cp.first ? 1 : 0) | (cp.last ? 2 : 0);
  if (all_safe) {  // uniform over the warpgroup
    flags |= 0xF0;
  } else {
    // per block: |column exponents| bounded, and row factors bounded above
    float m = fabsf(ref - l1), gmax = lam, rm = lane >= 1 ? lam : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
      rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, o));
    }
    if (lane == 0) {
      X.m[wq] = m;
      X.gmax[wq] = gmax;
      X.rm[wq] = rm;
      X.ref[wq] = ref;
    }
    if (!wg_sync(&s.wg_bar[p], wg_phase)) return false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float mx = X.rm[k];
#pragma unroll
      for (int k2 = k + 1; k2 < 4; ++k2) mx = fmaxf(mx, X.gmax[k2]);
      if (X.m[k] <= kSafeExp2 && mx - X.ref[k] <= kSafeExp2) flags |= 1 << (4 + k);
    }
  }
  if (i == 0) {
    sl.decay_end = exp2f(lam_end);
    sl.dskip = a.Dskip[cp.h * a.sD];
    sl.a0 = av;
    sl.g0 = ga;
    sl.n = cp.n;
    sl.flags = flags;
  }
  mbar_arrive(&s.scal_full[q]);
  li = lam;
  bi = be;
  return true;
}

// ------------------------------------------------------------------------------------
// One 32-column block of row i: full (below the diagonal), diagonal and above-diagonal
// blocks share one code path through the column limit il = i - 32 qd. The factor of
// element j is the block's row factor times its column factor.
__device__ __forceinline__ void mask_block(const uint32_t (&r)[32], uint32_t (&pk)[16], int qd, int i,
                                           const ScalSlot& sl, float li, float bi, float dk) {
  const float rowf = exp2f(li - sl.lam2[32 * qd + 1]);
  const int il = i - 32 * qd;
  const float4* cf4 = reinterpret_cast<const float4*>(sl.colf + 32 * qd);
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 c = cf4[e4];
    const float cc[4] = {c.x * rowf, c.y * rowf, c.z * rowf, c.w * rowf};
    float v[4];
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int jl = 4 * e4 + z;
      const float gij = __uint_as_float(r[jl]);
      const float off = jl == il ? fmaf(gij, bi, dk) : 0.f;
      v[z] = jl < il ? gij * cc[z] : off;
    }
    pk[2 * e4] = pack_bf16(v[0], v[1]);
    pk[2 * e4 + 1] = pack_bf16(v[2], v[3]);
  }
}

// The same block when its split exponents could leave the fp32 range: one exp2 per
// element. Rare (chunks with |ADT| above 2.5 or ADT above 0.6), so it is kept out of line
// and rolled; it reloads G from TMEM itself, so no register array crosses the call.
__device__ __noinline__ void mask_block_exact(uint32_t taddr_in, uint32_t taddr_out, int qd, int i,
                                              const ScalSlot& sl, float li, float bi, float dk) {
  uint32_t r[32];
  tmem_ld32(taddr_in, r);
  tmem_wait_ld();
  uint32_t pk[16];
  const int il = i - 32 * qd;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float v[2];
#pragma unroll
    for (int z = 0; z < 2; ++z) {
      const int jl = 2 * e + z, j = 32 * qd + jl;
      const float gij = __uint_as_float(r[jl]);
      v[z] = jl < il ? gij * (exp2f(li - sl.lam2[j + 1]) * sl.mu[j]) : (jl == il ? fmaf(gij, bi, dk) : 0.f);
    }
    pk[e] = pack_bf16(v[0], v[1]);
  }
  tmem_st16(taddr_out, pk);
}


// y = e^{lambda} Y1 + Y2 of chunk g, thread = row i
__device__ __forceinline__ void epilogue(const ChunkArgs& a, Smem& s, uint32_t tbase, int g, int nch, int warp, int i) {
  const int p = g & 1;
  const ChunkPos cp = chunk_pos(a, g, nch);
  const ScalSlot& sl = s.sc[g % NSC];
  const float sc = exp2f(sl.lam2[i]);
  const bool valid = i < cp.n;
  uint4* dst = reinterpret_cast<uint4*>(a.y + (int64_t)cp.b * a.sy.b + (int64_t)(cp.t0 + (valid ? i : 0)) * a.sy.l +
                                        (int64_t)cp.h * a.sy.h);
#pragma unroll
  for (int qt = 0; qt < 4; ++qt) {
    uint32_t y1[16], y2[16];
    tmem_ld16(lane_addr(tbase, warp, kColY1 + 16 * qt), y1);
    tmem_ld16(lane_addr(tbase, warp, col_y2(p) + 16 * qt), y2);
    tmem_wait_ld();
    if (qt == 3) {
      tc_fence_before();
      mbar_arrive(&s.y1_free);
      mbar_arrive(&s.y2_free[p]);
    }
    uint32_t outp[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      outp[e] = pack_bf16(fmaf(sc, __uint_as_float(y1[2 * e]), __uint_as_float(y2[2 * e])),
                          fmaf(sc, __uint_as_float(y1[2 * e + 1]), __uint_as_float(y2[2 * e + 1])));
    if (valid && a.y) {
      dst[2 * qt] = make_uint4(outp[0], outp[1], outp[2], outp[3]);
      dst[2 * qt + 1] = make_uint4(outp[4], outp[5], outp[6], outp[7]);
    }
  }
}

// ------------------------------------------------------------------------------------
// One chunk per mask warpgroup iteration: the chunk's scalars (scal_phase), the w o X tile
// for dK, G -> G' (TMEM, in place), then the epilogue. Warps 4-7 take the even chunks,
// warps 12-15 the odd ones (each chunk parity has its own TMEM columns), so two chunks are
// in flight. Thread i owns row i. Warp r (rows 32r..32r+31) sees column blocks b < r
// entirely below the diagonal, block r on it and blocks b > r above it (zeros, not read).
// The packed bf16 G' of block b lands in columns 16b..16b+15, which this thread has
// already read.
// ------------------------------------------------------------------------------------
__device__ void mask_role(const ChunkArgs& a, Smem& s, uint32_t tbase, int G, int nch, int warp, int i, int parity) {
  const int wr = warp & 3;
  uint32_t wg_phase = 0;
  RawRow raw;
  float li = 0.f, bi = 0.f, wk = 0.f;  // row i's lambda, beta and state weight of chunk g
  if (parity < G) {
    load_raw_row(a, chunk_pos(a, parity, nch), i, raw);
    if (!scal_phase(a, s, parity, nch, i, raw, wg_phase, li, bi, wk)) return;
    if (parity + 2 < G) load_raw_row(a, chunk_pos(a, parity + 2, nch), i, raw);
  }
  for (int g = parity; g < G; g += 2) {
    const int p = g & 1, q = g % NSC;
    // (w o x) row i of this chunk, for dK(g)
    if (!wait_or_flag(&s.x_full[p], (g >> 1) & 1)) return;
    if (!wait_or_flag(&s.xs_empty[p], ((g >> 1) & 1) ^ 1)) return;
    write_xs_row(s.xr[p], s.xs[p], wk, i);
    fence_proxy_async_smem();
    mbar_arrive(&s.xs_full[p]);
    // every row's slot entries written
    if (!wait_or_flag(&s.scal_full[q], (g / NSC) & 1)) return;
    if (!wait_or_flag(&s.g_full[p], (g >> 1) & 1)) return;
    tc_fence_after();
    const ScalSlot& sl = s.sc[q];
    const float dk = sl.dskip;
    const int flags = sl.flags;
#pragma unroll 1
    for (int qd = 0; qd <= wr; ++qd) {
      const uint32_t tin = lane_addr(tbase, warp, col_g(p) + 32 * qd);
      const uint32_t tout = lane_addr(tbase, warp, col_g(p) + 16 * qd);
      if ((flags >> (4 + qd)) & 1) {
        uint32_t r[32];
        tmem_ld32(tin, r);
        tmem_wait_ld();
        uint32_t pk[16];
        mask_block(r, pk, qd, i, sl, li, bi, dk);
        tmem_st16(tout, pk);
      } else {
        mask_block_exact(tin, tout, qd, i, sl, li, bi, dk);
      }
    }
    {
      uint32_t z[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) z[e] = 0u;
#pragma unroll 1
      for (int qd = wr + 1; qd < 4; ++qd) tmem_st16(lane_addr(tbase, warp, col_g(p) + 16 * qd), z);
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&s.gp_ready[p]);
    // the scalars of this warpgroup's next chunk, while Y1 / Y2 of this one run (its slot
    // was released by chunk g - 2)
    float li_n = 0.f, bi_n = 0.f, wk_n = 0.f;
    if (g + 2 < G) {
      if (!scal_phase(a, s, g + 2, nch, i, raw, wg_phase, li_n, bi_n, wk_n)) return;
      if (g + 4 < G) load_raw_row(a, chunk_pos(a, g + 4, nch), i, raw);
    }
    // this chunk's outputs
    if (!wait_or_flag(&s.y_full[p], (g >> 1) & 1)) return;
    if (!wait_or_flag(&s.y1_full[p], (g >> 1) & 1)) return;
    tc_fence_after();
    epilogue(a, s, tbase, g, nch, warp, i);
    mbar_arrive(&s.scal_empty[q]);
    li = li_n;
    bi = bi_n;
    wk = wk_n;
  }
}

// ------------------------------------------------------------------------------------
// warps 8-11: w o X (thread = row t) and the carried state (thread = state row d)
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void write_kbuf(Smem& s, int d, const float (&k)[kP]) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    uint4 v;
    v.x = pack_bf16(k[8 * cc + 0], k[8 * cc + 1]);
    v.y = pack_bf16(k[8 * cc + 2], k[8 * cc + 3]);
    v.z = pack_bf16(k[8 * cc + 4], k[8 * cc + 5]);
    v.w = pack_bf16(k[8 * cc + 6], k[8 * cc + 7]);
    *reinterpret_cast<uint4*>(s.kbuf + sw128_off(d, 8 * cc)) = v;
  }
}

__device__ __forceinline__ void init_state(const ChunkArgs& a, const ChunkPos& cp, float a0, float g0, int d,
                                           float (&k)[kP]) {
  const int64_t sb = ((int64_t)cp.b * a.H + cp.h) * kP * a.D;
  const bool dv = d < a.D;
#pragma unroll
  for (int pp = 0; pp < kP; ++pp) {
    float v = 0.f;
    if (a.h0 && dv) v = a0 * a.h0[sb + (int64_t)pp * a.D + d];
    if (a.bx0 && dv) v = fmaf(g0, a.bx0[sb + (int64_t)pp * a.D + d], v);
    k[pp] = v;
  }
}

__device__ __forceinline__ void store_h_last(const ChunkArgs& a, int b, int h, int d, const float (&k)[kP]) {
  if (d >= a.D) return;
  const int64_t sb = ((int64_t)b * a.H + h) * kP * a.D;
  for (int pp = 0; pp < kP; ++pp) a.h_last[sb + (int64_t)pp * a.D + d] = k[pp];
}


// chunk-start state row d (bf16, plain [d][p] rows of 128 B) for the backward
__device__ __forceinline__ void store_kstate(const ChunkArgs& a, const ChunkPos& cp, int nch, int d,
                                             const float (&k)[kP]) {
  const int64_t u = (int64_t)cp.b * a.H + cp.h;
  uint4* dst = reinterpret_cast<uint4*>(a.kst + (((u * nch + cp.c) * kD) + d) * kP);
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
    dst[cc] = make_uint4(pack_bf16(k[8 * cc + 0], k[8 * cc + 1]), pack_bf16(k[8 * cc + 2], k[8 * cc + 3]),
                         pack_bf16(k[8 * cc + 4], k[8 * cc + 5]), pack_bf16(k[8 * cc + 6], k[8 * cc + 7]));
}

// k = dec * k + dK, read in quarters
__device__ __forceinline__ void add_dk(uint32_t tbase, int warp, float dec, float (&k)[kP]) {
#pragma unroll
  for (int qt = 0; qt < 4; ++qt) {
    uint32_t r[16];
    tmem_ld16(lane_addr(tbase, warp, kColDK + 16 * qt), r);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; ++e) k[16 * qt + e] = fmaf(dec, k[16 * qt + e], __uint_as_float(r[e]));
  }
}

__device__ void state_role(const ChunkArgs& a, Smem& s, uint32_t tbase, int G, int nch, int warp, int d) {
  float k[kP];
  float prev_dec = 0.f;
  int prev_b = 0, prev_h = 0, prev_last = 0;
  for (int g = 0; g <= G; ++g) {
    // (1) fold dK(g-1) into the carried state (or finish the unit that g-1 closed)
    if (g > 0) {
      if (!wait_or_flag(&s.dk_full, (g - 1) & 1)) return;
      tc_fence_after();
      add_dk(tbase, warp, prev_dec, k);
      if (prev_last && a.h_last) store_h_last(a, prev_b, prev_h, d, k);
      tc_fence_before();
      mbar_arrive(&s.dk_free);
    }
    if (g == G) break;
    const int q = g % NSC;
    const ChunkPos cp = chunk_pos(a, g, nch);
    if (!wait_or_flag(&s.scal_full[q], (g / NSC) & 1)) return;
    const ScalSlot& sl = s.sc[q];
    // (2) k_c for this chunk -> kbuf
    if (cp.first) {
      if (a.h0 || a.bx0) {
        init_state(a, cp, sl.a0, sl.g0, d, k);
      } else {
#pragma unroll
        for (int pp = 0; pp < kP; ++pp) k[pp] = 0.f;
      }
    }
    // kbuf's previous reader is Y1(g-1)
    if (g > 0 && !wait_or_flag(&s.y1_full[(g - 1) & 1], ((g - 1) >> 1) & 1)) return;
    write_kbuf(s, d, k);
    fence_proxy_async_smem();
    mbar_arrive(&s.k_ready);
    if (a.kst) store_kstate(a, cp, nch, d, k);
    prev_dec = sl.decay_end;
    prev_last = cp.last;
    prev_b = cp.b;
    prev_h = cp.h;
    mbar_arrive(&s.scal_empty[q]);
  }
}

// ------------------------------------------------------------------------------------
// warp 1, one thread: the tcgen05 MMAs, in three streams, each in chunk order:
//   G  : G(c) = C B^T                 needs the C/B stage, and Y2(c-2) issued (G'(c-2) read:
//                                     the tensor pipe runs MMAs in issue order)
//   K  : dK(c) = B^T (w o X), then Y1(c) = C k_c^T
//        dK(c) needs w o X(c), the dK columns read (dK(c-1) consumed) and G(c) issued;
//        Y1(c) needs k_c and the Y1 columns read (epilogue of c-1); Y1(c) is the last
//        reader of the stage, so its commit frees it
//   Y2 : Y2(c) = G' X                 needs the mask of c, X(c) and w o X(c), the Y2
//                                     columns of c-2 read
// A single thread issuing dependent integer work runs at instruction latency, so the issue
// path is kept short: shared-memory descriptors are formed once and advanced by constant
// offsets, every group is unrolled, and a stream's readiness conditions are polled only
// until each has been seen to hold (sticky bits, reset when the group is issued).
// ------------------------------------------------------------------------------------
template <int NKD>
__device__ __forceinline__ void mma_role(Smem& s, uint32_t tbase, int G) {
  constexpr uint32_t I_G = idesc_bf16_f32(128, 128, false, false);
  constexpr uint32_t I_Y = idesc_bf16_f32(128, 64, false, true);
  constexpr uint32_t I_DK = idesc_bf16_f32(128, 64, true, true);
  // K-major tiles: +32 B per K step of 16, +one tile per 64 K elements; MN-major tiles:
  // +2048 B (16 rows) per K step. Descriptor addresses are in 16-byte units.
  constexpr uint64_t kTileU = kTileBytes >> 4;
  const uint64_t dC0 = sdesc_sw128(smem_u32(s.cb[0][0]), 16, 1024), dC1 = sdesc_sw128(smem_u32(s.cb[1][0]), 16, 1024);
  const uint64_t dB0 = sdesc_sw128(smem_u32(s.cb[0][2]), 16, 1024), dB1 = sdesc_sw128(smem_u32(s.cb[1][2]), 16, 1024);
  const uint64_t dBt0 = sdesc_sw128(smem_u32(s.cb[0][2]), kTileBytes, 1024);
  const uint64_t dBt1 = sdesc_sw128(smem_u32(s.cb[1][2]), kTileBytes, 1024);
  const uint64_t dXs0 = sdesc_sw128(smem_u32(s.xs[0]), kTileBytes, 1024);
  const uint64_t dXs1 = sdesc_sw128(smem_u32(s.xs[1]), kTileBytes, 1024);
  const uint64_t dX0 = sdesc_sw128(smem_u32(s.xr[0]), kTileBytes, 1024);
  const uint64_t dX1 = sdesc_sw128(smem_u32(s.xr[1]), kTileBytes, 1024);
  const uint64_t dKb = sdesc_sw128(smem_u32(s.kbuf), kTileBytes, 1024);
  int cg = 0, ck = 0, sk = 0, gb = 0;
  uint32_t rk = 0, ry = 0;  // sticky readiness bits of the K and Y2 streams
  uint32_t idle = 0;
  while (cg < G || ck < G || gb < G) {
    bool moved = false;
    if (cg < G && gb >= cg - 1 && mbar_test(&s.cb_full[cg & 1], (cg >> 1) & 1)) {
      const int p = cg & 1;
      const uint64_t a0 = p ? dC1 : dC0, b0 = p ? dB1 : dB0;
      const uint32_t d = tbase + col_g(p);
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < NKD; ++kk) {
        const uint64_t off = (uint64_t)(kk >> 2) * kTileU + (uint64_t)(kk & 3) * 2u;
        mma_ss(d, a0 + off, b0 + off, I_G, kk > 0);
      }
      mma_commit(&s.g_full[p]);
      ++cg;
      moved = true;
    }
    if (ck < G) {
      const int p = ck & 1;
      if (sk == 0) {
        if (!(rk & 1) && mbar_test(&s.xs_full[p], (ck >> 1) & 1)) rk |= 1;
        if (!(rk & 2) && mbar_test(&s.dk_free, (ck & 1) ^ 1)) rk |= 2;
        if (rk == 3 && cg > ck) {
          const uint64_t a0 = p ? dBt1 : dBt0, b0 = p ? dXs1 : dXs0;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) mma_ss(tbase + kColDK, a0 + (uint64_t)kk * 128u, b0 + (uint64_t)kk * 128u, I_DK, kk > 0);
          mma_commit(&s.dk_full);
          mma_commit(&s.xs_empty[p]);
          sk = 1;
          rk = 0;
          moved = true;
        }
      } else {
        if (!(rk & 1) && mbar_test(&s.k_ready, ck & 1)) rk |= 1;
        if (!(rk & 2) && mbar_test(&s.y1_free, (ck & 1) ^ 1)) rk |= 2;
        if (rk == 3) {
          const uint64_t a0 = p ? dC1 : dC0;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < NKD; ++kk)
            mma_ss(tbase + kColY1, a0 + (uint64_t)(kk >> 2) * kTileU + (uint64_t)(kk & 3) * 2u, dKb + (uint64_t)kk * 128u,
                   I_Y, kk > 0);
          mma_commit(&s.y1_full[p]);
          mma_commit(&s.cb_empty[p]);  // last reader of this C/B stage
          sk = 0;
          rk = 0;
          ++ck;
          moved = true;
        }
      }
    }
    if (gb < G) {
      const int p = gb & 1;
      const uint32_t ph = (gb >> 1) & 1;
      // (w o X(gb) written implies the mask warps are past their wait on X(gb), so X(gb+2)
      // cannot land in this slot before that wait)
      if (!(ry & 1) && mbar_test(&s.gp_ready[p], ph)) ry |= 1;
      if (!(ry & 2) && mbar_test(&s.x_full[p], ph)) ry |= 2;
      if (!(ry & 4) && mbar_test(&s.xs_full[p], ph)) ry |= 4;
      if (!(ry & 8) && mbar_test(&s.y2_free[p], ph ^ 1)) ry |= 8;
      if (ry == 15) {
        const uint64_t b0 = p ? dX1 : dX0;
        const uint32_t d = tbase + col_y2(p), a = tbase + col_g(p);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_ts(d, a + 8u * kk, b0 + (uint64_t)kk * 128u, I_Y, kk > 0);
        mma_commit(&s.y_full[p]);
        mma_commit(&s.x_empty[p]);
        ry = 0;
        ++gb;
        moved = true;
      }
    }
    if (moved) {
      idle = 0;
    } else {
      if (++idle > kIdleLimit) {
        atomicExch(&g_chunk_error, 1);
        break;
      }
      __nanosleep(32);
    }
  }
}

// ------------------------------------------------------------------------------------
template <int NKD>
__global__ void __launch_bounds__(kThreads, 1)
siso_chunk_fwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_B,
                      const __grid_constant__ CUtensorMap tm_C, ChunkArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base, derived from smem_raw so that accesses stay shared-space
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nch = (a.L + Q - 1) / Q;
  const int units = a.Bn * a.H;
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int G = my_units * nch;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s.cb_full[i], 1);
      mbar_init(&s.cb_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.x_full[i], 1);
      mbar_init(&s.x_empty[i], 1);
      mbar_init(&s.xs_full[i], 128);
      mbar_init(&s.xs_empty[i], 1);
      mbar_init(&s.wg_bar[i], 128);
    }
    mbar_init(&s.k_ready, 128);
    mbar_init(&s.y1_full[0], 1);
    mbar_init(&s.y1_full[1], 1);
    mbar_init(&s.y1_free, 128);
    mbar_init(&s.dk_full, 1);
    mbar_init(&s.dk_free, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.g_full[i], 1);
      mbar_init(&s.gp_ready[i], 128);
      mbar_init(&s.y_full[i], 1);
      mbar_init(&s.y2_free[i], 128);
    }
    for (int i = 0; i < NSC; ++i) {
      mbar_init(&s.scal_full[i], 128);
      mbar_init(&s.scal_empty[i], 2 * 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (a.D < kD) {
    // d_state 64: the upper halves of the C / B tiles are never loaded; they read as zero
    for (int i = tid; i < NS * 2 * (int)(kTileBytes / 16); i += kThreads) {
      const int st = i / (2 * (kTileBytes / 16)), rem = i % (2 * (kTileBytes / 16));
      const int t = rem < (int)(kTileBytes / 16) ? 1 : 3, off = rem % (kTileBytes / 16);
      reinterpret_cast<uint4*>(s.cb[st][t])[off] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;

  if (warp == 3) {
    // one producer thread polling two independent streams: the C/B ring (waits for dK of
    // two chunks back) and the X ring (waits for Y2 of two back)
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_B);
      prefetch_tensormap(&tm_C);
      int gc = 0, gx = 0;
      uint32_t idle = 0;
      while (gc < G || gx < G) {
        bool moved = false;
        if (gc < G && mbar_test(&s.cb_empty[gc % NS], ((gc / NS) & 1) ^ 1)) {
          const int st = gc % NS;
          const ChunkPos cp = chunk_pos(a, gc, nch);
          mbar_expect_tx(&s.cb_full[st], a.D == kD ? kCBBytes : kCBBytes / 2);
          tma_load_4d(s.cb[st][0], &tm_C, &s.cb_full[st], 0, cp.h, cp.t0, cp.b);
          tma_load_4d(s.cb[st][2], &tm_B, &s.cb_full[st], 0, cp.h, cp.t0, cp.b);
          if (a.D == kD) {
            tma_load_4d(s.cb[st][1], &tm_C, &s.cb_full[st], 64, cp.h, cp.t0, cp.b);
            tma_load_4d(s.cb[st][3], &tm_B, &s.cb_full[st], 64, cp.h, cp.t0, cp.b);
          }
          ++gc;
          moved = true;
        }
        if (gx < G && mbar_test(&s.x_empty[gx & 1], ((gx >> 1) & 1) ^ 1)) {
          const int xi = gx & 1;
          const ChunkPos cp = chunk_pos(a, gx, nch);
          mbar_expect_tx(&s.x_full[xi], kTileBytes);
          tma_load_4d(s.xr[xi], &tm_x, &s.x_full[xi], 0, cp.h, cp.t0, cp.b);
          ++gx;
          moved = true;
        }
        if (moved) {
          idle = 0;
        } else {
          if (++idle > kIdleLimit) {
            atomicExch(&g_chunk_error, 1);
            break;
          }
          __nanosleep(32);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) mma_role<NKD>(s, tbase, G);
  } else if (warp >= 4 && warp < 8) {
    mask_role(a, s, tbase, G, nch, warp, tid - 128, 0);
  } else if (warp >= 8 && warp < 12) {
    state_role(a, s, tbase, G, nch, warp, tid - 256);
  } else if (warp >= 12) {
    mask_role(a, s, tbase, G, nch, warp, tid - 384, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 lookup_encode() {
  cudaDriverEntryPointQueryResult q;
  void* p = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  return nullptr;
}
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = lookup_encode();  // thread-safe static init
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

PFN_cuTensorMapEncodeTiled_v12000 chunk_encode_fn() { return get_encode(); }
int chunk_tmap_4d(CUtensorMap* m, const void* base, int64_t inner, int64_t H, int64_t L, int64_t Bn, const Str3& st) {
  return make_map(m, base, inner, H, L, Bn, st);
}
int chunk_sm_count() {
  int n = 0;
  return device_sm_count(&n) == M3_OK ? n : 148;
}

bool siso_chunk_supported(const SisoParams& p, int xdt, int bcdt) {
  if (xdt != M3_BFLOAT16 || bcdt != M3_BFLOAT16) return false;
  if (p.P != kP || (p.D != kD && p.D != 64)) return false;
  if (!aligned16(p.x) || !aligned16(p.Bm) || !aligned16(p.Cm) || !aligned16(p.y)) return false;
  if (!strides_ok(p.sx) || !strides_ok(p.sB) || !strides_ok(p.sC) || !strides_ok(p.sy)) return false;
  if (!get_encode()) return false;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

int chunk_error_word(bool reset, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_chunk_error, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_chunk_error, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("chunk error word: ") + cudaGetErrorString(e));
  *out = v;
  return M3_OK;
}

int launch_siso_fwd_chunked(const SisoParams& p, int xdt, int bcdt, cudaStream_t s) {
  (void)xdt; (void)bcdt;
  CUtensorMap mx, mb, mc;
  M3_TRY(make_map(&mx, p.x, p.P, p.H, p.L, p.Bn, p.sx));
  M3_TRY(make_map(&mb, p.Bm, p.D, p.H, p.L, p.Bn, p.sB));
  M3_TRY(make_map(&mc, p.Cm, p.D, p.H, p.L, p.Bn, p.sC));
  ChunkArgs a{};
  a.Bn = p.Bn; a.L = p.L; a.H = p.H;
  a.D = p.D;
  a.adt = p.adt; a.sadt = p.sadt;
  a.dt = p.dt; a.sdt = p.sdt;
  a.trap = p.trap; a.strap = p.strap;
  a.Dskip = p.Dskip; a.sD = p.sD;
  a.h0 = p.h0; a.bx0 = p.bx0;
  a.y = reinterpret_cast<__nv_bfloat16*>(p.y); a.sy = p.sy;
  a.h_last = p.h_last;
  a.kst = reinterpret_cast<__nv_bfloat16*>(p.kstates);
  const size_t smem = sizeof(Smem) + 1024;
  // the shared-memory opt-in belongs to each device's context: set it once per device
  static std::atomic<bool> smem_set[2][kMaxDevices];
  const void* kfn = p.D == kD ? reinterpret_cast<const void*>(siso_chunk_fwd_kernel<8>)
                              : reinterpret_cast<const void*>(siso_chunk_fwd_kernel<4>);
  M3_TRY(ensure_dynamic_smem(kfn, smem, smem_set[p.D == kD ? 0 : 1]));
  int sms = 0;
  M3_TRY(device_sm_count(&sms));
  const int units = p.Bn * p.H;
  const int grid = units < sms ? units : sms;
  if (p.D == kD) siso_chunk_fwd_kernel<8><<<grid, kThreads, smem, s>>>(mx, mb, mc, a);
  else siso_chunk_fwd_kernel<4><<<grid, kThreads, smem, s>>>(mx, mb, mc, a);
  M3_TRY(check_launch("siso_chunk_fwd_kernel"));
  if (!p.bx_last) return M3_OK;
  bx_last_kernel<<<units, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(p.x), p.sx,
                                       reinterpret_cast<const __nv_bfloat16*>(p.Bm), p.sB, p.H, p.L, p.D, p.bx_last);
  return check_launch("bx_last_kernel");
}

}  // namespace m3
