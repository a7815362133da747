// Fused single-token decode step of one Mamba3 mixer: everything Mamba3.step
// (mamba3_ssm/layer.py:298-371) does between in_proj and out_proj, in one kernel.
// Three layouts, chosen per shape:
//   MIMO, d_state and headdim 64 / 128: a warp per (b, h), lane l owning the column pairs
//     2l, 2l+1 (vector loads and stores, the RoPE partner in the same lane, one sincos per
//     pair for every rank);
//   other MIMO shapes with d_state 32 / 64 / 128: a warp per (b, h), lane = column;
//   SISO and the remaining MIMO shapes: a CTA per (b, h) with the prologue (split of the
//     in_proj row, softplus / clamp / sigmoid, RMSNorm + bias of B and C, angle update and
//     RoPE) in shared memory.
// Each streams the fp32 state once (read old state, write new state).
#include "m3_common.cuh"
#include "decode_step.cuh"

namespace m3 {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxRD = 2048;  // R * D

struct StepSmem {
  float Bp[kMaxRD];
  float Cp[kMaxRD];
  float ss[2 * 8];  // sum of squares per (B|C, r)
  float ang[256];
  float xr[8];
  float yr[8];
  float scal[4];    // DT, decay, tr, D
};

// Prologue shared by SISO and MIMO: fills Bp/Cp (R x D, normed + bias + RoPE) and the
// per-head scalars, writes angle_out.
template <typename TZ>
__device__ void step_prologue(const StepParams& a, int b, int h, StepSmem& s) {
  const int tid = threadIdx.x, D = a.D, R = a.R, G = a.G, H = a.H;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)b * a.s_row;
  const int g = (int)(((int64_t)h * G) / H);
  const int off_B = 2 * a.d_inner, off_C = off_B + D * G * R, off_dt = off_C + D * G * R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  if (tid == 0) {
    const float DT = softplusf_(to_f32(row[off_dt + h]) + a.dt_bias[h]);
    const float A = -fminf(softplusf_(to_f32(row[off_A + h])), -a.A_floor);  // layer.py:317
    s.scal[0] = DT;
    s.scal[1] = expf(A * DT);
    s.scal[2] = sigmoidf_(to_f32(row[off_tr + h]));
    s.scal[3] = a.Dskip[h];
  }
  for (int i = tid; i < R * D; i += blockDim.x) {
    const int r = i / D, d = i - r * D;
    s.Bp[i] = to_f32(row[off_B + (r * G + g) * D + d]);
    s.Cp[i] = to_f32(row[off_C + (r * G + g) * D + d]);
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  for (int j = warp; j < 2 * R; j += nw) {
    const float* v = (j < R) ? (s.Bp + j * D) : (s.Cp + (j - R) * D);
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) acc = fmaf(v[d], v[d], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s.ss[j] = acc;
  }
  const float DT = s.scal[0];
  for (int i = tid; i < a.S; i += blockDim.x) {
    const int64_t ai = ((int64_t)b * H + h) * a.S + i;
    const float an = a.angle_in[ai] + to_f32(row[off_ang + i]) * DT;
    s.ang[i] = an;
    a.angle_out[ai] = an;
  }
  __syncthreads();
  // normalise + bias, then rotate pairs of the first rope_split dims
  const int npair = a.split / 2;
  const int per_r = npair + (D - a.split);
  for (int i = tid; i < R * per_r; i += blockDim.x) {
    const int r = i / per_r, k = i - r * per_r;
    // RMSNorm (ops.py:102-104): x / sqrt(mean(x^2) + eps) * weight
    const float rb = sqrtf(s.ss[r] / D + a.eps);
    const float rc = sqrtf(s.ss[R + r] / D + a.eps);
    const float* bb = a.B_bias + ((int64_t)h * R + r) * D;
    const float* cb = a.C_bias + ((int64_t)h * R + r) * D;
    float* Bv = s.Bp + r * D;
    float* Cv = s.Cp + r * D;
    if (k < npair) {
      const int d0 = 2 * k, d1 = d0 + 1;
      const float b0 = Bv[d0] / rb * a.B_norm_w[d0] + bb[d0];
      const float b1 = Bv[d1] / rb * a.B_norm_w[d1] + bb[d1];
      const float c0 = Cv[d0] / rc * a.C_norm_w[d0] + cb[d0];
      const float c1 = Cv[d1] / rc * a.C_norm_w[d1] + cb[d1];
      float sn, cs;
      sincosf(s.ang[k], &sn, &cs);
      Bv[d0] = b0 * cs - b1 * sn;
      Bv[d1] = b0 * sn + b1 * cs;
      Cv[d0] = c0 * cs - c1 * sn;
      Cv[d1] = c0 * sn + c1 * cs;
    } else {
      const int d = a.split + (k - npair);
      Bv[d] = Bv[d] / rb * a.B_norm_w[d] + bb[d];
      Cv[d] = Cv[d] / rc * a.C_norm_w[d] + cb[d];
    }
  }
  __syncthreads();
}

template <typename TZ>
__global__ void __launch_bounds__(kThreads) siso_step_kernel(StepParams a) {
  __shared__ StepSmem s;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  step_prologue<TZ>(a, b, h, s);
  const int D = a.D, P = a.P, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)b * a.s_row;
  const float DT = s.scal[0], decay = s.scal[1], tr = s.scal[2], Dk = s.scal[3];
  const int LPR = D / 4 < 32 ? D / 4 : 32;  // lanes per state row (float4 each)
  const int RPW = 32 / LPR;                  // rows per warp pass
  const int li = lane % LPR, rw = lane / LPR;
  const int64_t base = ((int64_t)b * a.H + h) * P * D;
  for (int p0 = warp * RPW; p0 < P; p0 += (blockDim.x >> 5) * RPW) {
    const int p = p0 + rw;
    const bool pv = p < P;
    const float xv = pv ? to_f32(row[a.d_inner + h * P + p]) : 0.f;
    float acc = 0.f;
    for (int d4 = li; 4 * d4 < D; d4 += LPR) {
      const int d = 4 * d4;
      if (pv) {
        const float4 hs = *reinterpret_cast<const float4*>(a.ssm_in + base + (int64_t)p * D + d);
        const float4 bp = *reinterpret_cast<const float4*>(a.bx_in + base + (int64_t)p * D + d);
        const float hk[4] = {hs.x, hs.y, hs.z, hs.w};
        const float pk[4] = {bp.x, bp.y, bp.z, bp.w};
        float ho[4], bo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float bxc = xv * s.Bp[d + k];
          const float blend = (1.0f - tr) * bxc + tr * 0.5f * (bxc + pk[k]);  // layer.py:362
          ho[k] = decay * hk[k] + DT * blend;                                  // layer.py:363-366
          bo[k] = bxc;
          acc = fmaf(s.Cp[d + k], ho[k], acc);
        }
        *reinterpret_cast<float4*>(a.ssm_out + base + (int64_t)p * D + d) = make_float4(ho[0], ho[1], ho[2], ho[3]);
        *reinterpret_cast<float4*>(a.bx_out + base + (int64_t)p * D + d) = make_float4(bo[0], bo[1], bo[2], bo[3]);
      }
    }
    for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (pv && li == 0) {
      const float y = acc + Dk * xv;
      const float z = to_f32(row[h * P + p]);
      st(reinterpret_cast<TZ*>(a.y) + (int64_t)b * a.s_y + h * P + p, y * (z * sigmoidf_(z)));
    }
  }
}

template <typename TZ>
__global__ void __launch_bounds__(kThreads) mimo_step_kernel(StepParams a) {
  __shared__ StepSmem s;
  __shared__ float sx[1024];
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  step_prologue<TZ>(a, b, h, s);
  const int D = a.D, P = a.P, R = a.R, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)b * a.s_row;
  const float DT = s.scal[0], decay = s.scal[1], tr = s.scal[2], Dk = s.scal[3];
  for (int p = tid; p < P; p += blockDim.x) sx[p] = to_f32(row[a.d_inner + h * P + p]);
  __syncthreads();
  // xr = mimo_x x   (layer.py:346)
  for (int r = warp; r < R; r += blockDim.x >> 5) {
    float acc = 0.f;
    for (int p = lane; p < P; p += 32) acc = fmaf(sx[p], a.mimo_x[((int64_t)h * R + r) * P + p], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s.xr[r] = acc;
  }
  __syncthreads();
  // state update; y_r partial sums per warp, added in warp order (deterministic)
  __shared__ float yw[kThreads / 32][8];
  const int64_t base = ((int64_t)b * a.H + h) * D;
  float yacc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) yacc[r] = 0.f;
  for (int d = tid; d < D; d += blockDim.x) {
    float bxc = 0.f;
    for (int r = 0; r < R; ++r) bxc = fmaf(s.xr[r], s.Bp[r * D + d], bxc);  // layer.py:347
    const float blend = (1.0f - tr) * bxc + tr * 0.5f * (bxc + a.bx_in[base + d]);
    const float hn = decay * a.ssm_in[base + d] + DT * blend;
    a.ssm_out[base + d] = hn;
    a.bx_out[base + d] = bxc;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < R) yacc[r] = fmaf(s.Cp[r * D + d], hn, yacc[r]);
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < R) {
      float v = yacc[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) yw[warp][r] = v;
    }
  }
  __syncthreads();
  if (tid < R) {
    float v = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) v += yw[w][tid];
    s.yr[tid] = v;
  }
  __syncthreads();
  // y = mimo_o^T (y_r + D xr), gated (layer.py:352-356)
  for (int p = tid; p < P; p += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < R; ++r)
      acc = fmaf(s.yr[r] + Dk * s.xr[r], a.mimo_o[((int64_t)h * R + r) * P + p], acc);
    const float z = to_f32(row[h * P + p]);
    st(reinterpret_cast<TZ*>(a.y) + (int64_t)b * a.s_y + h * P + p, acc * (z * sigmoidf_(z)));
  }
}

// ------------------------------------------------------------------------------------
// MIMO step, one warp per (b, h): 8 batch rows of one head per CTA. The head's parameters
// (B/C bias and norm weights, mimo_x, mimo_o) are staged once per CTA in shared memory;
// every per-row reduction is a warp shuffle. Lane l holds d = 32 k + l of each rank's
// B / C row (DL = D / 32 values per rank) and p = l + 32 j of x. Templates: DL, RM (rank
// rounded up to a power of two) and PJ (headdim / 32 rounded up), so the register
// arrays match the shape. Used when D % 32 == 0, R * D <= 512 and P <= 256.
// ------------------------------------------------------------------------------------
constexpr int kWarpRows = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Warp totals of N values at once (N a power of two <= 32), every lane receiving all N.
// Each butterfly step halves the values a lane carries: the lane whose `o` bit is set
// keeps the upper half and the partner the lower half, so N values cost
// N-1 + log2(32/N) shuffles plus N broadcasts instead of 5 N. Value k ends in the lanes
// whose top log2(N) bits spell k, i.e. lane k * 32 / N.
template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N], int lane) {
  if constexpr (N == 1) {
    v[0] = warp_sum(v[0]);
  } else {
#pragma unroll
    for (int n = N, o = 16; n > 1; n >>= 1, o >>= 1) {
      const bool up = lane & o;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? v[i] : v[i + n / 2];
        const float keep = up ? v[i + n / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    float t = v[0];
#pragma unroll
    for (int o = 16 / N; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
#pragma unroll
    for (int k = 0; k < N; ++k) v[k] = __shfl_sync(0xffffffffu, t, k * (32 / N));
  }
}

template <typename TZ, int DL, int RM, int PJ>
__global__ void __launch_bounds__(32 * kWarpRows) mimo_step_warp_kernel(StepParams a) {
  constexpr int NK = RM * DL;  // B / C values per lane
  constexpr int D = 32 * DL;
  extern __shared__ float wsm[];
  const int P = a.P, R = a.R, G = a.G, H = a.H;
  float* sBb = wsm;            // (R, D)
  float* sCb = sBb + R * D;    // (R, D)
  float* sBw = sCb + R * D;    // (D)
  float* sCw = sBw + D;        // (D)
  float* smx = sCw + D;        // (R, P)
  float* smo = smx + R * P;    // (R, P)
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int b = blockIdx.y * kWarpRows + (threadIdx.x >> 5);
  const bool active = b < a.Bn;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)(active ? b : 0) * a.s_row;
  const int g = (int)(((int64_t)h * G) / H);
  const int off_B = 2 * a.d_inner, off_C = off_B + D * G * R, off_dt = off_C + D * G * R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  // this row's operands: all loads independent, issued before the parameter barrier
  float Bv[NK], Cv[NK], xv[PJ], zv[PJ], hs[DL], bp[DL];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int r = k / DL, d = 32 * (k % DL) + lane;
    const bool v = r < R;
    Bv[k] = v ? to_f32(row[off_B + (r * G + g) * D + d]) : 0.f;
    Cv[k] = v ? to_f32(row[off_C + (r * G + g) * D + d]) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < PJ; ++j) {
    const int p = lane + 32 * j;
    const bool v = p < P;
    xv[j] = v ? to_f32(row[a.d_inner + h * P + p]) : 0.f;
    zv[j] = v ? to_f32(row[h * P + p]) : 0.f;
  }
  const int64_t sbase = ((int64_t)(active ? b : 0) * H + h) * D;
#pragma unroll
  for (int k = 0; k < DL; ++k) {
    hs[k] = active ? a.ssm_in[sbase + 32 * k + lane] : 0.f;
    bp[k] = active ? a.bx_in[sbase + 32 * k + lane] : 0.f;
  }
  const float dt_raw = to_f32(row[off_dt + h]), A_raw = to_f32(row[off_A + h]), tr_raw = to_f32(row[off_tr + h]);
  const int npair = a.split / 2;
  const int64_t abase = ((int64_t)(active ? b : 0) * H + h) * a.S;
  float ang_in[DL], ang_raw[DL];
#pragma unroll
  for (int k = 0; k < DL; ++k) {
    const int i = (32 * k + lane) >> 1;  // angle of the pair holding d = 32 k + lane
    ang_in[k] = i < npair && active ? a.angle_in[abase + i] : 0.f;
    ang_raw[k] = i < npair ? to_f32(row[off_ang + i]) : 0.f;
  }
  // head parameters into shared memory
  for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
    sBb[i] = a.B_bias[(int64_t)h * R * D + i];
    sCb[i] = a.C_bias[(int64_t)h * R * D + i];
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    sBw[i] = a.B_norm_w[i];
    sCw[i] = a.C_norm_w[i];
  }
  for (int i = threadIdx.x; i < R * P; i += blockDim.x) {
    smx[i] = a.mimo_x[(int64_t)h * R * P + i];
    smo[i] = a.mimo_o[(int64_t)h * R * P + i];
  }
  __syncthreads();
  if (!active) return;

  const float DT = softplusf_(dt_raw + a.dt_bias[h]);
  const float A = -fminf(softplusf_(A_raw), -a.A_floor);  // layer.py:317
  const float decay = expf(A * DT);
  const float tr = sigmoidf_(tr_raw);
  const float Dk = a.Dskip[h];
  // RMSNorm per rank over D (ops.py:102-104), then bias
  float rB[RM], rC[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) { rB[r] = 0.f; rC[r] = 0.f; }
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    rB[k / DL] = fmaf(Bv[k], Bv[k], rB[k / DL]);
    rC[k / DL] = fmaf(Cv[k], Cv[k], rC[k / DL]);
  }
  {
    float ss[2 * RM];
#pragma unroll
    for (int r = 0; r < RM; ++r) { ss[r] = rB[r]; ss[RM + r] = rC[r]; }
    warp_sum_n<2 * RM>(ss, lane);
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      rB[r] = rsqrtf(ss[r] / D + a.eps);
      rC[r] = rsqrtf(ss[RM + r] / D + a.eps);
    }
  }
  // RoPE angle of this lane's pairs: one sincos per d slot, shared by every rank
  float sn[DL], cs[DL];
#pragma unroll
  for (int k = 0; k < DL; ++k) {
    const float an = ang_in[k] + ang_raw[k] * DT;
    sincosf(an, &sn[k], &cs[k]);
  }
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int r = k / DL, kd = k % DL, d = 32 * kd + lane;
    if (r < R) {
      Bv[k] = Bv[k] * rB[r] * sBw[d] + sBb[r * D + d];
      Cv[k] = Cv[k] * rC[r] * sCw[d] + sCb[r * D + d];
    }
    // pairs (2i, 2i+1), i < split / 2: the partner sits in lane ^ 1
    const float pb = __shfl_xor_sync(0xffffffffu, Bv[k], 1);
    const float pc = __shfl_xor_sync(0xffffffffu, Cv[k], 1);
    if ((d >> 1) < npair) {
      if (lane & 1) {
        Bv[k] = pb * sn[kd] + Bv[k] * cs[kd];
        Cv[k] = pc * sn[kd] + Cv[k] * cs[kd];
      } else {
        Bv[k] = Bv[k] * cs[kd] - pb * sn[kd];
        Cv[k] = Cv[k] * cs[kd] - pc * sn[kd];
      }
    }
  }
  // angle update (layer.py:331-332); angle_out may alias angle_in, which every lane has read
  __syncwarp();
  for (int i = lane; i < a.S; i += 32) a.angle_out[abase + i] = a.angle_in[abase + i] + to_f32(row[off_ang + i]) * DT;
  // xr = mimo_x x (layer.py:346)
  float xr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < PJ; ++j) {
      const int p = lane + 32 * j;
      if (r < R && p < P) acc = fmaf(smx[r * P + p], xv[j], acc);
    }
    xr[r] = acc;
  }
  warp_sum_n<RM>(xr, lane);
  // state update (layer.py:347-351) and y_r = C_r h
  float yr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) yr[r] = 0.f;
#pragma unroll
  for (int k = 0; k < DL; ++k) {
    float bxc = 0.f;
#pragma unroll
    for (int r = 0; r < RM; ++r) bxc = fmaf(xr[r], Bv[r * DL + k], bxc);  // zero rows beyond R
    const float blend = (1.0f - tr) * bxc + tr * 0.5f * (bxc + bp[k]);
    const float hn = decay * hs[k] + DT * blend;
    a.ssm_out[sbase + 32 * k + lane] = hn;
    a.bx_out[sbase + 32 * k + lane] = bxc;
#pragma unroll
    for (int r = 0; r < RM; ++r) yr[r] = fmaf(Cv[r * DL + k], hn, yr[r]);
  }
  warp_sum_n<RM>(yr, lane);
#pragma unroll
  for (int r = 0; r < RM; ++r) yr[r] += Dk * xr[r];
  // y = mimo_o^T (y_r + D xr), gated by silu(z) (layer.py:352-356)
  TZ* yo = reinterpret_cast<TZ*>(a.y) + (int64_t)b * a.s_y + h * P;
#pragma unroll
  for (int j = 0; j < PJ; ++j) {
    const int p = lane + 32 * j;
    if (p < P) {
      float acc = 0.f;
#pragma unroll
      for (int r = 0; r < RM; ++r)
        if (r < R) acc = fmaf(yr[r], smo[r * P + p], acc);
      const float z = zv[j];
      st(yo + p, acc * (z * sigmoidf_(z)));
    }
  }
}

// ------------------------------------------------------------------------------------
// Lean warp-per-(b, h) MIMO step for d_state 64 / 128 and headdim 64 / 128 (the shapes of
// the LM presets): lane l owns the column pairs d = 2l, 2l+1 (+ 64 for d_state 128) and
// p = 2l, 2l+1 (+ 64), so every load and store is a 4- or 8-byte vector, the RoPE partner
// of a pair is in the same lane (no shuffles), and one sincos per lane and d-slot serves
// every rank. Head parameters are read through the read-only cache (the CTA's 8 warps
// are 8 batch rows of one head).
// ------------------------------------------------------------------------------------
template <typename T> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 ld(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float2 v) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
  }
};
template <> struct Pair<__half> {
  static __device__ __forceinline__ float2 ld(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
  }
  static __device__ __forceinline__ void st(__half* p, float2 v) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v.x, v.y);
  }
};
__device__ __forceinline__ float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }


template <typename TZ, int DP, int PP, int RM>
__global__ void __launch_bounds__(32 * kWarpRows) mimo_step_pair_kernel(StepParams a) {
  constexpr int D = 64 * DP, P = 64 * PP;
  const int R = a.R, G = a.G, H = a.H, S = a.S;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int b = blockIdx.y * kWarpRows + (threadIdx.x >> 5);
  if (b >= a.Bn) return;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)b * a.s_row;
  const int g = (int)(((int64_t)h * G) / H);
  const int off_B = 2 * a.d_inner, off_C = off_B + D * G * R, off_dt = off_C + D * G * R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  // this row's operands (all loads independent)
  float2 Bv[RM][DP], Cv[RM][DP], xv[PP], zv[PP], hs[DP], bp[DP];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int q = 0; q < DP; ++q) {
      const int d0 = 2 * lane + 64 * q;
      Bv[r][q] = r < R ? Pair<TZ>::ld(row + off_B + (r * G + g) * D + d0) : make_float2(0.f, 0.f);
      Cv[r][q] = r < R ? Pair<TZ>::ld(row + off_C + (r * G + g) * D + d0) : make_float2(0.f, 0.f);
    }
#pragma unroll
  for (int q = 0; q < PP; ++q) {
    const int p0 = 2 * lane + 64 * q;
    xv[q] = Pair<TZ>::ld(row + a.d_inner + h * P + p0);
    zv[q] = Pair<TZ>::ld(row + h * P + p0);
  }
  const int64_t sbase = ((int64_t)b * H + h) * D;
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    hs[q] = *reinterpret_cast<const float2*>(a.ssm_in + sbase + 2 * lane + 64 * q);
    bp[q] = *reinterpret_cast<const float2*>(a.bx_in + sbase + 2 * lane + 64 * q);
  }
  const int64_t abase = ((int64_t)b * H + h) * S;
  float ang_in[DP], ang_raw[DP];
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int i = lane + 32 * q;  // the pair's angle
    ang_in[q] = i < S ? a.angle_in[abase + i] : 0.f;
    ang_raw[q] = i < S ? to_f32(row[off_ang + i]) : 0.f;
  }
  const float dt_raw = to_f32(row[off_dt + h]), A_raw = to_f32(row[off_A + h]), tr_raw = to_f32(row[off_tr + h]);

  const float DT = softplusf_(dt_raw + __ldg(a.dt_bias + h));
  const float A = -fminf(softplusf_(A_raw), -a.A_floor);  // layer.py:317
  const float decay = expf(A * DT);
  const float tr = fast_sigmoid(tr_raw);
  const float Dk = __ldg(a.Dskip + h);
  // RMSNorm per rank over D (ops.py:102-104)
  float ss[2 * RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    float sb = 0.f, sc = 0.f;
#pragma unroll
    for (int q = 0; q < DP; ++q) {
      sb = fmaf(Bv[r][q].x, Bv[r][q].x, fmaf(Bv[r][q].y, Bv[r][q].y, sb));
      sc = fmaf(Cv[r][q].x, Cv[r][q].x, fmaf(Cv[r][q].y, Cv[r][q].y, sc));
    }
    ss[r] = sb;
    ss[RM + r] = sc;
  }
  warp_sum_n<2 * RM>(ss, lane);
  // angle update (layer.py:331-332) and the RoPE rotation of each owned pair
  float sn[DP], cs[DP];
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int i = lane + 32 * q;
    const float an = ang_in[q] + ang_raw[q] * DT;
    sincos_reduced(an, &sn[q], &cs[q]);
    if (i < S) a.angle_out[abase + i] = an;  // angle_out may alias angle_in: same lane, read above
  }
  // normalise, weight, bias, rotate
  const float* Bb = a.B_bias + (int64_t)h * R * D;
  const float* Cb = a.C_bias + (int64_t)h * R * D;
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int d0 = 2 * lane + 64 * q;
    const bool rot = lane + 32 * q < S;
    const float2 wb = ldg2(a.B_norm_w + d0), wc = ldg2(a.C_norm_w + d0);
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      if (r >= R) break;
      const float nb = rsqrtf(ss[r] * (1.0f / D) + a.eps), nc = rsqrtf(ss[RM + r] * (1.0f / D) + a.eps);
      const float2 bb = ldg2(Bb + r * D + d0), cb = ldg2(Cb + r * D + d0);
      float b0 = fmaf(Bv[r][q].x * nb, wb.x, bb.x), b1 = fmaf(Bv[r][q].y * nb, wb.y, bb.y);
      float c0 = fmaf(Cv[r][q].x * nc, wc.x, cb.x), c1 = fmaf(Cv[r][q].y * nc, wc.y, cb.y);
      if (rot) {
        const float rb0 = b0 * cs[q] - b1 * sn[q], rb1 = b0 * sn[q] + b1 * cs[q];
        const float rc0 = c0 * cs[q] - c1 * sn[q], rc1 = c0 * sn[q] + c1 * cs[q];
        b0 = rb0; b1 = rb1; c0 = rc0; c1 = rc1;
      }
      Bv[r][q] = make_float2(b0, b1);
      Cv[r][q] = make_float2(c0, c1);
    }
  }
  // xr = mimo_x x (layer.py:346)
  const float* mx = a.mimo_x + (int64_t)h * R * P;
  const float* mo = a.mimo_o + (int64_t)h * R * P;
  float xr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    float acc = 0.f;
    if (r < R) {
#pragma unroll
      for (int q = 0; q < PP; ++q) {
        const float2 m = ldg2(mx + r * P + 2 * lane + 64 * q);
        acc = fmaf(m.x, xv[q].x, fmaf(m.y, xv[q].y, acc));
      }
    }
    xr[r] = acc;
  }
  warp_sum_n<RM>(xr, lane);
  // state update (layer.py:347-351) and y_r = C_r h
  float yr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) yr[r] = 0.f;
  const float w1 = 1.0f - 0.5f * tr, w2 = 0.5f * tr;  // blend = w1 bx + w2 bx_prev
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    float2 bxc = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RM; ++r) {  // zero B rows beyond R
      bxc.x = fmaf(xr[r], Bv[r][q].x, bxc.x);
      bxc.y = fmaf(xr[r], Bv[r][q].y, bxc.y);
    }
    float2 hn;
    hn.x = fmaf(decay, hs[q].x, DT * fmaf(w1, bxc.x, w2 * bp[q].x));
    hn.y = fmaf(decay, hs[q].y, DT * fmaf(w1, bxc.y, w2 * bp[q].y));
    *reinterpret_cast<float2*>(a.ssm_out + sbase + 2 * lane + 64 * q) = hn;
    *reinterpret_cast<float2*>(a.bx_out + sbase + 2 * lane + 64 * q) = bxc;
#pragma unroll
    for (int r = 0; r < RM; ++r) yr[r] = fmaf(Cv[r][q].x, hn.x, fmaf(Cv[r][q].y, hn.y, yr[r]));
  }
  warp_sum_n<RM>(yr, lane);
  // y = mimo_o^T (y_r + D xr), gated by silu(z) (layer.py:352-356)
  TZ* yo = reinterpret_cast<TZ*>(a.y) + (int64_t)b * a.s_y + h * P;
#pragma unroll
  for (int q = 0; q < PP; ++q) {
    const int p0 = 2 * lane + 64 * q;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      if (r >= R) break;
      const float2 m = ldg2(mo + r * P + p0);
      const float yv = fmaf(Dk, xr[r], yr[r]);
      acc.x = fmaf(yv, m.x, acc.x);
      acc.y = fmaf(yv, m.y, acc.y);
    }
    const float2 z = zv[q];
    Pair<TZ>::st(yo + p0, make_float2(acc.x * (z.x * fast_sigmoid(z.x)), acc.y * (z.y * fast_sigmoid(z.y))));
  }
}

// ------------------------------------------------------------------------------------
// The same vector-pair layout with one B / C group (G = 1): a CTA takes one batch row and 8
// consecutive heads (warp = head). Work every head of the row shares is done once per CTA:
// warp 0 computes the RMSNorm factors of the row's B and C ranks and, on lanes 0-7, the
// per-head scalars (two softplus, decay, trapezoid weights), handed over through shared
// memory. RoPE is applied once per state pair instead of once per rank: the rotation is
// linear and the same for every rank, so Bx = rot(sum_r xr_r b_r) and
// C_r . h = c_r . rot^T(h), with b_r, c_r the normalised, weighted, biased rows.
// ------------------------------------------------------------------------------------
template <typename TZ, int DP, int PP, int RM>
__global__ void __launch_bounds__(32 * kWarpRows) mimo_step_row_kernel(StepParams a) {
  constexpr int D = 64 * DP, P = 64 * PP;
  const int R = a.R, H = a.H, S = a.S;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int h = blockIdx.x * kWarpRows + warp;
  if (h >= H) return;
  const int hh = h;
  const TZ* row = reinterpret_cast<const TZ*>(a.zxbcdt) + (int64_t)b * a.s_row;
  const int off_B = 2 * a.d_inner, off_C = off_B + D * R, off_dt = off_C + D * R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  // this (row, head)'s operands (all loads independent)
  float2 Bv[RM][DP], Cv[RM][DP], xv[PP], zv[PP], hs[DP], bp[DP];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int q = 0; q < DP; ++q) {
      const int d0 = 2 * lane + 64 * q;
      Bv[r][q] = r < R ? Pair<TZ>::ld(row + off_B + r * D + d0) : make_float2(0.f, 0.f);
      Cv[r][q] = r < R ? Pair<TZ>::ld(row + off_C + r * D + d0) : make_float2(0.f, 0.f);
    }
#pragma unroll
  for (int q = 0; q < PP; ++q) {
    const int p0 = 2 * lane + 64 * q;
    xv[q] = Pair<TZ>::ld(row + a.d_inner + hh * P + p0);
    zv[q] = Pair<TZ>::ld(row + hh * P + p0);
  }
  const int64_t sbase = ((int64_t)b * H + hh) * D;
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    hs[q] = *reinterpret_cast<const float2*>(a.ssm_in + sbase + 2 * lane + 64 * q);
    bp[q] = *reinterpret_cast<const float2*>(a.bx_in + sbase + 2 * lane + 64 * q);
  }
  const int64_t abase = ((int64_t)b * H + hh) * S;
  float ang_in[DP], ang_raw[DP];
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int i = lane + 32 * q;
    ang_in[q] = i < S ? a.angle_in[abase + i] : 0.f;
    ang_raw[q] = i < S ? to_f32(row[off_ang + i]) : 0.f;
  }
  // the row's norm factors, formed by every warp from the B / C rows it holds (no barrier:
  // the CTA's warps never wait on one another)
  float nrm[2 * RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    float sb = 0.f, sc = 0.f;
#pragma unroll
    for (int q = 0; q < DP; ++q) {
      sb = fmaf(Bv[r][q].x, Bv[r][q].x, fmaf(Bv[r][q].y, Bv[r][q].y, sb));
      sc = fmaf(Cv[r][q].x, Cv[r][q].x, fmaf(Cv[r][q].y, Cv[r][q].y, sc));
    }
    nrm[r] = sb;
    nrm[RM + r] = sc;
  }
  warp_sum_n<2 * RM>(nrm, lane);
#pragma unroll
  for (int k = 0; k < 2 * RM; ++k) nrm[k] = rsqrtf(nrm[k] * (1.0f / D) + a.eps);
  // this head's scalars (every lane, from broadcast loads)
  const float DT = softplusf_(to_f32(row[off_dt + hh]) + __ldg(a.dt_bias + hh));
  const float A = -fminf(softplusf_(to_f32(row[off_A + hh])), -a.A_floor);  // layer.py:317
  const float tr = fast_sigmoid(to_f32(row[off_tr + hh]));
  const float decay = expf(A * DT), w1 = 1.0f - 0.5f * tr, w2 = 0.5f * tr, Dk = __ldg(a.Dskip + hh);
  // angle update (layer.py:331-332); angle_out may alias angle_in: same lane, read above
  float sn[DP], cs[DP];
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int i = lane + 32 * q;
    const float an = ang_in[q] + ang_raw[q] * DT;
    sincos_reduced(an, &sn[q], &cs[q]);
    if (i < S) a.angle_out[abase + i] = an;
  }
  // normalise, weight, bias (the rotation comes once per pair below)
  const float* Bb = a.B_bias + (int64_t)h * R * D;
  const float* Cb = a.C_bias + (int64_t)h * R * D;
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const int d0 = 2 * lane + 64 * q;
    const float2 wb = ldg2(a.B_norm_w + d0), wc = ldg2(a.C_norm_w + d0);
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      if (r >= R) break;
      const float nb = nrm[r], nc = nrm[RM + r];
      const float2 bb = ldg2(Bb + r * D + d0), cb = ldg2(Cb + r * D + d0);
      Bv[r][q] = make_float2(fmaf(Bv[r][q].x * nb, wb.x, bb.x), fmaf(Bv[r][q].y * nb, wb.y, bb.y));
      Cv[r][q] = make_float2(fmaf(Cv[r][q].x * nc, wc.x, cb.x), fmaf(Cv[r][q].y * nc, wc.y, cb.y));
    }
  }
  // xr = mimo_x x (layer.py:346)
  const float* mx = a.mimo_x + (int64_t)h * R * P;
  const float* mo = a.mimo_o + (int64_t)h * R * P;
  float xr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    float acc = 0.f;
    if (r < R) {
#pragma unroll
      for (int q = 0; q < PP; ++q) {
        const float2 m = ldg2(mx + r * P + 2 * lane + 64 * q);
        acc = fmaf(m.x, xv[q].x, fmaf(m.y, xv[q].y, acc));
      }
    }
    xr[r] = acc;
  }
  warp_sum_n<RM>(xr, lane);
  // state update (layer.py:347-351) and y_r = C_r h = c_r . rot^T(h)
  float yr[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) yr[r] = 0.f;
#pragma unroll
  for (int q = 0; q < DP; ++q) {
    const bool rot = lane + 32 * q < S;
    float2 bxc = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RM; ++r) {  // zero B rows beyond R
      bxc.x = fmaf(xr[r], Bv[r][q].x, bxc.x);
      bxc.y = fmaf(xr[r], Bv[r][q].y, bxc.y);
    }
    if (rot) bxc = make_float2(bxc.x * cs[q] - bxc.y * sn[q], bxc.x * sn[q] + bxc.y * cs[q]);
    float2 hn;
    hn.x = fmaf(decay, hs[q].x, DT * fmaf(w1, bxc.x, w2 * bp[q].x));
    hn.y = fmaf(decay, hs[q].y, DT * fmaf(w1, bxc.y, w2 * bp[q].y));
    *reinterpret_cast<float2*>(a.ssm_out + sbase + 2 * lane + 64 * q) = hn;
    *reinterpret_cast<float2*>(a.bx_out + sbase + 2 * lane + 64 * q) = bxc;
    const float2 ht = rot ? make_float2(hn.x * cs[q] + hn.y * sn[q], hn.y * cs[q] - hn.x * sn[q]) : hn;
#pragma unroll
    for (int r = 0; r < RM; ++r) yr[r] = fmaf(Cv[r][q].x, ht.x, fmaf(Cv[r][q].y, ht.y, yr[r]));
  }
  warp_sum_n<RM>(yr, lane);
  // y = mimo_o^T (y_r + D xr), gated by silu(z) (layer.py:352-356)
  TZ* yo = reinterpret_cast<TZ*>(a.y) + (int64_t)b * a.s_y + h * P;
#pragma unroll
  for (int q = 0; q < PP; ++q) {
    const int p0 = 2 * lane + 64 * q;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      if (r >= R) break;
      const float2 m = ldg2(mo + r * P + p0);
      const float yv = fmaf(Dk, xr[r], yr[r]);
      acc.x = fmaf(yv, m.x, acc.x);
      acc.y = fmaf(yv, m.y, acc.y);
    }
    const float2 z = zv[q];
    Pair<TZ>::st(yo + p0, make_float2(acc.x * (z.x * fast_sigmoid(z.x)), acc.y * (z.y * fast_sigmoid(z.y))));
  }
}

template <typename TZ, int DP, int PP>
void launch_row_pp(const StepParams& p, cudaStream_t s) {
  const dim3 grid((p.H + kWarpRows - 1) / kWarpRows, p.Bn);
  if (p.R <= 1) mimo_step_row_kernel<TZ, DP, PP, 1><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else if (p.R <= 2) mimo_step_row_kernel<TZ, DP, PP, 2><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else if (p.R <= 4) mimo_step_row_kernel<TZ, DP, PP, 4><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else mimo_step_row_kernel<TZ, DP, PP, 8><<<grid, 32 * kWarpRows, 0, s>>>(p);
}

template <typename TZ, int DP, int PP>
void launch_pair_pp(const StepParams& p, cudaStream_t s) {
  const dim3 grid(p.H, (p.Bn + kWarpRows - 1) / kWarpRows);
  if (p.R <= 1) mimo_step_pair_kernel<TZ, DP, PP, 1><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else if (p.R <= 2) mimo_step_pair_kernel<TZ, DP, PP, 2><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else if (p.R <= 4) mimo_step_pair_kernel<TZ, DP, PP, 4><<<grid, 32 * kWarpRows, 0, s>>>(p);
  else mimo_step_pair_kernel<TZ, DP, PP, 8><<<grid, 32 * kWarpRows, 0, s>>>(p);
}

template <typename TZ>
void launch_pair(const StepParams& p, cudaStream_t s) {
  if (p.G == 1) {  // the row-per-CTA layout shares the group's norms between heads
    if (p.D == 64) {
      if (p.P == 64) launch_row_pp<TZ, 1, 1>(p, s);
      else launch_row_pp<TZ, 1, 2>(p, s);
    } else {
      if (p.P == 64) launch_row_pp<TZ, 2, 1>(p, s);
      else launch_row_pp<TZ, 2, 2>(p, s);
    }
    return;
  }
  if (p.D == 64) {
    if (p.P == 64) launch_pair_pp<TZ, 1, 1>(p, s);
    else launch_pair_pp<TZ, 1, 2>(p, s);
  } else {
    if (p.P == 64) launch_pair_pp<TZ, 2, 1>(p, s);
    else launch_pair_pp<TZ, 2, 2>(p, s);
  }
}

template <typename TZ, int DL, int RM>
void launch_warp_rm(const StepParams& p, cudaStream_t s) {
  const dim3 grid(p.H, (p.Bn + kWarpRows - 1) / kWarpRows);
  const size_t smem = sizeof(float) * (size_t)(2 * p.R * p.D + 2 * p.D + 2 * p.R * p.P);
  if (p.P <= 64) mimo_step_warp_kernel<TZ, DL, RM, 2><<<grid, 32 * kWarpRows, smem, s>>>(p);
  else mimo_step_warp_kernel<TZ, DL, RM, 8><<<grid, 32 * kWarpRows, smem, s>>>(p);
}

template <typename TZ, int DL>
void launch_warp_dl(const StepParams& p, cudaStream_t s) {
  if (p.R <= 1) launch_warp_rm<TZ, DL, 1>(p, s);
  else if (p.R <= 2) launch_warp_rm<TZ, DL, 2>(p, s);
  else if (p.R <= 4) launch_warp_rm<TZ, DL, 4>(p, s);
  else if constexpr (DL <= 2) launch_warp_rm<TZ, DL, 8>(p, s);
}

template <typename TZ>
void launch_warp(const StepParams& p, cudaStream_t s) {
  const int dl = p.D / 32;
  if (dl == 1) launch_warp_dl<TZ, 1>(p, s);
  else if (dl == 2) launch_warp_dl<TZ, 2>(p, s);
  else launch_warp_dl<TZ, 4>(p, s);
}

}  // namespace

inline bool aligned_to(const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

int launch_step(const StepParams& p, int zdt, bool mimo, cudaStream_t s) {
  if (p.R * p.D > kMaxRD || p.R > 8 || p.S > 256) return fail(M3_ERR_UNSUPPORTED, "step: mimo_rank*d_state above 2048, rank above 8 or more than 256 angles");
  if (mimo && p.P > 1024) return fail(M3_ERR_UNSUPPORTED, "step: headdim above 1024");
  if (!mimo && (p.D % 16 != 0 || (p.D & (p.D - 1)) != 0)) return fail(M3_ERR_UNSUPPORTED, "siso step: d_state must be a power of two >= 16");
  const dim3 grid(p.Bn * p.H);
  // warp-per-(b, h) MIMO kernel where its register layout fits (shared memory: head
  // parameters, at most 2*512 + 2*128 + 2*8*256 floats = 21.5 KB)
  const int dl = p.D / 32;
  const bool warp_mimo = mimo && p.D % 32 == 0 && (dl == 1 || dl == 2 || dl == 4) && p.R * dl <= 16 &&
                         p.P <= 256 && p.split <= p.D;
  // the vector-pair kernel: d_state and headdim 64 / 128, every row and state row starts on
  // an 8-byte boundary (pairs of 16-bit or 32-bit values)
  const int esz = zdt == M3_FLOAT32 ? 4 : 2;
  const bool pair_mimo = mimo && (p.D == 64 || p.D == 128) && (p.P == 64 || p.P == 128) && p.R <= 8 &&
                         2 * p.S <= p.D && p.split == 2 * p.S && (p.s_row % 2) == 0 && (p.s_y % 2) == 0 &&
                         (p.d_inner % 2) == 0 && aligned_to(p.zxbcdt, 2 * esz) && aligned_to(p.y, 2 * esz) &&
                         aligned_to(p.ssm_in, 8) && aligned_to(p.ssm_out, 8) && aligned_to(p.bx_in, 8) &&
                         aligned_to(p.bx_out, 8) && aligned_to(p.B_bias, 8) && aligned_to(p.C_bias, 8) &&
                         aligned_to(p.mimo_x, 8) && aligned_to(p.mimo_o, 8) && aligned_to(p.B_norm_w, 8) &&
                         aligned_to(p.C_norm_w, 8);
#define M3_STEP_LAUNCH(T)                                                          \
  do {                                                                             \
    if (pair_mimo) launch_pair<T>(p, s);                                            \
    else if (warp_mimo) launch_warp<T>(p, s);                                       \
    else if (mimo) mimo_step_kernel<T><<<grid, kThreads, 0, s>>>(p);               \
    else siso_step_kernel<T><<<grid, kThreads, 0, s>>>(p);                         \
  } while (0)
  if (zdt == M3_FLOAT32) M3_STEP_LAUNCH(float);
  else if (zdt == M3_BFLOAT16) M3_STEP_LAUNCH(__nv_bfloat16);
  else if (zdt == M3_FLOAT16) M3_STEP_LAUNCH(__half);
  else return fail(M3_ERR_UNSUPPORTED, "step: unsupported dtype");
#undef M3_STEP_LAUNCH
  return check_launch(mimo ? "mimo_step_kernel" : "siso_step_kernel");
}

}  // namespace m3
