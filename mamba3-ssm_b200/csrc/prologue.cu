// Fused prologue and gate of Mamba3.forward (mamba3_ssm/layer.py:180-266) for inference:
// everything between the in_proj GEMM and the scan, and the silu gate between the scan and
// out_proj, read straight from the in_proj output.
//
//   angle kernels (one CTA per (b, h); 128-step tiles, or segments when units are few):
//     DT = softplus(dd_dt + dt_bias), A = -min(softplus(dd_A), -A_floor) (layer.py:207),
//     ADT = A DT, trap logit copied to fp32, angles[b,l,h,i] = angle0[b,h,i] (the decode
//     cache's angle state, zero when absent) + sum_{l'<=l} angle_raw[b,l',i] DT
//   bc kernel (one warp per output row (b, l, B|C, r, h)): RMSNorm over d_state of the
//     row's group (ops.py:94-102), the head's bias, and the rotation of the pairs
//     (2i, 2i+1), i < rope_split / 2, by angles[b,l,h,i]
//     (ops.py:116-119, layer.py:229-244), written as B_proj / C_proj (B, L, R, H, D) in the
//     scan's operand dtype
//   gate kernel: out = y * silu(z) in the dtype of out (layer.py:262-266)
#include "m3_common.cuh"
#include "prologue.cuh"

namespace m3 {
namespace {

// Many (b, h) units (four or more per SM): one CTA per (b, h), thread = time step of a
// kAT-step tile. Each thread carries its step's
// angles 16 at a time in registers: a warp scan over the tile, the warp totals through
// shared memory (two barriers per 16 angles), then one (b, l, h) row of angles written as
// 16-byte vectors (the S angles of a row are contiguous).
template <typename TZ, int kAT>
__global__ void __launch_bounds__(kAT) prologue_angle_tile_kernel(PrologueParams a) {
  constexpr int kS = 16;
  __shared__ float wsum[kAT / 32][kS];
  __shared__ float carry[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  const int H = a.H, S = a.S;
  const int off_dt = 2 * a.d_inner + 2 * a.D * a.G * a.R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  const float dtb = a.dt_bias[h];
  const TZ* base = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb;
  const bool vec = (S % 4) == 0 && (reinterpret_cast<uintptr_t>(a.angles) & 15) == 0;
  for (int s0 = tid; s0 < S; s0 += kAT) carry[s0] = a.angle0 ? a.angle0[(int64_t)u * S + s0] : 0.f;
  __syncthreads();
  for (int l0 = 0; l0 < a.L; l0 += kAT) {
    const int l = l0 + tid;
    const bool v = l < a.L;
    const TZ* row = base + (int64_t)(v ? l : 0) * a.s_zl;
    float dtv = 0.f;
    const int64_t o = ((int64_t)b * a.L + l) * H + h;
    if (v) {
      dtv = softplusf_(to_f32(row[off_dt + h]) + dtb);
      const float A = -fminf(softplusf_(to_f32(row[off_A + h])), -a.A_floor);
      a.DT[o] = dtv;
      a.ADT[o] = A * dtv;
      a.trap[o] = to_f32(row[off_tr + h]);
    }
    for (int s0 = 0; s0 < S; s0 += kS) {
      float x[kS];
#pragma unroll
      for (int k = 0; k < kS; ++k) x[k] = (v && s0 + k < S) ? to_f32(row[off_ang + s0 + k]) * dtv : 0.f;
#pragma unroll
      for (int of = 1; of < 32; of <<= 1) {
#pragma unroll
        for (int k = 0; k < kS; ++k) {
          const float y = __shfl_up_sync(0xffffffffu, x[k], of);
          if (lane >= of) x[k] += y;
        }
      }
      if (lane == 31)
#pragma unroll
        for (int k = 0; k < kS; ++k) wsum[warp][k] = x[k];
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kS; ++k) {
        float pre = s0 + k < S ? carry[s0 + k] : 0.f;
        for (int w = 0; w < warp; ++w) pre += wsum[w][k];
        x[k] += pre;
      }
      if (v) {
        float* dst = a.angles + o * S + s0;
        if (vec && s0 + kS <= S) {
#pragma unroll
          for (int k = 0; k < kS; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
        } else {
#pragma unroll
          for (int k = 0; k < kS; ++k)
            if (s0 + k < S) dst[k] = x[k];
        }
      }
      __syncthreads();  // carry and wsum read by every thread before they change
      if (tid == kAT - 1)
#pragma unroll
        for (int k = 0; k < kS; ++k)
          if (s0 + k < S) carry[s0 + k] = x[k];
    }
    __syncthreads();
  }
}

// Few (b, h) units: one CTA per (b, h); warp w walks the w-th of the CTA's consecutive segments of T steps
// (T a multiple of 32) in slabs of 32 steps. Per slab each lane forms DT of one step (lane
// = step, one softplus per step); the walk over the slab's steps then runs with lane =
// angle (32 angles at a time), DT of step j handed over by a warp shuffle, so each step's
// angle_raw row and each row of angles is one contiguous access of the warp. Pass 1 sums
// each angle's increments angle_raw[l, i] DT[l] over the warp's segment; the segment totals
// meet in shared memory, where one thread per angle turns them into exclusive prefixes
// (starting from angle0). Pass 2 walks the segment again from that prefix, writing the
// running angles; its first angle group also writes DT, ADT and trap. No scratch memory, no
// waits between CTAs.
template <typename TZ>
__global__ void __launch_bounds__(1024) prologue_angle_kernel(PrologueParams a, int T) {
  constexpr int kB = 8;           // steps whose angle_raw loads are issued together
  __shared__ float tot[32][65];  // [segment][angle]: totals, then exclusive prefixes
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  const int H = a.H, S = a.S;
  const int off_dt = 2 * a.d_inner + 2 * a.D * a.G * a.R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  const float dtb = a.dt_bias[h];
  const TZ* base = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb;
  const int64_t szl = a.s_zl, HS = (int64_t)H * S;
  const int l0 = w * T, l1 = min(l0 + T, a.L);
  for (int s0 = 0; s0 < S; s0 += 32) {
    const int s = s0 + lane;
    float acc = 0.f;
    for (int ls = l0; ls < l1; ls += 32) {
      const int l = ls + lane, n = min(32, l1 - ls);
      const float dtl = l < l1 ? softplusf_(to_f32(base[(int64_t)l * szl + off_dt + h]) + dtb) : 0.f;
      const TZ* col = base + (int64_t)ls * szl + off_ang + (s < S ? s : 0);
      for (int j0 = 0; j0 < n; j0 += kB) {
        float xv[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) xv[k] = j0 + k < n ? to_f32(col[(int64_t)(j0 + k) * szl]) : 0.f;
#pragma unroll
        for (int k = 0; k < kB; ++k) acc = fmaf(xv[k], __shfl_sync(0xffffffffu, dtl, (j0 + k) & 31), acc);
      }
    }
    if (s < S) tot[w][s] = acc;
  }
  __syncthreads();
  if (threadIdx.x < S) {
    const int i = threadIdx.x;
    float run = a.angle0 ? a.angle0[(int64_t)u * S + i] : 0.f;
    for (int j = 0; j < W; ++j) {
      const float t = tot[j][i];
      tot[j][i] = run;
      run += t;
    }
  }
  __syncthreads();
  for (int s0 = 0; s0 < (S > 0 ? S : 1); s0 += 32) {  // S == 0: one pass for DT, ADT, trap
    const int s = s0 + lane;
    const bool sv = s < S;
    float run = sv ? tot[w][s] : 0.f;
    for (int ls = l0; ls < l1; ls += 32) {
      const int l = ls + lane, n = min(32, l1 - ls);
      const bool v = l < l1;
      const TZ* row = base + (int64_t)(v ? l : l0) * szl;
      const float dtl = v ? softplusf_(to_f32(row[off_dt + h]) + dtb) : 0.f;
      if (s0 == 0 && v) {
        const int64_t o = ((int64_t)b * a.L + l) * H + h;
        const float A = -fminf(softplusf_(to_f32(row[off_A + h])), -a.A_floor);
        a.DT[o] = dtl;
        a.ADT[o] = A * dtl;
        a.trap[o] = to_f32(row[off_tr + h]);
      }
      if (S == 0) continue;
      const TZ* col = base + (int64_t)ls * szl + off_ang + (sv ? s : 0);
      float* dst = a.angles + ((int64_t)b * a.L + ls) * HS + (int64_t)h * S + (sv ? s : 0);
      // the batch's loads first: each is independent of the angles stored before it
      for (int j0 = 0; j0 < n; j0 += kB) {
        float xv[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) xv[k] = j0 + k < n ? to_f32(col[(int64_t)(j0 + k) * szl]) : 0.f;
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          run = fmaf(xv[k], __shfl_sync(0xffffffffu, dtl, (j0 + k) & 31), run);
          if (sv && j0 + k < n) dst[(int64_t)(j0 + k) * HS] = run;
        }
      }
    }
  }
}

template <typename TO>
__device__ __forceinline__ void st_pair(TO* p, float v0, float v1) {
  p[0] = from_f32<TO>(v0);
  p[1] = from_f32<TO>(v1);
}
template <>
__device__ __forceinline__ void st_pair<__nv_bfloat16>(__nv_bfloat16* p, float v0, float v1) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v0, v1);
}
template <>
__device__ __forceinline__ void st_pair<float>(float* p, float v0, float v1) {
  *reinterpret_cast<float2*>(p) = make_float2(v0, v1);
}

// one warp per (b, l, r): lanes over the pairs (2k, 2k + 1) of d_state (PPL per lane). The
// group rows of B and C are loaded and normalised once (G == 1) or per head (G == H), then
// for every head: bias, one sin / cos per pair shared by B and C, rotate, store.
template <typename TZ, typename TO, int PPL>
__global__ void __launch_bounds__(256) prologue_bc_kernel(PrologueParams a) {
  const int R = a.R, G = a.G, D = a.D, H = a.H, S = a.S;
  const int half = D / 2, npair = a.split / 2, lane = threadIdx.x & 31;
  const int rowo = blockIdx.x;  // b * L + l
  const int r = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const int b = rowo / a.L, l = rowo - b * a.L;
  const TZ* zrow = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb + (int64_t)l * a.s_zl + 2 * a.d_inner;
  const int64_t RGD = (int64_t)R * G * D;
  float wb0[PPL], wb1[PPL], wc0[PPL], wc1[PPL];
#pragma unroll
  for (int j = 0; j < PPL; ++j) {
    const int k = min(lane + 32 * j, half - 1);
    wb0[j] = a.B_norm_w[2 * k]; wb1[j] = a.B_norm_w[2 * k + 1];
    wc0[j] = a.C_norm_w[2 * k]; wc1[j] = a.C_norm_w[2 * k + 1];
  }
  float b0[PPL], b1[PPL], c0[PPL], c1[PPL];  // normalised group rows
  for (int h = 0; h < H; ++h) {
    if (h == 0 || G != 1) {
      const int g = G == 1 ? 0 : h;
      const TZ* sb = zrow + (int64_t)(r * G + g) * D;
      const TZ* sc = sb + RGD;
      float ssb = 0.f, ssc = 0.f;
#pragma unroll
      for (int j = 0; j < PPL; ++j) {
        const int k = lane + 32 * j;
        const bool v = k < half;
        b0[j] = v ? to_f32(sb[2 * k]) : 0.f; b1[j] = v ? to_f32(sb[2 * k + 1]) : 0.f;
        c0[j] = v ? to_f32(sc[2 * k]) : 0.f; c1[j] = v ? to_f32(sc[2 * k + 1]) : 0.f;
        ssb = fmaf(b0[j], b0[j], fmaf(b1[j], b1[j], ssb));
        ssc = fmaf(c0[j], c0[j], fmaf(c1[j], c1[j], ssc));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ssb += __shfl_xor_sync(0xffffffffu, ssb, o);
        ssc += __shfl_xor_sync(0xffffffffu, ssc, o);
      }
      const float rb = 1.0f / sqrtf(ssb / (float)D + a.eps), rc = 1.0f / sqrtf(ssc / (float)D + a.eps);
#pragma unroll
      for (int j = 0; j < PPL; ++j) {
        b0[j] = b0[j] * rb * wb0[j]; b1[j] = b1[j] * rb * wb1[j];
        c0[j] = c0[j] * rc * wc0[j]; c1[j] = c1[j] * rc * wc1[j];
      }
    }
    const float* bb = a.B_bias + ((int64_t)h * R + r) * D;
    const float* cb = a.C_bias + ((int64_t)h * R + r) * D;
    const float* ang = a.angles + ((int64_t)rowo * H + h) * S;
    TO* ob = reinterpret_cast<TO*>(a.Bp) + (((int64_t)rowo * R + r) * H + h) * D;
    TO* oc = reinterpret_cast<TO*>(a.Cp) + (((int64_t)rowo * R + r) * H + h) * D;
#pragma unroll
    for (int j = 0; j < PPL; ++j) {
      const int k = lane + 32 * j;
      if (k < half) {
        const int d0 = 2 * k;
        const float2 bv = __ldg(reinterpret_cast<const float2*>(bb + d0));
        const float2 cv = __ldg(reinterpret_cast<const float2*>(cb + d0));
        float x0 = b0[j] + bv.x, x1 = b1[j] + bv.y;
        float y0 = c0[j] + cv.x, y1 = c1[j] + cv.y;
        if (k < npair) {
          float sn, cs;
          sincos_reduced(ang[k], &sn, &cs);
          const float t0 = x0 * cs - x1 * sn, u0 = y0 * cs - y1 * sn;
          x1 = x0 * sn + x1 * cs;
          y1 = y0 * sn + y1 * cs;
          x0 = t0;
          y0 = u0;
        }
        st_pair<TO>(ob + d0, x0, x1);
        st_pair<TO>(oc + d0, y0, y1);
      }
    }
  }
}

// thread = 8 consecutive elements of one (b, l, h) row (16-byte vectors when VEC)
template <typename T>
struct alignas(16) V8 {
  T e[8];
};

template <typename TY, typename TZ, typename TO, bool VEC>
__global__ void __launch_bounds__(256) gate_kernel(GateParams a) {
  const int nv = (a.P + 7) / 8;
  const int64_t n = a.rows * nv;
  const int LH = a.L * a.H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int p0 = (int)(i - r * nv) * 8;
    const int64_t b = r / LH;
    const int rem = (int)(r - b * LH);
    const int l = rem / a.H, h = rem - l * a.H;
    const TY* y = reinterpret_cast<const TY*>(a.y) + b * a.sy.b + (int64_t)l * a.sy.l + (int64_t)h * a.sy.h + p0;
    const TZ* z = reinterpret_cast<const TZ*>(a.z) + b * a.sz.b + (int64_t)l * a.sz.l + (int64_t)h * a.sz.h + p0;
    TO* o = reinterpret_cast<TO*>(a.out) + b * a.so.b + (int64_t)l * a.so.l + (int64_t)h * a.so.h + p0;
    if (VEC) {
      const V8<TY> yv = *reinterpret_cast<const V8<TY>*>(y);
      const V8<TZ> zv = *reinterpret_cast<const V8<TZ>*>(z);
      V8<TO> ov;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float zz = to_f32(zv.e[k]);
        ov.e[k] = from_f32<TO>(to_f32(yv.e[k]) * (zz * fast_sigmoid(zz)));
      }
      *reinterpret_cast<V8<TO>*>(o) = ov;
    } else {
      for (int k = 0; k < 8 && p0 + k < a.P; ++k) {
        const float zz = to_f32(z[k]);
        o[k] = from_f32<TO>(to_f32(y[k]) * (zz * fast_sigmoid(zz)));
      }
    }
  }
}

}  // namespace

int launch_prologue(const PrologueParams& p, int zdt, int odt, cudaStream_t s) {
  if (p.S > 64) return fail(M3_ERR_UNSUPPORTED, "prologue: more than 64 rope angles");
  if (p.D % 2 || p.D > 256 || p.R > 8) return fail(M3_ERR_UNSUPPORTED, "prologue: d_state odd or above 256, or rank above 8");
  if ((reinterpret_cast<uintptr_t>(p.B_bias) | reinterpret_cast<uintptr_t>(p.C_bias)) & 7)
    return fail(M3_ERR_UNSUPPORTED, "prologue: B_bias / C_bias must be 8-byte aligned");
  const unsigned ga = (unsigned)(p.Bn * p.H);
  if ((int64_t)p.Bn * p.L > 2147483647LL) return fail(M3_ERR_UNSUPPORTED, "prologue: batch * seqlen too large");
  const dim3 gb((unsigned)((int64_t)p.Bn * p.L), (unsigned)((p.R + 7) / 8));
  const int ppl = (p.D / 2 + 31) / 32;
  int sms = 148;
  if (device_sm_count(&sms) != M3_OK) sms = 148;
  // fewer than four (b, h) units per SM: the segment kernel, about 64 warps per SM over the
  // grid (at most 32 segments per unit, each whole slabs of 32 steps); else 128-step tiles
  const bool seg = (int64_t)ga < 4 * (int64_t)sms && p.L > 128;
  const int64_t want = std::min<int64_t>(32, std::max<int64_t>(1, ((int64_t)sms * 64 + ga - 1) / ga));
  const int T = (int)(((p.L + want - 1) / want + 31) / 32 * 32);
  const int nseg = (p.L + T - 1) / T;
#define M3_PRO(TZ, TO)                                                                  \
  do {                                                                                  \
    if (seg) prologue_angle_kernel<TZ><<<ga, 32 * nseg, 0, s>>>(p, T);                  \
    else prologue_angle_tile_kernel<TZ, 128><<<ga, 128, 0, s>>>(p);                     \
    M3_TRY(check_launch("prologue_angle_kernel"));                                      \
    if (!p.Bp) return M3_OK; /* angles and step scalars only */                         \
    const int th = 32 * (p.R < 8 ? p.R : 8);                                            \
    if (ppl == 1) prologue_bc_kernel<TZ, TO, 1><<<gb, th, 0, s>>>(p);                   \
    else if (ppl == 2) prologue_bc_kernel<TZ, TO, 2><<<gb, th, 0, s>>>(p);              \
    else prologue_bc_kernel<TZ, TO, 4><<<gb, th, 0, s>>>(p);                            \
    return check_launch("prologue_bc_kernel");                                          \
  } while (0)
  if (zdt == M3_BFLOAT16 && odt == M3_BFLOAT16) M3_PRO(__nv_bfloat16, __nv_bfloat16);
  if (zdt == M3_BFLOAT16 && odt == M3_FLOAT32) M3_PRO(__nv_bfloat16, float);
  if (zdt == M3_FLOAT32 && odt == M3_FLOAT32) M3_PRO(float, float);
  if (zdt == M3_FLOAT32 && odt == M3_BFLOAT16) M3_PRO(float, __nv_bfloat16);
  if (zdt == M3_FLOAT16 && odt == M3_FLOAT32) M3_PRO(__half, float);
  if (zdt == M3_FLOAT16 && odt == M3_FLOAT16) M3_PRO(__half, __half);
#undef M3_PRO
  return fail(M3_ERR_UNSUPPORTED, "prologue: unsupported dtype pair");
}

int launch_gate(const GateParams& p, int ydt, int zdt, int odt, cudaStream_t s) {
  const int64_t n = p.rows * ((p.P + 7) / 8);
  if (n == 0) return M3_OK;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  auto al = [](const void* ptr, const Str3& st, int es) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && (st.b * es) % 16 == 0 && (st.l * es) % 16 == 0 &&
           (st.h * es) % 16 == 0;
  };
#define M3_GATE(TY, TZ, TO)                                                                          \
  do {                                                                                               \
    const bool vec = p.P % 8 == 0 && al(p.y, p.sy, sizeof(TY)) && al(p.z, p.sz, sizeof(TZ)) &&       \
                     al(p.out, p.so, sizeof(TO));                                                    \
    if (vec) gate_kernel<TY, TZ, TO, true><<<grid, 256, 0, s>>>(p);                                  \
    else gate_kernel<TY, TZ, TO, false><<<grid, 256, 0, s>>>(p);                                     \
    return check_launch("gate_kernel");                                                              \
  } while (0)
  if (ydt == M3_BFLOAT16 && zdt == M3_BFLOAT16 && odt == M3_BFLOAT16) M3_GATE(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
  if (ydt == M3_FLOAT32 && zdt == M3_FLOAT32 && odt == M3_FLOAT32) M3_GATE(float, float, float);
  if (ydt == M3_FLOAT32 && zdt == M3_BFLOAT16 && odt == M3_BFLOAT16) M3_GATE(float, __nv_bfloat16, __nv_bfloat16);
  if (ydt == M3_BFLOAT16 && zdt == M3_BFLOAT16 && odt == M3_FLOAT32) M3_GATE(__nv_bfloat16, __nv_bfloat16, float);
  if (ydt == M3_FLOAT16 && zdt == M3_FLOAT16 && odt == M3_FLOAT16) M3_GATE(__half, __half, __half);
#undef M3_GATE
  return fail(M3_ERR_UNSUPPORTED, "gate: unsupported dtype combination");
}

}  // namespace m3
