// Fused prologue and gate of Mamba3.forward (mamba3_ssm/layer.py:180-266) for inference:
// everything between the in_proj GEMM and the scan, and the silu gate between the scan and
// out_proj, read straight from the in_proj output.
//
//   angle kernel (one warp per (b, h), lane = rotary angle, walks the sequence):
//     DT = softplus(dd_dt + dt_bias), A = -min(softplus(dd_A), -A_floor) (layer.py:207),
//     ADT = A DT, trap logit copied to fp32, angles[b,l,h,i] = sum_{l'<=l} angle_raw[b,l',i] DT
//   bc kernel (one CTA per (b, l) row): RMSNorm over d_state of every (r, g) row of B and C
//     (ops.py:94-102, once per group, not once per head), then per head the bias and the
//     rotation of the pairs (2i, 2i+1), i < rope_split / 2, by angles[b,l,h,i]
//     (ops.py:116-119, layer.py:229-244), written as B_proj / C_proj (B, L, R, H, D) in the
//     scan's operand dtype
//   gate kernel: out = y * silu(z) in the dtype of out (layer.py:262-266)
#include "m3_common.cuh"
#include "prologue.cuh"

namespace m3 {
namespace {

constexpr int kWarps = 4;

template <typename TZ>
__global__ void __launch_bounds__(32 * kWarps) prologue_angle_kernel(PrologueParams a) {
  const int lane = threadIdx.x & 31;
  const int u = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (u >= a.Bn * a.H) return;
  const int b = u / a.H, h = u - b * a.H;
  const int H = a.H, S = a.S;
  const int off_dt = 2 * a.d_inner + 2 * a.D * a.G * a.R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  const float dtb = a.dt_bias[h];
  float ang0 = 0.f, ang1 = 0.f;  // angles lane and lane + 32
  const TZ* base = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb;
#pragma unroll 4
  for (int l = 0; l < a.L; ++l) {
    const TZ* row = base + (int64_t)l * a.s_zl;
    const float dtv = softplusf_(to_f32(row[off_dt + h]) + dtb);
    const int64_t o = ((int64_t)b * a.L + l) * H + h;
    if (lane == 0) {
      const float A = -fminf(softplusf_(to_f32(row[off_A + h])), -a.A_floor);
      a.DT[o] = dtv;
      a.ADT[o] = A * dtv;
      a.trap[o] = to_f32(row[off_tr + h]);
    }
    if (lane < S) {
      ang0 = fmaf(to_f32(row[off_ang + lane]), dtv, ang0);
      a.angles[o * S + lane] = ang0;
    }
    if (lane + 32 < S) {
      ang1 = fmaf(to_f32(row[off_ang + lane + 32]), dtv, ang1);
      a.angles[o * S + lane + 32] = ang1;
    }
  }
}

template <typename TZ, typename TO>
__global__ void __launch_bounds__(128) prologue_bc_kernel(PrologueParams a) {
  extern __shared__ float psm[];
  const int b = blockIdx.y, l = blockIdx.x;
  const int R = a.R, G = a.G, D = a.D, H = a.H, S = a.S;
  const int RGD = R * G * D;
  float* raw = psm;              // [2][R][G][D]: B then C
  float* inv = raw + 2 * RGD;    // [2][R][G]
  const TZ* row = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb + (int64_t)l * a.s_zl;
  const int off_B = 2 * a.d_inner;
  for (int i = threadIdx.x; i < 2 * RGD; i += blockDim.x) raw[i] = to_f32(row[off_B + i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < 2 * R * G; j += blockDim.x >> 5) {
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss = fmaf(raw[j * D + d], raw[j * D + d], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) inv[j] = sqrtf(ss / (float)D + a.eps);
  }
  __syncthreads();
  const int half = D / 2, npair = a.split / 2;
  const int64_t rowo = ((int64_t)b * a.L + l);
  const float* angr = a.angles + rowo * H * S;
  // item = (m, r, h, pair): pair k covers d = 2k, 2k + 1
  const int items = 2 * R * H * half;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int k = it % half;
    int rest = it / half;
    const int h = rest % H;
    rest /= H;
    const int r = rest % R, m = rest / R;
    const int g = (int)(((int64_t)h * G) / H);
    const float* src = raw + ((m * R + r) * G + g) * D;
    const float rs = inv[(m * R + r) * G + g];
    const float* w = m ? a.C_norm_w : a.B_norm_w;
    const float* bias = (m ? a.C_bias : a.B_bias) + ((int64_t)h * R + r) * D;
    const int d0 = 2 * k, d1 = d0 + 1;
    float v0 = src[d0] / rs * w[d0] + bias[d0];
    float v1 = src[d1] / rs * w[d1] + bias[d1];
    if (k < npair) {
      float sn, cs;
      sincosf(angr[h * S + k], &sn, &cs);
      const float t0 = v0 * cs - v1 * sn;
      v1 = v0 * sn + v1 * cs;
      v0 = t0;
    }
    TO* out = reinterpret_cast<TO*>(m ? a.Cp : a.Bp) + ((rowo * R + r) * H + h) * D;
    out[d0] = from_f32<TO>(v0);
    out[d1] = from_f32<TO>(v1);
  }
}

template <typename TY, typename TZ, typename TO>
__global__ void __launch_bounds__(256) gate_kernel(GateParams a) {
  const int64_t n = (int64_t)a.rows * a.P;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / a.P;
    const int p = (int)(i - r * a.P);
    const int64_t b = r / ((int64_t)a.L * a.H), rem = r - b * a.L * a.H;
    const int64_t l = rem / a.H, h = rem - l * a.H;
    const float y = to_f32(reinterpret_cast<const TY*>(a.y)[b * a.sy.b + l * a.sy.l + h * a.sy.h + p]);
    const float z = to_f32(reinterpret_cast<const TZ*>(a.z)[b * a.sz.b + l * a.sz.l + h * a.sz.h + p]);
    reinterpret_cast<TO*>(a.out)[b * a.so.b + l * a.so.l + h * a.so.h + p] = from_f32<TO>(y * (z * sigmoidf_(z)));
  }
}

}  // namespace

int launch_prologue(const PrologueParams& p, int zdt, int odt, cudaStream_t s) {
  if (p.S > 64) return fail(M3_ERR_UNSUPPORTED, "prologue: more than 64 rope angles");
  if (p.D % 2) return fail(M3_ERR_UNSUPPORTED, "prologue: odd d_state");
  const size_t smem = sizeof(float) * (2 * (size_t)p.R * p.G * p.D + 2 * (size_t)p.R * p.G);
  if (smem > 48 * 1024) return fail(M3_ERR_UNSUPPORTED, "prologue: B/C rows too wide for shared memory");
  if (p.L > 65535) return fail(M3_ERR_UNSUPPORTED, "prologue: sequence above 65535");
  const unsigned ga = (unsigned)((p.Bn * p.H + kWarps - 1) / kWarps);
  const dim3 gb(p.L, p.Bn);
#define M3_PRO(TZ, TO)                                                        \
  do {                                                                        \
    prologue_angle_kernel<TZ><<<ga, 32 * kWarps, 0, s>>>(p);                  \
    M3_TRY(check_launch("prologue_angle_kernel"));                            \
    prologue_bc_kernel<TZ, TO><<<gb, 128, smem, s>>>(p);                      \
    return check_launch("prologue_bc_kernel");                                \
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
  const int64_t n = (int64_t)p.rows * p.P;
  if (n == 0) return M3_OK;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 32);
#define M3_GATE(TY, TZ, TO)                                          \
  do {                                                               \
    gate_kernel<TY, TZ, TO><<<grid, 256, 0, s>>>(p);                 \
    return check_launch("gate_kernel");                              \
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
