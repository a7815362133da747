// Backward of the fused prologue and of the silu gate of Mamba3.forward (the training path;
// mamba3_ssm/layer.py:180-266): the gradients autograd returns through the reference's
// prologue, given the scan's gradients.
//
//   bc kernel (CTA per tile of kRowsBC (b, l) rows, warp r = rank r, heads in a loop):
//     recompute the group row n = raw / rms * w and, per head, v = n + bias_h and the rotated
//     o = rot_theta(v) on the pairs i < S (theta = the forward's angles[b,l,h,i]); then
//       dv        = rot_theta^T(dB_proj)             the gradient before the rotation
//       dtheta_i += -dv1' o2 + dv2' o1               over B and C (dv' = dB_proj), ranks summed in
//                                                    shared memory, one write per (b, l, h, i)
//       dbias    += dv                               summed over the CTA's rows in shared memory,
//                                                    then a workspace slot per CTA
//       dn        = sum_h dv (one group) / dv (group per head)
//       draw      = (w dn) / rms - raw sum_d(w dn raw) / (D rms^3)   into d zxbcdt
//       dw       += dn raw / rms                     registers, then the CTA's slot
//   reduce kernel: the slots summed (a thread per output, 64 slots each, one atomic each)
//   angle kernel (CTA per (b, h), tiles of 128 steps from the end): q = suffix sums over l
//     of dtheta; dDT_ang[b,l,h] = sum_i q angle_raw[b,l,i]; dangle_raw[b,l,i] += q DT[b,l,h]
//     (atomics over heads into an fp32 buffer)
//   dt kernel (thread per (b, l, h)): dDT_total = dDT + A dADT + dDT_ang, with A the clamped
//     constant of layer.py:207 (so dd_A gets no gradient); dpre = dDT_total softplus'(dd_dt +
//     dt_bias) into d zxbcdt (dt column), the trap logit's gradient into its column, and the
//     dt_bias gradient (block sums, then atomics); the angle_raw columns from the fp32 buffer
//   gate kernel: dy = dout silu(z), dz = dout y silu'(z)
#include <algorithm>

#include "m3_common.cuh"
#include "prologue.cuh"
#include "sm100.cuh"

namespace m3 {
namespace {

constexpr int kRowsBC = 16;  // (b, l) rows per CTA of the bc kernel
constexpr int kATmax = 512;  // steps per tile of the angle kernel when (b, h) units are few (else 128)

template <typename T>
__device__ __forceinline__ float2 ld_pair(const T* p) {
  return make_float2(to_f32(p[0]), to_f32(p[1]));
}
template <>
__device__ __forceinline__ float2 ld_pair<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 ld_pair<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <typename T>
__device__ __forceinline__ void st_pair2(T* p, float a, float b) {
  p[0] = from_f32<T>(a);
  p[1] = from_f32<T>(b);
}

// Shared memory of the bc kernel: the bias gradients of the tile (H, R, D) for B and C and
// one row's angle gradients (H, S).
template <typename TZ, typename TO, int PPL>
__global__ void __launch_bounds__(256) prologue_bwd_bc_kernel(PrologueBwdParams a) {
  extern __shared__ float sm[];
  const int R = a.R, G = a.G, D = a.D, H = a.H, S = a.S;
  const int half = D / 2, npair = a.split / 2;
  const int lane = threadIdx.x & 31, r = threadIdx.x >> 5;
  const int HRD = H * R * D;
  float* sbB = sm;                 // (H, R, D)
  float* sbC = sm + HRD;           // (H, R, D)
  float* sang = sm + 2 * HRD;      // (H, S) of the current row
  float* swb = sang + H * S;       // (R, D) dw partials of B
  float* swc = swb + R * D;        // (R, D) of C
  for (int i = threadIdx.x; i < 2 * HRD + H * S; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const int64_t nrows = (int64_t)a.Bn * a.L;
  const int64_t RGD = (int64_t)R * G * D;
  float wb0[PPL], wb1[PPL], wc0[PPL], wc1[PPL];
  float dwb0[PPL], dwb1[PPL], dwc0[PPL], dwc1[PPL];
#pragma unroll
  for (int j = 0; j < PPL; ++j) {
    const int k = min(lane + 32 * j, half - 1);
    wb0[j] = a.B_norm_w[2 * k]; wb1[j] = a.B_norm_w[2 * k + 1];
    wc0[j] = a.C_norm_w[2 * k]; wc1[j] = a.C_norm_w[2 * k + 1];
    dwb0[j] = dwb1[j] = dwc0[j] = dwc1[j] = 0.f;
  }
  const int64_t ntiles = (nrows + kRowsBC - 1) / kRowsBC;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x)
  for (int t = 0; t < kRowsBC; ++t) {
    const int64_t rowo = tile * kRowsBC + t;  // b * L + l
    const bool rv = rowo < nrows;                              // uniform over the CTA
    if (rv) {
      const int64_t b = rowo / a.L, l = rowo - b * a.L;
      const TZ* zrow = reinterpret_cast<const TZ*>(a.zx) + b * a.s_zb + l * a.s_zl + 2 * a.d_inner;
      TZ* drow = reinterpret_cast<TZ*>(a.dzx) + b * a.s_dzb + l * a.s_dzl + 2 * a.d_inner;
      float rb0[PPL], rb1[PPL], rc0[PPL], rc1[PPL];  // raw group rows
      float rsb = 0.f, rsc = 0.f;                    // 1 / rms
      float db0[PPL], db1[PPL], dc0[PPL], dc1[PPL];  // dn (sum over the group's heads)
      // heads in batches of kHB: the batch's gradient pairs and angles are loaded into
      // registers before any of them is used, so their latencies overlap
      constexpr int kHB = 8 / PPL;
      for (int h0 = 0; h0 < H; h0 += kHB) {
        float2 gbv[kHB][PPL], gcv[kHB][PPL];
        float angv[kHB][PPL];
#pragma unroll
        for (int hh = 0; hh < kHB; ++hh) {
          const int h = h0 + hh;
          const TO* gB = reinterpret_cast<const TO*>(a.dBp) + ((rowo * R + r) * H + h) * D;
          const TO* gC = reinterpret_cast<const TO*>(a.dCp) + ((rowo * R + r) * H + h) * D;
          const float* ang = a.angles + (rowo * H + h) * S;
#pragma unroll
          for (int j = 0; j < PPL; ++j) {
            const int k = lane + 32 * j;
            const bool v = h < H && k < half;
            gbv[hh][j] = v ? ld_pair(gB + 2 * k) : make_float2(0.f, 0.f);
            gcv[hh][j] = v ? ld_pair(gC + 2 * k) : make_float2(0.f, 0.f);
            angv[hh][j] = v && k < npair ? __ldg(ang + k) : 0.f;
          }
        }
#pragma unroll
        for (int hh = 0; hh < kHB; ++hh) {
          const int h = h0 + hh;
          if (h >= H) break;
          const int g = G == 1 ? 0 : h;
          if (h == 0 || G != 1) {
            const TZ* sb = zrow + (int64_t)(r * G + g) * D;
            const TZ* sc = sb + RGD;
            float ssb = 0.f, ssc = 0.f;
#pragma unroll
            for (int j = 0; j < PPL; ++j) {
              const int k = lane + 32 * j;
              const bool v = k < half;
              rb0[j] = v ? to_f32(sb[2 * k]) : 0.f; rb1[j] = v ? to_f32(sb[2 * k + 1]) : 0.f;
              rc0[j] = v ? to_f32(sc[2 * k]) : 0.f; rc1[j] = v ? to_f32(sc[2 * k + 1]) : 0.f;
              ssb = fmaf(rb0[j], rb0[j], fmaf(rb1[j], rb1[j], ssb));
              ssc = fmaf(rc0[j], rc0[j], fmaf(rc1[j], rc1[j], ssc));
              db0[j] = db1[j] = dc0[j] = dc1[j] = 0.f;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              ssb += __shfl_xor_sync(0xffffffffu, ssb, o);
              ssc += __shfl_xor_sync(0xffffffffu, ssc, o);
            }
            rsb = 1.0f / sqrtf(ssb / (float)D + a.eps);
            rsc = 1.0f / sqrtf(ssc / (float)D + a.eps);
          }
          const float* bb = a.B_bias + ((int64_t)h * R + r) * D;
          const float* cb = a.C_bias + ((int64_t)h * R + r) * D;
          float* sbBh = sbB + ((int64_t)h * R + r) * D;
          float* sbCh = sbC + ((int64_t)h * R + r) * D;
#pragma unroll
          for (int j = 0; j < PPL; ++j) {
            const int k = lane + 32 * j;
            if (k < half) {
              const int d0 = 2 * k;
              float2 gb = gbv[hh][j], gc = gcv[hh][j];
              if (k < npair) {
                // o = rot(v) with v = n + bias; dtheta = -g1 o2 + g2 o1; dv = rot^T(g)
                const float2 bv = __ldg(reinterpret_cast<const float2*>(bb + d0));
                const float2 cv = __ldg(reinterpret_cast<const float2*>(cb + d0));
                const float x0 = rb0[j] * rsb * wb0[j] + bv.x, x1 = rb1[j] * rsb * wb1[j] + bv.y;
                const float y0 = rc0[j] * rsc * wc0[j] + cv.x, y1 = rc1[j] * rsc * wc1[j] + cv.y;
                float sn, cs;
                sincos_reduced(angv[hh][j], &sn, &cs);
                const float ob0 = x0 * cs - x1 * sn, ob1 = x0 * sn + x1 * cs;
                const float oc0 = y0 * cs - y1 * sn, oc1 = y0 * sn + y1 * cs;
                const float dth = (-gb.x * ob1 + gb.y * ob0) + (-gc.x * oc1 + gc.y * oc0);
                atomicAdd(&sang[h * S + k], dth);  // ranks of the row add up
                gb = make_float2(gb.x * cs + gb.y * sn, -gb.x * sn + gb.y * cs);
                gc = make_float2(gc.x * cs + gc.y * sn, -gc.x * sn + gc.y * cs);
              }
              sbBh[d0] += gb.x; sbBh[d0 + 1] += gb.y;  // warp r owns (h, r, :)
              sbCh[d0] += gc.x; sbCh[d0 + 1] += gc.y;
              db0[j] += gb.x; db1[j] += gb.y;
              dc0[j] += gc.x; dc1[j] += gc.y;
            }
          }
          if (h == H - 1 || G != 1) {
            // RMSNorm backward of group (r, g): draw = (w dn)/rms - raw sum(w dn raw)/(D rms^3)
            float pb = 0.f, pc = 0.f;
#pragma unroll
            for (int j = 0; j < PPL; ++j) {
              pb = fmaf(wb0[j] * db0[j], rb0[j], fmaf(wb1[j] * db1[j], rb1[j], pb));
              pc = fmaf(wc0[j] * dc0[j], rc0[j], fmaf(wc1[j] * dc1[j], rc1[j], pc));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              pb += __shfl_xor_sync(0xffffffffu, pb, o);
              pc += __shfl_xor_sync(0xffffffffu, pc, o);
            }
            const float kb = pb * rsb * rsb * rsb / (float)D, kc = pc * rsc * rsc * rsc / (float)D;
            TZ* ob = drow + (int64_t)(r * G + g) * D;
            TZ* oc = ob + RGD;
#pragma unroll
            for (int j = 0; j < PPL; ++j) {
              const int k = lane + 32 * j;
              if (k < half) {
                st_pair2(ob + 2 * k, wb0[j] * db0[j] * rsb - rb0[j] * kb, wb1[j] * db1[j] * rsb - rb1[j] * kb);
                st_pair2(oc + 2 * k, wc0[j] * dc0[j] * rsc - rc0[j] * kc, wc1[j] * dc1[j] * rsc - rc1[j] * kc);
                dwb0[j] = fmaf(db0[j], rb0[j] * rsb, dwb0[j]); dwb1[j] = fmaf(db1[j], rb1[j] * rsb, dwb1[j]);
                dwc0[j] = fmaf(dc0[j], rc0[j] * rsc, dwc0[j]); dwc1[j] = fmaf(dc1[j], rc1[j] * rsc, dwc1[j]);
              }
            }
          }
        }
      }
    }
    __syncthreads();  // the row's angle gradients complete
    if (rv) {
      float* dst = a.dtheta + rowo * H * S;
      for (int i = threadIdx.x; i < H * S; i += blockDim.x) {
        dst[i] = sang[i];
        sang[i] = 0.f;
      }
    }
    __syncthreads();
  }
  // the CTA's partials into its workspace slot: bias gradients (H, R, D) of B and C, then
  // the norm-weight gradients (D) of B and C (summed over the ranks); plain stores, summed
  // over the slots by bc_reduce_kernel
#pragma unroll
  for (int j = 0; j < PPL; ++j) {
    const int k = lane + 32 * j;
    if (k < half) {
      swb[r * D + 2 * k] = dwb0[j]; swb[r * D + 2 * k + 1] = dwb1[j];
      swc[r * D + 2 * k] = dwc0[j]; swc[r * D + 2 * k + 1] = dwc1[j];
    }
  }
  __syncthreads();
  float* slot = a.bc_part + (int64_t)blockIdx.x * (2 * HRD + 2 * D);
  for (int i = threadIdx.x; i < 2 * HRD; i += blockDim.x) slot[i] = sm[i];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float sb = 0.f, sc = 0.f;
    for (int rr = 0; rr < R; ++rr) {
      sb += swb[rr * D + d];
      sc += swc[rr * D + d];
    }
    slot[2 * HRD + d] = sb;
    slot[2 * HRD + D + d] = sc;
  }
}

// Sum of the bc kernel's workspace slots: thread = output (B bias, C bias, B norm weight, C
// norm weight, in slot order), grid.y = groups of kSlotsPerThread slots, one atomic per
// (output, group) into outputs cleared beforehand.
constexpr int kSlotsPerThread = 64;
__global__ void __launch_bounds__(256) bc_reduce_kernel(PrologueBwdParams a, int nslots) {
  const int HRD = a.H * a.R * a.D, W = 2 * HRD + 2 * a.D;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= W) return;
  const int s0 = blockIdx.y * kSlotsPerThread, s1 = min(s0 + kSlotsPerThread, nslots);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int sl = s0;
  for (; sl + 4 <= s1; sl += 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += a.bc_part[(int64_t)(sl + k) * W + o];
  }
  for (; sl < s1; ++sl) acc[0] += a.bc_part[(int64_t)sl * W + o];
  const float v = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  float* dst = o < HRD ? a.dB_bias + o
               : o < 2 * HRD ? a.dC_bias + (o - HRD)
               : o < 2 * HRD + a.D ? a.dB_norm_w + (o - 2 * HRD)
                                   : a.dC_norm_w + (o - 2 * HRD - a.D);
  atomicAdd(dst, v);
}

// The bc kernel for one B / C group (ngroups 1), a thread per (head, pair) slot of a row
// for every rank: the angle's sin / cos once per (row, head, pair) for all ranks and both B
// and C, dtheta summed in registers and written once, the bias gradients in thread-private
// shared-memory slots, dn (the sum over heads) through shared-memory atomics, one per
// (thread, rank, element) and row. CTAs stride over the rows; a row's dB / dC block, raw
// B / C group rows and angles arrive by bulk copies into one of two buffers while the CTA
// works on the row before (bounded waits). The RMSNorm backward of a row is a warp per
// (B or C, rank). Partial sums go to the CTA's workspace slot as in the general kernel.
constexpr int kBC1 = 256;
__device__ int g_prologue_error;  // set when a bounded wait gives up

struct Bc1Smem {
  uint32_t bias, gb[2], gc[2], zr[2], an[2], rs, sdn, swb, sdv, total;
};
__host__ __device__ inline uint32_t bc1_up(uint32_t v) { return (v + 127u) & ~127u; }
__host__ __device__ inline Bc1Smem bc1_smem(int H, int R, int D, int S, int ez, int eo) {
  Bc1Smem L;
  uint32_t o = 128;  // two mbarriers
  L.bias = o; o = bc1_up(o + (uint32_t)(2 * H * R * D * 4));
  for (int k = 0; k < 2; ++k) {
    L.gb[k] = o; o = bc1_up(o + (uint32_t)(R * H * D * eo));
    L.gc[k] = o; o = bc1_up(o + (uint32_t)(R * H * D * eo));
    L.zr[k] = o; o = bc1_up(o + (uint32_t)(2 * R * D * ez));
    L.an[k] = o; o = bc1_up(o + (uint32_t)(H * S * 4));
  }
  L.rs = o; o = bc1_up(o + (uint32_t)(2 * R * 4));
  L.sdn = o; o = bc1_up(o + (uint32_t)(2 * R * D * 4));
  L.swb = o; o = bc1_up(o + (uint32_t)(2 * R * D * 4));
  // per thread group (the threads whose slots share a pair, when the pairs of a row divide
  // the CTA): its sums over heads of dv, (group, B / C, R, D)
  L.sdv = o; o = bc1_up(o + (uint32_t)((kBC1 % (D / 2) == 0 ? kBC1 / (D / 2) : 0) * 2 * R * D * 4));
  L.total = o + 128;  // slack for aligning the base
  return L;
}

template <typename TZ, typename TO, int RT>
__global__ void __launch_bounds__(kBC1, 3) prologue_bwd_bc1_kernel(PrologueBwdParams a, Bc1Smem L) {
  extern __shared__ __align__(128) unsigned char bsm_raw[];
  unsigned char* bsm = bsm_raw + ((128u - (sm100::smem_u32(bsm_raw) & 127u)) & 127u);
  constexpr int R = RT;
  const int D = a.D, H = a.H, S = a.S, half = D / 2, npair = a.split / 2;
  const int np = H * half;  // (head, pair) slots of a row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(bsm);
  float4* sbias = reinterpret_cast<float4*>(bsm + L.bias);  // [r][slot]: (dB0, dB1, dC0, dC1)
  float* rs = reinterpret_cast<float*>(bsm + L.rs);         // (2, R): 1 / rms
  float* sdn = reinterpret_cast<float*>(bsm + L.sdn);       // (2, R, D): dn = sum over heads of dv
  float* swb = reinterpret_cast<float*>(bsm + L.swb);       // (2, R, D): norm-weight gradient partials
  float* sdv = reinterpret_cast<float*>(bsm + L.sdv);       // (groups, 2, R, D): dn partials per group
  // when the row's pairs divide the CTA, thread t's slots t, t + kBC1, ... share the pair
  // t mod half, and the groups of half threads add their dn partials through sdv (no atomics)
  const bool grouped = kBC1 % half == 0;
  const int ngrp = grouped ? kBC1 / half : 0, grp = grouped ? tid / half : 0;
  const int64_t RD = (int64_t)R * D;
  const uint32_t gbytes = (uint32_t)(R * H * D * sizeof(TO)), zbytes = (uint32_t)(2 * RD * sizeof(TZ)),
                 abytes = (uint32_t)(H * S * 4);
  const int64_t nrows = (int64_t)a.Bn * a.L;
  auto issue = [&](int64_t row, int kb) {
    const int64_t b = row / a.L, l = row - b * a.L;
    uint64_t* bar = &bars[kb];
    sm100::mbar_expect_tx(bar, 2 * gbytes + zbytes + abytes);
    sm100::bulk_load(bsm + (kb ? L.gb[1] : L.gb[0]), reinterpret_cast<const TO*>(a.dBp) + row * R * H * D, gbytes, bar);
    sm100::bulk_load(bsm + (kb ? L.gc[1] : L.gc[0]), reinterpret_cast<const TO*>(a.dCp) + row * R * H * D, gbytes, bar);
    sm100::bulk_load(bsm + (kb ? L.zr[1] : L.zr[0]),
                     reinterpret_cast<const TZ*>(a.zx) + b * a.s_zb + l * a.s_zl + 2 * a.d_inner, zbytes, bar);
    sm100::bulk_load(bsm + (kb ? L.an[1] : L.an[0]), a.angles + row * H * S, abytes, bar);
  };
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
  }
  for (int i = tid; i < R * np; i += kBC1) sbias[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = tid; i < 2 * R * D; i += kBC1) swb[i] = 0.f;
  __syncthreads();
  if (tid == 0 && blockIdx.x < nrows) issue(blockIdx.x, 0);
  uint32_t par0 = 0u, par1 = 0u;
  int k = 0;
  for (int64_t row = blockIdx.x; row < nrows; row += gridDim.x, k ^= 1) {
    __syncthreads();  // the previous row is done with the other buffer, rs and sdn
    if (tid == 0 && row + gridDim.x < nrows) issue(row + gridDim.x, k ^ 1);
    const uint32_t pk = k ? par1 : par0;
    if (!sm100::mbar_wait(&bars[k], pk, 1u << 24)) {  // give up: flag it, wait once more for the copies
      atomicExch(&g_prologue_error, 1);
      sm100::mbar_wait(&bars[k], pk, 1u << 24);
    }
    if (k) par1 ^= 1u; else par0 ^= 1u;
    const TO* gbs = reinterpret_cast<const TO*>(bsm + (k ? L.gb[1] : L.gb[0]));
    const TO* gcs = reinterpret_cast<const TO*>(bsm + (k ? L.gc[1] : L.gc[0]));
    const TZ* zr = reinterpret_cast<const TZ*>(bsm + (k ? L.zr[1] : L.zr[0]));  // B rows (R, D), then C rows (R, D)
    const float* an = reinterpret_cast<const float*>(bsm + (k ? L.an[1] : L.an[0]));
    const int64_t b = row / a.L, l = row - b * a.L;
    TZ* drow = reinterpret_cast<TZ*>(a.dzx) + b * a.s_dzb + l * a.s_dzl + 2 * a.d_inner;
    if (!grouped)
      for (int i = tid; i < 2 * R * D; i += kBC1) sdn[i] = 0.f;
    for (int it = warp; it < 2 * R; it += kBC1 / 32) {
      float ss = 0.f;
      for (int d = lane; d < D; d += 32) {
        const float v = to_f32(zr[it * D + d]);
        ss = fmaf(v, v, ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rs[it] = 1.0f / sqrtf(ss / (float)D + a.eps);
    }
    __syncthreads();
    float dnb0[R], dnb1[R], dnc0[R], dnc1[R];
    int kcur = -1;
#pragma unroll
    for (int r = 0; r < R; ++r) dnb0[r] = dnb1[r] = dnc0[r] = dnc1[r] = 0.f;
    for (int sl = tid, hg = grp; sl < np; sl += kBC1, hg += ngrp) {
      const int h = grouped ? hg : sl / half, kp = sl - h * half, d0 = 2 * kp;
      if (kp != kcur) {  // flush the running sums over heads of the previous pair
        if (kcur >= 0) {  // (only without groups: a grouped thread's slots share one pair)
#pragma unroll
          for (int r = 0; r < R; ++r) {
            atomicAdd(&sdn[r * D + 2 * kcur], dnb0[r]); atomicAdd(&sdn[r * D + 2 * kcur + 1], dnb1[r]);
            atomicAdd(&sdn[RD + r * D + 2 * kcur], dnc0[r]); atomicAdd(&sdn[RD + r * D + 2 * kcur + 1], dnc1[r]);
            dnb0[r] = dnb1[r] = dnc0[r] = dnc1[r] = 0.f;
          }
        }
        kcur = kp;
      }
      const bool rot = kp < npair;
      float sn = 0.f, cs = 1.f;
      if (rot) sincos_reduced(an[h * S + kp], &sn, &cs);
      const float2 wb = __ldg(reinterpret_cast<const float2*>(a.B_norm_w + d0));
      const float2 wc = __ldg(reinterpret_cast<const float2*>(a.C_norm_w + d0));
      float dth = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float2 g1 = ld_pair(gbs + ((int64_t)r * H + h) * D + d0), g2 = ld_pair(gcs + ((int64_t)r * H + h) * D + d0);
        if (rot) {
          // o = rot(v), v = n + bias; dv = rot^T(g); dtheta = -g1 o2 + g2 o1 = dv2 v1 - dv1 v2
          // (the rotation commutes with the quarter turn)
          g1 = make_float2(g1.x * cs + g1.y * sn, -g1.x * sn + g1.y * cs);
          g2 = make_float2(g2.x * cs + g2.y * sn, -g2.x * sn + g2.y * cs);
          const float2 bv = __ldg(reinterpret_cast<const float2*>(a.B_bias + ((int64_t)h * R + r) * D + d0));
          const float2 cv = __ldg(reinterpret_cast<const float2*>(a.C_bias + ((int64_t)h * R + r) * D + d0));
          const float rb = rs[r], rc = rs[R + r];
          const float2 zb = ld_pair(zr + r * D + d0), zc = ld_pair(zr + RD + r * D + d0);
          const float x0 = fmaf(zb.x * rb, wb.x, bv.x), x1 = fmaf(zb.y * rb, wb.y, bv.y);
          const float y0 = fmaf(zc.x * rc, wc.x, cv.x), y1 = fmaf(zc.y * rc, wc.y, cv.y);
          dth += fmaf(g1.y, x0, -g1.x * x1) + fmaf(g2.y, y0, -g2.x * y1);
        }
        float4 acc = sbias[r * np + sl];
        acc.x += g1.x; acc.y += g1.y; acc.z += g2.x; acc.w += g2.y;
        sbias[r * np + sl] = acc;
        dnb0[r] += g1.x; dnb1[r] += g1.y; dnc0[r] += g2.x; dnc1[r] += g2.y;
      }
      if (rot) a.dtheta[(row * H + h) * S + kp] = dth;
    }
    if (grouped) {
      // the group's sums over its heads; every thread of the CTA owns one (group, pair)
      const int kq = tid - grp * half;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        *reinterpret_cast<float2*>(&sdv[((size_t)grp * 2 * R + r) * D + 2 * kq]) = make_float2(dnb0[r], dnb1[r]);
        *reinterpret_cast<float2*>(&sdv[((size_t)grp * 2 * R + R + r) * D + 2 * kq]) = make_float2(dnc0[r], dnc1[r]);
      }
    } else if (kcur >= 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        atomicAdd(&sdn[r * D + 2 * kcur], dnb0[r]); atomicAdd(&sdn[r * D + 2 * kcur + 1], dnb1[r]);
        atomicAdd(&sdn[RD + r * D + 2 * kcur], dnc0[r]); atomicAdd(&sdn[RD + r * D + 2 * kcur + 1], dnc1[r]);
      }
    }
    __syncthreads();
    if (grouped) {
      for (int i = tid; i < 2 * R * D; i += kBC1) {
        float v = 0.f;
        for (int g2 = 0; g2 < ngrp; ++g2) v += sdv[(size_t)g2 * 2 * R * D + i];
        sdn[i] = v;
      }
      __syncthreads();
    }
    // RMSNorm backward of (B or C, rank): draw = (w dn) / rms - raw sum(w dn raw) / (D rms^3)
    for (int it = warp; it < 2 * R; it += kBC1 / 32) {
      const float* w = it < R ? a.B_norm_w : a.C_norm_w;
      const float rr = rs[it];
      float pb = 0.f;
      for (int d = lane; d < D; d += 32) pb = fmaf(__ldg(w + d) * sdn[it * D + d], to_f32(zr[it * D + d]), pb);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pb += __shfl_xor_sync(0xffffffffu, pb, o);
      const float kk = pb * rr * rr * rr / (float)D;
      for (int d = lane; d < D; d += 32) {
        const float dn = sdn[it * D + d], rv = to_f32(zr[it * D + d]);
        drow[it * D + d] = from_f32<TZ>(fmaf(__ldg(w + d) * dn, rr, -rv * kk));
        swb[it * D + d] = fmaf(dn, rv * rr, swb[it * D + d]);
      }
    }
  }
  // the CTA's partial sums into its slot: bias gradients (H, R, D) of B and C, then the
  // norm-weight gradients (D) of B and C
  __syncthreads();
  const int HRD = H * R * D;
  float* slot = a.bc_part + (int64_t)blockIdx.x * (2 * HRD + 2 * D);
  for (int i = tid; i < HRD; i += kBC1) {
    const int h = i / (R * D), rem = i - h * R * D, r = rem / D, d = rem - r * D;
    const float4 v = sbias[r * np + h * half + (d >> 1)];
    slot[i] = (d & 1) ? v.y : v.x;
    slot[HRD + i] = (d & 1) ? v.w : v.z;
  }
  for (int d = tid; d < D; d += kBC1) {
    float sb = 0.f, sc = 0.f;
    for (int r = 0; r < R; ++r) {
      sb += swb[r * D + d];
      sc += swb[RD + r * D + d];
    }
    slot[2 * HRD + d] = sb;
    slot[2 * HRD + D + d] = sc;
  }
}

// CTA per (b, h); thread = step of a 128-step tile walked from the end; suffix sums over l
// of dtheta[b,l,h,i] for the S angles, 16 at a time, carried between tiles
template <typename TZ, int kAT>
__global__ void __launch_bounds__(kAT) prologue_bwd_angle_kernel(PrologueBwdParams a) {
  constexpr int kS = 16;
  __shared__ float wsum[kAT / 32][kS];
  __shared__ float carry[64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int u = blockIdx.x, b = u / a.H, h = u - b * a.H;
  const int H = a.H, S = a.S;
  const int off_ang = 2 * a.d_inner + 2 * a.D * a.G * a.R + 3 * H;
  const TZ* base = reinterpret_cast<const TZ*>(a.zx) + (int64_t)b * a.s_zb;
  for (int s0 = tid; s0 < S; s0 += kAT) carry[s0] = 0.f;
  __syncthreads();
  const int ntile = (a.L + kAT - 1) / kAT;
  for (int tt = ntile - 1; tt >= 0; --tt) {
    const int l = tt * kAT + tid;
    const bool v = l < a.L;
    const int64_t o = ((int64_t)b * a.L + (v ? l : 0)) * H + h;
    const TZ* row = base + (int64_t)(v ? l : 0) * a.s_zl;
    const float dtv = v ? a.DT[o] : 0.f;
    float ddt = 0.f;
    for (int s0 = 0; s0 < S; s0 += kS) {
      float x[kS];
#pragma unroll
      for (int k = 0; k < kS; ++k) x[k] = (v && s0 + k < S) ? a.dtheta[o * S + s0 + k] : 0.f;
#pragma unroll
      for (int of = 1; of < 32; of <<= 1) {
#pragma unroll
        for (int k = 0; k < kS; ++k) {
          const float y = __shfl_down_sync(0xffffffffu, x[k], of);
          if (lane + of < 32) x[k] += y;
        }
      }
      if (lane == 0)
#pragma unroll
        for (int k = 0; k < kS; ++k) wsum[warp][k] = x[k];
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kS; ++k) {
        float post = s0 + k < S ? carry[s0 + k] : 0.f;
        for (int w = warp + 1; w < kAT / 32; ++w) post += wsum[w][k];
        x[k] += post;
      }
      if (v) {
#pragma unroll
        for (int k = 0; k < kS; ++k) {
          if (s0 + k < S) {
            ddt = fmaf(x[k], to_f32(row[off_ang + s0 + k]), ddt);
            atomicAdd(a.dangle_raw + ((int64_t)b * a.L + l) * S + s0 + k, x[k] * dtv);
          }
        }
      }
      __syncthreads();  // carry and wsum read by every thread before they change
      if (tid == 0)
#pragma unroll
        for (int k = 0; k < kS; ++k)
          if (s0 + k < S) carry[s0 + k] = x[k];
    }
    if (v) a.dDT_ang[o] = ddt;
    __syncthreads();
  }
}

// thread per (b, l, h)
template <typename TZ>
__global__ void __launch_bounds__(256) prologue_bwd_dt_kernel(PrologueBwdParams a) {
  __shared__ float sdb[256];
  const int64_t n = (int64_t)a.Bn * a.L * a.H;
  const int H = a.H, S = a.S;
  const int off_dt = 2 * a.d_inner + 2 * a.D * a.G * a.R;
  const int off_A = off_dt + H, off_tr = off_A + H, off_ang = off_tr + H;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float dpre = 0.f;
  int h = 0;
  if (i < n) {
    const int64_t bl = i / H;
    h = (int)(i - bl * H);
    const int64_t b = bl / a.L, l = bl - b * a.L;
    const TZ* row = reinterpret_cast<const TZ*>(a.zx) + b * a.s_zb + l * a.s_zl;
    TZ* drow = reinterpret_cast<TZ*>(a.dzx) + b * a.s_dzb + l * a.s_dzl;
    const float A = -fminf(softplusf_(to_f32(row[off_A + h])), -a.A_floor);
    const float pre = to_f32(row[off_dt + h]) + a.dt_bias[h];
    const float dDT = a.dDT[i] + A * a.dADT[i] + a.dDT_ang[i];
    dpre = dDT * (pre > 20.0f ? 1.0f : sigmoidf_(pre));
    drow[off_dt + h] = from_f32<TZ>(dpre);
    drow[off_A + h] = from_f32<TZ>(0.f);  // the clamp of layer.py:207 passes no gradient
    drow[off_tr + h] = from_f32<TZ>(a.dtrap[i]);
    if (h == 0)
      for (int k = 0; k < S; ++k) drow[off_ang + k] = from_f32<TZ>(a.dangle_raw[bl * S + k]);
  }
  // dt_bias: the block's sums per head (thread t of the block holds head (start + t) mod H),
  // then one atomic per head and block
  sdb[threadIdx.x] = dpre;
  __syncthreads();
  const int64_t start = (int64_t)blockIdx.x * blockDim.x;
  const int s0 = (int)(start % H);
  for (int hh = threadIdx.x; hh < H; hh += blockDim.x) {
    float sum = 0.f;
    for (int t = (hh - s0 + H) % H; t < (int)blockDim.x; t += H)
      if (start + t < n) sum += sdb[t];
    atomicAdd(a.ddt_bias + hh, sum);
  }
  (void)h;
}

template <typename TY, typename TZ, typename TD>
__global__ void __launch_bounds__(256) gate_bwd_kernel(GateBwdParams a) {
  const int64_t n = a.rows * a.P;
  const int LH = a.L * a.H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / a.P;
    const int p = (int)(i - r * a.P);
    const int64_t b = r / LH;
    const int rem = (int)(r - b * LH);
    const int l = rem / a.H, h = rem - l * a.H;
    const float yv = to_f32(reinterpret_cast<const TY*>(a.y)[b * a.sy.b + (int64_t)l * a.sy.l + (int64_t)h * a.sy.h + p]);
    const float zv = to_f32(reinterpret_cast<const TZ*>(a.z)[b * a.sz.b + (int64_t)l * a.sz.l + (int64_t)h * a.sz.h + p]);
    const float g = to_f32(reinterpret_cast<const TD*>(a.dout)[b * a.sd.b + (int64_t)l * a.sd.l + (int64_t)h * a.sd.h + p]);
    const float sg = sigmoidf_(zv);
    reinterpret_cast<TY*>(a.dy)[b * a.sdy.b + (int64_t)l * a.sdy.l + (int64_t)h * a.sdy.h + p] =
        from_f32<TY>(g * zv * sg);
    reinterpret_cast<TZ*>(a.dz)[b * a.sdz.b + (int64_t)l * a.sdz.l + (int64_t)h * a.sdz.h + p] =
        from_f32<TZ>(g * yv * sg * (1.0f + zv * (1.0f - sg)));
  }
}

// The gate backward on 16-byte groups of p (one dtype for all five tensors, rows and strides
// in whole 16-byte units): index arithmetic once per group, 16-byte loads and stores.
struct Div32 {
  uint32_t m, s;
};
inline Div32 make_div32(uint32_t d) {
  Div32 f;
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  f.s = s;
  f.m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);  // round-up multiplier (Granlund-Montgomery)
  return f;
}
__device__ __forceinline__ uint32_t div32(uint32_t x, Div32 f) { return (__umulhi(x, f.m) + x) >> f.s; }

template <typename T>
__global__ void __launch_bounds__(256) gate_bwd_vec_kernel(GateBwdParams a, Div32 fpc, Div32 fh, Div32 flh,
                                                           uint32_t ngroups) {
  constexpr int V = 16 / sizeof(T);
  const uint32_t PC = (uint32_t)a.P / V;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < ngroups; i += gridDim.x * blockDim.x) {
    const uint32_t r = div32(i, fpc), j = i - r * PC;
    const uint32_t b = div32(r, flh), rem = r - b * (uint32_t)(a.L * a.H);
    const uint32_t l = div32(rem, fh), h = rem - l * (uint32_t)a.H;
    const int64_t p = (int64_t)j * V;
    auto at = [&](const Str3& st) { return (int64_t)b * st.b + (int64_t)l * st.l + (int64_t)h * st.h + p; };
    const uint4 yw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.y) + at(a.sy));
    const uint4 zw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.z) + at(a.sz));
    const uint4 gw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.dout) + at(a.sd));
    const T* yv = reinterpret_cast<const T*>(&yw);
    const T* zv = reinterpret_cast<const T*>(&zw);
    const T* gv = reinterpret_cast<const T*>(&gw);
    uint4 dyw, dzw;
    T* dyv = reinterpret_cast<T*>(&dyw);
    T* dzv = reinterpret_cast<T*>(&dzw);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float y = to_f32(yv[e]), z = to_f32(zv[e]), g = to_f32(gv[e]);
      const float sg = sigmoidf_(z);
      dyv[e] = from_f32<T>(g * z * sg);
      dzv[e] = from_f32<T>(g * y * sg * (1.0f + z * (1.0f - sg)));
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.dy) + at(a.sdy)) = dyw;
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.dz) + at(a.sdz)) = dzw;
  }
}

template <typename T>
bool gate_vec_ok(const GateBwdParams& p) {
  const int64_t e = sizeof(T), V = 16 / e;
  auto al = [&](const void* q, const Str3& st) {
    return reinterpret_cast<uintptr_t>(q) % 16 == 0 && (st.b * e) % 16 == 0 && (st.l * e) % 16 == 0 &&
           (st.h * e) % 16 == 0;
  };
  return p.P % V == 0 && p.rows * (p.P / V) < (int64_t(1) << 31) && al(p.y, p.sy) && al(p.z, p.sz) &&
         al(p.dout, p.sd) && al(p.dy, p.sdy) && al(p.dz, p.sdz);
}

template <typename T>
int launch_gate_bwd_vec(const GateBwdParams& p, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const uint32_t ng = (uint32_t)(p.rows * (p.P / V));
  const unsigned grid = (unsigned)std::min<int64_t>((ng + 255) / 256, 148 * 16);
  gate_bwd_vec_kernel<T><<<grid, 256, 0, s>>>(p, make_div32((uint32_t)(p.P / V)), make_div32((uint32_t)p.H),
                                              make_div32((uint32_t)(p.L * p.H)), ng);
  return check_launch("gate_bwd_vec_kernel");
}

}  // namespace

int prologue_error_word(bool reset, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_prologue_error, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_prologue_error, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("prologue error word: ") + cudaGetErrorString(e));
  *out = v;
  return M3_OK;
}

// Slots of the bc kernel's partial sums: one per CTA, at most 1024 and at most 32 MB.
int64_t bc_slots(int64_t rows, int64_t H, int64_t R, int64_t D) {
  const int64_t W = 2 * H * R * D + 2 * D;
  const int64_t cap = std::max<int64_t>(1, std::min<int64_t>(1024, (int64_t(32) << 20) / (4 * W)));
  return std::max<int64_t>(1, std::min<int64_t>((rows + kRowsBC - 1) / kRowsBC, cap));
}

size_t prologue_bwd_workspace_bytes(int64_t Bn, int64_t L, int64_t H, int64_t S, int64_t R, int64_t D) {
  // dtheta (B, L, H, S), dDT_ang (B, L, H), dangle_raw (B, L, S), then the bc kernel's
  // partial-sum slots, all fp32
  const int64_t rows = Bn * L;
  return sizeof(float) * (size_t)(rows * (H * S + H + S) + bc_slots(rows, H, R, D) * (2 * H * R * D + 2 * D));
}

// Launch of the slot-per-thread bc kernel: as many CTAs as fit on the device at once, at
// most `slots` (each CTA writes one slot); *used = the CTAs launched.
template <typename K>
int bc1_launch(K k, const PrologueBwdParams& p, const Bc1Smem& L, unsigned slots, unsigned* used,
               cudaStream_t s) {
  const size_t smem = L.total;
  static LaunchCache lc[16];  // per instantiation of this launcher: one per kernel pointer below
  static std::atomic<const void*> keys[16];
  const void* kp = reinterpret_cast<const void*>(k);
  int slot = -1;
  for (int i = 0; i < 16 && slot < 0; ++i) {
    const void* cur = keys[i].load(std::memory_order_acquire);
    if (cur == kp) slot = i;
    else if (cur == nullptr) {
      const void* expect = nullptr;
      if (keys[i].compare_exchange_strong(expect, kp) || expect == kp) slot = i;
    }
  }
  if (slot < 0) return fail(M3_ERR_UNSUPPORTED, "prologue backward: launch cache full");
  int resident = 1;
  M3_TRY(kernel_residency(kp, kBC1, smem, &lc[slot], &resident));
  *used = std::min<unsigned>(slots, (unsigned)resident);
  k<<<*used, kBC1, smem, s>>>(p, L);
  return check_launch("prologue_bwd_bc1_kernel");
}

int launch_prologue_bwd(const PrologueBwdParams& p0, float* ws, int zdt, int odt, cudaStream_t s) {
  PrologueBwdParams p = p0;
  if (p.S > 64) return fail(M3_ERR_UNSUPPORTED, "prologue backward: more than 64 rope angles");
  if (p.D % 2 || p.D > 256 || p.R > 8) return fail(M3_ERR_UNSUPPORTED, "prologue backward: d_state or rank");
  if ((reinterpret_cast<uintptr_t>(p.B_bias) | reinterpret_cast<uintptr_t>(p.C_bias)) & 7)
    return fail(M3_ERR_UNSUPPORTED, "prologue backward: B_bias / C_bias must be 8-byte aligned");
  const int64_t rows = (int64_t)p.Bn * p.L;
  p.dtheta = ws;
  p.dDT_ang = ws + rows * p.H * p.S;
  p.dangle_raw = p.dDT_ang + rows * p.H;
  p.bc_part = p.dangle_raw + rows * p.S;
  const int64_t nslots = bc_slots(rows, p.H, p.R, p.D);
  const int W = 2 * p.H * p.R * p.D + 2 * p.D;
  const size_t zero_bytes = sizeof(float) * (size_t)(rows * p.S);
  cudaError_t e = cudaMemsetAsync(p.dangle_raw, 0, zero_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.dB_bias, 0, sizeof(float) * (size_t)p.H * p.R * p.D, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.dC_bias, 0, sizeof(float) * (size_t)p.H * p.R * p.D, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.dB_norm_w, 0, sizeof(float) * (size_t)p.D, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.dC_norm_w, 0, sizeof(float) * (size_t)p.D, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.ddt_bias, 0, sizeof(float) * (size_t)p.H, s);
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("prologue backward memset: ") + cudaGetErrorString(e));
  const size_t smem = sizeof(float) * (size_t)(2 * p.H * p.R * p.D + p.H * p.S + 2 * p.R * p.D);
  if (smem > 200 * 1024) return fail(M3_ERR_UNSUPPORTED, "prologue backward: nheads * rank * d_state too large");
  const unsigned gbc = (unsigned)nslots;
  // one B / C group and a power-of-two rank up to 8: the slot-per-thread kernel
  // one B / C group, a power-of-two rank up to 8, and every row's blocks on 16-byte
  // boundaries in whole 16-byte units (bulk copies): the slot-per-thread kernel
  const int ez = zdt == M3_FLOAT32 ? 4 : 2, eo = odt == M3_FLOAT32 ? 4 : 2;
  const Bc1Smem L1 = bc1_smem(p.H, p.R, p.D, p.S, ez, eo);
  auto a16 = [](int64_t v) { return v % 16 == 0; };
  const bool bc1 = p.G == 1 && (p.R == 1 || p.R == 2 || p.R == 4 || p.R == 8) && L1.total <= 200 * 1024 &&
                   ((reinterpret_cast<uintptr_t>(p.B_norm_w) | reinterpret_cast<uintptr_t>(p.C_norm_w)) & 7) == 0 &&
                   a16((int64_t)p.R * p.H * p.D * eo) && a16(2 * (int64_t)p.R * p.D * ez) &&
                   a16((int64_t)p.H * p.S * 4) && p.S > 0 && a16(p.s_zb * ez) && a16(p.s_zl * ez) &&
                   a16(2 * (int64_t)p.d_inner * ez) &&
                   ((reinterpret_cast<uintptr_t>(p.zx) | reinterpret_cast<uintptr_t>(p.dBp) |
                     reinterpret_cast<uintptr_t>(p.dCp) | reinterpret_cast<uintptr_t>(p.angles)) & 15) == 0;
  const int ppl = (p.D / 2 + 31) / 32;
  const unsigned gdt = (unsigned)((rows * p.H + 255) / 256);
  int nsm = 148;
  if (device_sm_count(&nsm) != M3_OK) nsm = 148;
  const bool wide = (int64_t)p.Bn * p.H < 4 * (int64_t)nsm && p.L > 128;
#define M3_PBWD(TZ, TO)                                                                                  \
  do {                                                                                                   \
    unsigned used = gbc;                                                                                 \
    if (bc1) {                                                                                           \
      auto k1 = p.R == 1 ? prologue_bwd_bc1_kernel<TZ, TO, 1>                                            \
                         : p.R == 2 ? prologue_bwd_bc1_kernel<TZ, TO, 2>                                 \
                                    : p.R == 4 ? prologue_bwd_bc1_kernel<TZ, TO, 4> : prologue_bwd_bc1_kernel<TZ, TO, 8>; \
      M3_TRY(bc1_launch(k1, p, L1, gbc, &used, s));                                                   \
    } else {                                                                                             \
      auto kbc = ppl == 1 ? prologue_bwd_bc_kernel<TZ, TO, 1>                                            \
                          : (ppl == 2 ? prologue_bwd_bc_kernel<TZ, TO, 2> : prologue_bwd_bc_kernel<TZ, TO, 4>); \
      if (smem > 48 * 1024) {                                                                            \
        cudaError_t ea = cudaFuncSetAttribute(kbc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (ea != cudaSuccess) return fail(M3_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(ea)); \
      }                                                                                                  \
      kbc<<<gbc, 32 * p.R, smem, s>>>(p);                                                                \
      M3_TRY(check_launch("prologue_bwd_bc_kernel"));                                                    \
    }                                                                                                    \
    bc_reduce_kernel<<<dim3((unsigned)((W + 255) / 256), (unsigned)((used + kSlotsPerThread - 1) / kSlotsPerThread)), \
                       256, 0, s>>>(p, (int)used);                                                        \
    M3_TRY(check_launch("bc_reduce_kernel"));                                                            \
    if (wide) prologue_bwd_angle_kernel<TZ, kATmax><<<(unsigned)(p.Bn * p.H), kATmax, 0, s>>>(p);         \
    else prologue_bwd_angle_kernel<TZ, 128><<<(unsigned)(p.Bn * p.H), 128, 0, s>>>(p);                   \
    M3_TRY(check_launch("prologue_bwd_angle_kernel"));                                                   \
    prologue_bwd_dt_kernel<TZ><<<gdt, 256, 0, s>>>(p);                                                   \
    return check_launch("prologue_bwd_dt_kernel");                                                       \
  } while (0)
  if (zdt == M3_BFLOAT16 && odt == M3_BFLOAT16) M3_PBWD(__nv_bfloat16, __nv_bfloat16);
  if (zdt == M3_BFLOAT16 && odt == M3_FLOAT32) M3_PBWD(__nv_bfloat16, float);
  if (zdt == M3_FLOAT32 && odt == M3_FLOAT32) M3_PBWD(float, float);
  if (zdt == M3_FLOAT16 && odt == M3_FLOAT32) M3_PBWD(__half, float);
#undef M3_PBWD
  return fail(M3_ERR_UNSUPPORTED, "prologue backward: unsupported dtype pair");
}

int launch_gate_bwd(const GateBwdParams& p, int ydt, int zdt, int ddt, cudaStream_t s) {
  const int64_t n = p.rows * p.P;
  if (n == 0) return M3_OK;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
#define M3_GB(TY, TZ, TD)                                \
  do {                                                   \
    gate_bwd_kernel<TY, TZ, TD><<<grid, 256, 0, s>>>(p); \
    return check_launch("gate_bwd_kernel");              \
  } while (0)
  if (ydt == zdt && zdt == ddt && (int64_t)p.L * p.H < (int64_t(1) << 31)) {
    if (ydt == M3_BFLOAT16 && gate_vec_ok<__nv_bfloat16>(p)) return launch_gate_bwd_vec<__nv_bfloat16>(p, s);
    if (ydt == M3_FLOAT32 && gate_vec_ok<float>(p)) return launch_gate_bwd_vec<float>(p, s);
    if (ydt == M3_FLOAT16 && gate_vec_ok<__half>(p)) return launch_gate_bwd_vec<__half>(p, s);
  }
  if (ydt == M3_BFLOAT16 && zdt == M3_BFLOAT16 && ddt == M3_BFLOAT16) M3_GB(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
  if (ydt == M3_FLOAT32 && zdt == M3_FLOAT32 && ddt == M3_FLOAT32) M3_GB(float, float, float);
  if (ydt == M3_FLOAT16 && zdt == M3_FLOAT16 && ddt == M3_FLOAT16) M3_GB(__half, __half, __half);
#undef M3_GB
  return fail(M3_ERR_UNSUPPORTED, "gate backward: unsupported dtype combination");
}

}  // namespace m3
