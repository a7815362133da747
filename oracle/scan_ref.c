/*
 * CPU restatement of the reference's SISO scan loop, in fp32 C with OpenMP over the
 * independent (batch, head) units. Test infrastructure and CPU baseline only: nothing in
 * the product links or loads it.
 *
 * It follows mamba3_ssm/ops.py:142-177 of Aiyoniganmaaiya/mamba3-ssm v0.2.1 step for
 * step in fp32: decay = exp(ADT), dt = DT, tr = sigmoid(trap) (ops.py:146-148); for every
 * timestep Bx = x (x) B, blend = (1-tr) Bx + tr * 0.5 * (Bx + Bx_prev), h = decay h +
 * dt blend, y = C.h + D x, Bx_prev = Bx (ops.py:166-175). Pinned against the reference's
 * golden fixtures by tests/test_oracle_golden.py.
 *
 * Layouts (contiguous): x, y (B,L,H,P); Bm, Cm (B,L,H,D); adt, dt, trap (B,L,H); Dk (H).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int m3_ref_siso_fwd(const float* x, const float* Bm, const float* Cm, const float* adt, const float* dtp,
                    const float* trap, const float* Dk, float* y, int nb, int L, int H, int P, int D,
                    int nthreads) {
  if (nthreads > 0) {
#ifdef _OPENMP
    omp_set_num_threads(nthreads);
#endif
  }
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : bad)
  for (int u = 0; u < nb * H; ++u) {
    const int b = u / H, hh = u % H;
    float* h = (float*)calloc((size_t)P * D, sizeof(float));
    float* bxp = (float*)calloc((size_t)P * D, sizeof(float));
    if (!h || !bxp) {
      bad += 1;
      free(h);
      free(bxp);
      continue;
    }
    for (int t = 0; t < L; ++t) {
      const size_t s = ((size_t)b * L + t) * H + hh;
      const float decay = expf(adt[s]);
      const float dt = dtp[s];
      const float tr = 1.0f / (1.0f + expf(-trap[s]));
      const float* xt = x + s * P;
      const float* Bt = Bm + s * D;
      const float* Ct = Cm + s * D;
      float* yt = y + s * P;
      for (int p = 0; p < P; ++p) {
        const float xv = xt[p];
        float* hp = h + (size_t)p * D;
        float* bp = bxp + (size_t)p * D;
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) {
          const float bx = xv * Bt[d];
          const float blend = (1.0f - tr) * bx + tr * 0.5f * (bx + bp[d]);
          const float hn = decay * hp[d] + dt * blend;
          hp[d] = hn;
          bp[d] = bx;
          acc += Ct[d] * hn;
        }
        yt[p] = acc + Dk[hh] * xv;
      }
    }
    free(h);
    free(bxp);
  }
  return bad;
}

int m3_ref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
