/* CPU mirror of the device's exp_pair (bitnetrs_b200/csrc/common.cuh), the
 * same float operations in the same order with the same pair tables, used by
 * tests/test_exp_pair_cpu.py to check it against the host libm's expf:
 *   exp_pair_mirror STRIDE
 * visits every STRIDE-th float of [-87, 0] (STRIDE 1: all of them) and
 * prints how many non-candidates round differently from expf (must be 0)
 * and the largest distance of hi + lo from exp(x) * 2^S (long double), in
 * float ulps.  Build with -ffp-contract=off so no multiply-add is fused. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float en_hi[88], en_lo[88], en_s[88], fj_hi[128], fj_lo[128];

static void tables(void) {
  for (int k = 0; k < 88; ++k) {
    long double v = expl(-(long double)k);
    int S = (int)lrintl((long double)k * 1.442695040888963407359924681L);
    long double w = ldexpl(v, S);
    en_hi[k] = (float)w;
    en_lo[k] = (float)(w - (long double)en_hi[k]);
    en_s[k] = (float)S;
  }
  for (int j = 0; j < 128; ++j) {
    long double v = expl(-(long double)j / 128.0L);
    fj_hi[j] = (float)v;
    fj_lo[j] = (float)(v - (long double)fj_hi[j]);
  }
}

static uint32_t fb(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float bf(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* 1: candidate, 0: not, with *f, the pair and S for the error check */
static int exp_pair(float x, float* f, float* phi, float* plo, int* s_out) {
  const float n = ceilf(x);
  const float fr = x - n;
  const float jf = ceilf(fr * 128.0f);
  const float r = fr - jf * 0.0078125f;
  float q = fmaf(r, 0x1.111112p-7f, 0x1.555556p-5f);
  q = fmaf(q, r, 0x1.555556p-3f);
  q = fmaf(q, r, 0.5f);
  q = q * (r * r);
  const float a_hi = 1.0f + r;
  const float a_lo = (r - (a_hi - 1.0f)) + q;
  const int k = (int)(-n), j = (int)(-jf);
  const float p = en_hi[k] * fj_hi[j];
  float pe = fmaf(en_hi[k], fj_hi[j], -p);
  pe = fmaf(en_hi[k], fj_lo[j], pe);
  pe = fmaf(en_lo[k], fj_hi[j], pe);
  const float y = p * a_hi;
  float ye = fmaf(p, a_hi, -y);
  ye = fmaf(p, a_lo, ye);
  ye = fmaf(pe, a_hi, ye);
  const float hi = y + ye;
  const float lo = ye - (hi - y);
  const int S = (int)en_s[k];
  const uint32_t hb = fb(hi);
  *f = bf(hb - ((uint32_t)S << 23));
  *phi = hi;
  *plo = lo;
  *s_out = S;
  float ulp = bf((hb & 0x7f800000u) - (23u << 23));
  if (lo < 0.0f && (hb & 0x7fffffu) == 0u) ulp = ulp * 0.5f;
  return fabsf(lo) > 0.497f * ulp;
}

int main(int argc, char** argv) {
  const uint32_t stride = argc > 1 ? (uint32_t)atoi(argv[1]) : 1u;
  tables();
  long n = 0, cand = 0, bad = 0;
  double maxerr = 0.0;
  for (uint32_t u = 0x80000000u; u <= fb(-87.0f); u += stride) {
    const float x = bf(u);
    float f, hi, lo;
    int S;
    const int c = exp_pair(x, &f, &hi, &lo, &S);
    ++n;
    const long double ex = ldexpl(expl((long double)x), S);
    const long double ulp = ldexpl(1.0L, (int)((fb(hi) >> 23) & 0xff) - 127 - 23);
    const double e = (double)(fabsl(((long double)hi + (long double)lo) - ex) / ulp);
    if (e > maxerr) maxerr = e;
    if (c)
      ++cand;
    else if (fb(expf(x)) != fb(f))
      ++bad;
  }
  printf("checked %ld candidates %ld non_candidate_mismatches %ld max_err_ulp %.6g\n", n, cand, bad, maxerr);
  return bad != 0;
}
