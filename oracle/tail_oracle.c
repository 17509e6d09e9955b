/*
 * C restatement of verbo's logits producer tail - TEST INFRASTRUCTURE ONLY.
 *
 * Session::Impl::batch ends (src/session.cpp:163-169) with
 *   rmsnorm(x_i, model.norm, xb_i)          for every output row i,
 *   act(head, xb)                           quant_act per row for Q8/Q4 heads,
 *   matmul(head, act, out)                  one dot product per (row, vocab id).
 * This file restates the reference's SCALAR build (CMake option VERBO_SCALAR,
 * which defines VERBO_FORCE_SCALAR): the dot products accumulate in the order
 * of the scalar loops of src/kernels.cpp, so the result is bit-identical to
 * that build; the AVX2 build sums the same terms in another order.
 *
 * Rounding follows that build as g++ compiles it (-O3, x86-64-v3): the
 * rmsnorm sum of squares and dot_f32 round every product and every sum, while
 * the block accumulate of dot_q8/dot_q4, r += (scale_w * scale_x) * sum, is
 * contracted into one fused multiply-add (found by calling the reference's
 * compiled dot_q8 on seeded blocks).  This file is built with
 * -ffp-contract=off and writes that one FMA out as fmaf.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "oracle.h"

enum { kBlk = 32 }; /* quantisation block, src/kernels.hpp:11 */

/* binary16 bits -> float, exactly (h2f, src/kernels.cpp:38): every half is a
   small integer times a power of two, which ldexpf represents exactly. */
static float half_bits_to_float(uint16_t h) {
  const int e = (h >> 10) & 0x1F;
  const int m = h & 0x3FF;
  float v;
  if (e == 31)
    v = m ? NAN : INFINITY;
  else if (e == 0)
    v = ldexpf((float)m, -24);
  else
    v = ldexpf((float)(m | 0x400), e - 25);
  return (h & 0x8000) ? -v : v;
}

/* rmsnorm, src/session.cpp:14-19: the sum of squares in index order, one
   rounding per product and per sum; r = 1/sqrt(mean + eps); w * (x * r). */
static void rms_norm_row(const float* x, const float* w, float* out, int n, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float p = x[i] * x[i];
    ss = ss + p;
  }
  const float r = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; ++i) out[i] = w[i] * (x[i] * r);
}

/* quant_act, src/kernels.cpp:106 (scalar branch): per 32-block d = amax/127,
   q = nearbyint(v / d) through the reciprocal, no clamp. */
static void quant_row(const float* v, int n, int8_t* q, float* s) {
  for (int b = 0; b < n / kBlk; ++b) {
    const float* x = v + b * kBlk;
    float amax = 0.0f;
    for (int i = 0; i < kBlk; ++i) {
      const float a = fabsf(x[i]);
      if (amax < a) amax = a; /* std::max(amax, a): a NaN never replaces amax */
    }
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    s[b] = d;
    for (int i = 0; i < kBlk; ++i) {
      const float t = nearbyintf(x[i] * id);
      q[b * kBlk + i] = isnan(t) ? (int8_t)0 : (int8_t)(int)t;
    }
  }
}

/* dot_q8 / dot_q4 / dot_f32, src/kernels.cpp:576-606 (scalar build): an exact
   integer sum per block, then r = fma(scale_w * scale_x, sum, r) in block
   order; dot_f32 rounds the product and the sum separately. */
static float dot_q8_row(const int8_t* w, const uint16_t* ws, const int8_t* x, const float* xs, int nb) {
  float r = 0.0f;
  for (int b = 0; b < nb; ++b) {
    int32_t acc = 0;
    for (int i = 0; i < kBlk; ++i) acc += (int32_t)w[b * kBlk + i] * (int32_t)x[b * kBlk + i];
    const float c = half_bits_to_float(ws[b]) * xs[b];
    r = fmaf(c, (float)acc, r);
  }
  return r;
}

static float dot_q4_row(const uint8_t* w, const uint16_t* ws, const int8_t* x, const float* xs, int nb) {
  float r = 0.0f;
  for (int b = 0; b < nb; ++b) {
    int32_t acc = 0;
    for (int i = 0; i < kBlk / 2; ++i) {
      const int lo = (w[b * (kBlk / 2) + i] & 0x0F) - 8;
      const int hi = (w[b * (kBlk / 2) + i] >> 4) - 8;
      acc += lo * x[b * kBlk + i] + hi * x[b * kBlk + i + kBlk / 2];
    }
    const float c = half_bits_to_float(ws[b]) * xs[b];
    r = fmaf(c, (float)acc, r);
  }
  return r;
}

static float dot_f32_row(const float* a, const float* b, int n) {
  float r = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float p = a[i] * b[i];
    r = r + p;
  }
  return r;
}

int oracle_logits_tail(int dtype, int vocab, int dim, const void* q, const uint16_t* s, const float* norm,
                       float eps, const float* x, int n, long long ldx, float* out, long long ld, int8_t* xq,
                       float* xs) {
  if (dtype < 0 || dtype > 2 || vocab < 1 || dim < kBlk || dim % kBlk || n < 0 || ldx < dim || ld < vocab) return -1;
  if (!q || !norm || (n && (!x || !out)) || (dtype != 0 && !s)) return -1;
  const int nb = dim / kBlk;
  float xb[dim];
  int8_t aq[dim];
  float as[nb];
  for (int i = 0; i < n; ++i) {
    rms_norm_row(x + (long long)i * ldx, norm, xb, dim, eps);
    if (dtype != 0) {
      quant_row(xb, dim, aq, as);
      if (xq) memcpy(xq + (long long)i * dim, aq, (size_t)dim);
      if (xs) memcpy(xs + (long long)i * nb, as, sizeof(float) * (size_t)nb);
    }
    float* o = out + (long long)i * ld;
    for (int r = 0; r < vocab; ++r) {
      if (dtype == 0)
        o[r] = dot_f32_row((const float*)q + (long long)r * dim, xb, dim);
      else if (dtype == 1)
        o[r] = dot_q8_row((const int8_t*)q + (long long)r * dim, s + (long long)r * nb, aq, as, nb);
      else
        o[r] = dot_q4_row((const uint8_t*)q + (long long)r * (dim / 2), s + (long long)r * nb, aq, as, nb);
    }
  }
  return 0;
}
