/* Plain-C restatement of the Wan attention-prep arithmetic (see prep_ref.h).
 * TEST INFRASTRUCTURE ONLY. */
#include "prep_ref.h"

#include <math.h>
#include <string.h>

float ref_bf16_to_float(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

uint16_t ref_float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

void ref_rms_norm_row(const uint16_t* x, const uint16_t* w, int n, float eps, uint16_t* out) {
  double ssq = 0.0;
  for (int i = 0; i < n; ++i) {
    const double v = ref_bf16_to_float(x[i]);
    ssq += v * v;
  }
  const float mean = (float)(ssq / n);
  const float rstd = 1.0f / sqrtf(mean + eps);
  for (int i = 0; i < n; ++i) {
    const float scaled = ref_bf16_to_float(x[i]) * rstd;
    out[i] = ref_float_to_bf16(scaled * ref_bf16_to_float(w[i]));
  }
}

void ref_rope_row(const uint16_t* x, const float* cos, const float* sin, int heads, int head_dim, uint16_t* out) {
  for (int h = 0; h < heads; ++h) {
    const uint16_t* xh = x + h * head_dim;
    uint16_t* oh = out + h * head_dim;
    for (int i = 0; i < head_dim; i += 2) {
      const float e = ref_bf16_to_float(xh[i]);
      const float o = ref_bf16_to_float(xh[i + 1]);
      const float a = e * cos[i];
      const float b = o * sin[i + 1];
      const float c = e * sin[i];
      const float d = o * cos[i + 1];
      oh[i] = ref_float_to_bf16(a - b);
      oh[i + 1] = ref_float_to_bf16(c + d);
    }
  }
}

void ref_token_table(const float* table, int head_dim, int t_dim, int h_dim, int f, int r, int c, float* out) {
  for (int j = 0; j < head_dim; ++j) {
    const int row = j < t_dim ? f : (j < t_dim + h_dim ? r : c);
    out[j] = table[(long)row * head_dim + j];
  }
}

int ref_bf16_ulps(uint16_t a, uint16_t b) {
  /* map the sign-magnitude encoding onto a monotonic integer line */
  const int ia = (a & 0x8000u) ? -(int)(a & 0x7fffu) : (int)a;
  const int ib = (b & 0x8000u) ? -(int)(b & 0x7fffu) : (int)b;
  return ia > ib ? ia - ib : ib - ia;
}
