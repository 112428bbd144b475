/*
 * A plain-C consumer of the C ABI (include/physis_b200.h, include/physis_b200_ltx.h): no
 * Python, no torch -- what an engine binding the library from C or C++ does.
 *
 *   consumer validate   host-only: ABI version and the ps_*_validate status codes
 *                       (makes no CUDA call; runs without a GPU)
 *   consumer run        one fused ps_qk_norm_rope_kv call on device buffers from
 *                       cudaMalloc, checked against the C restatement in oracle/c
 *
 * Exit status 0 when every check holds.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "physis_b200.h"
#include "physis_b200_ltx.h"
#include "prep_ref.h"

enum { H = 2, D = 128, C = H * D, GH = 3, GW = 4, T = GH * GW, CAP = 2, OFFSET = 5, TABLE_ROWS = 16 };
enum { T_DIM = 44, H_DIM = 42, W_DIM = 42 };

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAIL: %s (%s)\n", what, ps_error_message());
    ++failures;
  }
}

static uint32_t lcg = 12345u;
static float next_uniform(void) { /* in [-2, 2) */
  lcg = lcg * 1664525u + 1013904223u;
  return ((lcg >> 8) * (1.0f / 16777216.0f)) * 4.0f - 2.0f;
}

static void fill_args(ps_qk_prep_args* a, const ps_seq* seq) {
  memset(a, 0, sizeof *a);
  a->dtype = PS_BF16;
  a->heads = H;
  a->head_dim = D;
  a->table_mode = PS_TABLE_AXES;
  a->t_dim = T_DIM;
  a->h_dim = H_DIM;
  a->w_dim = W_DIM;
  a->n_seqs = 1;
  a->eps = 1e-6f;
  a->in_rows = T;
  a->q_stride = a->k_stride = a->v_stride = C;
  a->q_out_stride = a->k_out_stride = a->v_out_stride = a->k_pre_stride = C;
  a->table_rows = TABLE_ROWS;
  a->kv_out_rows = CAP * T;
  a->seqs = seq;
}

static int validate_mode(void) {
  expect(ps_abi_version() == PS_ABI_VERSION, "ABI version");
  /* fake, 16-byte aligned addresses: validation never dereferences them */
  char* base = (char*)(uintptr_t)(1ull << 40);
  ps_seq seq = {0, T, GH, GW, OFFSET, 0, 0, CAP, OFFSET % CAP, PS_SEQ_PREP, 0};
  ps_qk_prep_args a;
  fill_args(&a, &seq);
  a.q = base; a.k = base + 0x100000; a.v = base + 0x200000;
  a.q_weight = base + 0x300000; a.k_weight = base + 0x310000;
  a.cos = (const float*)(base + 0x400000); a.sin = (const float*)(base + 0x410000);
  a.q_out = base + 0x500000; a.k_out = base + 0x600000; a.v_out = base + 0x700000;
  expect(ps_qk_prep_validate(&a) == PS_OK, "valid fused prep accepted");
  a.q = base + 8;
  expect(ps_qk_prep_validate(&a) == PS_ERR_ALIGN, "misaligned q rejected");
  a.q = base;
  a.kv_out_rows = T;
  expect(ps_qk_prep_validate(&a) == PS_ERR_BOUNDS, "ring rows beyond kv_out_rows rejected");

  const int64_t xs[3] = {T * C, C, D}, ts[2] = {0, D};
  expect(ps_rope_validate(PS_BF16, base, xs, (const float*)(base + 0x400000), (const float*)(base + 0x410000), ts,
                          base + 0x500000, xs, 1, T, H, D) == PS_OK, "valid rope accepted");
  expect(ps_rope_validate(7, base, xs, (const float*)(base + 0x400000), (const float*)(base + 0x410000), ts,
                          base + 0x500000, xs, 1, T, H, D) == PS_ERR_DTYPE, "bad rope dtype rejected");
  const int64_t tts[3] = {0, D / 2, T * D / 2};
  expect(ps_rope_tables_validate(PS_BF16, PS_ROPE_SPLIT, base, xs, (const float*)(base + 0x400000),
                                 (const float*)(base + 0x410000), tts, base + 0x500000, xs, 1, T, H, D) == PS_OK,
         "valid table rotation accepted");
  printf("validate: %s\n", failures ? "FAILED" : "ok");
  return failures ? 1 : 0;
}

/* Per-axis RoPE tables [TABLE_ROWS, D] (t|h|w column segments, pair-duplicated). */
static void make_tables(float* cos_t, float* sin_t) {
  const int dims[3] = {T_DIM, H_DIM, W_DIM};
  for (int row = 0; row < TABLE_ROWS; ++row) {
    int col = 0;
    for (int axis = 0; axis < 3; ++axis) {
      const int d = dims[axis];
      for (int j = 0; j < d / 2; ++j) {
        const double angle = row * pow(10000.0, -2.0 * j / d);
        cos_t[row * D + col] = cos_t[row * D + col + 1] = (float)cos(angle);
        sin_t[row * D + col] = sin_t[row * D + col + 1] = (float)sin(angle);
        col += 2;
      }
    }
  }
}

#define CHECK_CUDA(call)                                                   \
  do {                                                                     \
    cudaError_t e_ = (call);                                               \
    if (e_ != cudaSuccess) {                                               \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));          \
      return 2;                                                            \
    }                                                                      \
  } while (0)

static int run_mode(void) {
  static uint16_t q[T * C], k[T * C], v[T * C], wq[C], wk[C];
  static uint16_t q_out[T * C], k_pre[T * C], ring_k[CAP * T * C], ring_v[CAP * T * C];
  static float cos_t[TABLE_ROWS * D], sin_t[TABLE_ROWS * D];
  for (int i = 0; i < T * C; ++i) {
    q[i] = ref_float_to_bf16(next_uniform());
    k[i] = ref_float_to_bf16(next_uniform());
    v[i] = ref_float_to_bf16(next_uniform());
  }
  for (int i = 0; i < C; ++i) {
    wq[i] = ref_float_to_bf16(0.5f + 0.25f * (next_uniform() + 2.0f));
    wk[i] = ref_float_to_bf16(0.5f + 0.25f * (next_uniform() + 2.0f));
  }
  make_tables(cos_t, sin_t);

  const size_t row_bytes = C * sizeof(uint16_t), tab_bytes = sizeof cos_t;
  void *dq, *dk, *dv, *dwq, *dwk, *dcos, *dsin, *dq_out, *dk_pre, *dring_k, *dring_v;
  CHECK_CUDA(cudaMalloc(&dq, T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dk, T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dv, T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dwq, row_bytes));
  CHECK_CUDA(cudaMalloc(&dwk, row_bytes));
  CHECK_CUDA(cudaMalloc(&dcos, tab_bytes));
  CHECK_CUDA(cudaMalloc(&dsin, tab_bytes));
  CHECK_CUDA(cudaMalloc(&dq_out, T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dk_pre, T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dring_k, CAP * T * row_bytes));
  CHECK_CUDA(cudaMalloc(&dring_v, CAP * T * row_bytes));
  CHECK_CUDA(cudaMemcpy(dq, q, T * row_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dk, k, T * row_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dv, v, T * row_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwq, wq, row_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwk, wk, row_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dcos, cos_t, tab_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dsin, sin_t, tab_bytes, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemset(dring_k, 0, CAP * T * row_bytes));
  CHECK_CUDA(cudaMemset(dring_v, 0, CAP * T * row_bytes));

  const int slot = OFFSET % CAP;
  ps_seq seq = {0, T, GH, GW, OFFSET, 0, 0, CAP, slot, PS_SEQ_PREP, 0};
  ps_qk_prep_args a;
  fill_args(&a, &seq);
  a.q = dq; a.k = dk; a.v = dv; a.q_weight = dwq; a.k_weight = dwk;
  a.cos = (const float*)dcos; a.sin = (const float*)dsin;
  a.q_out = dq_out; a.k_out = dring_k; a.v_out = dring_v; a.k_pre = dk_pre;
  const int32_t status = ps_qk_norm_rope_kv(&a, NULL);
  expect(status == PS_OK, "fused launch accepted");
  CHECK_CUDA(cudaDeviceSynchronize());
  CHECK_CUDA(cudaMemcpy(q_out, dq_out, T * row_bytes, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(k_pre, dk_pre, T * row_bytes, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(ring_k, dring_k, CAP * T * row_bytes, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(ring_v, dring_v, CAP * T * row_bytes, cudaMemcpyDeviceToHost));
  uint32_t timeouts = 1;
  expect(ps_device_timeouts(&timeouts, 1) == PS_OK && timeouts == 0, "no bounded wait ran out");

  int worst_norm = 0, differ = 0, rot_exact = 1, v_exact = 1, untouched = 1;
  double worst_q = 0.0;
  uint16_t norm_ref[C], rot_ref[C], qn_ref[C], q_ref[C];
  float ct[D], st[D];
  for (int l = 0; l < T; ++l) {
    const int f = l / (GH * GW), r = (l / GW) % GH, c = l % GW;
    ref_token_table(cos_t, D, T_DIM, H_DIM, OFFSET + f, r, c, ct);
    ref_token_table(sin_t, D, T_DIM, H_DIM, OFFSET + f, r, c, st);
    const int ring_row = slot * T + l;
    /* RMSNorm(K): within one bf16 ulp of the restatement */
    ref_rms_norm_row(k + l * C, wk, C, 1e-6f, norm_ref);
    for (int i = 0; i < C; ++i) {
      const int u = ref_bf16_ulps(norm_ref[i], k_pre[l * C + i]);
      if (u > worst_norm) worst_norm = u;
      differ += u != 0;
    }
    /* RoPE of the kernel's own normalised K, placed at the ring slot: bit-exact */
    ref_rope_row(k_pre + l * C, ct, st, H, D, rot_ref);
    rot_exact &= memcmp(rot_ref, ring_k + ring_row * C, row_bytes) == 0;
    /* V at the ring slot: bit-exact; the other slot untouched */
    v_exact &= memcmp(v + l * C, ring_v + ring_row * C, row_bytes) == 0;
    for (int i = 0; i < C; ++i) untouched &= ring_v[((1 - slot) * T + l) * C + i] == 0;
    /* Q: within 2^-6 of each pair's magnitude of the restatement */
    ref_rms_norm_row(q + l * C, wq, C, 1e-6f, qn_ref);
    ref_rope_row(qn_ref, ct, st, H, D, q_ref);
    for (int i = 0; i < C; i += 2) {
      const double e = ref_bf16_to_float(qn_ref[i]), o = ref_bf16_to_float(qn_ref[i + 1]);
      const double mag = sqrt(e * e + o * o) + 1e-30;
      for (int j = 0; j < 2; ++j) {
        const double diff = fabs((double)ref_bf16_to_float(q_ref[i + j]) - ref_bf16_to_float(q_out[l * C + i + j]));
        if (diff / mag > worst_q) worst_q = diff / mag;
      }
    }
  }
  expect(worst_norm <= 1, "normalised K within 1 bf16 ulp");
  expect(differ <= T * C / 100, "few normalised K values differ");
  expect(rot_exact, "rotated K at the ring slot bit-exact");
  expect(v_exact, "V at the ring slot bit-exact");
  expect(untouched, "the other ring slot untouched");
  expect(worst_q <= 1.0 / 64.0, "rotated Q within 2^-6 of its pair magnitude");
  printf("run: K norm <= %d ulp (%d of %d differ), rotated K %s, V %s, Q worst %.2e of the pair: %s\n", worst_norm,
         differ, T * C, rot_exact ? "exact" : "DIFFERS", v_exact ? "exact" : "DIFFERS", worst_q,
         failures ? "FAILED" : "ok");
  cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dwq); cudaFree(dwk); cudaFree(dcos); cudaFree(dsin);
  cudaFree(dq_out); cudaFree(dk_pre); cudaFree(dring_k); cudaFree(dring_v);
  return failures ? 1 : 0;
}

int main(int argc, char** argv) {
  if (argc == 2 && strcmp(argv[1], "validate") == 0) return validate_mode();
  if (argc == 2 && strcmp(argv[1], "run") == 0) return run_mode();
  fprintf(stderr, "usage: %s validate|run\n", argv[0]);
  return 2;
}
