// Fused Q/K RMSNorm + 3D RoPE + K/V history-ring write for sm_100a.
//
// One launch covers every token of up to PS_MAX_SEQS sequences (streams, batch
// members of WanDiT.block_batch, or varlen members).  A "row group" of tpr
// threads owns one token row of C = H*D elements at a time:
//   * thread lt of the group owns the 16-byte vector dvec = lt % vph of every
//     head it covers (vph = vectors per head), heads head0 + i*hstep for
//     i < V, so its head-dim slice -- and therefore its cos/sin values -- is
//     the same for all of its V heads and is loaded once per token;
//   * sum(x^2) over the whole row (the reference's RMSNorm spans all heads,
//     wan.py:104-105) is reduced with xor shuffles inside power-of-two lane
//     segments, then across segments through shared memory in a fixed order,
//     so every thread of the group obtains bit-identical sums;
//   * V copies, Q/K loads and stores are 128-bit, coalesced along the row.
// The path is purely elementwise + row reduction, so it is bound by HBM
// bandwidth: 12*C bytes per token (read q,k,v; write q', k'-slot, v-slot) for
// bf16.  No tensor cores, no TMA: the row-group loads are already full-line
// coalesced, and the per-axis cos/sin rows (<= a few KB per CTA) stay in L1.

#include <stdio.h>
#include <string.h>

#include "ps_common.cuh"

namespace ps {
namespace {

struct DevSeq {
  int64_t row0;       // token_start
  int64_t table_row;  // PS_TABLE_TOKENS row of token 0
  int64_t ring_row;   // ring slot 0 row in k_out / v_out
  int32_t hw;         // grid_h * grid_w
  int32_t gw;
  int32_t frame_offset;
  int32_t ring_frames;
  int32_t ring_slot0;
  int32_t _pad;
};

enum : int32_t {
  kHasQ = 1,
  kHasK = 2,
  kHasV = 4,
  kNormQ = 8,
  kNormK = 16,
  kKPre = 32,
  kKOut = 64,
};

struct KParams {
  const void* q;
  const void* k;
  const void* v;
  const void* wq;
  const void* wk;
  const float* cos;
  const float* sin;
  void* q_out;
  void* k_out;
  void* v_out;
  void* k_pre;
  int64_t q_stride, k_stride, v_stride, q_out_stride, k_out_stride, v_out_stride, k_pre_stride;
  int32_t head_dim;
  int32_t C;
  int32_t tpr;    // threads per row group
  int32_t rows;   // row groups per CTA
  int32_t vph;    // 16-byte vectors per head
  int32_t hstep;  // heads between a thread's consecutive vectors = tpr / vph
  int32_t seg;    // shuffle segment (largest power of two dividing tpr, <= 32)
  int32_t nseg;   // tpr / seg
  int32_t tp;     // pairs of the frame axis
  int32_t thp;    // pairs of the frame + row axes
  int32_t table_mode;
  int32_t flags;
  int32_t n_seqs;
  int32_t total;  // tokens over all sequences
  float eps;
  float c_f;      // (float)C
  int32_t cum[PS_MAX_SEQS + 1];
  DevSeq seq[PS_MAX_SEQS];
};
static_assert(sizeof(KParams) <= 4096, "kernel parameters must fit the classic 4 KB space");

// CTA size cap: 512 threads leave 128 registers per thread, enough for the
// V <= 8 vectors of Q and K a thread holds while the row sum is reduced.
constexpr int kMaxThreads = 512;

template <typename T, int V>
__global__ void __launch_bounds__(kMaxThreads) qk_prep_kernel(const __grid_constant__ KParams p) {
  using VT = Vec16<T>;
  constexpr int E = VT::kElems;  // elements per 16-byte vector
  constexpr int P = E / 2;       // rotation pairs per vector
  extern __shared__ float2 partials[];  // [rows][nseg] (sum q^2, sum k^2)

  const int rg = threadIdx.x / p.tpr;
  const int lt = threadIdx.x - rg * p.tpr;
  const int dvec = lt % p.vph;
  const int head0 = lt / p.vph;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * p.rows + rg;
  const bool active = g < p.total;
  const int flags = p.flags;

  // Sequence of token g: last s with cum[s] <= g (uniform per row group).
  int s = 0;
  if (active) {
    int lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cum[mid] <= g) lo = mid; else hi = mid - 1;
    }
    s = lo;
  }
  const DevSeq& sq = p.seq[s];
  const int l = active ? static_cast<int>(g - p.cum[s]) : 0;
  const int64_t row = sq.row0 + l;
  const int f = l / sq.hw;
  const int rr = l - f * sq.hw;

  int elem_off[V];
#pragma unroll
  for (int i = 0; i < V; ++i) elem_off[i] = (head0 + i * p.hstep) * p.head_dim + dvec * E;

  const T* qrow = static_cast<const T*>(p.q) + row * p.q_stride;
  const T* krow = static_cast<const T*>(p.k) + row * p.k_stride;
  const T* vrow = static_cast<const T*>(p.v) + row * p.v_stride;

  uint4 qv[V], kv[V];
  if (active) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (flags & kHasQ) qv[i] = ld_stream(qrow + elem_off[i]);
      if (flags & kHasK) kv[i] = ld_stream(krow + elem_off[i]);
    }
  }

  // Destination row of K / V: ring slot of the token's frame.
  int64_t kv_row = 0;
  if (active && (flags & (kKOut | kHasV))) {
    int slot = sq.ring_slot0 + f;
    slot = slot % sq.ring_frames;
    kv_row = sq.ring_row + static_cast<int64_t>(slot) * sq.hw + rr;
  }

  if (active && (flags & kHasV)) {
    uint4 vv[V];
#pragma unroll
    for (int i = 0; i < V; ++i) vv[i] = ld_stream(vrow + elem_off[i]);
    T* vout = static_cast<T*>(p.v_out) + kv_row * p.v_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) st_vec(vout + elem_off[i], vv[i]);
  }

  // cos / sin of this thread's P pairs.
  float ce[P], co[P], se[P], so[P];
  if (active && (flags & (kHasQ | kHasK))) {
    int64_t trow_t, trow_h, trow_w;
    if (p.table_mode == PS_TABLE_AXES) {
      const int hh = rr / sq.gw;
      trow_t = sq.frame_offset + f;
      trow_h = hh;
      trow_w = rr - hh * sq.gw;
    } else {
      trow_t = trow_h = trow_w = sq.table_row + l;
    }
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int pair = dvec * P + j;
      const int64_t trow = pair < p.tp ? trow_t : (pair < p.thp ? trow_h : trow_w);
      const float2 c = __ldg(reinterpret_cast<const float2*>(p.cos + trow * p.head_dim + 2 * pair));
      const float2 sn = __ldg(reinterpret_cast<const float2*>(p.sin + trow * p.head_dim + 2 * pair));
      ce[j] = c.x;
      co[j] = c.y;
      se[j] = sn.x;
      so[j] = sn.y;
    }
  }

  // Row sums of squares (fp32).
  float ssq_q = 0.f, ssq_k = 0.f;
  if (active) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float x[E];
      if (flags & kNormQ) {
        VT::unpack(qv[i], x);
#pragma unroll
        for (int e = 0; e < E; ++e) ssq_q = fmaf(x[e], x[e], ssq_q);
      }
      if (flags & kNormK) {
        VT::unpack(kv[i], x);
#pragma unroll
        for (int e = 0; e < E; ++e) ssq_k = fmaf(x[e], x[e], ssq_k);
      }
    }
  }
  if (flags & (kNormQ | kNormK)) {
    for (int o = p.seg >> 1; o > 0; o >>= 1) {
      ssq_q += __shfl_xor_sync(0xffffffffu, ssq_q, o);
      ssq_k += __shfl_xor_sync(0xffffffffu, ssq_k, o);
    }
    if (p.nseg > 1) {
      if ((lt % p.seg) == 0) partials[rg * p.nseg + lt / p.seg] = make_float2(ssq_q, ssq_k);
      __syncthreads();
      float sum_q = 0.f, sum_k = 0.f;
      for (int i = 0; i < p.nseg; ++i) {
        const float2 t = partials[rg * p.nseg + i];
        sum_q += t.x;
        sum_k += t.y;
      }
      ssq_q = sum_q;
      ssq_k = sum_k;
    }
  }
  if (!active) return;

  // rstd = 1 / sqrt(mean(x^2) + eps), each step IEEE-rounded (torch.rsqrt on CPU).
  const float rstd_q = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssq_q, p.c_f), p.eps)));
  const float rstd_k = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssq_k, p.c_f), p.eps)));

  if (flags & kHasQ) {
    T* qout = static_cast<T*>(p.q_out) + row * p.q_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float x[E], y[E];
      VT::unpack(qv[i], x);
      if (flags & kNormQ) {
        float w[E];
        VT::unpack(ld_keep(static_cast<const T*>(p.wq) + elem_off[i]), w);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = VT::round(__fmul_rn(__fmul_rn(x[e], rstd_q), w[e]));
      }
#pragma unroll
      for (int j = 0; j < P; ++j)
        rotate_pair(x[2 * j], x[2 * j + 1], ce[j], co[j], se[j], so[j], y[2 * j], y[2 * j + 1]);
      st_vec(qout + elem_off[i], VT::pack(y));
    }
  }
  if (flags & kHasK) {
    T* kout = static_cast<T*>(p.k_out) + kv_row * p.k_out_stride;
    T* kpre = static_cast<T*>(p.k_pre) + row * p.k_pre_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float x[E], y[E];
      VT::unpack(kv[i], x);
      if (flags & kNormK) {
        float w[E];
        VT::unpack(ld_keep(static_cast<const T*>(p.wk) + elem_off[i]), w);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = VT::round(__fmul_rn(__fmul_rn(x[e], rstd_k), w[e]));
        if (flags & kKPre) st_vec(kpre + elem_off[i], VT::pack(x));
      } else if (flags & kKPre) {
        st_vec(kpre + elem_off[i], kv[i]);
      }
      if (flags & kKOut) {
#pragma unroll
        for (int j = 0; j < P; ++j)
          rotate_pair(x[2 * j], x[2 * j + 1], ce[j], co[j], se[j], so[j], y[2 * j], y[2 * j + 1]);
        st_vec(kout + elem_off[i], VT::pack(y));
      }
    }
  }
}

struct Plan {
  KParams params;
  int V;
  int threads;
  int64_t blocks;
  size_t smem;
  int elem_size;
};

static int pow2_segment(int tpr) {
  int seg = 1;
  while (seg < 32 && (tpr % (seg * 2)) == 0) seg *= 2;
  return seg;
}

static bool supported_v(int v) { return v == 1 || v == 2 || v == 3 || v == 4 || v == 5 || v == 6 || v == 8; }

// Chooses heads-per-thread V: prefer V >= 2 with a warp-multiple row group of
// at most 256 threads (several loads in flight per thread, few registers),
// then any warp-multiple group, then any group that fits a CTA.
static int choose_v(int heads, int vph) {
  const int order[] = {2, 3, 4, 5, 6, 8, 1};
  for (int v : order)
    if (heads % v == 0 && (vph * (heads / v)) % 32 == 0 && vph * (heads / v) <= 256) return v;
  for (int v : order)
    if (heads % v == 0 && (vph * (heads / v)) % 32 == 0 && vph * (heads / v) <= kMaxThreads) return v;
  for (int v : order)
    if (heads % v == 0 && vph * (heads / v) <= kMaxThreads) return v;
  return 0;
}

static int check_ptr(const void* p, const char* name) {
  if (!p) return fail(PS_ERR_NULL, "%s is NULL", name);
  if (!aligned16(p)) return fail(PS_ERR_ALIGN, "%s is not 16-byte aligned", name);
  return PS_OK;
}

static int check_stride(int64_t stride, int64_t C, int es, const char* name) {
  if (stride < C) return fail(PS_ERR_SHAPE, "%s row stride %lld is below C=%lld", name, (long long)stride, (long long)C);
  if ((stride * es) % 16) return fail(PS_ERR_ALIGN, "%s row stride %lld elements is not a multiple of 16 bytes", name, (long long)stride);
  return PS_OK;
}

static int build_plan(const ps_qk_prep_args* a, Plan* plan) {
  clear_error();
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  if (a->dtype != PS_BF16 && a->dtype != PS_F32) return fail(PS_ERR_DTYPE, "dtype %d is not PS_BF16 or PS_F32", a->dtype);
  const int es = a->dtype == PS_BF16 ? 2 : 4;
  const int E = 16 / es;
  if (a->heads < 1 || a->head_dim < 2 || (a->head_dim % 2)) return fail(PS_ERR_SHAPE, "heads=%d head_dim=%d invalid", a->heads, a->head_dim);
  if (a->head_dim % E) return fail(PS_ERR_ALIGN, "head_dim=%d: a head must be whole 16-byte vectors", a->head_dim);
  const int64_t C = static_cast<int64_t>(a->heads) * a->head_dim;
  const int vph = a->head_dim / E;

  const bool has_q = a->q != nullptr, has_k = a->k != nullptr, has_v = a->v != nullptr;
  if (!has_q && !has_k && !has_v) return fail(PS_ERR_NULL, "q, k and v are all NULL");
  const bool norm_q = has_q && a->q_weight != nullptr;
  const bool norm_k = has_k && a->k_weight != nullptr;
  if (a->q_weight && !has_q) return fail(PS_ERR_SHAPE, "q_weight given without q");
  if (a->k_weight && !has_k) return fail(PS_ERR_SHAPE, "k_weight given without k");
  if (a->k_pre && !has_k) return fail(PS_ERR_SHAPE, "k_pre given without k");
  if (a->k_out && !has_k) return fail(PS_ERR_SHAPE, "k_out given without k");
  if (a->v_out && !has_v) return fail(PS_ERR_SHAPE, "v_out given without v");
  if ((norm_q || norm_k) && !(a->eps >= 0.f)) return fail(PS_ERR_SHAPE, "eps must be >= 0");
  int rc;
  if (has_q) {
    if ((rc = check_ptr(a->q, "q")) || (rc = check_stride(a->q_stride, C, es, "q")) ||
        (rc = check_ptr(a->q_out, "q_out")) || (rc = check_stride(a->q_out_stride, C, es, "q_out")))
      return rc;
    if (norm_q && (rc = check_ptr(a->q_weight, "q_weight"))) return rc;
  }
  if (has_k) {
    if ((rc = check_ptr(a->k, "k")) || (rc = check_stride(a->k_stride, C, es, "k"))) return rc;
    if (!a->k_out && !a->k_pre) return fail(PS_ERR_NULL, "k given without k_out or k_pre");
    if (a->k_out && ((rc = check_ptr(a->k_out, "k_out")) || (rc = check_stride(a->k_out_stride, C, es, "k_out"))))
      return rc;
    if (norm_k && (rc = check_ptr(a->k_weight, "k_weight"))) return rc;
    if (a->k_pre && ((rc = check_ptr(a->k_pre, "k_pre")) || (rc = check_stride(a->k_pre_stride, C, es, "k_pre"))))
      return rc;
  }
  if (has_v) {
    if ((rc = check_ptr(a->v, "v")) || (rc = check_stride(a->v_stride, C, es, "v")) ||
        (rc = check_ptr(a->v_out, "v_out")) || (rc = check_stride(a->v_out_stride, C, es, "v_out")))
      return rc;
  }
  const bool rotate = has_q || has_k;
  if (rotate) {
    if ((rc = check_ptr(a->cos, "cos")) || (rc = check_ptr(a->sin, "sin"))) return rc;
    if (a->table_rows < 1) return fail(PS_ERR_SHAPE, "table_rows=%lld", (long long)a->table_rows);
    if (a->table_mode != PS_TABLE_TOKENS && a->table_mode != PS_TABLE_AXES)
      return fail(PS_ERR_SHAPE, "table_mode %d unknown", a->table_mode);
    if (a->table_mode == PS_TABLE_AXES) {
      if (a->t_dim < 0 || a->h_dim < 0 || a->w_dim < 0 || (a->t_dim | a->h_dim | a->w_dim) & 1 ||
          a->t_dim + a->h_dim + a->w_dim != a->head_dim)
        return fail(PS_ERR_SHAPE, "axis split %d/%d/%d must be even parts of head_dim=%d", a->t_dim, a->h_dim,
                    a->w_dim, a->head_dim);
    }
  }
  if (a->n_seqs < 1) return fail(PS_ERR_SHAPE, "n_seqs=%d", a->n_seqs);
  if (a->n_seqs > PS_MAX_SEQS) return fail(PS_ERR_TOO_MANY_SEQS, "n_seqs=%d exceeds PS_MAX_SEQS=%d", a->n_seqs, PS_MAX_SEQS);
  if (!a->seqs) return fail(PS_ERR_NULL, "seqs is NULL");
  if (a->in_rows < 0) return fail(PS_ERR_SHAPE, "in_rows=%lld", (long long)a->in_rows);

  int V = a->heads_per_thread;
  if (V == 0) V = choose_v(a->heads, vph);
  if (V <= 0 || a->heads % V) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d does not divide heads=%d", V, a->heads);
  if (!supported_v(V)) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d not compiled (1,2,3,4,5,6,8)", V);
  const int tpr = vph * (a->heads / V);
  if (tpr > kMaxThreads) return fail(PS_ERR_UNSUPPORTED, "row group of %d threads exceeds a CTA", tpr);
  int rows = tpr >= 256 ? 1 : 256 / tpr;
  while ((rows * tpr) % 32) ++rows;
  if (rows * tpr > kMaxThreads) return fail(PS_ERR_UNSUPPORTED, "cannot tile %d-thread rows into whole warps", tpr);

  KParams& k = plan->params;
  memset(&k, 0, sizeof(k));
  k.q = a->q; k.k = a->k; k.v = a->v; k.wq = norm_q ? a->q_weight : nullptr; k.wk = norm_k ? a->k_weight : nullptr;
  k.cos = a->cos; k.sin = a->sin;
  k.q_out = a->q_out; k.k_out = a->k_out; k.v_out = a->v_out; k.k_pre = a->k_pre;
  k.q_stride = a->q_stride; k.k_stride = a->k_stride; k.v_stride = a->v_stride;
  k.q_out_stride = a->q_out_stride; k.k_out_stride = a->k_out_stride; k.v_out_stride = a->v_out_stride;
  k.k_pre_stride = a->k_pre_stride;
  k.head_dim = a->head_dim;
  k.C = static_cast<int32_t>(C);
  k.tpr = tpr;
  k.rows = rows;
  k.vph = vph;
  k.hstep = tpr / vph;
  k.seg = pow2_segment(tpr);
  k.nseg = tpr / k.seg;
  if (a->table_mode == PS_TABLE_AXES) {
    k.tp = a->t_dim / 2;
    k.thp = (a->t_dim + a->h_dim) / 2;
  } else {
    k.tp = k.thp = a->head_dim;  // every pair reads the token row
  }
  k.table_mode = a->table_mode;
  const bool k_out = has_k && a->k_out != nullptr;
  k.flags = (has_q ? kHasQ : 0) | (has_k ? kHasK : 0) | (has_v ? kHasV : 0) | (norm_q ? kNormQ : 0) |
            (norm_k ? kNormK : 0) | (a->k_pre ? kKPre : 0) | (k_out ? kKOut : 0);
  k.n_seqs = a->n_seqs;
  k.eps = a->eps;
  k.c_f = static_cast<float>(C);

  int64_t total = 0;
  for (int s = 0; s < a->n_seqs; ++s) {
    const ps_seq& q = a->seqs[s];
    if (q.n_tokens < 0 || q.grid_h < 1 || q.grid_w < 1)
      return fail(PS_ERR_SHAPE, "seq %d: n_tokens=%d grid=%dx%d", s, q.n_tokens, q.grid_h, q.grid_w);
    const int64_t hw = static_cast<int64_t>(q.grid_h) * q.grid_w;
    if (hw > INT32_MAX || q.n_tokens % hw)
      return fail(PS_ERR_SHAPE, "seq %d: n_tokens=%d is not whole frames of %lld tokens", s, q.n_tokens, (long long)hw);
    const int64_t frames = q.n_tokens / hw;
    if (q.token_start < 0 || q.token_start + q.n_tokens > a->in_rows)
      return fail(PS_ERR_BOUNDS, "seq %d: rows [%lld, %lld) outside in_rows=%lld", s, (long long)q.token_start,
                  (long long)(q.token_start + q.n_tokens), (long long)a->in_rows);
    if (rotate && q.n_tokens > 0) {
      if (a->table_mode == PS_TABLE_AXES) {
        if (q.frame_offset < 0 || q.frame_offset + frames > a->table_rows || q.grid_h > a->table_rows ||
            q.grid_w > a->table_rows)
          return fail(PS_ERR_BOUNDS, "seq %d: positions (frames %d..%lld, %dx%d) exceed table_rows=%lld", s,
                      q.frame_offset, (long long)(q.frame_offset + frames - 1), q.grid_h, q.grid_w,
                      (long long)a->table_rows);
      } else if (q.table_row < 0 || q.table_row + q.n_tokens > a->table_rows) {
        return fail(PS_ERR_BOUNDS, "seq %d: table rows [%lld, %lld) exceed table_rows=%lld", s, (long long)q.table_row,
                    (long long)(q.table_row + q.n_tokens), (long long)a->table_rows);
      }
    }
    if (((has_k && a->k_out) || has_v) && q.n_tokens > 0) {
      if (q.ring_frames < 1 || q.ring_slot0 < 0 || q.ring_slot0 >= q.ring_frames)
        return fail(PS_ERR_BOUNDS, "seq %d: ring slot %d outside [0, %d)", s, q.ring_slot0, q.ring_frames);
      if (frames > q.ring_frames)
        return fail(PS_ERR_BOUNDS, "seq %d: %lld frames would overwrite each other in a ring of %d", s, (long long)frames,
                    q.ring_frames);
      if (q.ring_row < 0 || q.ring_row + static_cast<int64_t>(q.ring_frames) * hw > a->kv_out_rows)
        return fail(PS_ERR_BOUNDS, "seq %d: ring rows [%lld, %lld) outside kv_out_rows=%lld", s, (long long)q.ring_row,
                    (long long)(q.ring_row + q.ring_frames * hw), (long long)a->kv_out_rows);
    }
    k.cum[s] = static_cast<int32_t>(total);
    DevSeq& d = k.seq[s];
    d.row0 = q.token_start;
    d.table_row = q.table_row;
    d.ring_row = q.ring_row;
    d.hw = static_cast<int32_t>(hw);
    d.gw = q.grid_w;
    d.frame_offset = q.frame_offset;
    d.ring_frames = q.ring_frames > 0 ? q.ring_frames : 1;
    d.ring_slot0 = q.ring_slot0;
    total += q.n_tokens;
    if (total > INT32_MAX) return fail(PS_ERR_SHAPE, "more than 2^31-1 tokens in one call");
  }
  k.cum[a->n_seqs] = static_cast<int32_t>(total);
  k.total = static_cast<int32_t>(total);

  plan->V = V;
  plan->threads = rows * tpr;
  plan->blocks = (total + rows - 1) / rows;
  plan->smem = k.nseg > 1 ? static_cast<size_t>(rows) * k.nseg * sizeof(float2) : 0;
  plan->elem_size = es;
  return PS_OK;
}

template <typename T>
static cudaError_t launch_typed(const Plan& plan, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(plan.blocks)), block(plan.threads);
  switch (plan.V) {
    case 1: qk_prep_kernel<T, 1><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 2: qk_prep_kernel<T, 2><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 3: qk_prep_kernel<T, 3><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 4: qk_prep_kernel<T, 4><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 5: qk_prep_kernel<T, 5><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 6: qk_prep_kernel<T, 6><<<grid, block, plan.smem, stream>>>(plan.params); break;
    case 8: qk_prep_kernel<T, 8><<<grid, block, plan.smem, stream>>>(plan.params); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_qk_prep_validate(const ps_qk_prep_args* args) {
  ps::Plan plan;
  return ps::build_plan(args, &plan);
}

extern "C" int32_t ps_qk_norm_rope_kv(const ps_qk_prep_args* args, void* stream) {
  ps::Plan plan;
  const int rc = ps::build_plan(args, &plan);
  if (rc != PS_OK) return rc;
  if (plan.blocks == 0) return PS_OK;
  if (plan.blocks > 0x7fffffffLL) return ps::fail(PS_ERR_UNSUPPORTED, "grid of %lld CTAs", (long long)plan.blocks);
  const cudaError_t err = plan.elem_size == 2
                              ? ps::launch_typed<__nv_bfloat16>(plan, static_cast<cudaStream_t>(stream))
                              : ps::launch_typed<float>(plan, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "qk_prep launch: %s", cudaGetErrorString(err));
  return PS_OK;
}
