// Self-attention prep with explicit per-(token, head) RoPE tables: the LTX-2.5
// video processor (physisserve/models/ltx2.py:66-95).
//
// table_prep_kernel: one row group of tpr threads per token row.  A thread owns
// one table slice (E = 16 bytes of activations) of V heads; in the split style
// it holds both partners of every pair (element i of the first half and i of
// the second half of a head, the same table slice), in the interleaved style
// the pairs sit inside its own vector.  All loads (V, Q, K, then the table
// slices) are issued before the row reduction, V is stored as soon as it has
// arrived, and the rotation runs on packed fp32 pairs.
//
// rope_tables_kernel: the rotation alone on a strided [B, L, H, D] view (the
// window rope, ltx2.py:77); one thread per (token, slice) walking a chunk of
// heads with every x and table load of the chunk in flight.

#include <cstring>

#include "physis_b200_ltx.h"
#include "ps_common.cuh"

namespace ps {
namespace {

constexpr int kTMaxThreads = 512;
constexpr int kTCtaThreads = 256;
constexpr int kTHasQ = 1, kTHasK = 2, kTHasV = 4, kTNormQ = 8, kTNormK = 16, kTKPre = 32, kTKOut = 64;

struct TParams {
  const void* q;
  const void* k;
  const void* v;
  int64_t q_stride, k_stride, v_stride;
  const void* wq;
  const void* wk;
  const float* cos;
  const float* sin;
  int64_t tb, tt, th;  // table strides of batch, token, head
  void* q_out;
  void* k_pre;
  void* k_out;
  void* v_out;
  int64_t q_out_stride, k_pre_stride, k_out_stride, v_out_stride;
  uint64_t tok_magic;  // division by tokens
  int32_t flags, w_f32, head_dim, tokens, total;
  int32_t tpr, rows, slices, hstep, seg, nseg;  // slices: table slices per head
  float eps, c_f;
  int64_t kv_row0[PS_MAX_SEQS];
};

// E weights starting at element `off`, as fp32 pairs.
template <int E>
__device__ __forceinline__ void load_weights(const void* w, bool f32, int64_t off, f32x2* out) {
  if (f32) {
    const float* wf = static_cast<const float*>(w) + off;
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(wf + e));
      out[e / 2] = f2_make(v.x, v.y);
      out[e / 2 + 1] = f2_make(v.z, v.w);
    }
  } else {
    const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(w) + off;
    if constexpr (E == 8) {
      Pairs16<__nv_bfloat16>::unpack(ld_keep(wb), out);
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(wb));
      out[0] = f2_make(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u));
      out[1] = f2_make(__uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    }
  }
}

// E table entries starting at `t` as fp32 pairs.
template <int E>
__device__ __forceinline__ void load_table(const float* t, f32x2* out) {
#pragma unroll
  for (int e = 0; e < E; e += 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(t + e));
    out[e / 2] = f2_make(v.x, v.y);
    out[e / 2 + 1] = f2_make(v.z, v.w);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack_pairs(const f32x2* v) {
  constexpr int P = Pairs16<T>::kPairs;
  float lo[P], hi[P];
#pragma unroll
  for (int j = 0; j < P; ++j) f2_split(v[j], lo[j], hi[j]);
  return Pairs16<T>::pack(lo, hi);
}

// Interleaved: pair (e, o) with table pairs (c[2i], c[2i+1]), (s[2i], s[2i+1]):
// (rn(rn(e*c0) - rn(o*s0)), rn(rn(o*c1) + rn(e*s1))).
__device__ __forceinline__ f32x2 rotate_interleaved(f32x2 x, f32x2 c, f32x2 s) {
  float a0, a1, b0, b1;
  f2_split(f2_mul(x, c), a0, a1);
  f2_split(f2_mul(f2_swap(x), s), b0, b1);
  return f2_make(__fsub_rn(a0, b0), __fadd_rn(a1, b1));
}

// Split: partners a (element i) and b (element i + D/2) with the table pair at i:
// (rn(rn(a*c) - rn(b*s)), rn(rn(b*c) + rn(a*s))), two elements per packed lane.  The
// products are packed; the difference and the sum are scalar IEEE operations.
__device__ __forceinline__ void rotate_split(f32x2 a, f32x2 b, f32x2 c, f32x2 s, f32x2& lo, f32x2& hi) {
  float ac0, ac1, bs0, bs1, bc0, bc1, as0, as1;
  f2_split(f2_mul(a, c), ac0, ac1);
  f2_split(f2_mul(b, s), bs0, bs1);
  f2_split(f2_mul(b, c), bc0, bc1);
  f2_split(f2_mul(a, s), as0, as1);
  lo = f2_make(__fsub_rn(ac0, bs0), __fsub_rn(ac1, bs1));
  hi = f2_make(__fadd_rn(bc0, as0), __fadd_rn(bc1, as1));
}

template <typename T, int STYLE, int V>
__global__ void __launch_bounds__(kTMaxThreads) table_prep_kernel(const __grid_constant__ TParams p) {
  using PT = Pairs16<T>;
  constexpr int E = Vec16<T>::kElems;
  constexpr int P = PT::kPairs;
  constexpr int NV = STYLE == PS_ROPE_SPLIT ? 2 : 1;  // vectors per head per thread
  extern __shared__ float2 tparts[];                  // [rows][nseg]
  const int flags = p.flags;
  const int rg = threadIdx.x / p.tpr;
  const int lt = threadIdx.x - rg * p.tpr;
  const int slice = lt % p.slices;
  const int head0 = lt / p.slices;
  const int r0 = blockIdx.x * p.rows + rg;
  const bool active = r0 < p.total;
  const int row = active ? r0 : 0;
  const int half = p.head_dim / 2;

  int off[V][NV];
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int n = 0; n < NV; ++n) off[i][n] = (head0 + i * p.hstep) * p.head_dim + n * half + slice * E;

  uint4 qv[V][NV], kv[V][NV], vv[V][NV];
  f32x2 cs[V][P], sn[V][P];
  const uint32_t b = div_by(static_cast<uint32_t>(row), p.tok_magic);
  const int t = row - static_cast<int>(b) * p.tokens;
  if (active) {
    const T* vrow = static_cast<const T*>(p.v) + row * p.v_stride;
    const T* qrow = static_cast<const T*>(p.q) + row * p.q_stride;
    const T* krow = static_cast<const T*>(p.k) + row * p.k_stride;
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int n = 0; n < NV; ++n) {
        if (flags & kTHasV) vv[i][n] = ld_stream(vrow + off[i][n]);
        if (flags & kTHasQ) qv[i][n] = ld_stream(qrow + off[i][n]);
        if (flags & kTHasK) kv[i][n] = ld_stream(krow + off[i][n]);
      }
    if (flags & (kTHasQ | kTKOut)) {
      const int64_t tab0 = static_cast<int64_t>(b) * p.tb + static_cast<int64_t>(t) * p.tt + slice * E;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int64_t h = head0 + i * p.hstep;
        load_table<E>(p.cos + tab0 + h * p.th, cs[i]);
        load_table<E>(p.sin + tab0 + h * p.th, sn[i]);
      }
    }
  }
  const int64_t kv_row = p.kv_row0[b] + t;
  if (active && (flags & kTHasV)) {
    T* vout = static_cast<T*>(p.v_out) + kv_row * p.v_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int n = 0; n < NV; ++n) st_vec(vout + off[i][n], vv[i][n]);
  }

  float sq = 0.f, sk = 0.f;
  if (active && (flags & (kTNormQ | kTNormK))) {
    f32x2 aq = 0, ak = 0;
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int n = 0; n < NV; ++n) {
        f32x2 x[P];
        if (flags & kTNormQ) {
          PT::unpack(qv[i][n], x);
#pragma unroll
          for (int j = 0; j < P; ++j) aq = f2_fma(x[j], x[j], aq);
        }
        if (flags & kTNormK) {
          PT::unpack(kv[i][n], x);
#pragma unroll
          for (int j = 0; j < P; ++j) ak = f2_fma(x[j], x[j], ak);
        }
      }
    float a, c;
    f2_split(aq, a, c);
    sq = a + c;
    f2_split(ak, a, c);
    sk = a + c;
  }
  if (flags & (kTNormQ | kTNormK)) {
    for (int o = p.seg >> 1; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    if (p.nseg > 1) {
      float2* parts = tparts + rg * p.nseg;
      if ((lt % p.seg) == 0) parts[lt / p.seg] = make_float2(sq, sk);
      __syncthreads();
      float a = 0.f, c = 0.f;
      for (int i = 0; i < p.nseg; ++i) {
        const float2 v2 = parts[i];
        a += v2.x;
        c += v2.y;
      }
      sq = a;
      sk = c;
    }
  }
  if (!active) return;
  const float rq = rstd_of(sq, p.c_f, p.eps), rk = rstd_of(sk, p.c_f, p.eps);
  const f32x2 rq2 = f2_make(rq, rq), rk2 = f2_make(rk, rk);

  // Normalised (rounded) pairs of one head's vectors, then the rotation.
  auto prepare = [&](const uint4 (&src)[NV], const void* w, bool norm, f32x2 r2, int i, f32x2 (&x)[NV][P]) {
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      PT::unpack(src[n], x[n]);
      if (norm) {
        f32x2 wv[P];
        load_weights<E>(w, p.w_f32, off[i][n], wv);
#pragma unroll
        for (int j = 0; j < P; ++j) x[n][j] = PT::round(f2_mul(f2_mul(x[n][j], r2), wv[j]));
      }
    }
  };
  auto rotate = [&](const f32x2 (&x)[NV][P], int i, f32x2 (&y)[NV][P]) {
#pragma unroll
    for (int j = 0; j < P; ++j) {
      if constexpr (STYLE == PS_ROPE_SPLIT) {
        rotate_split(x[0][j], x[NV - 1][j], cs[i][j], sn[i][j], y[0][j], y[NV - 1][j]);
      } else {
        y[0][j] = rotate_interleaved(x[0][j], cs[i][j], sn[i][j]);
      }
    }
  };

  if (flags & kTHasQ) {
    T* qout = static_cast<T*>(p.q_out) + row * p.q_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      f32x2 x[NV][P], y[NV][P];
      prepare(qv[i], p.wq, flags & kTNormQ, rq2, i, x);
      rotate(x, i, y);
#pragma unroll
      for (int n = 0; n < NV; ++n) st_vec(qout + off[i][n], pack_pairs<T>(y[n]));
    }
  }
  if (flags & kTHasK) {
    T* kpre = static_cast<T*>(p.k_pre) + row * p.k_pre_stride;
    T* kout = static_cast<T*>(p.k_out) + kv_row * p.k_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      f32x2 x[NV][P], y[NV][P];
      prepare(kv[i], p.wk, flags & kTNormK, rk2, i, x);
      if (flags & kTKPre) {
#pragma unroll
        for (int n = 0; n < NV; ++n)
          st_vec(kpre + off[i][n], (flags & kTNormK) ? pack_pairs<T>(x[n]) : kv[i][n]);
      }
      if (flags & kTKOut) {
        rotate(x, i, y);
#pragma unroll
        for (int n = 0; n < NV; ++n) st_vec(kout + off[i][n], pack_pairs<T>(y[n]));
      }
    }
  }
}

// ------------------------------------------------------------------------------------
// Strided rotation with explicit tables
// ------------------------------------------------------------------------------------
constexpr int kRtHeads = 4;  // heads one thread rotates

struct RtParams {
  const void* x;
  const float* cos;
  const float* sin;
  void* out;
  int64_t xb, xl, xh, ob, ol, oh, tb, tl, th;
  uint64_t slice_magic, l_magic;
  uint32_t slices, L, tokens;
  int32_t heads, heads_per_block, head_dim;
};

template <typename T, int STYLE>
__global__ void __launch_bounds__(kTCtaThreads) rope_tables_kernel(const __grid_constant__ RtParams p) {
  using PT = Pairs16<T>;
  constexpr int E = Vec16<T>::kElems;
  constexpr int P = PT::kPairs;
  constexpr int NV = STYLE == PS_ROPE_SPLIT ? 2 : 1;
  const uint32_t gid = blockIdx.x * kTCtaThreads + threadIdx.x;
  const uint32_t token = div_by(gid, p.slice_magic);
  if (token >= p.tokens) return;
  const uint32_t slice = gid - token * p.slices;
  const uint32_t b = div_by(token, p.l_magic);
  const uint32_t l = token - b * p.L;
  const int h0 = blockIdx.y * p.heads_per_block;
  const int nh = min(p.heads - h0, p.heads_per_block);
  const int64_t e0 = static_cast<int64_t>(slice) * E;
  const int half = p.head_dim / 2;

  const T* xp = static_cast<const T*>(p.x) + b * p.xb + l * p.xl + h0 * p.xh + e0;
  const float* cp = p.cos + b * p.tb + l * p.tl + h0 * p.th + e0;
  const float* sp = p.sin + b * p.tb + l * p.tl + h0 * p.th + e0;
  uint4 xv[kRtHeads][NV];
  f32x2 cs[kRtHeads][P], sn[kRtHeads][P];
#pragma unroll
  for (int u = 0; u < kRtHeads; ++u) {
    if (u < nh) {
#pragma unroll
      for (int n = 0; n < NV; ++n) xv[u][n] = ld_stream(xp + u * p.xh + n * half);
      load_table<E>(cp + u * p.th, cs[u]);
      load_table<E>(sp + u * p.th, sn[u]);
    }
  }
  T* op = static_cast<T*>(p.out) + b * p.ob + l * p.ol + h0 * p.oh + e0;
#pragma unroll
  for (int u = 0; u < kRtHeads; ++u) {
    if (u >= nh) break;
    f32x2 x[NV][P], y[NV][P];
#pragma unroll
    for (int n = 0; n < NV; ++n) PT::unpack(xv[u][n], x[n]);
#pragma unroll
    for (int j = 0; j < P; ++j) {
      if constexpr (STYLE == PS_ROPE_SPLIT) {
        rotate_split(x[0][j], x[NV - 1][j], cs[u][j], sn[u][j], y[0][j], y[NV - 1][j]);
      } else {
        y[0][j] = rotate_interleaved(x[0][j], cs[u][j], sn[u][j]);
      }
    }
#pragma unroll
    for (int n = 0; n < NV; ++n) st_vec(op + u * p.oh + n * half, pack_pairs<T>(y[n]));
  }
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
int device_sms() {
  static int cached = 0;
  if (cached > 0) return cached;
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      n > 0)
    cached = n;
  return n > 0 ? n : 148;
}

bool valid_tpr(int tpr) {
  if (tpr <= 0 || tpr > kTMaxThreads) return false;
  if (tpr < 32) return (tpr & (tpr - 1)) == 0;
  return tpr % 32 == 0;
}

int check_rows(const void* p, int64_t stride, int64_t C, int es, const char* name) {
  if (!aligned16(p)) return fail(PS_ERR_ALIGN, "%s is not 16-byte aligned", name);
  if (stride < C) return fail(PS_ERR_SHAPE, "%s row stride %lld is below C=%lld", name, (long long)stride, (long long)C);
  if ((stride * es) % 16) return fail(PS_ERR_ALIGN, "%s row stride is not a multiple of 16 bytes", name);
  return PS_OK;
}

struct TPlan {
  TParams k;
  int es = 2, style = 0, V = 1, threads = 0;
  int64_t blocks = 0;
  size_t smem = 0;
};

int build_table_plan(const ps_table_prep_args* a, TPlan* plan) {
  clear_error();
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  if (a->dtype != PS_BF16 && a->dtype != PS_F32) return fail(PS_ERR_DTYPE, "dtype %d is not PS_BF16 or PS_F32", a->dtype);
  if (a->weight_dtype != PS_BF16 && a->weight_dtype != PS_F32)
    return fail(PS_ERR_DTYPE, "weight_dtype %d is not PS_BF16 or PS_F32", a->weight_dtype);
  if (a->style != PS_ROPE_SPLIT && a->style != PS_ROPE_INTERLEAVED) return fail(PS_ERR_SHAPE, "style %d unknown", a->style);
  if (a->reserved != 0) return fail(PS_ERR_SHAPE, "reserved must be 0");
  const int es = a->dtype == PS_BF16 ? 2 : 4;
  const int E = 16 / es;
  const int D = a->head_dim;
  if (a->heads < 1 || D < 2 || (D % 2)) return fail(PS_ERR_SHAPE, "heads=%d head_dim=%d invalid", a->heads, D);
  const int unit = a->style == PS_ROPE_SPLIT ? 2 * E : E;
  if (D % unit)
    return fail(PS_ERR_ALIGN, "head_dim=%d: the %s style needs whole 16-byte vectors per %s", D,
                a->style == PS_ROPE_SPLIT ? "split" : "interleaved", a->style == PS_ROPE_SPLIT ? "half head" : "head");
  const int64_t C = static_cast<int64_t>(a->heads) * D;
  if (C > (1 << 20)) return fail(PS_ERR_UNSUPPORTED, "C=%lld too large", (long long)C);
  if (a->batch < 0 || a->tokens < 0) return fail(PS_ERR_SHAPE, "batch=%d tokens=%d", a->batch, a->tokens);
  if (a->batch > PS_MAX_SEQS) return fail(PS_ERR_TOO_MANY_SEQS, "batch=%d exceeds %d", a->batch, PS_MAX_SEQS);
  const int64_t total = static_cast<int64_t>(a->batch) * a->tokens;
  if (total > 0x7fffffffLL) return fail(PS_ERR_UNSUPPORTED, "%lld rows", (long long)total);
  if (!(a->eps >= 0.f)) return fail(PS_ERR_SHAPE, "eps must be >= 0");

  int flags = 0;
  if (a->q) flags |= kTHasQ;
  if (a->k) flags |= kTHasK;
  if (a->v) flags |= kTHasV;
  if (a->q && a->q_weight) flags |= kTNormQ;
  if (a->k && a->k_weight) flags |= kTNormK;
  if (a->k && a->k_pre) flags |= kTKPre;
  if (a->k && a->k_out) flags |= kTKOut;
  if (!(flags & (kTHasQ | kTHasK | kTHasV))) return fail(PS_ERR_NULL, "no role: q, k and v are all NULL");
  if ((flags & kTHasQ) && !a->q_out) return fail(PS_ERR_NULL, "q is set but q_out is NULL");
  if ((flags & kTHasK) && !(flags & (kTKPre | kTKOut))) return fail(PS_ERR_NULL, "k is set but k_pre and k_out are NULL");
  if ((flags & kTHasV) && !a->v_out) return fail(PS_ERR_NULL, "v is set but v_out is NULL");
  if (a->q_weight && !a->q) return fail(PS_ERR_NULL, "q_weight without q");
  if (a->k_weight && !a->k) return fail(PS_ERR_NULL, "k_weight without k");
  int rc;
  if ((flags & kTHasQ) && ((rc = check_rows(a->q, a->q_stride, C, es, "q")) || (rc = check_rows(a->q_out, a->q_out_stride, C, es, "q_out"))))
    return rc;
  if ((flags & kTHasK) && (rc = check_rows(a->k, a->k_stride, C, es, "k"))) return rc;
  if ((flags & kTKPre) && (rc = check_rows(a->k_pre, a->k_pre_stride, C, es, "k_pre"))) return rc;
  if ((flags & kTKOut) && (rc = check_rows(a->k_out, a->k_out_stride, C, es, "k_out"))) return rc;
  if ((flags & kTHasV) && ((rc = check_rows(a->v, a->v_stride, C, es, "v")) || (rc = check_rows(a->v_out, a->v_out_stride, C, es, "v_out"))))
    return rc;
  if ((a->q_weight && !aligned16(a->q_weight)) || (a->k_weight && !aligned16(a->k_weight)))
    return fail(PS_ERR_ALIGN, "norm weights must be 16-byte aligned");
  const bool rotates = flags & (kTHasQ | kTKOut);
  if (rotates) {
    if (!a->cos || !a->sin) return fail(PS_ERR_NULL, "cos/sin tables are NULL");
    if (!aligned16(a->cos) || !aligned16(a->sin)) return fail(PS_ERR_ALIGN, "cos/sin must be 16-byte aligned");
    if (a->tab_batch_stride < 0 || a->tab_token_stride < 0 || a->tab_head_stride < 0 || (a->tab_batch_stride % 4) ||
        (a->tab_token_stride % 4) || (a->tab_head_stride % 4))
      return fail(PS_ERR_ALIGN, "table strides must be non-negative multiples of 16 bytes");
    const int64_t width = a->style == PS_ROPE_SPLIT ? D / 2 : D;
    if (total > 0) {
      const int64_t last = (a->batch - 1) * a->tab_batch_stride + static_cast<int64_t>(a->tokens - 1) * a->tab_token_stride +
                           static_cast<int64_t>(a->heads - 1) * a->tab_head_stride + width;
      if (last > a->tab_elems)
        return fail(PS_ERR_BOUNDS, "tables need %lld elements, tab_elems is %lld", (long long)last, (long long)a->tab_elems);
    }
  }
  TParams& k = plan->k;
  memset(&k, 0, sizeof(k));
  for (int b = 0; b < a->batch; ++b) {
    const int64_t r0 = a->kv_row0 ? a->kv_row0[b] : static_cast<int64_t>(b) * a->tokens;
    if ((flags & (kTKOut | kTHasV)) && (r0 < 0 || r0 + a->tokens > a->kv_out_rows))
      return fail(PS_ERR_BOUNDS, "member %d: kv rows [%lld, %lld) outside [0, %lld)", b, (long long)r0,
                  (long long)(r0 + a->tokens), (long long)a->kv_out_rows);
    k.kv_row0[b] = r0;
  }

  const int slices = a->style == PS_ROPE_SPLIT ? D / (2 * E) : D / E;
  int V = a->heads_per_thread;
  if (V == 0) {
    // The row group closest to 256 threads from below (measured best for both styles at
    // the LTX-2 shape: split V=1, interleaved V=2), else the smallest valid one.
    int best = 0, best_tpr = 0;
    for (int cand = 1; cand <= 2; ++cand) {
      if (a->heads % cand) continue;
      const int t = slices * (a->heads / cand);
      if (!valid_tpr(t)) continue;
      const bool better = best == 0 || (t <= kTCtaThreads && (best_tpr > kTCtaThreads || t > best_tpr)) ||
                          (t > kTCtaThreads && best_tpr > kTCtaThreads && t < best_tpr);
      if (better) {
        best = cand;
        best_tpr = t;
      }
    }
    V = best ? best : 1;
  }
  if (V != 1 && V != 2) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d not compiled (1, 2)", V);
  if (a->heads % V) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d does not divide heads=%d", V, a->heads);
  const int tpr = slices * (a->heads / V);
  if (!valid_tpr(tpr))
    return fail(PS_ERR_UNSUPPORTED, "row group of %d threads is neither a power of two below 32 nor whole warps up to %d",
                tpr, kTMaxThreads);
  const int rows = tpr >= kTCtaThreads ? 1 : kTCtaThreads / tpr;

  k.q = a->q; k.k = a->k; k.v = a->v;
  k.q_stride = a->q_stride; k.k_stride = a->k_stride; k.v_stride = a->v_stride;
  k.wq = a->q_weight; k.wk = a->k_weight;
  k.cos = a->cos; k.sin = a->sin;
  k.tb = a->tab_batch_stride; k.tt = a->tab_token_stride; k.th = a->tab_head_stride;
  k.q_out = a->q_out; k.k_pre = a->k_pre; k.k_out = a->k_out; k.v_out = a->v_out;
  k.q_out_stride = a->q_out_stride; k.k_pre_stride = a->k_pre_stride;
  k.k_out_stride = a->k_out_stride; k.v_out_stride = a->v_out_stride;
  k.tok_magic = div_magic(static_cast<uint32_t>(a->tokens > 0 ? a->tokens : 1));
  k.flags = flags;
  k.w_f32 = a->weight_dtype == PS_F32;
  k.head_dim = D;
  k.tokens = a->tokens;
  k.total = static_cast<int32_t>(total);
  k.tpr = tpr;
  k.rows = rows;
  k.slices = slices;
  k.hstep = tpr / slices;
  k.seg = tpr < 32 ? tpr : 32;
  k.nseg = tpr / k.seg;
  k.eps = a->eps;
  k.c_f = static_cast<float>(C);
  plan->es = es;
  plan->style = a->style;
  plan->V = V;
  plan->threads = rows * tpr;
  plan->blocks = (total + rows - 1) / rows;
  plan->smem = k.nseg > 1 ? static_cast<size_t>(rows) * k.nseg * sizeof(float2) : 0;
  return PS_OK;
}

template <typename T, int STYLE>
int launch_table(const TPlan& plan, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(plan.blocks));
  if (plan.V == 2)
    table_prep_kernel<T, STYLE, 2><<<grid, plan.threads, plan.smem, s>>>(plan.k);
  else
    table_prep_kernel<T, STYLE, 1><<<grid, plan.threads, plan.smem, s>>>(plan.k);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(PS_ERR_LAUNCH, "table prep launch: %s", cudaGetErrorString(err));
  return PS_OK;
}

int build_rope_tables(int32_t dtype, int32_t style, const void* x, const int64_t* xs, const float* cos, const float* sin,
                      const int64_t* ts, void* out, const int64_t* os, int64_t B, int64_t L, int64_t H, int64_t D,
                      RtParams* p, int* es_out) {
  clear_error();
  if (dtype != PS_BF16 && dtype != PS_F32) return fail(PS_ERR_DTYPE, "dtype %d is not PS_BF16 or PS_F32", dtype);
  if (style != PS_ROPE_SPLIT && style != PS_ROPE_INTERLEAVED) return fail(PS_ERR_SHAPE, "style %d unknown", style);
  const int es = dtype == PS_BF16 ? 2 : 4;
  const int E = 16 / es;
  if (!x || !cos || !sin || !out || !xs || !os || !ts) return fail(PS_ERR_NULL, "a pointer argument is NULL");
  if (!aligned16(x) || !aligned16(out) || !aligned16(cos) || !aligned16(sin))
    return fail(PS_ERR_ALIGN, "x, out, cos and sin must be 16-byte aligned");
  if (B < 0 || L < 0 || H < 0 || D < 2 || (D % 2))
    return fail(PS_ERR_SHAPE, "shape [%lld,%lld,%lld,%lld]", (long long)B, (long long)L, (long long)H, (long long)D);
  const int unit = style == PS_ROPE_SPLIT ? 2 * E : E;
  if (D % unit) return fail(PS_ERR_ALIGN, "head_dim=%lld is not whole 16-byte vectors per rotated part", (long long)D);
  for (int i = 0; i < 3; ++i) {
    if (xs[i] < 0 || os[i] < 0 || (xs[i] * es) % 16 || (os[i] * es) % 16)
      return fail(PS_ERR_ALIGN, "strides must be non-negative multiples of 16 bytes");
    if (ts[i] < 0 || (ts[i] % 4)) return fail(PS_ERR_ALIGN, "table strides must be non-negative multiples of 16 bytes");
  }
  const int64_t slices = style == PS_ROPE_SPLIT ? D / (2 * E) : D / E;
  const int64_t tokens = B * L;
  if (tokens > 0xffffffffLL || tokens * slices > 0xfffffe00LL || L > 0xffffffffLL || H > 0x7fffffffLL || D > 0x7fffffffLL)
    return fail(PS_ERR_UNSUPPORTED, "shape exceeds 32-bit thread indexing");
  p->x = x; p->cos = cos; p->sin = sin; p->out = out;
  p->xb = xs[0]; p->xl = xs[1]; p->xh = xs[2];
  p->ob = os[0]; p->ol = os[1]; p->oh = os[2];
  p->tb = ts[0]; p->tl = ts[1]; p->th = ts[2];
  p->slices = static_cast<uint32_t>(slices);
  p->slice_magic = div_magic(p->slices);
  p->L = static_cast<uint32_t>(L > 0 ? L : 1);
  p->l_magic = div_magic(p->L);
  p->tokens = (B > 0 && L > 0 && H > 0) ? static_cast<uint32_t>(tokens) : 0;
  p->heads = static_cast<int32_t>(H);
  p->heads_per_block = 1;
  p->head_dim = static_cast<int32_t>(D);
  *es_out = es;
  return PS_OK;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_table_prep_validate(const ps_table_prep_args* args) {
  ps::TPlan plan;
  return ps::build_table_plan(args, &plan);
}

extern "C" int32_t ps_qk_norm_rope_tables(const ps_table_prep_args* args, void* stream) {
  ps::TPlan plan;
  const int rc = ps::build_table_plan(args, &plan);
  if (rc != PS_OK) return rc;
  if (plan.blocks == 0) return PS_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (plan.es == 2)
    return plan.style == PS_ROPE_SPLIT ? ps::launch_table<__nv_bfloat16, PS_ROPE_SPLIT>(plan, s)
                                       : ps::launch_table<__nv_bfloat16, PS_ROPE_INTERLEAVED>(plan, s);
  return plan.style == PS_ROPE_SPLIT ? ps::launch_table<float, PS_ROPE_SPLIT>(plan, s)
                                     : ps::launch_table<float, PS_ROPE_INTERLEAVED>(plan, s);
}

extern "C" int32_t ps_rope_tables_validate(int32_t dtype, int32_t style, const void* x, const int64_t* x_strides,
                                           const float* cos, const float* sin, const int64_t* tab_strides, void* out,
                                           const int64_t* out_strides, int64_t B, int64_t L, int64_t H, int64_t D) {
  ps::RtParams p;
  int es = 0;
  return ps::build_rope_tables(dtype, style, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D, &p, &es);
}

extern "C" int32_t ps_rope_tables(int32_t dtype, int32_t style, const void* x, const int64_t* x_strides,
                                  const float* cos, const float* sin, const int64_t* tab_strides, void* out,
                                  const int64_t* out_strides, int64_t B, int64_t L, int64_t H, int64_t D,
                                  void* stream) {
  ps::RtParams p;
  int es = 0;
  const int rc = ps::build_rope_tables(dtype, style, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D,
                                       &p, &es);
  if (rc != PS_OK) return rc;
  if (p.tokens == 0) return PS_OK;
  // Head chunks of at most kRtHeads, split further until the grid fills the GPU.
  const int64_t threads_x = static_cast<int64_t>(p.tokens) * p.slices;
  const int64_t target = static_cast<int64_t>(ps::device_sms()) * 2048;
  int64_t split = (p.heads + ps::kRtHeads - 1) / ps::kRtHeads;
  const int64_t want = (target + threads_x - 1) / threads_x;
  if (want > split) split = want < p.heads ? want : p.heads;
  p.heads_per_block = static_cast<int32_t>((p.heads + split - 1) / split);
  split = (p.heads + p.heads_per_block - 1) / p.heads_per_block;
  const int64_t blocks = (threads_x + ps::kTCtaThreads - 1) / ps::kTCtaThreads;
  if (blocks > 0x7fffffffLL || split > 65535)
    return ps::fail(PS_ERR_UNSUPPORTED, "grid of %lld x %lld CTAs", (long long)blocks, (long long)split);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(split));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (es == 2) {
    if (style == PS_ROPE_SPLIT)
      ps::rope_tables_kernel<__nv_bfloat16, PS_ROPE_SPLIT><<<grid, ps::kTCtaThreads, 0, s>>>(p);
    else
      ps::rope_tables_kernel<__nv_bfloat16, PS_ROPE_INTERLEAVED><<<grid, ps::kTCtaThreads, 0, s>>>(p);
  } else {
    if (style == PS_ROPE_SPLIT)
      ps::rope_tables_kernel<float, PS_ROPE_SPLIT><<<grid, ps::kTCtaThreads, 0, s>>>(p);
    else
      ps::rope_tables_kernel<float, PS_ROPE_INTERLEAVED><<<grid, ps::kTCtaThreads, 0, s>>>(p);
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "rope tables launch: %s", cudaGetErrorString(err));
  return PS_OK;
}
