// Strided drop-in for the reference's _rope(x, cosine, sine) (wan.py:58-63).
//
// Used where the reference layout must be kept exactly: the window RoPE of
// _Attention (wan.py:109), whose input is the transposed view
// [B, window_tokens, H, D] of the concatenated pre-RoPE K window, and the Q
// RoPE with per-token tables.  Each thread rotates two 16-byte vectors (8
// bf16 or 4 fp32 elements each); the three outer dimensions are visited in
// the order of decreasing x stride so that consecutive threads touch
// consecutive memory for any permutation of [B, L, H].

#include "ps_common.cuh"

namespace ps {
namespace {

constexpr int kVecsPerThread = 2;

struct RopeParams {
  const void* x;
  const float* cos;
  const float* sin;
  void* out;
  int64_t n[3];        // outer dimension sizes, outermost first
  int64_t xs[3];       // x element strides of those dimensions
  int64_t os[3];       // out element strides
  int64_t ts[3];       // table element strides (0 for the head dimension)
  int64_t total_vecs;  // n0*n1*n2*vph
  int32_t vph;         // 16-byte vectors per head
};

template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const __grid_constant__ RopeParams p) {
  using VT = Vec16<T>;
  constexpr int E = VT::kElems;
  constexpr int P = E / 2;
  const int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * kVecsPerThread;

  uint4 xv[kVecsPerThread];
  int64_t xo[kVecsPerThread], oo[kVecsPerThread], to[kVecsPerThread];
  bool ok[kVecsPerThread];
#pragma unroll
  for (int u = 0; u < kVecsPerThread; ++u) {
    const int64_t idx = base + u;
    ok[u] = idx < p.total_vecs;
    const int64_t id = ok[u] ? idx : 0;
    const int64_t dv = id % p.vph;
    int64_t rest = id / p.vph;
    const int64_t i2 = rest % p.n[2];
    rest /= p.n[2];
    const int64_t i1 = rest % p.n[1];
    const int64_t i0 = rest / p.n[1];
    xo[u] = i0 * p.xs[0] + i1 * p.xs[1] + i2 * p.xs[2] + dv * E;
    oo[u] = i0 * p.os[0] + i1 * p.os[1] + i2 * p.os[2] + dv * E;
    to[u] = i0 * p.ts[0] + i1 * p.ts[1] + i2 * p.ts[2] + dv * E;
    if (ok[u]) xv[u] = ld_stream(static_cast<const T*>(p.x) + xo[u]);
  }
#pragma unroll
  for (int u = 0; u < kVecsPerThread; ++u) {
    if (!ok[u]) continue;
    float c[E], s[E], x[E], y[E];
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 cv = __ldg(reinterpret_cast<const float4*>(p.cos + to[u] + e));
      const float4 sv = __ldg(reinterpret_cast<const float4*>(p.sin + to[u] + e));
      c[e] = cv.x; c[e + 1] = cv.y; c[e + 2] = cv.z; c[e + 3] = cv.w;
      s[e] = sv.x; s[e + 1] = sv.y; s[e + 2] = sv.z; s[e + 3] = sv.w;
    }
    VT::unpack(xv[u], x);
#pragma unroll
    for (int j = 0; j < P; ++j)
      rotate_pair(x[2 * j], x[2 * j + 1], c[2 * j], c[2 * j + 1], s[2 * j], s[2 * j + 1], y[2 * j], y[2 * j + 1]);
    st_vec(static_cast<T*>(p.out) + oo[u], VT::pack(y));
  }
}

static int build(int32_t dtype, const void* x, const int64_t* x_strides, const float* cos, const float* sin,
                 const int64_t* tab_strides, void* out, const int64_t* out_strides, int64_t B, int64_t L, int64_t H,
                 int64_t D, RopeParams* p, int* es_out) {
  clear_error();
  if (dtype != PS_BF16 && dtype != PS_F32) return fail(PS_ERR_DTYPE, "dtype %d is not PS_BF16 or PS_F32", dtype);
  const int es = dtype == PS_BF16 ? 2 : 4;
  const int E = 16 / es;
  if (!x || !cos || !sin || !out || !x_strides || !out_strides || !tab_strides)
    return fail(PS_ERR_NULL, "a pointer argument is NULL");
  if (!aligned16(x) || !aligned16(out) || !aligned16(cos) || !aligned16(sin))
    return fail(PS_ERR_ALIGN, "x, out, cos and sin must be 16-byte aligned");
  if (B < 0 || L < 0 || H < 0 || D < 2 || (D % 2)) return fail(PS_ERR_SHAPE, "shape [%lld,%lld,%lld,%lld]", (long long)B,
                                                              (long long)L, (long long)H, (long long)D);
  if (D % E) return fail(PS_ERR_ALIGN, "head_dim=%lld: a head must be whole 16-byte vectors", (long long)D);
  for (int i = 0; i < 3; ++i) {
    if (x_strides[i] < 0 || out_strides[i] < 0 || (x_strides[i] * es) % 16 || (out_strides[i] * es) % 16)
      return fail(PS_ERR_ALIGN, "strides must be non-negative multiples of 16 bytes");
  }
  if (tab_strides[0] < 0 || tab_strides[1] < 0 || (tab_strides[0] * 4) % 16 || (tab_strides[1] * 4) % 16)
    return fail(PS_ERR_ALIGN, "table strides must be non-negative multiples of 16 bytes");
  // Order the outer dimensions by decreasing x stride (stable).
  int64_t n[3] = {B, L, H};
  int64_t xs[3] = {x_strides[0], x_strides[1], x_strides[2]};
  int64_t os[3] = {out_strides[0], out_strides[1], out_strides[2]};
  int64_t ts[3] = {tab_strides[0], tab_strides[1], 0};
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j + 1 < 3 - i; ++j)
      if (xs[j] < xs[j + 1]) {
        int64_t t;
        t = n[j]; n[j] = n[j + 1]; n[j + 1] = t;
        t = xs[j]; xs[j] = xs[j + 1]; xs[j + 1] = t;
        t = os[j]; os[j] = os[j + 1]; os[j + 1] = t;
        t = ts[j]; ts[j] = ts[j + 1]; ts[j + 1] = t;
      }
  for (int i = 0; i < 3; ++i) {
    p->n[i] = n[i] > 0 ? n[i] : 1;
    p->xs[i] = xs[i];
    p->os[i] = os[i];
    p->ts[i] = ts[i];
  }
  p->x = x;
  p->cos = cos;
  p->sin = sin;
  p->out = out;
  p->vph = static_cast<int32_t>(D / E);
  p->total_vecs = (B > 0 && L > 0 && H > 0) ? B * L * H * (D / E) : 0;
  *es_out = es;
  return PS_OK;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_rope_validate(int32_t dtype, const void* x, const int64_t* x_strides, const float* cos,
                                    const float* sin, const int64_t* tab_strides, void* out,
                                    const int64_t* out_strides, int64_t B, int64_t L, int64_t H, int64_t D) {
  ps::RopeParams p;
  int es;
  return ps::build(dtype, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D, &p, &es);
}

extern "C" int32_t ps_rope(int32_t dtype, const void* x, const int64_t* x_strides, const float* cos, const float* sin,
                           const int64_t* tab_strides, void* out, const int64_t* out_strides, int64_t B, int64_t L,
                           int64_t H, int64_t D, void* stream) {
  ps::RopeParams p;
  int es;
  const int rc = ps::build(dtype, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D, &p, &es);
  if (rc != PS_OK) return rc;
  if (p.total_vecs == 0) return PS_OK;
  const int threads = 256;
  const int64_t per_block = static_cast<int64_t>(threads) * ps::kVecsPerThread;
  const int64_t blocks = (p.total_vecs + per_block - 1) / per_block;
  if (blocks > 0x7fffffffLL) return ps::fail(PS_ERR_UNSUPPORTED, "grid of %lld CTAs", (long long)blocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (es == 2)
    ps::rope_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), threads, 0, s>>>(p);
  else
    ps::rope_kernel<float><<<static_cast<unsigned>(blocks), threads, 0, s>>>(p);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "rope launch: %s", cudaGetErrorString(err));
  return PS_OK;
}
