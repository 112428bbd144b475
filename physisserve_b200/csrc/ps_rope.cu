// Strided drop-in for the reference's _rope(x, cosine, sine) (wan.py:58-63).
//
// Used where the reference layout must be kept exactly: the window RoPE of
// _Attention (wan.py:109), whose input is the transposed view
// [B, window_tokens, H, D] of the concatenated pre-RoPE K window, and the Q
// RoPE with per-token tables.  The tables depend on the token (b, l) only, so
// a thread owns one 16-byte slice (8 bf16 or 4 fp32 elements) of one token and
// walks up to kMaxHeads heads with it: the cos/sin slice is loaded once per
// token and head chunk instead of once per head, all of the chunk's x loads are
// in flight before the first rotation, and the only divisions are two
// magic-number ones per thread.  Consecutive threads cover consecutive slices of
// a token, then consecutive tokens, so every warp reads and writes whole
// head rows for any strides of [B, L, H].

#include "ps_common.cuh"

namespace ps {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxHeads = 8;  // heads one thread rotates (the chunk along H)

int sm_count() {
  static int cached = 0;
  if (cached > 0) return cached;
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      n > 0)
    cached = n;
  return n > 0 ? n : 148;
}

struct RopeParams {
  const void* x;
  const float* cos;
  const float* sin;
  void* out;
  int64_t xb, xl, xh;  // x element strides of B, L, H
  int64_t ob, ol, oh;  // out element strides
  int64_t tb, tl;      // table element strides of B, L (H broadcasts)
  uint64_t vph_magic;  // division by vph
  uint64_t l_magic;    // division by L
  uint32_t vph;        // 16-byte slices per head
  uint32_t L;
  uint32_t tokens;     // B * L
  int32_t heads;
  int32_t heads_per_block;  // chunk of H one blockIdx.y covers (<= kMaxHeads)
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 4) rope_kernel(const __grid_constant__ RopeParams p) {
  using PT = Pairs16<T>;
  constexpr int E = Vec16<T>::kElems;
  constexpr int P = PT::kPairs;
  const uint32_t gid = blockIdx.x * kThreads + threadIdx.x;
  const uint32_t token = div_by(gid, p.vph_magic);
  if (token >= p.tokens) return;
  const uint32_t dv = gid - token * p.vph;
  const uint32_t b = div_by(token, p.l_magic);
  const uint32_t l = token - b * p.L;
  const int h0 = blockIdx.y * p.heads_per_block;
  const int nh = min(p.heads - h0, p.heads_per_block);
  const int64_t e0 = static_cast<int64_t>(dv) * E;

  const T* xp = static_cast<const T*>(p.x) + b * p.xb + l * p.xl + h0 * p.xh + e0;
  uint4 xv[kMaxHeads];
#pragma unroll
  for (int u = 0; u < kMaxHeads; ++u)
    if (u < nh) xv[u] = ld_stream(xp + u * p.xh);

  const int64_t t0 = b * p.tb + l * p.tl + e0;
  f32x2 c[P], sn[P];
#pragma unroll
  for (int e = 0; e < E; e += 4) {
    const float4 cv = __ldg(reinterpret_cast<const float4*>(p.cos + t0 + e));
    const float4 sv = __ldg(reinterpret_cast<const float4*>(p.sin + t0 + e));
    c[e / 2] = f2_make(cv.x, cv.y);
    c[e / 2 + 1] = f2_make(cv.z, cv.w);
    sn[e / 2] = f2_make(sv.x, sv.y);
    sn[e / 2 + 1] = f2_make(sv.z, sv.w);
  }

  T* op = static_cast<T*>(p.out) + b * p.ob + l * p.ol + h0 * p.oh + e0;
#pragma unroll
  for (int u = 0; u < kMaxHeads; ++u) {
    if (u >= nh) break;
    f32x2 x[P];
    float lo[P], hi[P];
    PT::unpack(xv[u], x);
#pragma unroll
    for (int j = 0; j < P; ++j) rotate_f2(x[j], c[j], sn[j], lo[j], hi[j]);
    st_vec(op + u * p.oh, PT::pack(lo, hi));
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
  const int64_t vph = D / E;
  const int64_t tokens = B * L;
  if (tokens > 0xffffffffLL || tokens * vph > 0xfffffe00LL || L > 0xffffffffLL || H > 0x7fffffffLL)
    return fail(PS_ERR_UNSUPPORTED, "shape [%lld,%lld,%lld,%lld] exceeds 32-bit thread indexing", (long long)B,
                (long long)L, (long long)H, (long long)D);
  p->x = x;
  p->cos = cos;
  p->sin = sin;
  p->out = out;
  p->xb = x_strides[0];
  p->xl = x_strides[1];
  p->xh = x_strides[2];
  p->ob = out_strides[0];
  p->ol = out_strides[1];
  p->oh = out_strides[2];
  p->tb = tab_strides[0];
  p->tl = tab_strides[1];
  p->vph = static_cast<uint32_t>(vph);
  p->vph_magic = div_magic(static_cast<uint32_t>(vph));
  p->L = static_cast<uint32_t>(L > 0 ? L : 1);
  p->l_magic = div_magic(p->L);
  p->tokens = (B > 0 && L > 0 && H > 0) ? static_cast<uint32_t>(tokens) : 0;
  p->heads = static_cast<int32_t>(H);
  p->heads_per_block = 1;
  *es_out = es;
  return PS_OK;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_rope_validate(int32_t dtype, const void* x, const int64_t* x_strides, const float* cos,
                                    const float* sin, const int64_t* tab_strides, void* out,
                                    const int64_t* out_strides, int64_t B, int64_t L, int64_t H, int64_t D) {
  ps::RopeParams p;
  int es = 0;
  return ps::build(dtype, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D, &p, &es);
}

extern "C" int32_t ps_rope(int32_t dtype, const void* x, const int64_t* x_strides, const float* cos, const float* sin,
                           const int64_t* tab_strides, void* out, const int64_t* out_strides, int64_t B, int64_t L,
                           int64_t H, int64_t D, void* stream) {
  ps::RopeParams p;
  int es = 0;
  const int rc = ps::build(dtype, x, x_strides, cos, sin, tab_strides, out, out_strides, B, L, H, D, &p, &es);
  if (rc != PS_OK) return rc;
  if (p.tokens == 0) return PS_OK;
  // Head chunks: at most kMaxHeads per thread, and enough chunks that the grid
  // fills the GPU (two CTAs of kThreads per SM slot of 2048 threads) when the
  // window is short; chunks are balanced so no blockIdx.y row runs a short tail.
  const int64_t threads_x = static_cast<int64_t>(p.tokens) * p.vph;
  const int64_t target = static_cast<int64_t>(ps::sm_count()) * 2048;
  int64_t split = (p.heads + ps::kMaxHeads - 1) / ps::kMaxHeads;
  const int64_t want = (target + threads_x - 1) / threads_x;
  if (want > split) split = want < p.heads ? want : p.heads;
  p.heads_per_block = static_cast<int32_t>((p.heads + split - 1) / split);
  split = (p.heads + p.heads_per_block - 1) / p.heads_per_block;
  const int64_t blocks = (threads_x + ps::kThreads - 1) / ps::kThreads;
  if (blocks > 0x7fffffffLL || split > 65535)
    return ps::fail(PS_ERR_UNSUPPORTED, "grid of %lld x %lld CTAs", (long long)blocks, (long long)split);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(split));
  const int threads = ps::kThreads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (es == 2)
    ps::rope_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(p);
  else
    ps::rope_kernel<float><<<grid, threads, 0, s>>>(p);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "rope launch: %s", cudaGetErrorString(err));
  return PS_OK;
}
