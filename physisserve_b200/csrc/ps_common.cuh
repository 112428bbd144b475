// Shared device helpers of the sm_100a attention-prep kernels: 16-byte vector
// traits for bf16 / fp32 rows and the host-side error slot behind
// ps_error_message().
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "physis_b200.h"

namespace ps {

// Records a formatted message for ps_error_message() and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the calling thread's message.
void clear_error();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A 16-byte vector of activations: 8 bf16 or 4 fp32 elements.  Conversions to and
// from fp32 pairs live in Pairs16 below.
template <typename T> struct Vec16;
template <> struct Vec16<__nv_bfloat16> { static constexpr int kElems = 8; };
template <> struct Vec16<float> { static constexpr int kElems = 4; };

// Read-once activation loads: read-only path without L1 allocation, so the
// streamed rows do not displace the RoPE tables / weights held in L1.  Volatile
// keeps every load of a row where it is written -- ahead of the first use -- so a
// thread has all of its row's 16-byte vectors in flight at once.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Reused loads (weights, tables): read-only path, cached.
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Division by a per-sequence constant d >= 1 with a host-computed magic number
// m = floor((2^64 - 1) / d) + 1 (m = 0 encodes d == 1): floor(n / d) =
// umulhi64(n, m) exactly for all n, d < 2^32, since n*m / 2^64 exceeds n / d by
// less than n / 2^64 < 1 / d.
__host__ __device__ inline uint64_t div_magic(uint32_t d) {
  return d <= 1 ? 0 : (~0ull) / d + 1;
}
__device__ __forceinline__ uint32_t div_by(uint32_t n, uint64_t magic) {
  return magic == 0 ? n : static_cast<uint32_t>(__umul64hi(static_cast<uint64_t>(n), magic));
}

__device__ __forceinline__ void st_vec(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// Programmatic dependent launch.  pdl_wait blocks the calling thread until the
// grids this one was launched to depend on have completed and their writes are
// visible (it returns at once for a grid launched in ordinary stream order);
// pdl_trigger lets a dependent grid be scheduled once every CTA of this grid has
// triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100's paired FP32 instructions).  Each lane of
// a pair is rounded exactly as the scalar IEEE operation would round it.
// ---------------------------------------------------------------------------
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 f2_make(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(f32x2 v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// A 16-byte vector as P = E/2 element pairs (even, odd) in fp32x2 registers,
// and back with one rounding to the element type.
template <typename T> struct Pairs16;

template <> struct Pairs16<__nv_bfloat16> {
  static constexpr int kPairs = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, f32x2* x) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = f2_make(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t pack_pair(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* lo, const float* hi) {
    return make_uint4(pack_pair(lo[0], hi[0]), pack_pair(lo[1], hi[1]), pack_pair(lo[2], hi[2]),
                      pack_pair(lo[3], hi[3]));
  }
  // Rounds each lane of a pair to bf16 and widens it back (exactly).
  __device__ __forceinline__ static f32x2 round(f32x2 v) {
    float a, b;
    f2_split(v, a, b);
    const uint32_t u = pack_pair(a, b);
    return f2_make(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
};

template <> struct Pairs16<float> {
  static constexpr int kPairs = 2;
  __device__ __forceinline__ static void unpack(const uint4& u, f32x2* x) {
    x[0] = f2_make(__uint_as_float(u.x), __uint_as_float(u.y));
    x[1] = f2_make(__uint_as_float(u.z), __uint_as_float(u.w));
  }
  __device__ __forceinline__ static uint4 pack(const float* lo, const float* hi) {
    return make_uint4(__float_as_uint(lo[0]), __float_as_uint(hi[0]), __float_as_uint(lo[1]), __float_as_uint(hi[1]));
  }
  __device__ __forceinline__ static f32x2 round(f32x2 v) { return v; }
};

// The RMSNorm weights of one 16-byte activation vector starting at element `off`,
// as fp32 pairs: one 16-byte load of T, or E/4 float4 loads when the weights are
// kept in fp32 (`w_f32`; fp32 activations always have fp32 weights).
template <typename T>
__device__ __forceinline__ void load_weight_pairs(const void* w, bool w_f32, int64_t off, f32x2* out) {
  constexpr int E = Vec16<T>::kElems;
  if (sizeof(T) == 2 && w_f32) {
    const float* wf = static_cast<const float*>(w) + off;
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(wf + e));
      out[e / 2] = f2_make(v.x, v.y);
      out[e / 2 + 1] = f2_make(v.z, v.w);
    }
  } else {
    Pairs16<T>::unpack(ld_keep(static_cast<const T*>(w) + off), out);
  }
}

__device__ __forceinline__ f32x2 f2_swap(f32x2 v) {
  float a, b;
  f2_split(v, a, b);
  return f2_make(b, a);
}

// RMSNorm's 1 / sqrt(mean(x^2) + eps), each step IEEE-rounded (torch's CPU rsqrt is
// 1/sqrt).
__device__ __forceinline__ float rstd_of(float ssq, float c, float eps) {
  return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssq, c), eps)));
}

// The even/odd rotation of one element pair exactly as _rope evaluates it
// (wan.py:61-62): pair (e, o) with cos pair (cos[2i], cos[2i+1]) and sin pair
// (sin[2i], sin[2i+1]); two packed products and a scalar difference and sum, each
// rounded separately in fp32 (no fused multiply-add may form).
__device__ __forceinline__ void rotate_f2(f32x2 x, f32x2 c, f32x2 sn, float& lo, float& hi) {
  float m1e, m1o, m2e, m2o;
  f2_split(f2_mul(x, c), m1e, m1o);   // (e*cos[2i], o*cos[2i+1])
  f2_split(f2_mul(x, sn), m2e, m2o);  // (e*sin[2i], o*sin[2i+1])
  lo = __fsub_rn(m1e, m2o);
  hi = __fadd_rn(m1o, m2e);
}

}  // namespace ps
