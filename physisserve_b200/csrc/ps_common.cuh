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

// A 16-byte vector of activations: 8 bf16 or 4 fp32 elements, converted to and
// from fp32 registers.  bf16 -> fp32 is exact; fp32 -> bf16 rounds to nearest
// even (the rounding of a PyTorch bf16 store).
template <typename T> struct Vec16;

template <> struct Vec16<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  // Rounds an fp32 value to the element type and back (exact widening).
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <> struct Vec16<float> {
  static constexpr int kElems = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float round(float x) { return x; }
};

// Read-once activation loads: read-only path without L1 allocation, so the
// streamed rows do not displace the RoPE tables / weights held in L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Reused loads (weights, tables): read-only path, cached.
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void st_vec(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// The even/odd rotation of one element pair exactly as _rope evaluates it
// (wan.py:61-62): each product and the difference/sum rounded separately in
// fp32, so no fused multiply-add may form.
__device__ __forceinline__ void rotate_pair(float e, float o, float cos_e, float cos_o, float sin_e,
                                            float sin_o, float& out_e, float& out_o) {
  out_e = __fsub_rn(__fmul_rn(e, cos_e), __fmul_rn(o, sin_o));
  out_o = __fadd_rn(__fmul_rn(e, sin_e), __fmul_rn(o, cos_o));
}

}  // namespace ps
