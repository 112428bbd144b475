// Attention over the K/V history ring on sm_100a: tcgen05 tensor cores, TMEM accumulators,
// TMA tile loads.
//
// The window of a Wan block call (sink + recent chunks + the chunk, already rotated in
// the ring, rows [0, kv_tokens) of each member) is attended by the chunk's rotated
// queries: out = softmax(scale * Q K^T) V per (member, head), non-causal, the SDPA call of
// the reference processor (models/wan.py:110) without the window concatenation of its
// cache (engine/kv_cache.py:51-56).
//
// Work units are (member, head, 128-row query tile); each unit runs over the window's
// 128-row key tiles.  The (unit, key tile) pairs are cut into G equal contiguous ranges,
// one per persistent CTA (G = SMs), so every SM gets the same number of tile pairs
// whatever the unit count (156 units of the 1.3B block call would otherwise take two
// waves on 148 SMs with the second nearly empty).  A unit whose key tiles span two or
// more CTAs leaves partial results (unnormalised O rows, running max and sum) in the
// workspace; combine_kernel merges them.
//
// CTA of 6 warps, one CTA per SM:
//   warp 0    TMA producer: Q tile once per unit segment, K and V tiles through 2-stage
//             rings, all 128-byte swizzled ({64 columns, 128 rows} boxes);
//   warp 1    owns the tensor memory (512 columns: O, two S buffers) and issues the MMAs:
//             S_t = Q K_t^T into S[t%2], then O += P_{t-1} V_{t-1}, so the tensor core
//             works on the next scores while the softmax warps exponentiate;
//   warps 2-5 softmax, one query row per thread (TMEM lane = row): S row from TMEM, row
//             max, exp2, row sum, P row (bf16) into a swizzled shared-memory tile that
//             the next MMA reads as its A operand.  O is rescaled in TMEM only when a
//             row's max grows by more than 2^8 (the probabilities are exact for any
//             fixed reference; a stale one only has to keep them in range).
// All waits are bounded (~2 s of %globaltimer): a wait that runs out counts itself in
// g_attn_timeouts, raises the CTA's abort flag, every role leaves its loop, the producer
// drains its loads, the MMA warp waits for its MMAs and frees the tensor memory.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "physis_b200_attention.h"
#include "ps_common.cuh"

namespace ps {

__device__ unsigned int g_attn_timeouts;

namespace {

constexpr int kBM = 128;         // query rows per tile (MMA M, TMEM lanes)
constexpr int kBN = 128;         // key rows per tile (MMA N of S, K of P V)
constexpr int kD = 128;          // head dim (MMA K of S, N of P V)
constexpr int kTile = kBM * kD * 2;       // bytes of one 128 x 128 bf16 tile (two 16 KB halves)
constexpr int kHalf = kTile / 2;          // one {64 columns, 128 rows} swizzled box
constexpr int kKStages = 2, kVStages = 2, kPBufs = 2;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kColO = 0, kColS = 128;     // TMEM columns of O and of S buffer 0 (buffer 1 at 256)
constexpr unsigned long long kAttnWaitNs = 2000000000ull;

// Shared memory (from a 1024-byte aligned base): Q | K stages | V stages | P buffers | barriers.
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;
constexpr int kOffV = kOffK + kKStages * kTile;
constexpr int kOffP = kOffV + kVStages * kTile;
constexpr int kOffBar = kOffP + kPBufs * kTile;
enum Bar {
  kQFull, kQEmpty, kKFull0, kKEmpty0 = kKFull0 + kKStages, kVFull0 = kKEmpty0 + kKStages,
  kVEmpty0 = kVFull0 + kVStages, kSFull0 = kVEmpty0 + kVStages, kSEmpty0 = kSFull0 + 2, kPFull0 = kSEmpty0 + 2,
  kPEmpty0 = kPFull0 + kPBufs, kMmaDone = kPEmpty0 + kPBufs, kNumBars
};
constexpr int kOffTmem = kOffBar + 8 * kNumBars;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemBytes = kOffAbort + 4 + 1024;  // + slack to align the base to 1024 bytes
static_assert(kSmemBytes <= 227 * 1024, "attention tiles exceed shared memory");

struct AParams {
  int32_t H, Lq, Lk, qtiles, nkv, G;
  int64_t W;             // (unit, key tile) pairs
  float scale_log2;      // softmax scale * log2(e)
  void* out;
  int64_t out_member_stride, out_row_stride;
  float* ws_o;           // [2G][128][128] unnormalised O of partial segments
  float2* ws_ml;         // [2G][128] (running max in log2 units, sum)
};

// ---------------------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of `bar`; gives up when the CTA aborted or after kAttnWaitNs
// (then raises the abort flag and, if `count`, counts the timeout).  A parity names the
// phase waited for only while the barrier has not run more than one phase past the
// previous wait of the same thread: every wait below follows its barrier's phases in order.
__device__ __noinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, bool count = true) {
  if (bar_try(bar, parity)) return true;
  const unsigned long long start = now_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (bar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (now_ns() - start > kAttnWaitNs) {
      if (count) atomicAdd(&g_attn_timeouts, 1u);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrives on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], bf16 in, fp32 accumulate.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc ? 1u : 0u)
      : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory matrix descriptor of a 128-byte swizzled tile (sm_100 format: start address,
// leading / stride byte offsets in 16-byte units, version 1, swizzle mode 2 = 128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: fp32 D, bf16 A and B, A K-major, B K-major
// (b_mn = 0) or MN-major (b_mn = 1), M = 128, N = 128.
__host__ __device__ constexpr uint32_t mma_idesc(uint32_t b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

// ---------------------------------------------------------------------------------------
// The attention kernel
// ---------------------------------------------------------------------------------------
struct Segment {
  int b, h, qt;
  int j0, j1;       // key tiles [j0, j1) of the unit
  bool complete;    // the segment covers every key tile of its unit
  int slot;         // workspace slot of a partial segment
};

// The segments of CTA `cta`: its contiguous range of (unit, key tile) pairs, unit by unit.
struct SegmentWalker {
  const AParams& p;
  int64_t pos, end, first_unit;
  int cta;
  __device__ SegmentWalker(const AParams& params, int c) : p(params), cta(c) {
    pos = static_cast<int64_t>(c) * p.W / p.G;
    end = static_cast<int64_t>(c + 1) * p.W / p.G;
    first_unit = pos / p.nkv;
  }
  __device__ bool next(Segment& s) {
    if (pos >= end) return false;
    const int64_t u = pos / p.nkv;
    s.j0 = static_cast<int>(pos - u * p.nkv);
    const int64_t stop = end - u * p.nkv;
    s.j1 = stop < p.nkv ? static_cast<int>(stop) : p.nkv;
    s.complete = s.j0 == 0 && s.j1 == p.nkv;
    s.slot = 2 * cta + (u == first_unit ? 0 : 1);
    const int64_t bh = u / p.qtiles;
    s.qt = static_cast<int>(u - bh * p.qtiles);
    s.b = static_cast<int>(bh / p.H);
    s.h = static_cast<int>(bh - static_cast<int64_t>(s.b) * p.H);
    pos = u * p.nkv + s.j1;
    return true;
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const __grid_constant__ AParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = saddr(smem);
  const uint32_t bars = sbase + kOffBar;
  auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    bar_init(bar(kQFull), 1);
    bar_init(bar(kQEmpty), 1);
    for (int s = 0; s < kKStages; ++s) {
      bar_init(bar(kKFull0 + s), 1);
      bar_init(bar(kKEmpty0 + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      bar_init(bar(kVFull0 + s), 1);
      bar_init(bar(kVEmpty0 + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      bar_init(bar(kSFull0 + s), 1);
      bar_init(bar(kSEmpty0 + s), 4);       // one arrive per softmax warp
      bar_init(bar(kPFull0 + s), 128);      // every softmax thread
      bar_init(bar(kPEmpty0 + s), 1);
    }
    bar_init(bar(kMmaDone), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Every role runs its loop with the whole warp (the warp stays converged for the
  // .sync.aligned tensor-memory instructions and the final barrier); lane 0 issues the TMA
  // copies, MMAs and commits.  A warp-wide wait succeeds only if it succeeded on every lane.
  auto warp_wait = [&](int i, int parity) {
    return __all_sync(0xffffffffu, bar_wait(bar(i), parity, abort_flag, lane == 0));
  };
  const bool leader = lane == 0;
  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    SegmentWalker walk(p, blockIdx.x);
    Segment sg;
    int t = 0, seg = 0, q_issued = 0;
    int last_k[kKStages], last_v[kVStages];
    for (int s = 0; s < kKStages; ++s) last_k[s] = -1;
    for (int s = 0; s < kVStages; ++s) last_v[s] = -1;
    bool ok = true;
    while (ok && walk.next(sg)) {
      if (seg > 0 && !(ok = warp_wait(kQEmpty, (seg - 1) & 1))) break;
      const int col = sg.h * kD;
      if (leader) {
        bar_expect_tx(bar(kQFull), kTile);
        tma_load(sbase + kOffQ, &tq, col, sg.qt * kBM, sg.b, bar(kQFull));
        tma_load(sbase + kOffQ + kHalf, &tq, col + 64, sg.qt * kBM, sg.b, bar(kQFull));
      }
      ++q_issued;
      for (int j = sg.j0; j < sg.j1; ++j, ++t) {
        const int sk = t % kKStages, sv = t % kVStages;
        if (t >= kKStages && !(ok = warp_wait(kKEmpty0 + sk, ((t / kKStages) & 1) ^ 1))) break;
        if (leader) {
          bar_expect_tx(bar(kKFull0 + sk), kTile);
          tma_load(sbase + kOffK + sk * kTile, &tk, col, j * kBN, sg.b, bar(kKFull0 + sk));
          tma_load(sbase + kOffK + sk * kTile + kHalf, &tk, col + 64, j * kBN, sg.b, bar(kKFull0 + sk));
        }
        last_k[sk] = t;
        if (t >= kVStages && !(ok = warp_wait(kVEmpty0 + sv, ((t / kVStages) & 1) ^ 1))) break;
        if (leader) {
          bar_expect_tx(bar(kVFull0 + sv), kTile);
          tma_load(sbase + kOffV + sv * kTile, &tv, col, j * kBN, sg.b, bar(kVFull0 + sv));
          tma_load(sbase + kOffV + sv * kTile + kHalf, &tv, col + 64, j * kBN, sg.b, bar(kVFull0 + sv));
        }
        last_v[sv] = t;
      }
      ++seg;
    }
    // Every load issued must have landed before the CTA may exit (bounded as well).
    if (leader) {
      volatile int never = 0;
      for (int s = 0; s < kKStages; ++s)
        if (last_k[s] >= 0) bar_wait(bar(kKFull0 + s), (last_k[s] / kKStages) & 1, &never);
      for (int s = 0; s < kVStages; ++s)
        if (last_v[s] >= 0) bar_wait(bar(kVFull0 + s), (last_v[s] / kVStages) & 1, &never);
      if (q_issued > 0) bar_wait(bar(kQFull), (q_issued - 1) & 1, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    const uint32_t id_s = mma_idesc(0), id_pv = mma_idesc(1);
    SegmentWalker walk(p, blockIdx.x);
    Segment sg;
    int t = 0, seg = 0;
    bool ok = true;
    // O += P_tt V_tt (first: overwrite O).
    auto pv = [&](int tt, bool first) -> bool {
      const int sv = tt % kVStages, pb = tt & 1;
      if (!warp_wait(kPFull0 + pb, (tt >> 1) & 1)) return false;
      if (!warp_wait(kVFull0 + sv, (tt / kVStages) & 1)) return false;
      tc_fence_after();
      if (leader) {
        const uint32_t pa = sbase + kOffP + pb * kTile, va = sbase + kOffV + sv * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // A = P (K-major: keys along the swizzled rows); B = V (MN-major: the head dim along
          // the rows, its two 64-column halves 16 KB apart, 8-row key groups 1 KB apart).
          const uint64_t a = smem_desc(pa + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc(va + kk * 16 * 128, kHalf, 1024);
          tc_mma(tmem + kColO, a, b, id_pv, !(first && kk == 0));
        }
        tc_commit(bar(kVEmpty0 + sv));
        tc_commit(bar(kPEmpty0 + pb));   // also tells the softmax warps that O holds P_tt V_tt
      }
      __syncwarp();
      return true;
    };
    while (ok && walk.next(sg)) {
      if (!(ok = warp_wait(kQFull, seg & 1))) break;
      for (int j = sg.j0; j < sg.j1; ++j, ++t) {
        const int sk = t % kKStages, sb = t & 1;
        if (!(ok = warp_wait(kKFull0 + sk, (t / kKStages) & 1))) break;
        if (t >= 2 && !(ok = warp_wait(kSEmpty0 + sb, ((t >> 1) & 1) ^ 1))) break;
        tc_fence_after();
        if (leader) {
          const uint32_t qa = sbase + kOffQ, ka = sbase + kOffK + sk * kTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            tc_mma(tmem + kColS + sb * 128, smem_desc(qa + off, 16, 1024), smem_desc(ka + off, 16, 1024), id_s, kk > 0);
          }
          tc_commit(bar(kKEmpty0 + sk));
          tc_commit(bar(kSFull0 + sb));
          if (j == sg.j1 - 1) tc_commit(bar(kQEmpty));
        }
        __syncwarp();
        if (j > sg.j0 && !(ok = pv(t - 1, j - 1 == sg.j0))) break;
      }
      if (!ok) break;
      if (!(ok = pv(t - 1, sg.j1 - 1 == sg.j0))) break;
      ++seg;
    }
    if (leader) tc_commit(bar(kMmaDone));
    __syncwarp();
  } else {
    // ------------------------------- softmax warps -------------------------------
    const int quarter = warp & 3;               // the TMEM lanes this warp may access
    const int row = quarter * 32 + lane;        // query row of the tile = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    SegmentWalker walk(p, blockIdx.x);
    Segment sg;
    int t = 0;
    bool ok = true;
    while (ok && walk.next(sg)) {
      float m = -INFINITY, l = 0.f;
      for (int j = sg.j0; j < sg.j1; ++j, ++t) {
        const int sb = t & 1;
        if (!(ok = warp_wait(kSFull0 + sb, (t >> 1) & 1))) break;
        tc_fence_after();
        uint32_t s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + kColS + sb * 128 + 32 * c, s + 32 * c);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (leader) bar_arrive(bar(kSEmpty0 + sb));
        const int valid = p.Lk - j * kBN;  // keys of this tile inside the window
        if (valid < kBN) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= valid) s[i] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          mx0 = fmaxf(mx0, __uint_as_float(s[i]));
          mx1 = fmaxf(mx1, __uint_as_float(s[i + 1]));
          mx2 = fmaxf(mx2, __uint_as_float(s[i + 2]));
          mx3 = fmaxf(mx3, __uint_as_float(s[i + 3]));
        }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * p.scale_log2;
        const float m_new = fmaxf(m, mx);
        const bool grow = m_new > m + 8.f;
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? fast_exp2(m - m_new) : 1.f;
          if (grow) {
            l *= alpha;
            m = m_new;
          }
          if (j > sg.j0) {
            // O holds this segment's earlier tiles: rescale it once P_{t-1} V_{t-1} has landed
            // (P buffer (t-1)%2 released; its previous phase, P_{t-3} V_{t-3}, was waited for
            // before P_{t-1} was written).
            if (!(ok = warp_wait(kPEmpty0 + ((t - 1) & 1), ((t - 1) >> 1) & 1))) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld32(lane_addr + kColO + 32 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st32(lane_addr + kColO + 32 * c, o);
            }
            tmem_wait_st();
          }
        }
        // Probabilities, their sum, and the bf16 P row in the 128-byte swizzled K-major layout.
        if (t >= 2 && !(ok = warp_wait(kPEmpty0 + sb, ((t >> 1) & 1) ^ 1))) break;
        unsigned char* prow = smem + kOffP + sb * kTile + (row >> 3) * 1024 + (row & 7) * 128;
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x0 = fast_exp2(fmaf(__uint_as_float(s[8 * c + 2 * e]), p.scale_log2, -m));
            const float x1 = fast_exp2(fmaf(__uint_as_float(s[8 * c + 2 * e + 1]), p.scale_log2, -m));
            l0 += x0;
            l1 += x1;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
            w[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
          const int half = c >> 3, chunk = (c & 7) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + half * kHalf + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l += l0 + l1;
        tc_fence_before();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bar_arrive(bar(kPFull0 + sb));
      }
      if (!ok) break;
      // Epilogue of the segment: O once its last tile's P V has landed.
      if (!(ok = warp_wait(kPEmpty0 + ((t - 1) & 1), ((t - 1) >> 1) & 1))) break;
      tc_fence_after();
      const int q_row = sg.qt * kBM + row;
      const bool live = q_row < p.Lq;
      if (sg.complete) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + sg.b * p.out_member_stride +
                             static_cast<int64_t>(q_row) * p.out_row_stride + sg.h * kD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + kColO + 32 * c, o);
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(o[8 * v + 2 * e]) * inv,
                                                          __uint_as_float(o[8 * v + 2 * e + 1]) * inv);
                w[e] = *reinterpret_cast<uint32_t*>(&h2);
              }
              *reinterpret_cast<uint4*>(dst + 32 * c + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      } else {
        float* dst = p.ws_o + (static_cast<int64_t>(sg.slot) * kBM + row) * kD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + kColO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<uint4*>(dst + 32 * c + 4 * v) = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
        p.ws_ml[static_cast<int64_t>(sg.slot) * kBM + row] = make_float2(m, l);
      }
      tc_fence_before();
    }
  }

  // Teardown: every role has left its loop; wait for the MMAs in flight, free the tensor memory.
  __syncthreads();
  if (warp == 1) {
    if (leader) {
      volatile int never = 0;
      bar_wait(bar(kMmaDone), 0, &never);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Merges the partial segments of the units whose key tiles were split between CTAs:
// out = sum_i 2^(m_i - m) O_i / sum_i 2^(m_i - m) l_i with m = max_i m_i.  One CTA per unit;
// a unit that one CTA finished is skipped.
__global__ void __launch_bounds__(256) combine_kernel(const __grid_constant__ AParams p) {
  const int64_t u = blockIdx.x;
  const int64_t first = u * p.nkv, last = first + p.nkv - 1;
  auto cta_of = [&](int64_t pos) {
    int64_t c = pos * p.G / p.W;
    while (c + 1 < p.G && (c + 1) * p.W / p.G <= pos) ++c;
    while (c > 0 && c * p.W / p.G > pos) --c;
    return c;
  };
  const int64_t c_lo = cta_of(first), c_hi = cta_of(last);
  if (c_lo == c_hi) return;
  const int row = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int64_t bh = u / p.qtiles;
  const int qt = static_cast<int>(u - bh * p.qtiles);
  const int b = static_cast<int>(bh / p.H), h = static_cast<int>(bh - static_cast<int64_t>(b) * p.H);
  const int q_row = qt * kBM + row;
  if (q_row >= p.Lq) return;
  float m = -INFINITY;
  for (int64_t c = c_lo; c <= c_hi; ++c) {
    const int64_t slot = 2 * c + ((c * p.W / p.G) / p.nkv == u ? 0 : 1);
    m = fmaxf(m, p.ws_ml[slot * kBM + row].x);
  }
  float acc[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = 0.f;
  float l = 0.f;
  for (int64_t c = c_lo; c <= c_hi; ++c) {
    const int64_t slot = 2 * c + ((c * p.W / p.G) / p.nkv == u ? 0 : 1);
    const float2 ml = p.ws_ml[slot * kBM + row];
    const float w = exp2f(ml.x - m);
    l += w * ml.y;
    const float4* src = reinterpret_cast<const float4*>(p.ws_o + (slot * kBM + row) * kD + half * 64);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 x = src[i];
      acc[4 * i] += w * x.x;
      acc[4 * i + 1] += w * x.y;
      acc[4 * i + 2] += w * x.z;
      acc[4 * i + 3] += w * x.w;
    }
  }
  const float inv = 1.f / l;
  __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + b * p.out_member_stride +
                       static_cast<int64_t>(q_row) * p.out_row_stride + h * kD + half * 64;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[8 * v + 2 * e] * inv, acc[8 * v + 2 * e + 1] * inv);
      w[e] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(dst + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
struct APlan {
  AParams params;
  int64_t units;
  int64_t ws_bytes;
};

static int sm_count_attn() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      n > 0)
    return n;
  return 148;
}

static int check_rows(const void* ptr, int64_t member_stride, int64_t row_stride, int64_t C, int B, int64_t rows,
                      const char* name) {
  if (!ptr) return fail(PS_ERR_NULL, "%s is NULL", name);
  if (!aligned16(ptr)) return fail(PS_ERR_ALIGN, "%s is not 16-byte aligned", name);
  if (row_stride < C) return fail(PS_ERR_SHAPE, "%s row stride %lld is below C=%lld", name, (long long)row_stride, (long long)C);
  if ((row_stride * 2) % 16 || (member_stride * 2) % 16)
    return fail(PS_ERR_ALIGN, "%s strides must be multiples of 16 bytes", name);
  if (B > 1 && member_stride < rows * row_stride)
    return fail(PS_ERR_SHAPE, "%s member stride %lld overlaps %lld rows", name, (long long)member_stride, (long long)rows);
  return PS_OK;
}

static int build_attn(const ps_attn_args* a, APlan* plan, bool host_only) {
  clear_error();
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  if (a->dtype != PS_BF16) return fail(PS_ERR_DTYPE, "attention takes bf16 (dtype %d)", a->dtype);
  if (a->head_dim != kD) return fail(PS_ERR_UNSUPPORTED, "head_dim=%d: the attention kernel is built for 128", a->head_dim);
  if (a->heads < 1 || a->batch < 1 || a->q_tokens < 0 || a->kv_tokens < 1)
    return fail(PS_ERR_SHAPE, "heads=%d batch=%d q_tokens=%d kv_tokens=%d", a->heads, a->batch, a->q_tokens,
                a->kv_tokens);
  if (a->ctas < 0) return fail(PS_ERR_SHAPE, "ctas=%d", a->ctas);
  const int64_t C = static_cast<int64_t>(a->heads) * kD;
  int rc;
  if ((rc = check_rows(a->q, a->q_member_stride, a->q_row_stride, C, a->batch, a->q_tokens, "q")) ||
      (rc = check_rows(a->k, a->k_member_stride, a->k_row_stride, C, a->batch, a->kv_tokens, "k")) ||
      (rc = check_rows(a->v, a->v_member_stride, a->v_row_stride, C, a->batch, a->kv_tokens, "v")) ||
      (rc = check_rows(a->out, a->out_member_stride, a->out_row_stride, C, a->batch, a->q_tokens, "out")))
    return rc;
  AParams& p = plan->params;
  memset(&p, 0, sizeof(p));
  p.H = a->heads;
  p.Lq = a->q_tokens;
  p.Lk = a->kv_tokens;
  p.qtiles = (a->q_tokens + kBM - 1) / kBM;
  p.nkv = (a->kv_tokens + kBN - 1) / kBN;
  plan->units = static_cast<int64_t>(a->batch) * a->heads * p.qtiles;
  p.W = plan->units * p.nkv;
  int G = a->ctas > 0 ? a->ctas : (host_only ? 148 : sm_count_attn());
  if (p.W < G) G = static_cast<int>(p.W > 0 ? p.W : 1);
  p.G = G;
  const double scale = a->scale > 0.f ? a->scale : 1.0 / sqrt(static_cast<double>(kD));
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.out = a->out;
  p.out_member_stride = a->out_member_stride;
  p.out_row_stride = a->out_row_stride;
  plan->ws_bytes = static_cast<int64_t>(2 * G) * kBM * (kD * 4 + 8);
  if (!host_only || a->workspace) {
    if (plan->units > 0 && (!a->workspace || a->workspace_bytes < plan->ws_bytes))
      return fail(PS_ERR_NULL, "workspace of %lld bytes needed (ps_attention_workspace), %lld given",
                  (long long)plan->ws_bytes, (long long)a->workspace_bytes);
    if (a->workspace && !aligned16(a->workspace)) return fail(PS_ERR_ALIGN, "workspace is not 16-byte aligned");
  }
  p.ws_o = static_cast<float*>(a->workspace);
  p.ws_ml = reinterpret_cast<float2*>(static_cast<unsigned char*>(a->workspace) +
                                      static_cast<int64_t>(2 * G) * kBM * kD * 4);
  return PS_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// {64 columns, 128 rows, 1 member} boxes of a [members, rows, C] bf16 tensor, 128-byte swizzle;
// rows beyond `rows` read as zero.
static int make_map(CUtensorMap* map, const void* base, int64_t C, int64_t rows, int B, int64_t row_stride,
                    int64_t member_stride, const char* name) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (!encode) return fail(PS_ERR_LAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(B)};
  const int64_t mstride = B > 1 ? member_stride : rows * row_stride;
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2), static_cast<cuuint64_t>(mstride * 2)};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kBM), 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PS_ERR_LAUNCH, "tensor map of %s: CUresult %d", name, static_cast<int>(r));
  return PS_OK;
}

static cudaError_t allow_attn_smem() {
  static int done_dev[64];
  static std::mutex lock;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> guard(lock);
  if (dev >= 0 && dev < 64 && done_dev[dev]) return cudaSuccess;
  err = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (err == cudaSuccess && dev >= 0 && dev < 64) done_dev[dev] = 1;
  return err;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_attention_workspace(const ps_attn_args* args, int64_t* bytes) {
  if (!bytes) return ps::fail(PS_ERR_NULL, "bytes is NULL");
  ps::APlan plan;
  ps_attn_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  const int rc = ps::build_attn(&a, &plan, true);
  if (rc != PS_OK) return rc;
  int G = args->ctas > 0 ? args->ctas : ps::sm_count_attn();
  if (plan.params.W < G) G = static_cast<int>(plan.params.W > 0 ? plan.params.W : 1);
  *bytes = static_cast<int64_t>(2 * G) * ps::kBM * (ps::kD * 4 + 8);
  return PS_OK;
}

extern "C" int32_t ps_attention_validate(const ps_attn_args* args) {
  ps::APlan plan;
  return ps::build_attn(args, &plan, true);
}

extern "C" int32_t ps_ring_attention(const ps_attn_args* args, void* stream) {
  ps::APlan plan;
  int rc = ps::build_attn(args, &plan, false);
  if (rc != PS_OK) return rc;
  if (plan.units == 0) return PS_OK;
  const int64_t C = static_cast<int64_t>(args->heads) * ps::kD;
  CUtensorMap tq, tk, tv;
  if ((rc = ps::make_map(&tq, args->q, C, args->q_tokens, args->batch, args->q_row_stride, args->q_member_stride, "q")) ||
      (rc = ps::make_map(&tk, args->k, C, args->kv_tokens, args->batch, args->k_row_stride, args->k_member_stride, "k")) ||
      (rc = ps::make_map(&tv, args->v, C, args->kv_tokens, args->batch, args->v_row_stride, args->v_member_stride, "v")))
    return rc;
  cudaError_t err = ps::allow_attn_smem();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "attention smem opt-in: %s", cudaGetErrorString(err));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ps::attention_kernel<<<plan.params.G, ps::kThreads, ps::kSmemBytes, s>>>(tq, tk, tv, plan.params);
  err = cudaGetLastError();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "attention launch: %s", cudaGetErrorString(err));
  // The combine launch is needed when a CTA boundary falls inside a unit's key tiles.
  bool split = false;
  for (int c = 1; c < plan.params.G && !split; ++c)
    split = (static_cast<int64_t>(c) * plan.params.W / plan.params.G) % plan.params.nkv != 0;
  if (split) {
    ps::combine_kernel<<<static_cast<unsigned>(plan.units), 256, 0, s>>>(plan.params);
    err = cudaGetLastError();
    if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "attention combine launch: %s", cudaGetErrorString(err));
  }
  return PS_OK;
}

extern "C" int32_t ps_attention_timeouts(uint32_t* count, int32_t reset) {
  ps::clear_error();
  if (!count) return ps::fail(PS_ERR_NULL, "count is NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(count, ps::g_attn_timeouts, sizeof(uint32_t));
  if (err == cudaSuccess && reset) {
    const uint32_t zero = 0;
    err = cudaMemcpyToSymbol(ps::g_attn_timeouts, &zero, sizeof(uint32_t));
  }
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "reading the timeout counter: %s", cudaGetErrorString(err));
  return PS_OK;
}
