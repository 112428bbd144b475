// Attention over the K/V history ring on sm_100a: tcgen05 tensor cores, TMEM accumulators,
// TMA tile loads.
//
// The window of a Wan block call (sink + recent chunks + the chunk, already rotated in
// the ring, rows [0, kv_tokens) of each member) is attended by the chunk's rotated
// queries: out = softmax(scale * Q K^T) V per (member, head), non-causal, the SDPA call of
// the reference processor (models/wan.py:110) without the window concatenation of its
// cache (engine/kv_cache.py:51-56).
//
// A unit is (member, head, 256-row query block) = two 128-row query tiles that share every
// K/V tile the CTA loads.  The window's 128-row key tiles of a unit are cut into S equal
// chunks; a piece is (key chunk, unit), pieces are numbered chunk-major and CTA g runs
// pieces g, g + G, g + 2G, ...  so the CTAs of one round hold the same key chunk of
// consecutive units -- the query blocks of a few heads -- and walk those keys in step: each
// K/V tile comes from DRAM once and from L2 for the other query blocks of its head.  The host
// picks S so that the pieces fill whole rounds of the SMs (156 query tiles of the 1.3B block
// call do not divide over 148 SMs).  With S > 1 every piece leaves partial results
// (unnormalised O rows, running max and sum) in the workspace; combine_kernel merges them.
//
// CTA of 10 warps, one CTA per SM:
//   warp 0     TMA producer: the two Q tiles once per piece, K and V tiles through 2-stage
//              rings, all 128-byte swizzled ({64 columns, 128 rows} boxes);
//   warp 1     owns the tensor memory (512 columns: O0 | S0 | O1 | S1) and issues the MMAs
//              in the order PV0(t), S0(t+1), PV1(t), S1(t+1): while one softmax warpgroup
//              exponentiates, the tensor core works for the other;
//   warps 2-5  softmax of query tile 0, warps 6-9 of tile 1: one query row per thread (TMEM
//              lane = row).  A thread loads its S row, takes the row max, writes the bf16
//              probabilities P back into the S columns it has read (P V then takes A from
//              tensor memory), and adds up the row sum.  O is rescaled in tensor memory only
//              when a row's max grows by more than 2^8 (the probabilities are exact for any
//              fixed reference; a stale one only has to keep them in range).
// tcgen05.mma operations of one thread complete in issue order, so a commit after S_i(t+1)
// also reports P_i(t) V(t) done, and S_i(t+1) may overwrite the P_i(t) columns it follows.
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
constexpr int kQTiles = 2;       // query tiles per unit (per CTA)
constexpr int kTile = kBM * kD * 2;       // bytes of one 128 x 128 bf16 tile (two 16 KB halves)
constexpr int kHalf = kTile / 2;          // one {64 columns, 128 rows} swizzled box
constexpr int kKStages = 2, kVStages = 2;
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr unsigned long long kAttnWaitNs = 2000000000ull;
constexpr int kMaxChunks = 16;

// TMEM columns of query tile i: O_i at 256*i, S_i / P_i at 256*i + 128.
__host__ __device__ constexpr int col_o(int i) { return 256 * i; }
__host__ __device__ constexpr int col_s(int i) { return 256 * i + 128; }

// Shared memory (from a 1024-byte aligned base): Q tiles | K stages | V stages | barriers.
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQTiles * kTile;
constexpr int kOffV = kOffK + kKStages * kTile;
constexpr int kOffBar = kOffV + kVStages * kTile;
enum Bar {
  kQFull, kQEmpty, kKFull0, kKEmpty0 = kKFull0 + kKStages, kVFull0 = kKEmpty0 + kKStages,
  kVEmpty0 = kVFull0 + kVStages, kSFull0 = kVEmpty0 + kVStages, kPFull0 = kSFull0 + kQTiles,
  kOFinal0 = kPFull0 + kQTiles, kMmaDone = kOFinal0 + kQTiles, kNumBars
};
constexpr int kOffTmem = kOffBar + 8 * kNumBars;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemBytes = kOffAbort + 4 + 1024;  // + slack to align the base to 1024 bytes
static_assert(kSmemBytes <= 227 * 1024, "attention tiles exceed shared memory");

struct AParams {
  int32_t H, Lq, Lk, qblocks, nkv, G;
  int32_t chunks;        // key chunks per unit (S)
  int64_t units;         // (member, head, 256-row query block) units
  int64_t pieces;        // units * chunks
  float scale_log2;      // softmax scale * log2(e)
  void* out;
  int64_t out_member_stride, out_row_stride;
  float* ws_o;           // [pieces][2][128][128] unnormalised O of the pieces (chunks > 1)
  float2* ws_ml;         // [pieces][2][128] (running max in log2 units, sum)
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
// Non-blocking test of phase `parity` (no suspension, unlike try_wait).
__device__ __forceinline__ bool bar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M x 16 bf16) packed two per 32-bit column.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc ? 1u : 0u)
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
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
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
struct Piece {
  int b, h, qb;
  int j0, j1;       // key tiles [j0, j1)
  bool two;         // query tile 1 holds rows below Lq
  int64_t index;    // piece number (workspace slot)
};

__device__ __forceinline__ void piece_of(const AParams& p, int64_t index, Piece& pc) {
  const int64_t c = index / p.units;
  const int64_t u = index - c * p.units;
  const int64_t bh = u / p.qblocks;
  pc.qb = static_cast<int>(u - bh * p.qblocks);
  pc.b = static_cast<int>(bh / p.H);
  pc.h = static_cast<int>(bh - static_cast<int64_t>(pc.b) * p.H);
  pc.j0 = static_cast<int>(c * p.nkv / p.chunks);
  pc.j1 = static_cast<int>((c + 1) * p.nkv / p.chunks);
  pc.two = (pc.qb * 2 + 1) * kBM < p.Lq;
  pc.index = index;
}

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
    for (int i = 0; i < kQTiles; ++i) {
      bar_init(bar(kSFull0 + i), 1);
      bar_init(bar(kPFull0 + i), 128);      // every softmax thread of the tile
      bar_init(bar(kOFinal0 + i), 1);
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
  // The phase waited for has often completed already (the MMA warp's operands arrive while it
  // issues the previous step): a non-blocking test returns in a few cycles, where the blocking
  // path (a call, try_wait) measured ~300 cycles even for a completed phase -- cycles in which
  // the tensor core ran dry.
  auto warp_wait = [&](int i, int parity) -> bool {
    if (__all_sync(0xffffffffu, bar_test(bar(i), parity))) return true;
    return __all_sync(0xffffffffu, bar_wait(bar(i), parity, abort_flag, lane == 0));
  };
  const bool leader = lane == 0;
  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    int t = 0, n_pieces = 0;
    int last_k[kKStages], last_v[kVStages];
    for (int s = 0; s < kKStages; ++s) last_k[s] = -1;
    for (int s = 0; s < kVStages; ++s) last_v[s] = -1;
    bool ok = true;
    Piece pc;
    for (int64_t index = blockIdx.x; ok && index < p.pieces; index += p.G) {
      piece_of(p, index, pc);
      if (n_pieces > 0 && !(ok = warp_wait(kQEmpty, (n_pieces - 1) & 1))) break;
      const int col = pc.h * kD;
      if (leader) {
        bar_expect_tx(bar(kQFull), pc.two ? 2 * kTile : kTile);
        for (int i = 0; i < (pc.two ? 2 : 1); ++i) {
          const int row = (2 * pc.qb + i) * kBM;
          tma_load(sbase + kOffQ + i * kTile, &tq, col, row, pc.b, bar(kQFull));
          tma_load(sbase + kOffQ + i * kTile + kHalf, &tq, col + 64, row, pc.b, bar(kQFull));
        }
      }
      ++n_pieces;
      for (int j = pc.j0; j < pc.j1; ++j, ++t) {
        const int sk = t % kKStages, sv = t % kVStages;
        if (t >= kKStages && !(ok = warp_wait(kKEmpty0 + sk, ((t / kKStages) & 1) ^ 1))) break;
        if (leader) {
          bar_expect_tx(bar(kKFull0 + sk), kTile);
          tma_load(sbase + kOffK + sk * kTile, &tk, col, j * kBN, pc.b, bar(kKFull0 + sk));
          tma_load(sbase + kOffK + sk * kTile + kHalf, &tk, col + 64, j * kBN, pc.b, bar(kKFull0 + sk));
        }
        last_k[sk] = t;
        if (t >= kVStages && !(ok = warp_wait(kVEmpty0 + sv, ((t / kVStages) & 1) ^ 1))) break;
        if (leader) {
          bar_expect_tx(bar(kVFull0 + sv), kTile);
          tma_load(sbase + kOffV + sv * kTile, &tv, col, j * kBN, pc.b, bar(kVFull0 + sv));
          tma_load(sbase + kOffV + sv * kTile + kHalf, &tv, col + 64, j * kBN, pc.b, bar(kVFull0 + sv));
        }
        last_v[sv] = t;
      }
    }
    // Every load issued must have landed before the CTA may exit (bounded as well).
    if (leader) {
      volatile int never = 0;
      for (int s = 0; s < kKStages; ++s)
        if (last_k[s] >= 0) bar_wait(bar(kKFull0 + s), (last_k[s] / kKStages) & 1, &never);
      for (int s = 0; s < kVStages; ++s)
        if (last_v[s] >= 0) bar_wait(bar(kVFull0 + s), (last_v[s] / kVStages) & 1, &never);
      if (n_pieces > 0) bar_wait(bar(kQFull), (n_pieces - 1) & 1, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    const uint32_t id_s = mma_idesc(0), id_pv = mma_idesc(1);
    int t = 0, t1 = 0, n_pieces = 0;  // key tiles (all / with query tile 1), pieces
    bool ok = true;
    Piece pc;
    // Descriptors of every Q tile and K / V stage, made once.  The eight K=16 steps of an MMA
    // chain differ from its first descriptor by constant address offsets: the address field
    // holds addr >> 4 and shared addresses stay below 2^18, so adding offset >> 4 cannot carry
    // out of it.  The tensor core takes an M=128 N=128 K=16 step in ~64 cycles; any dependent
    // work between issues (rebuilding a 64-bit descriptor) measured ~100 cycles per step on an
    // SMSP shared with two softmax warps, so the chains below issue back to back.
    // (Two of each: picked by a select, never by indexing a local array.)
    static_assert(kQTiles == 2 && kKStages == 2 && kVStages == 2, "descriptor selects assume two of each");
    const uint64_t q_desc0 = smem_desc(sbase + kOffQ, 16, 1024), q_desc1 = q_desc0 + (kTile >> 4);
    const uint64_t k_desc0 = smem_desc(sbase + kOffK, 16, 1024), k_desc1 = k_desc0 + (kTile >> 4);
    const uint64_t v_desc0 = smem_desc(sbase + kOffV, kHalf, 1024), v_desc1 = v_desc0 + (kTile >> 4);
    // S_i = Q_i K^T of key tile tt (K stage tt % kKStages) into the S_i columns: step kk reads
    // head-dim columns [16 kk, 16 kk + 16), 32 bytes into a 128-byte swizzled row, the second
    // 64 columns in the other 16 KB half.
    auto issue_s = [&](int i, int tt) {
      const uint64_t qd = i ? q_desc1 : q_desc0, kd = (tt & 1) ? k_desc1 : k_desc0;
      const uint32_t d = tmem + col_s(i);
      tc_mma(d, qd, kd, id_s, false);
#pragma unroll
      for (int kk = 1; kk < 8; ++kk) {
        const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4);
        tc_mma(d, qd + off, kd + off, id_s, true);
      }
    };
    // O_i (+)= P_i V of key tile tt: A = P_i from tensor memory (bf16 pairs packed in the S_i
    // columns, 8 columns per 16 keys), B = V (MN-major: the head dim along the swizzled rows,
    // its two 64-column halves 16 KB apart, 8-row key groups 1 KB apart; step kk starts 16 key
    // rows = 2 KB further).
    auto issue_pv = [&](int i, int tt, bool first) {
      const uint64_t vd = (tt & 1) ? v_desc1 : v_desc0;
      const uint32_t d = tmem + col_o(i), a = tmem + col_s(i);
      tc_mma_ts(d, a, vd, id_pv, !first);
#pragma unroll
      for (int kk = 1; kk < 8; ++kk) tc_mma_ts(d, a + kk * 8, vd + static_cast<uint64_t>(kk * 128), id_pv, true);
    };
    // The loop runs on lane 0 alone.  The tensor core keeps almost no issued MMAs queued, so
    // the gaps between chains are tensor-pipe idle time: a warp-wide barrier test, reconvergence
    // and __syncwarp between chains measured ~14 cycles per MMA more than back-to-back issue
    // (78 against 64), and ~25 more inside this kernel.  A single thread waits with plain
    // barrier tests and goes straight on to the next chain.
    auto wait1 = [&](int i, int parity) -> bool {
      return bar_test(bar(i), parity) || bar_wait(bar(i), parity, abort_flag, true);
    };
    if (leader) {
      for (int64_t index = blockIdx.x; ok && index < p.pieces; index += p.G) {
        piece_of(p, index, pc);
        const int nq = pc.two ? 2 : 1;
        if (!(ok = wait1(kQFull, n_pieces & 1))) break;
        ++n_pieces;
        // Prologue: S of the piece's first key tile for both query tiles.
        if (!(ok = wait1(kKFull0 + t % kKStages, (t / kKStages) & 1))) break;
        tc_fence_after();
        for (int i = 0; i < nq; ++i) {
          issue_s(i, t);
          tc_commit(bar(kSFull0 + i));
        }
        tc_commit(bar(kKEmpty0 + t % kKStages));
        const int n = pc.j1 - pc.j0;
        for (int jj = 0; jj < n; ++jj, ++t) {
          const bool more = jj + 1 < n;
          // The loads of V(t) and K(t+1) landed long ago (two-stage rings): test them first, so
          // that PV0(t) -> S0(t+1) and PV1(t) -> S1(t+1) issue back to back and the only waits
          // between chains are for the softmax warps' probabilities.
          if (!(ok = wait1(kVFull0 + t % kVStages, (t / kVStages) & 1))) break;
          if (more && !(ok = wait1(kKFull0 + (t + 1) % kKStages, ((t + 1) / kKStages) & 1))) break;
          // P_0 V for this key tile, then S_0 of the next one.
          if (!(ok = wait1(kPFull0, t & 1))) break;  // query tile 0 takes part in every key tile
          tc_fence_after();
          issue_pv(0, t, jj == 0);
          if (more) {
            issue_s(0, t + 1);
            tc_commit(bar(kSFull0));
          } else {
            tc_commit(bar(kOFinal0));
          }
          if (nq == 1) {
            tc_commit(bar(kVEmpty0 + t % kVStages));
            if (more) tc_commit(bar(kKEmpty0 + (t + 1) % kKStages));
            else tc_commit(bar(kQEmpty));
          } else {
            if (!(ok = wait1(kPFull0 + 1, t1 & 1))) break;
            ++t1;
            tc_fence_after();
            issue_pv(1, t, jj == 0);
            if (!more) {
              tc_commit(bar(kVEmpty0 + t % kVStages));
              tc_commit(bar(kOFinal0 + 1));
              tc_commit(bar(kQEmpty));
            } else {
              issue_s(1, t + 1);
              tc_commit(bar(kVEmpty0 + t % kVStages));
              tc_commit(bar(kSFull0 + 1));
              tc_commit(bar(kKEmpty0 + (t + 1) % kKStages));
            }
          }
        }
      }
    }
    __syncwarp();
    if (leader) tc_commit(bar(kMmaDone));
    __syncwarp();
  } else {
    // ------------------------------- softmax warps -------------------------------
    const int qi = (warp - 2) >> 2;             // query tile of this warpgroup
    const int quarter = warp & 3;               // the TMEM lanes this warp may access
    const int row = quarter * 32 + lane;        // query row of the tile = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_addr = lane_addr + col_s(qi), o_addr = lane_addr + col_o(qi);
    int n_tiles = 0, n_pieces = 0;              // key tiles / pieces this warpgroup has processed
    bool ok = true;
    Piece pc;
    for (int64_t index = blockIdx.x; ok && index < p.pieces; index += p.G) {
      piece_of(p, index, pc);
      if (qi == 1 && !pc.two) continue;         // query tile 1 past Lq: nothing to do
      float m = -INFINITY, l = 0.f;
      for (int j = pc.j0; j < pc.j1; ++j, ++n_tiles) {
        if (!(ok = warp_wait(kSFull0 + qi, n_tiles & 1))) break;
        tc_fence_after();
        uint32_t s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + 32 * c, s + 32 * c);
        tmem_wait_ld();
        const int valid = p.Lk - j * kBN;  // keys of this tile inside the window
        if (valid < kBN) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= valid) s[i] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = __uint_as_float(s[e]);
#pragma unroll
        for (int i = 8; i < 128; i += 8)
#pragma unroll
          for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], __uint_as_float(s[i + e]));
        const float row_max =
            fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
            p.scale_log2;
        const float m_new = fmaxf(m, row_max);
        const bool grow = m_new > m + 8.f;
        const float alpha = grow ? fast_exp2(m - m_new) : 1.f;
        if (grow) {
          l *= alpha;
          m = m_new;
        }
        // Probabilities (bf16 pairs, even key in the low half) over the S columns already read.
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float x0 = fast_exp2(fmaf(__uint_as_float(s[32 * h + 2 * c]), p.scale_log2, -m));
            const float x1 = fast_exp2(fmaf(__uint_as_float(s[32 * h + 2 * c + 1]), p.scale_log2, -m));
            ls[(c & 1) * 2] += x0;
            ls[(c & 1) * 2 + 1] += x1;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
            pk[c] = *reinterpret_cast<uint32_t*>(&h2);
          }
          tmem_st16(s_addr + 16 * h, pk);
        }
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        // O holds this piece's earlier tiles: bring it to the new reference.  P_i V of the
        // previous tile has completed (the commit of S_i for this tile follows it).
        if (__any_sync(0xffffffffu, grow) && j > pc.j0) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(o_addr + 32 * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + 32 * c, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        bar_arrive(bar(kPFull0 + qi));
      }
      if (!ok) break;
      // Epilogue of the piece: O once the piece's last P V has landed.
      if (!(ok = warp_wait(kOFinal0 + qi, n_pieces & 1))) break;
      ++n_pieces;
      tc_fence_after();
      const int q_row = (2 * pc.qb + qi) * kBM + row;
      const bool live = q_row < p.Lq;
      if (p.chunks == 1) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + pc.b * p.out_member_stride +
                             static_cast<int64_t>(q_row) * p.out_row_stride + pc.h * kD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
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
        const int64_t slot = pc.index * kQTiles + qi;
        float* dst = p.ws_o + (slot * kBM + row) * kD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<uint4*>(dst + 32 * c + 4 * v) = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
        p.ws_ml[slot * kBM + row] = make_float2(m, l);
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

// Merges the key chunks of every (unit, query tile): out = sum_c 2^(m_c - m) O_c /
// sum_c 2^(m_c - m) l_c with m = max_c m_c.  One CTA per (unit, query tile), a row per
// thread pair.
__global__ void __launch_bounds__(256) combine_kernel(const __grid_constant__ AParams p) {
  const int64_t u = blockIdx.x >> 1;
  const int qi = blockIdx.x & 1;
  const int row = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int64_t bh = u / p.qblocks;
  const int qb = static_cast<int>(u - bh * p.qblocks);
  const int b = static_cast<int>(bh / p.H), h = static_cast<int>(bh - static_cast<int64_t>(b) * p.H);
  const int q_row = (2 * qb + qi) * kBM + row;
  if (q_row >= p.Lq) return;
  float m = -INFINITY;
  for (int c = 0; c < p.chunks; ++c) m = fmaxf(m, p.ws_ml[((c * p.units + u) * kQTiles + qi) * kBM + row].x);
  float acc[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = 0.f;
  float l = 0.f;
  for (int c = 0; c < p.chunks; ++c) {
    const int64_t slot = (c * p.units + u) * kQTiles + qi;
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

// Key chunks per unit: the S (1..16) with the least modelled time, in key-tile times of one
// CTA: whole rounds of pieces (a piece = its key tiles + ~2 tiles of set-up and epilogue), and
// with S > 1 the partial results: ~3 tile times for a CTA to write a piece's 128 KB, and the
// combine pass reading them all (~8 MB per tile time over the whole GPU).
static int choose_chunks(int64_t units, int nkv, int max_ctas) {
  int best = 1;
  double best_cost = 0;
  for (int c = 1; c <= kMaxChunks && c <= nkv; ++c) {
    const int64_t pieces = units * c;
    const int64_t G = pieces < max_ctas ? pieces : max_ctas;
    const int64_t rounds = (pieces + G - 1) / G;
    double cost = static_cast<double>(rounds) * ((nkv + c - 1) / c + 2);
    if (c > 1) cost += 3.0 * rounds + static_cast<double>(pieces) * kQTiles * kBM * kD * 4 / 8.0e6;
    if (c == 1 || cost < best_cost) {
      best = c;
      best_cost = cost;
    }
  }
  return best;
}

static int64_t workspace_bytes(int64_t pieces, int chunks) {
  return chunks > 1 ? pieces * kQTiles * kBM * (kD * 4 + 8) : 0;
}

static int build_attn(const ps_attn_args* a, APlan* plan, bool host_only) {
  clear_error();
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  if (a->dtype != PS_BF16) return fail(PS_ERR_DTYPE, "attention takes bf16 (dtype %d)", a->dtype);
  if (a->head_dim != kD) return fail(PS_ERR_UNSUPPORTED, "head_dim=%d: the attention kernel is built for 128", a->head_dim);
  if (a->heads < 1 || a->batch < 1 || a->q_tokens < 0 || a->kv_tokens < 1)
    return fail(PS_ERR_SHAPE, "heads=%d batch=%d q_tokens=%d kv_tokens=%d", a->heads, a->batch, a->q_tokens,
                a->kv_tokens);
  if (a->ctas < 0 || a->key_chunks < 0 || a->key_chunks > kMaxChunks)
    return fail(PS_ERR_SHAPE, "ctas=%d key_chunks=%d (0..%d)", a->ctas, a->key_chunks, kMaxChunks);
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
  p.qblocks = (a->q_tokens + kQTiles * kBM - 1) / (kQTiles * kBM);
  p.nkv = (a->kv_tokens + kBN - 1) / kBN;
  p.units = static_cast<int64_t>(a->batch) * a->heads * p.qblocks;
  const int max_ctas = a->ctas > 0 ? a->ctas : (host_only ? 148 : sm_count_attn());
  int chunks = a->key_chunks > 0 ? a->key_chunks : choose_chunks(p.units, p.nkv, max_ctas);
  if (chunks > p.nkv) chunks = p.nkv;
  p.chunks = chunks;
  p.pieces = p.units * chunks;
  p.G = static_cast<int32_t>(p.pieces < max_ctas ? (p.pieces > 0 ? p.pieces : 1) : max_ctas);
  const double scale = a->scale > 0.f ? a->scale : 1.0 / sqrt(static_cast<double>(kD));
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.out = a->out;
  p.out_member_stride = a->out_member_stride;
  p.out_row_stride = a->out_row_stride;
  plan->ws_bytes = workspace_bytes(p.pieces, chunks);
  if (!host_only || a->workspace) {
    if (plan->ws_bytes > 0 && (!a->workspace || a->workspace_bytes < plan->ws_bytes))
      return fail(PS_ERR_NULL, "workspace of %lld bytes needed (ps_attention_workspace), %lld given",
                  (long long)plan->ws_bytes, (long long)a->workspace_bytes);
    if (a->workspace && !aligned16(a->workspace)) return fail(PS_ERR_ALIGN, "workspace is not 16-byte aligned");
  }
  p.ws_o = static_cast<float*>(a->workspace);
  p.ws_ml = reinterpret_cast<float2*>(static_cast<unsigned char*>(a->workspace) +
                                      p.pieces * kQTiles * kBM * kD * 4);
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

// ---------------------------------------------------------------------------------------
// ps_ring_attention_static: the partial results in a scratch array inside the library
// ---------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_attn_scratch[PS_ATTN_STATIC_SCRATCH_BYTES];

// Device address of g_attn_scratch on the current device, looked up once per device.
static int static_scratch(void** ptr) {
  static void* addr[256];
  static bool known[256];
  static std::mutex lock;
  int dev = 0;
  const cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(PS_ERR_LAUNCH, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= 256) return fail(PS_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> guard(lock);
  if (!known[dev]) {
    void* a = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&a, g_attn_scratch);
    if (e != cudaSuccess) return fail(PS_ERR_LAUNCH, "address of the attention scratch array: %s", cudaGetErrorString(e));
    addr[dev] = a;
    known[dev] = true;
  }
  *ptr = addr[dev];
  return PS_OK;
}

// The key chunks of the fastest modelled split (the model of choose_chunks) whose partial
// results fit `cap` bytes.
static int choose_chunks_within(int64_t units, int nkv, int max_ctas, int64_t cap) {
  int best = 1;
  double best_cost = 0;
  for (int c = 1; c <= kMaxChunks && c <= nkv; ++c) {
    const int64_t pieces = units * c;
    if (workspace_bytes(pieces, c) > cap) continue;
    const int64_t G = pieces < max_ctas ? pieces : max_ctas;
    const int64_t rounds = (pieces + G - 1) / G;
    double cost = static_cast<double>(rounds) * ((nkv + c - 1) / c + 2);
    if (c > 1) cost += 3.0 * rounds + static_cast<double>(pieces) * kQTiles * kBM * kD * 4 / 8.0e6;
    if (c == 1 || cost < best_cost) {
      best = c;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_ring_attention_static(const ps_attn_args* args, void* stream) {
  ps::clear_error();
  if (!args) return ps::fail(PS_ERR_NULL, "args is NULL");
  ps_attn_args a = *args;
  if (a.q_tokens > 0 && a.head_dim == ps::kD && a.heads > 0 && a.batch > 0 && a.kv_tokens > 0) {
    const int64_t qblocks = (static_cast<int64_t>(a.q_tokens) + ps::kQTiles * ps::kBM - 1) / (ps::kQTiles * ps::kBM);
    const int64_t units = static_cast<int64_t>(a.batch) * a.heads * qblocks;
    const int nkv = (a.kv_tokens + ps::kBN - 1) / ps::kBN;
    const int max_ctas = a.ctas > 0 ? a.ctas : ps::sm_count_attn();
    if (a.key_chunks == 0) {
      a.key_chunks = ps::choose_chunks_within(units, nkv, max_ctas, PS_ATTN_STATIC_SCRATCH_BYTES);
    } else {
      const int chunks = a.key_chunks < nkv ? a.key_chunks : nkv;
      const int64_t need = ps::workspace_bytes(units * chunks, chunks);
      if (need > static_cast<int64_t>(PS_ATTN_STATIC_SCRATCH_BYTES))
        return ps::fail(PS_ERR_UNSUPPORTED,
                        "key_chunks=%d needs %lld bytes of scratch; the library's static scratch holds %u "
                        "(use fewer key chunks, or ps_ring_attention with a workspace)",
                        a.key_chunks, (long long)need, PS_ATTN_STATIC_SCRATCH_BYTES);
    }
  }
  void* scratch = nullptr;
  const int rc = ps::static_scratch(&scratch);
  if (rc != PS_OK) return rc;
  a.workspace = scratch;
  a.workspace_bytes = PS_ATTN_STATIC_SCRATCH_BYTES;
  return ps_ring_attention(&a, stream);
}

extern "C" int32_t ps_attention_workspace(const ps_attn_args* args, int64_t* bytes) {
  if (!bytes) return ps::fail(PS_ERR_NULL, "bytes is NULL");
  if (!args) return ps::fail(PS_ERR_NULL, "args is NULL");
  ps::APlan plan;
  ps_attn_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (a.ctas == 0) a.ctas = ps::sm_count_attn();
  const int rc = ps::build_attn(&a, &plan, true);
  if (rc != PS_OK) return rc;
  *bytes = plan.ws_bytes;
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
  if (plan.params.units == 0) return PS_OK;
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
  if (plan.params.chunks > 1) {
    ps::combine_kernel<<<static_cast<unsigned>(plan.params.units * ps::kQTiles), 256, 0, s>>>(plan.params);
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
