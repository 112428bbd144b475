// Fused Q/K RMSNorm + 3D RoPE + K/V history-ring write for sm_100a.
//
// One launch covers every token of up to PS_MAX_SEQS sequences (streams, batch
// members of WanDiT.block_batch, or varlen members).  The work per token row
// (C = H*D elements of each of q, k, v) is:
//   * sum(x^2) over the whole row of q and of k (the reference's RMSNorm spans
//     all heads, wan.py:104-105), y = (x * rstd) * w rounded to the element type;
//   * RoPE of each element pair of y with the token's cos/sin (wan.py:58-63);
//   * rotated q to q_out, rotated k and the untouched v to the ring slot of the
//     token's frame.
// It is HBM-bound: 12*C bytes per token (read q,k,v; write q', k'-slot, v-slot)
// for bf16.  Two kernels implement it:
//
// bulk_kernel (automatic for rows of >= 8 KB) -- a persistent CTA per SM.  One producer thread streams
//   whole q/k/v rows into a ring of shared-memory stages with cp.async.bulk
//   (the TMA bulk-copy engine) completing on per-stage mbarriers; consumer row
//   groups normalise and rotate q and k in place in shared memory, and the rows
//   leave with cp.async.bulk stores (v goes global -> smem -> ring without
//   touching registers).  Loads of the next stages are in flight while a stage
//   is computed, so latency is hidden without holding rows in registers.
// rows_kernel (automatic for narrower rows) -- one row group per token with 128-bit
//   register loads, small CTAs of whole row groups; a row this short leaves too few bytes
//   per bulk copy for the staged pipeline to pay off (measured: an 8-stream 1.3B launch
//   39 us here, 78 us through the bulk kernel).
//
// Inside a row group of tpr threads, thread lt owns the 16-byte vector
// dvec = lt % vph of each of its V heads (head0 + i*hstep, vph = vectors per
// head), so its head-dim slice -- and its cos/sin values -- is the same for all
// of its heads.  Row sums are reduced with xor shuffles inside power-of-two lane
// segments, then across segments through shared memory in a fixed order, so
// every thread of the group obtains bit-identical sums.
//
// Every wait on an mbarrier is bounded by a deadline of ~2 s of %globaltimer;
// a wait that runs out bumps a device counter (ps_device_timeouts) and the CTA
// drains its own copies and returns instead of spinning.

#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "ps_common.cuh"

namespace ps {

// Count of bounded waits that ran out, per device (read by ps_device_timeouts).
__device__ unsigned int g_wait_timeouts;

namespace {

struct DevSeq {
  int64_t row0;       // token_start
  int64_t table_row;  // PS_TABLE_TOKENS row of token 0
  int64_t ring_row;   // ring slot 0 row in k_out / v_out
  uint64_t hw_magic;  // div_magic(hw)
  uint64_t gw_magic;  // div_magic(gw)
  int32_t hw;         // grid_h * grid_w
  int32_t gw;
  int32_t frame_offset;
  int32_t ring_frames;
  int32_t ring_slot0;
  int32_t kind;       // ps_seq_kind
};

enum : int32_t {
  kHasQ = 1,
  kHasK = 2,
  kHasV = 4,
  kNormQ = 8,
  kNormK = 16,
  kKPre = 32,
  kKOut = 64,
  kSinkSeqs = 128,  // some sequences are PS_SEQ_SINK (rows kernel only)
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
  const void* k_sink;
  int64_t q_stride, k_stride, v_stride, q_out_stride, k_out_stride, v_out_stride, k_pre_stride, k_sink_stride;
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
  int32_t w_f32;  // RMSNorm weights are fp32
  int32_t early;  // PS_LAUNCH_PDL_EARLY_INPUTS: inputs are read before the grid-dependency wait
  float eps;
  float c_f;      // (float)C
  // bulk_kernel only
  int32_t stages;       // shared-memory stages per CTA
  int32_t row_bytes;    // C * element size
  int32_t stage_bytes;  // bytes of one stage (q | k | v rows)
  int32_t load_bytes;   // bytes the producer loads into a stage
  int32_t defer;        // store groups a row group keeps in flight before freeing stages (0..7)
  int32_t vstages;      // shared-memory V stages per CTA
  int32_t vdepth;       // V stores kept in flight by the V drain (1..min(vstages - 1, 7))
  int32_t vstage_bytes;
  int32_t off_abort, off_partials, off_meta, off_vmeta, off_stages, off_vstages;
  int32_t cum[PS_MAX_SEQS + 1];
  DevSeq seq[PS_MAX_SEQS];
};
// Up to 32764 bytes of kernel parameters are accepted by the CUDA 12.1+ driver on
// Volta and newer; this stays well inside that limit.
static_assert(sizeof(KParams) <= 8192, "kernel parameters too large");

// CTA size cap of rows_kernel: 512 threads leave 128 registers per thread, enough
// for the V <= 8 vectors of Q and K a thread holds while the row sum is reduced.
constexpr int kMaxThreads = 512;
constexpr int kRowsCtaThreads = 64;  // rows_kernel CTA size target
// bulk_kernel: consumer threads per CTA at most (plus one producer warp).
constexpr int kBulkMaxConsumers = 384;
constexpr int kBulkMaxGroups = 15;           // named barriers 1..15
constexpr int kBulkSmemBudget = 227 * 1024;  // dynamic shared memory per CTA (sm_100 maximum)
constexpr unsigned long long kWaitNs = 2000000000ull;

// ------------------------------------------------------------------------------------
// Token decode and per-thread RoPE coefficients (shared by both kernels)
// ------------------------------------------------------------------------------------
struct Token {
  int64_t row;     // row in q/k/v/q_out/k_pre
  int64_t kv_row;  // ring row of k_out/v_out
  int64_t trow_t, trow_h, trow_w;  // table rows of the frame / row / column segments
};

__device__ __forceinline__ int find_seq(const KParams& p, int g) {
  int lo = 0, hi = p.n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cum[mid] <= g) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ Token decode_in(const KParams& p, int s, int g) {
  const DevSeq& sq = p.seq[s];
  const int l = g - p.cum[s];
  const int f = static_cast<int>(div_by(static_cast<uint32_t>(l), sq.hw_magic));
  const int rr = l - f * sq.hw;
  Token t;
  t.row = sq.row0 + l;
  int slot = sq.ring_slot0 + f;  // slot0 < ring_frames and f < frames <= ring_frames
  if (slot >= sq.ring_frames) slot -= sq.ring_frames;
  t.kv_row = sq.ring_row + static_cast<int64_t>(slot) * sq.hw + rr;
  if (p.table_mode == PS_TABLE_AXES) {
    const int hh = static_cast<int>(div_by(static_cast<uint32_t>(rr), sq.gw_magic));
    t.trow_t = sq.frame_offset + f;
    t.trow_h = hh;
    t.trow_w = rr - hh * sq.gw;
  } else {
    t.trow_t = t.trow_h = t.trow_w = sq.table_row + l;
  }
  return t;
}

// Reduces (sum q^2, sum k^2) over the tpr threads of a row group; every thread of the
// group receives bit-identical sums.  `sync` orders the shared partials.
template <typename Sync>
__device__ __forceinline__ void reduce_row(const KParams& p, float2* partials, int lt, float& sq, float& sk,
                                           Sync sync) {
  for (int o = p.seg >> 1; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
  }
  if (p.nseg > 1) {
    if ((lt % p.seg) == 0) partials[lt / p.seg] = make_float2(sq, sk);
    sync();
    float a = 0.f, b = 0.f;
    for (int i = 0; i < p.nseg; ++i) {
      const float2 t = partials[i];
      a += t.x;
      b += t.y;
    }
    sq = a;
    sk = b;
  }
}

// ------------------------------------------------------------------------------------
// rows_kernel: one row group per token, register loads
// ------------------------------------------------------------------------------------
// Flag sets with specialised kernels (the remaining combinations run the generic
// instantiation, FLAGS = 0, which reads the flags at run time).
constexpr int kModeRing = kHasQ | kHasK | kHasV | kNormQ | kNormK | kKOut;  // ring layout prep
constexpr int kModeRef = kHasQ | kHasK | kNormQ | kNormK | kKPre;           // reference-layout prep
constexpr int kModeSink = kHasK | kKOut;                                    // sink re-rotation

template <typename T, int V, int FLAGS>
__global__ void __launch_bounds__(kMaxThreads) rows_kernel(const __grid_constant__ KParams p) {
  using PT = Pairs16<T>;
  constexpr int E = Vec16<T>::kElems;
  constexpr int P = PT::kPairs;
  extern __shared__ float2 partials[];  // [rows][nseg]
  const int flags = FLAGS ? FLAGS : p.flags;

  const int rg = threadIdx.x / p.tpr;
  const int lt = threadIdx.x - rg * p.tpr;
  const int dvec = lt % p.vph;
  const int head0 = lt / p.vph;
  const int g0 = blockIdx.x * p.rows + rg;
  const bool active = g0 < p.total;
  const int g = active ? g0 : 0;
  // The row first, so the loads are issued before the rest of the decode.
  const int sidx = find_seq(p, g);
  const int64_t row = p.seq[sidx].row0 + (g - p.cum[sidx]);
  // A relocated sink's token: K only, read pre-RoPE from k_sink, no RMSNorm (row group uniform).
  const bool sink = (flags & kSinkSeqs) && p.seq[sidx].kind == PS_SEQ_SINK;
  const bool do_q = (flags & kHasQ) && !sink;
  const bool do_v = (flags & kHasV) && !sink;
  const bool norm_q = (flags & kNormQ) && !sink;
  const bool norm_k = (flags & kNormK) && !sink;
  const bool kpre = (flags & kKPre) && !sink;

  int elem_off[V];
#pragma unroll
  for (int i = 0; i < V; ++i) elem_off[i] = (head0 + i * p.hstep) * p.head_dim + dvec * E;

  if (!p.early) pdl_wait();
  uint4 qv[V], kv[V], vv[V];
  if (active) {
    const T* qrow = static_cast<const T*>(p.q) + row * p.q_stride;
    const T* krow = sink ? static_cast<const T*>(p.k_sink) + row * p.k_sink_stride
                         : static_cast<const T*>(p.k) + row * p.k_stride;
    const T* vrow = static_cast<const T*>(p.v) + row * p.v_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (do_q) qv[i] = ld_stream(qrow + elem_off[i]);
      if (flags & kHasK) kv[i] = ld_stream(krow + elem_off[i]);
      if (do_v) vv[i] = ld_stream(vrow + elem_off[i]);
    }
  }
  const Token t = decode_in(p, sidx, g);
  f32x2 cc[P], ss[P];
  if (active && (flags & (kHasQ | kHasK))) {
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int pair = dvec * P + j;
      const int64_t trow = pair < p.tp ? t.trow_t : (pair < p.thp ? t.trow_h : t.trow_w);
      cc[j] = __ldg(reinterpret_cast<const unsigned long long*>(p.cos + trow * p.head_dim + 2 * pair));
      ss[j] = __ldg(reinterpret_cast<const unsigned long long*>(p.sin + trow * p.head_dim + 2 * pair));
    }
  }
  // Every load of this thread is in flight: a dependent launch may be scheduled.
  pdl_trigger();
  if (p.early) pdl_wait();  // the previous kernel's writes to the outputs must land first
  if (active && do_v) {
    T* vout = static_cast<T*>(p.v_out) + t.kv_row * p.v_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) st_vec(vout + elem_off[i], vv[i]);
  }

  float ssq_q = 0.f, ssq_k = 0.f;
  if (active && (norm_q || norm_k)) {
    f32x2 aq = 0, ak = 0;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      f32x2 x[P];
      if (norm_q) {
        PT::unpack(qv[i], x);
#pragma unroll
        for (int j = 0; j < P; ++j) aq = f2_fma(x[j], x[j], aq);
      }
      if (norm_k) {
        PT::unpack(kv[i], x);
#pragma unroll
        for (int j = 0; j < P; ++j) ak = f2_fma(x[j], x[j], ak);
      }
    }
    float a, b;
    f2_split(aq, a, b);
    ssq_q = a + b;
    f2_split(ak, a, b);
    ssq_k = a + b;
  }
  if (flags & (kNormQ | kNormK)) reduce_row(p, partials + rg * p.nseg, lt, ssq_q, ssq_k, [] { __syncthreads(); });
  if (!active) return;
  const float rq = rstd_of(ssq_q, p.c_f, p.eps);
  const float rk = rstd_of(ssq_k, p.c_f, p.eps);
  const f32x2 rq2 = f2_make(rq, rq), rk2 = f2_make(rk, rk);

  if (do_q) {
    T* qout = static_cast<T*>(p.q_out) + t.row * p.q_out_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      f32x2 x[P], w[P];
      PT::unpack(qv[i], x);
      if (norm_q) {
        load_weight_pairs<T>(p.wq, p.w_f32, elem_off[i], w);
#pragma unroll
        for (int j = 0; j < P; ++j) x[j] = PT::round(f2_mul(f2_mul(x[j], rq2), w[j]));
      }
      float lo[P], hi[P];
#pragma unroll
      for (int j = 0; j < P; ++j) rotate_f2(x[j], cc[j], ss[j], lo[j], hi[j]);
      st_vec(qout + elem_off[i], PT::pack(lo, hi));
    }
  }
  if (flags & kHasK) {
    T* kout = static_cast<T*>(p.k_out) + t.kv_row * p.k_out_stride;
    T* kpre_row = static_cast<T*>(p.k_pre) + t.row * p.k_pre_stride;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      f32x2 x[P], w[P];
      PT::unpack(kv[i], x);
      if (norm_k) {
        load_weight_pairs<T>(p.wk, p.w_f32, elem_off[i], w);
#pragma unroll
        for (int j = 0; j < P; ++j) x[j] = PT::round(f2_mul(f2_mul(x[j], rk2), w[j]));
      }
      float lo[P], hi[P];
      if (kpre) {
#pragma unroll
        for (int j = 0; j < P; ++j) f2_split(x[j], lo[j], hi[j]);
        st_vec(kpre_row + elem_off[i], norm_k ? PT::pack(lo, hi) : kv[i]);
      }
      if (flags & kKOut) {
#pragma unroll
        for (int j = 0; j < P; ++j) rotate_f2(x[j], cc[j], ss[j], lo[j], hi[j]);
        st_vec(kout + elem_off[i], PT::pack(lo, hi));
      }
    }
  }
}

// ------------------------------------------------------------------------------------
// bulk_kernel: persistent CTAs, TMA bulk copies through a ring of smem stages
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `parity` to complete, giving up after `limit_ns`.
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > limit_ns) {
      atomicAdd(&g_wait_timeouts, 1u);
      return false;
    }
  }
}

// Self-test of the bounded wait: thread 0 waits on an mbarrier that expects one arrival
// nobody makes; the wait gives up after `limit_ns`, counts itself in g_wait_timeouts and
// the kernel returns.  Nothing else is touched.
__global__ void wait_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_wait(&bar, 0, limit_ns);
  }
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(smem_dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(smem_src)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Waits until at most n (0..7) committed bulk groups still read shared memory.
__device__ __forceinline__ void bulk_wait_read_upto(int n) {
  switch (n) {
    case 0: bulk_wait_read<0>(); break;
    case 1: bulk_wait_read<1>(); break;
    case 2: bulk_wait_read<2>(); break;
    case 3: bulk_wait_read<3>(); break;
    case 4: bulk_wait_read<4>(); break;
    case 5: bulk_wait_read<5>(); break;
    case 6: bulk_wait_read<6>(); break;
    default: bulk_wait_read<7>(); break;
  }
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Per-stage token record written by the producer before it arrives on the stage's
// full barrier (the arrive releases it to the waiting consumers).
struct StageMeta {
  int64_t row;
  int64_t kv_row;
  int64_t trow_t, trow_h, trow_w;
};


// bulk_kernel: warp 0 lane 0 is the producer, warp 1 lane 0 drains the V ring,
// warps 2.. are the consumer row groups.
//
// Shared memory (offsets in KParams): full/empty mbarriers of the S q|k stages,
// vfull/vempty of the SV v stages, per-group abort flags and reduction partials,
// the StageMeta of every q|k stage and the ring row of every v stage, then the
// stages.  V rows never wait for q/k compute: they are loaded into their own
// ring and stored back out by warp 1 as soon as they land, so a q|k stage holds
// two rows, not three, while it is being computed.
//
// The consumer side works on whole rows in shared memory with a runtime loop
// over its vectors (vector vi = lt + j*tpr of the row), so its registers do not
// grow with the head count and one or two warps finish a token:
//   pass 1 -- sum of squares of q and k (packed fp32x2 FMAs);
//   pass 2 -- y = round((x*rstd)*w), rotated with two packed products and two
//             scalar adds per pair, written back in place.
// A thread's vectors all sit at the same head-dim slice (tpr is a multiple of
// the vectors per head), so its cos/sin pairs are loaded once per token.
template <typename T, int FLAGS>
__global__ void __launch_bounds__(kBulkMaxConsumers + 64, 1) bulk_kernel(const __grid_constant__ KParams p) {
  using PT = Pairs16<T>;
  constexpr int E = Vec16<T>::kElems;
  constexpr int P = PT::kPairs;
  extern __shared__ __align__(128) unsigned char smem[];
  const int S = p.stages;
  const int SV = p.vstages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  uint64_t* vfull = empty + S;
  uint64_t* vempty = vfull + SV;
  int* abort_flag = reinterpret_cast<int*>(smem + p.off_abort);                // [groups]
  float2* partials_base = reinterpret_cast<float2*>(smem + p.off_partials);    // [groups][nseg]
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + p.off_meta);           // [S]
  int64_t* vmeta = reinterpret_cast<int64_t*>(smem + p.off_vmeta);             // [SV]
  unsigned char* qk_stages = smem + p.off_stages;
  unsigned char* v_stages = smem + p.off_vstages;

  const int flags = FLAGS ? FLAGS : p.flags;
  const bool has_qk = (flags & (kHasQ | kHasK)) != 0;
  const int G = gridDim.x;
  const int n_local = p.total > static_cast<int>(blockIdx.x) ? (p.total - 1 - static_cast<int>(blockIdx.x)) / G + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    for (int r = 0; r < p.rows; ++r) abort_flag[r] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (threadIdx.x < 32) {
    // ---------------- producer ----------------
    if (threadIdx.x != 0) pdl_trigger();
    if (threadIdx.x == 0) {
      if (!p.early) pdl_wait();
      const T* qb = static_cast<const T*>(p.q);
      const T* kb = static_cast<const T*>(p.k);
      const T* vb = static_cast<const T*>(p.v);
      int issued = 0, vissued = 0;
      int cursor = 0;  // sequence of the current token: tokens only move forward
      for (int i = 0; i < n_local; ++i) {
        const int g = static_cast<int>(blockIdx.x) + i * G;
        while (cursor + 1 < p.n_seqs && p.cum[cursor + 1] <= g) ++cursor;
        const Token t = decode_in(p, cursor, g);
        if (flags & kHasV) {
          const int sv = i % SV;
          if (i >= SV && !mbar_wait(&vempty[sv], ((i / SV) & 1) ^ 1)) break;
          vmeta[sv] = t.kv_row;
          mbar_arrive_expect_tx(&vfull[sv], p.row_bytes);
          bulk_load(v_stages + static_cast<size_t>(sv) * p.vstage_bytes, vb + t.row * p.v_stride, p.row_bytes,
                    &vfull[sv]);
          vissued = i + 1;
        }
        if (has_qk) {
          const int s = i % S;
          if (i >= S && !mbar_wait(&empty[s], ((i / S) & 1) ^ 1)) break;
          meta[s] = StageMeta{t.row, t.kv_row, t.trow_t, t.trow_h, t.trow_w};
          unsigned char* st = qk_stages + static_cast<size_t>(s) * p.stage_bytes;
          mbar_arrive_expect_tx(&full[s], p.load_bytes);
          if (flags & kHasQ) bulk_load(st, qb + t.row * p.q_stride, p.row_bytes, &full[s]);
          if (flags & kHasK) bulk_load(st + p.row_bytes, kb + t.row * p.k_stride, p.row_bytes, &full[s]);
          issued = i + 1;
        }
        if (i == 0) pdl_trigger();  // loads are in flight: a dependent launch may be scheduled
      }
      if (n_local == 0) pdl_trigger();
      // Drain: every load issued must have landed before the CTA may exit.
      for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) mbar_wait(&full[i % S], (i / S) & 1);
      for (int i = vissued - SV > 0 ? vissued - SV : 0; i < vissued; ++i) mbar_wait(&vfull[i % SV], (i / SV) & 1);
    }
    return;
  }
  // Every other thread writes outputs: wait for the kernel this one depends on (if any).
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x < 64) {
    // ---------------- V ring: store each row as soon as it lands ----------------
    if (threadIdx.x == 32 && (flags & kHasV)) {
      T* vout = static_cast<T*>(p.v_out);
      // Up to `depth` stores stay in flight; a stage is freed once its store has read it.
      const int depth = p.vdepth;
      int released = 0;
      int stored = 0;
      for (int i = 0; i < n_local; ++i) {
        const int sv = i % SV;
        if (!mbar_wait(&vfull[sv], (i / SV) & 1)) break;
        bulk_store(vout + vmeta[sv] * p.v_out_stride, v_stages + static_cast<size_t>(sv) * p.vstage_bytes,
                   p.row_bytes);
        bulk_commit();
        stored = i + 1;
        bulk_wait_read_upto(depth);
        for (; released < stored - depth; ++released) mbar_arrive(&vempty[released % SV]);
      }
      bulk_wait_read<0>();
      for (; released < stored; ++released) mbar_arrive(&vempty[released % SV]);
      bulk_wait_all();
    }
    return;
  }
  if (!has_qk) return;

  // ---------------- consumers ----------------
  const int ct = threadIdx.x - 64;
  const int rg = ct / p.tpr;
  const int lt = ct - rg * p.tpr;
  const int dvec = lt % p.vph;
  const bool leader = lt == 0;
  float2* partials = partials_base + rg * p.nseg;
  volatile int* aborted = abort_flag + rg;
  const int bar_id = 1 + rg;
  auto sync = [&] { named_sync(bar_id, p.tpr); };
  const int nvec = p.C / E;  // 16-byte vectors per row
  // Leader: up to p.defer of this group's store groups stay in flight; k-th token of
  // the group is i = rg + k*groups, its stage i % S is freed once its stores read it.
  int released = 0, committed = 0;

  for (int i = rg; i < n_local; i += p.rows) {
    const int s = i % S;
    if (!mbar_wait(&full[s], (i / S) & 1)) *aborted = 1;
    const StageMeta t = meta[s];
    unsigned char* st = qk_stages + static_cast<size_t>(s) * p.stage_bytes;
    T* sq = reinterpret_cast<T*>(st);
    T* sk = reinterpret_cast<T*>(st + p.row_bytes);

    // cos / sin of this thread's pairs: (cos[2i], cos[2i+1]) and (sin[2i], sin[2i+1]).
    f32x2 cc[P], ss[P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int pair = dvec * P + j;
      const int64_t trow = pair < p.tp ? t.trow_t : (pair < p.thp ? t.trow_h : t.trow_w);
      cc[j] = __ldg(reinterpret_cast<const unsigned long long*>(p.cos + trow * p.head_dim + 2 * pair));
      ss[j] = __ldg(reinterpret_cast<const unsigned long long*>(p.sin + trow * p.head_dim + 2 * pair));
    }

    // Pass 1: sums of squares.
    f32x2 aq0 = 0, aq1 = 0, ak0 = 0, ak1 = 0;
    if (flags & (kNormQ | kNormK)) {
#pragma unroll 2
      for (int vi = lt; vi < nvec; vi += p.tpr) {
        const int off = vi * E;
        f32x2 x[P];
        if (flags & kNormQ) {
          PT::unpack(*reinterpret_cast<const uint4*>(sq + off), x);
#pragma unroll
          for (int j = 0; j < P; j += 2) {
            aq0 = f2_fma(x[j], x[j], aq0);
            if (j + 1 < P) aq1 = f2_fma(x[j + 1], x[j + 1], aq1);
          }
        }
        if (flags & kNormK) {
          PT::unpack(*reinterpret_cast<const uint4*>(sk + off), x);
#pragma unroll
          for (int j = 0; j < P; j += 2) {
            ak0 = f2_fma(x[j], x[j], ak0);
            if (j + 1 < P) ak1 = f2_fma(x[j + 1], x[j + 1], ak1);
          }
        }
      }
    }
    float ssq_q, ssq_k;
    {
      float a, b, c, d;
      f2_split(aq0, a, b);
      f2_split(aq1, c, d);
      ssq_q = (a + b) + (c + d);
      f2_split(ak0, a, b);
      f2_split(ak1, c, d);
      ssq_k = (a + b) + (c + d);
    }
    if ((flags & (kNormQ | kNormK)) && p.nseg > 1) {
      reduce_row(p, partials, lt, ssq_q, ssq_k, sync);
    } else {
      if (flags & (kNormQ | kNormK)) reduce_row(p, partials, lt, ssq_q, ssq_k, sync);
      sync();  // orders the abort vote when the reduction needed no barrier
    }
    if (*aborted) break;  // every thread of the group passed the same barrier
    const float rq = rstd_of(ssq_q, p.c_f, p.eps);
    const float rk = rstd_of(ssq_k, p.c_f, p.eps);
    const f32x2 rq2 = f2_make(rq, rq), rk2 = f2_make(rk, rk);
    T* kpre = static_cast<T*>(p.k_pre) + t.row * p.k_pre_stride;

    // Pass 2: normalise, round, rotate, write back in place.
#pragma unroll 2
    for (int vi = lt; vi < nvec; vi += p.tpr) {
      const int off = vi * E;
      if (flags & kHasQ) {
        f32x2 x[P], w[P];
        PT::unpack(*reinterpret_cast<const uint4*>(sq + off), x);
        if (flags & kNormQ) {
          load_weight_pairs<T>(p.wq, p.w_f32, off, w);
#pragma unroll
          for (int j = 0; j < P; ++j) x[j] = PT::round(f2_mul(f2_mul(x[j], rq2), w[j]));
        }
        float lo[P], hi[P];
#pragma unroll
        for (int j = 0; j < P; ++j) rotate_f2(x[j], cc[j], ss[j], lo[j], hi[j]);
        *reinterpret_cast<uint4*>(sq + off) = PT::pack(lo, hi);
      }
      if (flags & kHasK) {
        f32x2 x[P], w[P];
        const uint4 raw = *reinterpret_cast<const uint4*>(sk + off);
        PT::unpack(raw, x);
        if (flags & kNormK) {
          load_weight_pairs<T>(p.wk, p.w_f32, off, w);
#pragma unroll
          for (int j = 0; j < P; ++j) x[j] = PT::round(f2_mul(f2_mul(x[j], rk2), w[j]));
        }
        if (flags & kKPre) {
          float lo[P], hi[P];
#pragma unroll
          for (int j = 0; j < P; ++j) f2_split(x[j], lo[j], hi[j]);
          st_vec(kpre + off, (flags & kNormK) ? PT::pack(lo, hi) : raw);
        }
        if (flags & kKOut) {
          float lo[P], hi[P];
#pragma unroll
          for (int j = 0; j < P; ++j) rotate_f2(x[j], cc[j], ss[j], lo[j], hi[j]);
          *reinterpret_cast<uint4*>(sk + off) = PT::pack(lo, hi);
        }
      }
    }
    fence_async_smem();
    sync();
    if (leader) {
      if (flags & kHasQ) bulk_store(static_cast<T*>(p.q_out) + t.row * p.q_out_stride, sq, p.row_bytes);
      if (flags & kKOut) bulk_store(static_cast<T*>(p.k_out) + t.kv_row * p.k_out_stride, sk, p.row_bytes);
      bulk_commit();
      ++committed;
      // A stage is free once its stores have read it (the global writes complete
      // asynchronously); the newest p.defer store groups may still be reading.
      bulk_wait_read_upto(p.defer);
      for (; released < committed - p.defer; ++released) mbar_arrive(&empty[(rg + released * p.rows) % S]);
    }
  }
  if (leader) {
    bulk_wait_read<0>();
    for (; released < committed; ++released) mbar_arrive(&empty[(rg + released * p.rows) % S]);
    bulk_wait_all();
  }
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
struct Plan {
  KParams params;
  int kernel;  // PS_KERNEL_ROWS or PS_KERNEL_BULK
  int V;
  int threads;
  int64_t blocks;
  size_t smem;
  int elem_size;
  int launch;  // ps_launch
};

// build_plan's answer for a call with PS_SEQ_SINK sequences that the bulk kernel would run:
// the caller splits it into a launch of the chunk's sequences and a K-only launch of the sinks.
constexpr int kNeedsSplit = -1;

static int pow2_segment(int tpr) {
  int seg = 1;
  while (seg < 32 && (tpr % (seg * 2)) == 0) seg *= 2;
  return seg;
}

static bool supported_v(int v) { return v == 1 || v == 2 || v == 3 || v == 4 || v == 5 || v == 6 || v == 8; }

// Chooses heads-per-thread V for rows_kernel: the most heads per thread (up to 6, the
// largest count that fits the register budget without spilling) that keeps the row group
// a whole number of warps.  More heads per thread means fewer threads per token, so the
// per-token work -- sequence lookup, position decode, row reduction, rstd -- is shared by
// fewer threads.  Measured on B200 (percent of the HBM copy peak): C=1536 bf16 V=6 (32
// threads) 98%, V=3 (64) 89%, V=2 (96) 84%; C=3072 V=6 (64) 93%, V=3 (128) 87%.
static int choose_v(int heads, int vph, int max_threads, bool warp_multiple) {
  const int order[] = {6, 5, 4, 3, 2, 1, 8};
  for (int v : order)
    if (heads % v == 0 && (vph * (heads / v)) % 32 == 0 && vph * (heads / v) <= 256) return v;
  for (int v : order)
    if (heads % v == 0 && (vph * (heads / v)) % 32 == 0 && vph * (heads / v) <= max_threads) return v;
  if (warp_multiple) return 0;
  for (int v : order)
    if (heads % v == 0 && vph * (heads / v) <= max_threads) return v;
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

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      n > 0)
    return n;
  return 148;
}

// Validates a call and fills its launch plan.  Sequences of kind PS_SEQ_SINK are accepted
// when `allow_sinks` (they read K from k_sink; one rows-kernel launch covers them with the
// chunk's sequences, see kNeedsSplit for the bulk kernel).
static int build_plan(const ps_qk_prep_args* a, Plan* plan, bool host_only, bool allow_sinks) {
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  if (a->dtype != PS_BF16 && a->dtype != PS_F32) return fail(PS_ERR_DTYPE, "dtype %d is not PS_BF16 or PS_F32", a->dtype);
  if (a->weight_f32 != 0 && a->weight_f32 != 1) return fail(PS_ERR_DTYPE, "weight_f32=%d is not 0 or 1", a->weight_f32);
  if (a->launch < PS_LAUNCH_STREAM || a->launch > PS_LAUNCH_PDL_EARLY_INPUTS)
    return fail(PS_ERR_SHAPE, "launch mode %d unknown", a->launch);
  if (a->n_seqs < 1) return fail(PS_ERR_SHAPE, "n_seqs=%d", a->n_seqs);
  if (a->n_seqs > PS_MAX_SEQS) return fail(PS_ERR_TOO_MANY_SEQS, "n_seqs=%d exceeds PS_MAX_SEQS=%d", a->n_seqs, PS_MAX_SEQS);
  if (!a->seqs) return fail(PS_ERR_NULL, "seqs is NULL");
  int n_sink = 0;
  for (int s = 0; s < a->n_seqs; ++s) {
    if (a->seqs[s].kind != PS_SEQ_PREP && a->seqs[s].kind != PS_SEQ_SINK)
      return fail(PS_ERR_SHAPE, "seq %d: kind %d unknown", s, a->seqs[s].kind);
    n_sink += a->seqs[s].kind == PS_SEQ_SINK;
  }
  if (n_sink && !allow_sinks) return fail(PS_ERR_SHAPE, "sink sequences are not accepted here");
  const int es = a->dtype == PS_BF16 ? 2 : 4;
  const int E = 16 / es;
  if (a->heads < 1 || a->head_dim < 2 || (a->head_dim % 2)) return fail(PS_ERR_SHAPE, "heads=%d head_dim=%d invalid", a->heads, a->head_dim);
  if (a->head_dim % E) return fail(PS_ERR_ALIGN, "head_dim=%d: a head must be whole 16-byte vectors", a->head_dim);
  const int64_t C = static_cast<int64_t>(a->heads) * a->head_dim;
  if (C > (1 << 20)) return fail(PS_ERR_UNSUPPORTED, "C=%lld too large", (long long)C);
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
  if (n_sink) {
    if (!a->k_sink) return fail(PS_ERR_NULL, "sink sequences need k_sink");
    if ((rc = check_ptr(a->k_sink, "k_sink")) || (rc = check_stride(a->k_sink_stride, C, es, "k_sink"))) return rc;
    if (!a->k_out) return fail(PS_ERR_NULL, "sink sequences need k_out");
    if (a->k_sink_rows < 0) return fail(PS_ERR_SHAPE, "k_sink_rows=%lld", (long long)a->k_sink_rows);
  }
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
  if (a->in_rows < 0) return fail(PS_ERR_SHAPE, "in_rows=%lld", (long long)a->in_rows);
  if (a->kernel != PS_KERNEL_AUTO && a->kernel != PS_KERNEL_ROWS && a->kernel != PS_KERNEL_BULK)
    return fail(PS_ERR_SHAPE, "kernel %d unknown", a->kernel);

  KParams& k = plan->params;
  memset(&k, 0, sizeof(k));
  const bool k_out = has_k && a->k_out != nullptr;
  k.flags = (has_q ? kHasQ : 0) | (has_k ? kHasK : 0) | (has_v ? kHasV : 0) | (norm_q ? kNormQ : 0) |
            (norm_k ? kNormK : 0) | (a->k_pre ? kKPre : 0) | (k_out ? kKOut : 0) | (n_sink ? kSinkSeqs : 0);
  int64_t total = 0;
  for (int s = 0; s < a->n_seqs; ++s) {
    const ps_seq& q = a->seqs[s];
    if (q.n_tokens < 0 || q.grid_h < 1 || q.grid_w < 1)
      return fail(PS_ERR_SHAPE, "seq %d: n_tokens=%d grid=%dx%d", s, q.n_tokens, q.grid_h, q.grid_w);
    const int64_t hw = static_cast<int64_t>(q.grid_h) * q.grid_w;
    if (hw > INT32_MAX || q.n_tokens % hw)
      return fail(PS_ERR_SHAPE, "seq %d: n_tokens=%d is not whole frames of %lld tokens", s, q.n_tokens, (long long)hw);
    const int64_t frames = q.n_tokens / hw;
    const bool sink = q.kind == PS_SEQ_SINK;
    const int64_t src_rows = sink ? a->k_sink_rows : a->in_rows;
    if (q.token_start < 0 || q.token_start + q.n_tokens > src_rows)
      return fail(PS_ERR_BOUNDS, "seq %d: rows [%lld, %lld) outside %s=%lld", s, (long long)q.token_start,
                  (long long)(q.token_start + q.n_tokens), sink ? "k_sink_rows" : "in_rows", (long long)src_rows);
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
    if ((k_out || has_v) && q.n_tokens > 0) {
      if (q.ring_frames < 1 || q.ring_slot0 < 0 || q.ring_slot0 >= q.ring_frames)
        return fail(PS_ERR_BOUNDS, "seq %d: ring slot %d outside [0, %d)", s, q.ring_slot0, q.ring_frames);
      if (frames > q.ring_frames)
        return fail(PS_ERR_BOUNDS, "seq %d: %lld frames would overwrite each other in a ring of %d", s, (long long)frames,
                    q.ring_frames);
      if (q.ring_row < 0 || q.ring_row + static_cast<int64_t>(q.ring_frames) * hw > a->kv_out_rows)
        return fail(PS_ERR_BOUNDS, "seq %d: ring rows [%lld, %lld) outside kv_out_rows=%lld", s, (long long)q.ring_row,
                    (long long)(q.ring_row + q.ring_frames * hw), (long long)a->kv_out_rows);
    }
    if (q.n_tokens >= (1 << 30)) return fail(PS_ERR_UNSUPPORTED, "seq %d: sizes beyond 2^30 tokens", s);
    k.cum[s] = static_cast<int32_t>(total);
    DevSeq& d = k.seq[s];
    d.hw_magic = div_magic(static_cast<uint32_t>(hw));
    d.gw_magic = div_magic(static_cast<uint32_t>(q.grid_w));
    d.row0 = q.token_start;
    d.table_row = q.table_row;
    d.ring_row = q.ring_row;
    d.hw = static_cast<int32_t>(hw);
    d.gw = q.grid_w;
    d.frame_offset = q.frame_offset;
    d.ring_frames = q.ring_frames > 0 ? q.ring_frames : 1;
    d.ring_slot0 = q.ring_slot0;
    d.kind = q.kind;
    total += q.n_tokens;
    if (total > (1 << 30)) return fail(PS_ERR_SHAPE, "more than 2^30 tokens in one call");
  }
  k.cum[a->n_seqs] = static_cast<int32_t>(total);
  k.total = static_cast<int32_t>(total);
  k.n_seqs = a->n_seqs;

  // Kernel and tiling.
  const int row_bytes = static_cast<int>(C * es);
  const int qk_stage_bytes = (2 * row_bytes + 127) & ~127;
  const int v_stage_bytes = (row_bytes + 127) & ~127;
  const int nvec = static_cast<int>(C / E);
  // The bulk pipeline is the faster kernel for rows of 8 KB and more (B200, C=5120 bf16: 95%
  // vs 91% of the HBM copy peak); on narrower rows the register-load kernel wins (C=3072:
  // 93% vs 81%, C=1536: 98% vs 47%).
  const bool bulk_shape = (32 % vph) == 0 && row_bytes >= 8192 &&
                          2048 + 4 * qk_stage_bytes + 2 * v_stage_bytes <= kBulkSmemBudget;
  int kernel = a->kernel;
  if (kernel == PS_KERNEL_AUTO) kernel = bulk_shape ? PS_KERNEL_BULK : PS_KERNEL_ROWS;
  if (a->release < 0 || a->release > 8) return fail(PS_ERR_SHAPE, "release mode %d unknown", a->release);
  if (a->vdepth < 0 || a->vdepth > 7) return fail(PS_ERR_SHAPE, "vdepth %d outside 0..7", a->vdepth);

  k.q = a->q; k.k = a->k; k.v = a->v; k.wq = norm_q ? a->q_weight : nullptr; k.wk = norm_k ? a->k_weight : nullptr;
  k.cos = a->cos; k.sin = a->sin;
  k.q_out = a->q_out; k.k_out = a->k_out; k.v_out = a->v_out; k.k_pre = a->k_pre;
  k.k_sink = n_sink ? a->k_sink : nullptr;
  k.k_sink_stride = a->k_sink_stride;
  k.w_f32 = a->dtype == PS_BF16 && a->weight_f32 == 1;
  k.early = a->launch == PS_LAUNCH_PDL_EARLY_INPUTS;
  plan->launch = a->launch;
  k.q_stride = a->q_stride; k.k_stride = a->k_stride; k.v_stride = a->v_stride;
  k.q_out_stride = a->q_out_stride; k.k_out_stride = a->k_out_stride; k.v_out_stride = a->v_out_stride;
  k.k_pre_stride = a->k_pre_stride;
  k.head_dim = a->head_dim;
  k.C = static_cast<int32_t>(C);
  k.vph = vph;
  if (a->table_mode == PS_TABLE_AXES) {
    k.tp = a->t_dim / 2;
    k.thp = (a->t_dim + a->h_dim) / 2;
  } else {
    k.tp = k.thp = a->head_dim;  // every pair reads the token row
  }
  k.table_mode = a->table_mode;
  k.eps = a->eps;
  k.c_f = static_cast<float>(C);
  plan->kernel = kernel;
  plan->elem_size = es;
  if (kernel == PS_KERNEL_BULK && n_sink) return kNeedsSplit;

  if (kernel == PS_KERNEL_ROWS) {
    int V = a->heads_per_thread;
    if (V == 0) V = choose_v(a->heads, vph, kMaxThreads, false);
    if (V <= 0 || a->heads % V) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d does not divide heads=%d", V, a->heads);
    if (!supported_v(V)) return fail(PS_ERR_UNSUPPORTED, "heads_per_thread=%d not compiled (1,2,3,4,5,6,8)", V);
    const int tpr = vph * (a->heads / V);
    if (tpr > kMaxThreads) return fail(PS_ERR_UNSUPPORTED, "row group of %d threads exceeds a CTA", tpr);
    // Small CTAs (>= 64 threads, whole warps): the last partial wave of a launch spreads over
    // more SMs.  Measured against 256-thread CTAs: config 2's 1 560-token launch 8.3 -> 7.3 us,
    // an 8-stream config-5 launch 40.0 -> 39.1 us, config 4 138.7 -> 136.1 us.
    int rows = tpr >= kRowsCtaThreads ? 1 : kRowsCtaThreads / tpr;
    while ((rows * tpr) % 32) ++rows;
    if (rows * tpr > kMaxThreads) return fail(PS_ERR_UNSUPPORTED, "cannot tile %d-thread rows into whole warps", tpr);
    k.tpr = tpr;
    k.hstep = tpr / vph;
    k.seg = pow2_segment(tpr);
    k.nseg = tpr / k.seg;
    k.rows = rows;
    plan->V = V;
    plan->threads = rows * tpr;
    plan->blocks = (total + rows - 1) / rows;
    plan->smem = k.nseg > 1 ? static_cast<size_t>(rows) * k.nseg * sizeof(float2) : 0;
    return PS_OK;
  }

  // Bulk kernel.  A row group of tpr threads (whole warps; named barriers count
  // warps) owns a token; thread lt covers vectors lt, lt + tpr, ... of the row, all
  // at head-dim slice lt % vph, which needs tpr to be a multiple of vph.
  if ((32 % vph) != 0)
    return fail(PS_ERR_UNSUPPORTED, "bulk kernel needs the vectors of a head (%d) to divide a warp", vph);
  int tpr = a->row_threads;
  if (tpr == 0) tpr = nvec >= 512 ? 64 : 32;
  if (tpr < 32 || tpr % 32 || tpr > kBulkMaxConsumers)
    return fail(PS_ERR_UNSUPPORTED, "row_threads=%d must be a multiple of 32 up to %d", tpr, kBulkMaxConsumers);
  k.tpr = tpr;
  k.hstep = 0;
  k.seg = 32;
  k.nseg = tpr / 32;
  // Shared memory: four V stages (they are short-lived), q|k stages the rest.  With the V
  // drain keeping vdepth = vstages - 2 stores in flight, exactly two V stages stay free for
  // the producer: one starves the V loads, three or more let V run ahead of Q/K (B200, C=5120:
  // 124 us vs 154 us and 128-133 us per 767 MB launch).
  int vstages = has_v ? (a->vstages > 0 ? a->vstages : 4) : 0;
  if (has_v && vstages < 2) vstages = 2;
  if (vstages > 32) vstages = 32;
  auto header = [&](int S, int SV, int groups) {
    int off = 16 * S + 16 * SV;         // mbarriers
    off += 64;                          // abort flags
    off += 8 * groups * k.nseg;         // partials
    off += static_cast<int>(sizeof(StageMeta)) * S + 8 * SV;
    return (off + 127) & ~127;
  };
  int groups = a->groups;
  const int room = kBulkSmemBudget - vstages * v_stage_bytes - header(64, vstages, kBulkMaxGroups);
  const int max_stages_fit = room / qk_stage_bytes;
  if (groups <= 0) {
    // Six row groups measured best on B200 for C = 1536 .. 5120 (one token in flight
    // per group; more groups only add stages held by compute).
    groups = 6;
    if (groups > max_stages_fit - 2) groups = max_stages_fit - 2;
    if (groups < 1) groups = 1;
  }
  if (groups > kBulkMaxGroups) groups = kBulkMaxGroups;
  while (groups > 1 && groups * tpr > kBulkMaxConsumers) --groups;
  int stages = a->stages;
  if (stages <= 0) stages = (kBulkSmemBudget - vstages * v_stage_bytes - header(64, vstages, groups)) / qk_stage_bytes;
  if (stages > 64) stages = 64;
  const int head = header(stages, vstages, groups);
  const size_t layout = static_cast<size_t>(head) + static_cast<size_t>(stages) * qk_stage_bytes +
                        static_cast<size_t>(vstages) * v_stage_bytes;
  // Store groups each row group keeps in flight (release mode 1 + depth, 0 = automatic:
  // as deep as the stages allow while one stage per group stays free for loading).
  int depth = a->release > 0 ? a->release - 1 : (stages - 2 * groups) / groups;
  if (depth < 0) depth = 0;
  if (depth > 7) depth = 7;
  if (stages < groups * (depth + 1) + 1 || layout > static_cast<size_t>(kBulkSmemBudget))
    return fail(PS_ERR_UNSUPPORTED, "%d stages of %d bytes for %d row groups do not fit shared memory", stages,
                qk_stage_bytes, groups);
  k.defer = depth;
  k.rows = groups;
  k.stages = stages;
  k.vstages = vstages;  // 0 without a V role
  int vdepth = a->vdepth > 0 ? a->vdepth : vstages - 2;
  if (vdepth > vstages - 1) vdepth = vstages - 1;
  if (vdepth < 1) vdepth = 1;
  k.vdepth = vdepth;
  k.row_bytes = row_bytes;
  k.stage_bytes = qk_stage_bytes;
  k.vstage_bytes = v_stage_bytes;
  k.load_bytes = row_bytes * ((has_q ? 1 : 0) + (has_k ? 1 : 0));
  k.off_abort = 16 * stages + 16 * vstages;
  k.off_partials = k.off_abort + 64;
  k.off_meta = k.off_partials + 8 * groups * k.nseg;
  k.off_vmeta = k.off_meta + static_cast<int>(sizeof(StageMeta)) * stages;
  k.off_stages = head;
  k.off_vstages = head + stages * qk_stage_bytes;
  plan->V = 0;
  plan->threads = 64 + groups * tpr;
  plan->smem = layout;
  int ctas = host_only ? 148 : sm_count();
  if (a->ctas_per_sm > 1) ctas *= a->ctas_per_sm;
  plan->blocks = total < ctas ? total : ctas;
  return PS_OK;
}

// Opts a bulk_kernel instantiation into its dynamic shared memory once per device.
static cudaError_t allow_smem(const void* fn, int bytes) {
  struct Entry {
    const void* fn;
    int device;
    int bytes;
  };
  static Entry cache[64];
  static int used = 0;
  static std::mutex lock;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> guard(lock);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].device == dev && cache[i].bytes >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess && used < 64) cache[used++] = Entry{fn, dev, bytes};
  return err;
}

// Launches `fn` in the call's ps_launch order (programmatic dependent launch or plain).
static cudaError_t launch_kernel(void (*fn)(KParams), const Plan& plan, dim3 grid, dim3 block, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (plan.launch != PS_LAUNCH_STREAM) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, fn, plan.params);
}

template <typename T, int FLAGS>
static void (*rows_fn(int V))(KParams) {
  switch (V) {
    case 1: return rows_kernel<T, 1, FLAGS>;
    case 2: return rows_kernel<T, 2, FLAGS>;
    case 3: return rows_kernel<T, 3, FLAGS>;
    case 4: return rows_kernel<T, 4, FLAGS>;
    case 5: return rows_kernel<T, 5, FLAGS>;
    case 6: return rows_kernel<T, 6, FLAGS>;
    case 8: return rows_kernel<T, 8, FLAGS>;
    default: return nullptr;
  }
}

// Flag sets of the chunk prep with relocated sinks in the same launch (rows kernel).
constexpr int kModeRingSink = kModeRing | kSinkSeqs;

template <typename T>
static cudaError_t launch_typed(const Plan& plan, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(plan.blocks)), block(plan.threads);
  if (plan.kernel == PS_KERNEL_ROWS) {
    void (*fn)(KParams) = nullptr;
    switch (plan.params.flags) {
      case kModeRing: fn = rows_fn<T, kModeRing>(plan.V); break;
      case kModeRingSink: fn = rows_fn<T, kModeRingSink>(plan.V); break;
      case kModeRef: fn = rows_fn<T, kModeRef>(plan.V); break;
      case kModeSink: fn = rows_fn<T, kModeSink>(plan.V); break;
      default: fn = rows_fn<T, 0>(plan.V); break;
    }
    if (!fn) return cudaErrorInvalidValue;
    return launch_kernel(fn, plan, grid, block, stream);
  }
  void (*fn)(KParams) = bulk_kernel<T, 0>;
  switch (plan.params.flags) {
    case kModeRing: fn = bulk_kernel<T, kModeRing>; break;
    case kModeRef: fn = bulk_kernel<T, kModeRef>; break;
    case kModeSink: fn = bulk_kernel<T, kModeSink>; break;
    default: break;
  }
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(fn), static_cast<int>(plan.smem));
  if (err != cudaSuccess) return err;
  return launch_kernel(fn, plan, grid, block, stream);
}

// The launches of one ps_qk_norm_rope_kv call: one, or two when the bulk kernel runs a call
// with sink sequences (the chunk's sequences, then the sinks as a K-only launch).
struct Calls {
  Plan plan[2];
  int n = 0;
  std::vector<ps_seq> seqs[2];
};

// The K-only call that re-rotates the sink sequences of `a` (all of kind PS_SEQ_SINK in `sinks`).
static ps_qk_prep_args sink_call(const ps_qk_prep_args* a, std::vector<ps_seq>& sinks) {
  ps_qk_prep_args c = *a;
  c.q = nullptr; c.q_weight = nullptr; c.q_out = nullptr;
  c.v = nullptr; c.v_out = nullptr;
  c.k_weight = nullptr; c.k_pre = nullptr;
  c.k = a->k_sink; c.k_stride = a->k_sink_stride; c.in_rows = a->k_sink_rows;
  c.k_sink = nullptr;
  for (ps_seq& q : sinks) q.kind = PS_SEQ_PREP;
  c.seqs = sinks.data();
  c.n_seqs = static_cast<int32_t>(sinks.size());
  return c;
}

static int plan_calls(const ps_qk_prep_args* a, Calls* calls, bool host_only) {
  clear_error();
  calls->n = 0;
  if (!a) return fail(PS_ERR_NULL, "args is NULL");
  int n_sink = 0;
  if (a->seqs && a->n_seqs >= 1 && a->n_seqs <= PS_MAX_SEQS)
    for (int s = 0; s < a->n_seqs; ++s) n_sink += a->seqs[s].kind == PS_SEQ_SINK;
  if (n_sink > 0 && n_sink == a->n_seqs) {
    // Sinks only: the specialised K-only launch reading k_sink.
    if (!a->k_sink) return fail(PS_ERR_NULL, "sink sequences need k_sink");
    calls->seqs[1].assign(a->seqs, a->seqs + a->n_seqs);
    const ps_qk_prep_args c = sink_call(a, calls->seqs[1]);
    const int rc = build_plan(&c, &calls->plan[0], host_only, false);
    if (rc == PS_OK) calls->n = 1;
    return rc;
  }
  int rc = build_plan(a, &calls->plan[0], host_only, true);
  if (rc != kNeedsSplit) {
    if (rc == PS_OK) calls->n = 1;
    return rc;
  }
  // Bulk kernel with sink sequences: the chunk's sequences, then the sinks.
  calls->seqs[0].clear();
  calls->seqs[1].clear();
  for (int s = 0; s < a->n_seqs; ++s) calls->seqs[a->seqs[s].kind == PS_SEQ_SINK ? 1 : 0].push_back(a->seqs[s]);
  ps_qk_prep_args main_call = *a;
  main_call.seqs = calls->seqs[0].data();
  main_call.n_seqs = static_cast<int32_t>(calls->seqs[0].size());
  main_call.k_sink = nullptr;
  const ps_qk_prep_args sinks = sink_call(a, calls->seqs[1]);
  if ((rc = build_plan(&main_call, &calls->plan[0], host_only, false)) != PS_OK) return rc;
  if ((rc = build_plan(&sinks, &calls->plan[1], host_only, false)) != PS_OK) return rc;
  calls->n = 2;
  return PS_OK;
}

}  // namespace
}  // namespace ps

extern "C" int32_t ps_qk_prep_validate(const ps_qk_prep_args* args) {
  ps::Calls calls;
  return ps::plan_calls(args, &calls, true);
}

extern "C" int32_t ps_qk_norm_rope_kv(const ps_qk_prep_args* args, void* stream) {
  ps::Calls calls;
  const int rc = ps::plan_calls(args, &calls, false);
  if (rc != PS_OK) return rc;
  for (int i = 0; i < calls.n; ++i) {
    const ps::Plan& plan = calls.plan[i];
    if (plan.blocks == 0) continue;
    if (plan.blocks > 0x7fffffffLL) return ps::fail(PS_ERR_UNSUPPORTED, "grid of %lld CTAs", (long long)plan.blocks);
    const cudaError_t err = plan.elem_size == 2
                                ? ps::launch_typed<__nv_bfloat16>(plan, static_cast<cudaStream_t>(stream))
                                : ps::launch_typed<float>(plan, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "qk_prep launch: %s", cudaGetErrorString(err));
  }
  return PS_OK;
}

extern "C" int32_t ps_wait_selftest(uint32_t limit_us, void* stream) {
  ps::clear_error();
  if (limit_us < 1 || limit_us > 1000000)
    return ps::fail(PS_ERR_SHAPE, "limit_us=%u outside [1, 1000000]", limit_us);
  ps::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(1000ull * limit_us);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "wait self-test launch: %s", cudaGetErrorString(err));
  return PS_OK;
}

extern "C" int32_t ps_device_timeouts(uint32_t* count, int32_t reset) {
  ps::clear_error();
  if (!count) return ps::fail(PS_ERR_NULL, "count is NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(count, ps::g_wait_timeouts, sizeof(uint32_t));
  if (err == cudaSuccess && reset) {
    const uint32_t zero = 0;
    err = cudaMemcpyToSymbol(ps::g_wait_timeouts, &zero, sizeof(uint32_t));
  }
  if (err != cudaSuccess) return ps::fail(PS_ERR_LAUNCH, "reading the timeout counter: %s", cudaGetErrorString(err));
  return PS_OK;
}
