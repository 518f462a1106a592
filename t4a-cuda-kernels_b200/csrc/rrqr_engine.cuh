// The column engine of the RRQR kernels (F32/F64 columns with unit row stride), sm_100a.
//
// One thread block owns one column task.  Its work is built from phases, each run by
// the whole block:
//   ring_dot      <v, t> * coeff over rows [0, rows) with v_0 = 1 (the reflector's
//                 implicit leading one), folded by the reference's 32-lane chain (lane l
//                 visits rows l, l + 32, ...) from segments that bulk copies stage in
//                 shared memory;
//   update_direct t = fma(-v, d, t) over the same rows with 16-byte global loads and
//                 stores by every thread, tracking the largest finite modulus and a
//                 non-finite flag of rows [1, rows);
//   peak_direct   the largest modulus of a column read directly by every thread;
//   scaled_norm   the reference's chain of (|x| / scale)^2: helper warps load x straight
//                 from global memory, divide, and fill shared-memory buffers that the
//                 chain warp folds.
// The chains run in one warp in the reference's visiting order, so every norm, dot and
// update has the reference's bits; the staging, the direct vector phases and the
// division of work between warps are this library's.
//
// Roles in a block of kColThreads threads:
//   warp 0       the chain warp;
//   warps 1..3   producers: lane 0 of warp 1 + k issues the bulk copies of ring stage k
//                (a bulk copy costs its issuing warp about the same time whatever its
//                size, so three warps keep three copies going);
//   warps 4..11  helpers (the scaled magnitudes of scaled_norm);
//   every warp   the direct phases.
// The dot's ring has kColStages stages of kColStageBytes with two mbarriers each: `full`
// (the stage's copies landed) and `empty` (the chain warp released it).  Ring position p
// uses stage p % kColStages for the (p / kColStages)-th time, so the parity of every wait
// is a function of p alone.  scaled_norm views the same bytes as kNormBufs buffers with
// their own `ready` / `freed` mbarriers; a block runs at most one scaled_norm.  Every
// wait is bounded; one that runs out stops the block's remaining staged work and sets
// bit 1 of the status word, and a stopped block writes no result it did not finish.
//
// Segment placement: element e of a segment sits at slot sh + e, where sh * sizeof(F) is
// the operand's address modulo 16 at its first row, so the 16-byte-aligned bytes covering
// a segment copy to slot 0.  No byte outside the operand's rows is copied: the partial
// 16-byte groups at the operand's two ends are loaded element by element.
#pragma once

#include "rrqr_core.cuh"

namespace t4a {
namespace rrqr {

constexpr int kColThreads = 384;
constexpr int kColWarps = kColThreads / 32;
constexpr int kColProducers = 3;
constexpr int kColStages = kColProducers;  // producer k issues every copy of stage k
constexpr int kColHelperWarp0 = 1 + kColProducers;
constexpr int kColHelpers = kColThreads - 32 * kColHelperWarp0;
constexpr int kColStageBytes = 32768;
// try_wait rounds of a staged-data wait before it gives up (a build may lower it: the
// tests build the library once with 0, so that every such wait runs out at once).
#ifndef T4A_STAGE_WAIT_LIMIT
#define T4A_STAGE_WAIT_LIMIT (1u << 20)
#endif
constexpr unsigned kColWaitLimit = T4A_STAGE_WAIT_LIMIT;
// Rounds of the exit drain, which waits for the bulk copies still in flight so that none
// lands in shared memory after the block is gone: separate, and never lowered.
constexpr unsigned kColDrainLimit = 1u << 22;
constexpr unsigned kColSuspendNs = 1000;

// scaled_norm's buffers: the ring's bytes viewed as kNormBufs buffers of kNormSeg elements.
constexpr int kNormBufs = 6;
// Largest thread-block cluster of the clustered column pass (the portable limit).
constexpr int kMaxCluster = 8;

template <typename F>
struct ColSmem {
  static constexpr int kPad = 16 / static_cast<int>(sizeof(F));
  static constexpr int kSeg1 = kColStageBytes / static_cast<int>(sizeof(F));  // norm: elements per segment
  static constexpr int kSeg2 = kSeg1 / 2;                                      // dot: per operand
  static constexpr int kRegion2 = kSeg2 + kPad;                                // dot: slots of one operand
  static constexpr int kStage = kSeg1 + 2 * kPad;
  static constexpr int kNormSeg = kColStages * kSeg1 / kNormBufs;  // scaled_norm: elements per buffer
  F raw[kColStages][kStage];
  unsigned long long full[kColStages];
  unsigned long long empty[kColStages];
  unsigned long long ready[kNormBufs];  // scaled_norm: buffer b filled by the helpers
  unsigned long long freed[kNormBufs];  // scaled_norm: buffer b folded by the chain warp
  F red[kColWarps];
  int bad[kColWarps];
  F cpeak[kMaxCluster];  // clustered pass, leader: each rank's block peak and flag
  int cbad[kMaxCluster];
  F dot;
  int abort;
  int last;  // this block drew the pass's last ticket
};

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

// Bounded wait for the phase of parity `parity` of an mbarrier; false when it ran out.
__device__ __forceinline__ bool bar_wait(const unsigned long long* bar, unsigned parity,
                                         unsigned limit = kColWaitLimit) {
  const unsigned addr = smem_addr(bar);
  for (unsigned it = 0; it < limit; ++it) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "n"(kColSuspendNs)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void bar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Orders this thread's generic-proxy writes before later bulk copies (async proxy).
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- thread-block clusters (the clustered column pass) -------------------------------
// This block's rank in its cluster (0 in a launch without clusters).
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every block of the cluster: the writes before it (shared memory of
// any block of the cluster, and global memory) are visible to the reads after it.  A
// hardware barrier: each block of a cluster is resident until it exits, and every thread
// of the clustered pass reaches each barrier exactly once.
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of `p` (this block's shared memory) in block `rank`.
__device__ __forceinline__ unsigned cluster_addr(const void* p, unsigned rank) {
  unsigned a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ double cluster_load(const double* p, unsigned rank) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(cluster_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ float cluster_load(const float* p, unsigned rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ int cluster_load(const int* p, unsigned rank) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(cluster_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_store(double* p, unsigned rank, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(cluster_addr(p, rank)), "d"(v) : "memory");
}
__device__ __forceinline__ void cluster_store(float* p, unsigned rank, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr(p, rank)), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_store(int* p, unsigned rank, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(cluster_addr(p, rank)), "r"(v) : "memory");
}

__device__ __forceinline__ int stage_of(long long p) { return static_cast<int>(p % kColStages); }
__device__ __forceinline__ unsigned parity_of(long long p) { return static_cast<unsigned>((p / kColStages) & 1); }

template <typename F>
__device__ __forceinline__ void fail(ColSmem<F>& sm, long long* status) {
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  atomicOr(reinterpret_cast<unsigned long long*>(status), 2ull);
}
template <typename F>
__device__ __forceinline__ bool aborted(ColSmem<F>& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort) != 0;
}

// Producer index of this thread (lane 0 of warps 1 .. kColProducers), or -1.
__device__ __forceinline__ int producer_index() {
  const int warp = threadIdx.x >> 5;
  return (threadIdx.x & 31) == 0 && warp >= 1 && warp <= kColProducers ? warp - 1 : -1;
}

template <typename F>
__device__ __forceinline__ void engine_init(ColSmem<F>& sm) {
  if (threadIdx.x == 0) {
    for (int q = 0; q < kColStages; ++q) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sm.full[q])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sm.empty[q])) : "memory");
    }
    for (int q = 0; q < kNormBufs; ++q) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&sm.ready[q])), "n"(kColHelpers / 32)
                   : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sm.freed[q])) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.abort = 0;
  }
  __syncthreads();
}

// One staged operand: rows [0, rows) from `base`, `seg` elements per segment, placed at
// slot `region` + sh of a stage.
template <typename F>
struct Operand {
  const F* base;
  long long rows;
  int seg;
  int sh;
  int region;
};

template <typename F>
__device__ __forceinline__ Operand<F> operand(const F* base, long long rows, int seg, int region) {
  return Operand<F>{base, rows, seg, static_cast<int>((reinterpret_cast<unsigned long long>(base) & 15) / sizeof(F)),
                    region};
}

// Producer: the copies of segment g of every operand into stage st.  Bytes at the
// operands' ends that share a 16-byte group with rows outside [0, rows) are loaded one
// element at a time; the rest goes by bulk copies completing on `full[st]`.
template <typename F, int Ops>
__device__ __forceinline__ void issue_segment(ColSmem<F>& sm, const Operand<F>* ops, int st, long long g) {
  constexpr unsigned long long es = sizeof(F);
  unsigned long long c0[Ops], c1[Ops], g0[Ops];
  unsigned tx = 0;
  bool edges = false;
#pragma unroll
  for (int o = 0; o < Ops; ++o) {
    const unsigned long long lo = reinterpret_cast<unsigned long long>(ops[o].base);
    const unsigned long long hi = reinterpret_cast<unsigned long long>(ops[o].base + ops[o].rows);
    const unsigned long long w0 = (lo + 15) & ~15ull, w1 = hi & ~15ull;
    const long long e0 = g * ops[o].seg;
    const long long e1 = ops[o].rows < e0 + ops[o].seg ? ops[o].rows : e0 + ops[o].seg;
    g0[o] = reinterpret_cast<unsigned long long>(ops[o].base + e0);
    const unsigned long long g1 = reinterpret_cast<unsigned long long>(ops[o].base + e1);
    c0[o] = (g0[o] & ~15ull) > w0 ? (g0[o] & ~15ull) : w0;
    c1[o] = ((g1 + 15) & ~15ull) < w1 ? ((g1 + 15) & ~15ull) : w1;
    if (c1[o] < c0[o]) c1[o] = c0[o];
    F* slots = sm.raw[st] + ops[o].region + ops[o].sh;
    for (unsigned long long x = g0[o]; x < g1 && x < c0[o]; x += es) {
      slots[(x - g0[o]) / es] = *reinterpret_cast<const F*>(x);
      edges = true;
    }
    for (unsigned long long x = c1[o] > g0[o] ? c1[o] : g0[o]; x < g1; x += es) {
      slots[(x - g0[o]) / es] = *reinterpret_cast<const F*>(x);
      edges = true;
    }
    tx += static_cast<unsigned>(c1[o] - c0[o]);
  }
  if (edges) fence_async_shared();
  const unsigned bar = smem_addr(&sm.full[st]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
#pragma unroll
  for (int o = 0; o < Ops; ++o) {
    if (c1[o] > c0[o]) {
      const unsigned dst = smem_addr(sm.raw[st] + ops[o].region + ops[o].sh) +
                           static_cast<unsigned>(static_cast<long long>(c0[o]) - static_cast<long long>(g0[o]));
      asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                   "l"(c0[o]), "r"(static_cast<unsigned>(c1[o] - c0[o])), "r"(bar)
                   : "memory");
    }
  }
}

// A producer's state: the last ring position it issued (-1: none).
struct Producer {
  int k;
  long long last;
};

__device__ __forceinline__ Producer producer_start() { return Producer{producer_index(), -1}; }

// Producer k's part of a ring phase at positions [base, base + nseg): the positions of
// stage k, each after the stage's previous use was released.  false: a wait ran out.
template <typename F, int Ops>
__device__ __forceinline__ bool produce(ColSmem<F>& sm, Producer& pr, const Operand<F>* ops, long long base,
                                        long long nseg) {
  long long p = base + ((pr.k - base % kColStages) % kColStages + kColStages) % kColStages;
  for (; p < base + nseg; p += kColStages) {
    if (aborted(sm)) return true;
    if (p >= kColStages && !bar_wait(&sm.empty[pr.k], parity_of(p - kColStages))) return false;
    issue_segment<F, Ops>(sm, ops, pr.k, p - base);
    pr.last = p;
  }
  return true;
}

// Producer exit: waits (bounded) for its copy still in flight, so that no bulk copy
// writes the block's shared memory after the block exits.
template <typename F>
__device__ __forceinline__ void drain(ColSmem<F>& sm, const Producer& pr, long long* status) {
  if (pr.k < 0 || pr.last < 0) return;
  if (!bar_wait(&sm.full[pr.k], parity_of(pr.last), kColDrainLimit))
    atomicOr(reinterpret_cast<unsigned long long*>(status), 2ull);
}

// Chain folds over one full segment (N elements per lane) in shared memory: loads run
// kAhead elements ahead of the dependent fma.
constexpr int kAhead = 8;
// lead_one: the segment's element 0 (lane 0's first) takes v = 1, the reflector's
// implicit leading one, instead of the stored value.
template <typename F, int N>
__device__ __forceinline__ F fold_products(const F* bv, const F* bt, int lane, F acc, bool lead_one = false) {
  F xv[kAhead], xt[kAhead];
#pragma unroll
  for (int k = 0; k < kAhead; ++k) {
    xv[k] = bv[lane + 32 * k];
    xt[k] = bt[lane + 32 * k];
  }
  if (lead_one && lane == 0) xv[0] = F(1);
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const F v = xv[k % kAhead], t = xt[k % kAhead];
    if (k + kAhead < N) {
      xv[k % kAhead] = bv[lane + 32 * (k + kAhead)];
      xt[k % kAhead] = bt[lane + 32 * (k + kAhead)];
    }
    acc = fma_rn(v, t, acc);
  }
  return acc;
}
template <typename F, int N>
__device__ __forceinline__ F fold_squares(const F* b, int lane, F acc) {
  F x[kAhead];
#pragma unroll
  for (int k = 0; k < kAhead; ++k) x[k] = b[lane + 32 * k];
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const F v = x[k % kAhead];
    if (k + kAhead < N) x[k % kAhead] = b[lane + 32 * (k + kAhead)];
    acc = fma_rn(v, v, acc);
  }
  return acc;
}

// <v, t> * coeff over rows [0, rows), v_0 = 1 (or v_0 as stored when !lead_one: a row
// block that does not hold the reflector's leading row), at ring positions [base, base +
// nseg) (nseg = dot_segments(rows)); the result goes to every thread (0 in a stopped
// block).
template <typename F>
__device__ __forceinline__ long long dot_segments(long long rows) {
  return (rows + ColSmem<F>::kSeg2 - 1) / ColSmem<F>::kSeg2;
}
template <typename F>
__device__ __forceinline__ F ring_dot(ColSmem<F>& sm, Producer& pr, long long base, const F* v, const F* t,
                                      long long rows, F coeff, long long* status, bool lead_one = true) {
  using S = ColSmem<F>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nseg = dot_segments<F>(rows);
  const Operand<F> ops[2] = {operand(v, rows, S::kSeg2, 0), operand(t, rows, S::kSeg2, S::kRegion2)};
  if (pr.k >= 0) {
    if (!produce<F, 2>(sm, pr, ops, base, nseg)) fail(sm, status);
  } else if (warp == 0) {
    F acc = F(0);
    // The chain checks the stop flag once: a producer that stops leaves a stage unfilled,
    // and the chain's bounded wait on it then runs out.
    const long long count = __any_sync(kAllLanes, aborted(sm)) ? 0 : nseg;
    for (long long g = 0; g < count; ++g) {
      const long long p = base + g;
      const int st = stage_of(p);
      if (!__all_sync(kAllLanes, bar_wait(&sm.full[st], parity_of(p)))) {
        if (lane == 0) fail(sm, status);
        break;
      }
      const F* bv = sm.raw[st] + ops[0].sh;
      const F* bt = sm.raw[st] + S::kRegion2 + ops[1].sh;
      const long long e0 = g * S::kSeg2;
      if (e0 + S::kSeg2 <= rows) {
        acc = fold_products<F, S::kSeg2 / 32>(bv, bt, lane, acc, g == 0 && lead_one);
      } else if (g == 0) {
        const int len = static_cast<int>(rows);
        for (int i = lane; i < len; i += 32) acc = fma_rn(i == 0 && lead_one ? F(1) : bv[i], bt[i], acc);
      } else {
        const int len = static_cast<int>(rows - e0);
        for (int i = lane; i < len; i += 32) acc = fma_rn(bv[i], bt[i], acc);
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.empty[st]);
    }
    const F d = butterfly(acc, AddOp()) * coeff;
    if (lane == 0) sm.dot = d;
  }
  __syncthreads();
  return aborted(sm) ? F(0) : sm.dot;
}

// Running maximum of finite moduli and the non-finite flag.
template <typename F>
__device__ __forceinline__ void track(F value, F* peak, bool* flagged) {
  const F m = modulus(value);
  const bool nf = nonfinite(m);
  *flagged = *flagged || nf;
  *peak = (!nf && m > *peak) ? m : *peak;
}

// 16-byte vectors of F for the direct phases.
template <typename F> struct Vec16;
template <> struct Vec16<double> {
  using V = double2;
  static constexpr int kW = 2;
};
template <> struct Vec16<float> {
  using V = float4;
  static constexpr int kW = 4;
};

template <typename F>
__device__ __forceinline__ F& elem(typename Vec16<F>::V& x, int i) {
  return reinterpret_cast<F*>(&x)[i];
}

// Rows [0, rows) of a column split for 16-byte access: `lead` rows before the first
// 16-byte boundary, `body` whole 16-byte groups, then the tail.
template <typename F>
struct Split16 {
  long long lead, body, tail0;
};
template <typename F>
__device__ __forceinline__ Split16<F> split16(const F* x, long long rows) {
  const long long head = static_cast<long long>((16 - (reinterpret_cast<unsigned long long>(x) & 15)) & 15) /
                         static_cast<long long>(sizeof(F));
  Split16<F> s;
  s.lead = head < rows ? head : rows;
  s.body = (rows - s.lead) / Vec16<F>::kW;
  s.tail0 = s.lead + s.body * Vec16<F>::kW;
  return s;
}

// t = fma(-v, d, t) over rows [0, rows) (v_0 = 1 unless !lead_one), by every thread, with
// 16-byte loads and stores where v and t share their alignment.  The 16-byte groups are
// taken from the last one down, so the lowest rows, which a following ring phase reads
// first, are the most recently written.  kTrack: the largest finite modulus and the
// non-finite flag of the updated rows other than the implicit-one row go to *peak /
// *flagged.
template <bool kTrack, typename F>
__device__ __forceinline__ void update_direct(const F* v, F* t, long long rows, F d, F* peak, bool* flagged,
                                              bool lead_one = true) {
  const long long one = lead_one ? 0 : -1;  // the row whose v is the implicit 1 (none: -1)
  using V = typename Vec16<F>::V;
  constexpr int kW = Vec16<F>::kW;
  const long long tid = threadIdx.x;
  const bool paired = ((reinterpret_cast<unsigned long long>(v) ^ reinterpret_cast<unsigned long long>(t)) & 15) == 0;
  Split16<F> sp = split16(t, rows);
  if (!paired) {
    sp.body = 0;
    sp.tail0 = sp.lead;
  }
  const long long edge = sp.lead + (rows - sp.tail0);
  for (long long i = tid; i < edge; i += kColThreads) {
    const long long r = i < sp.lead ? i : sp.tail0 + (i - sp.lead);
    const F nt = fma_rn(-(r == one ? F(1) : v[r]), d, t[r]);
    t[r] = nt;
    if (kTrack && r != one) track(nt, peak, flagged);
  }
  const V* vv = reinterpret_cast<const V*>(v + sp.lead);
  V* tv = reinterpret_cast<V*>(t + sp.lead);
  constexpr int kU = 4;  // groups in flight per thread
  for (long long q0 = sp.body - 1 - tid; q0 >= 0; q0 -= kU * kColThreads) {
    V xv[kU], xt[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long q = q0 - static_cast<long long>(u) * kColThreads;
      if (q >= 0) {
        xv[u] = vv[q];
        xt[u] = tv[q];
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long q = q0 - static_cast<long long>(u) * kColThreads;
      if (q < 0) continue;
#pragma unroll
      for (int e = 0; e < kW; ++e) {
        const long long r = sp.lead + q * kW + e;
        const F nt = fma_rn(-(r == one ? F(1) : elem<F>(xv[u], e)), d, elem<F>(xt[u], e));
        elem<F>(xt[u], e) = nt;
        if (kTrack && r != one) track(nt, peak, flagged);
      }
      tv[q] = xt[u];
    }
  }
}

// x = x / divisor over rows [0, rows), IEEE division per element, by every thread:
// 16-byte loads and stores, kU groups per thread loaded before any is divided, so the
// loads of a thread overlap instead of each waiting out its own latency.
template <typename F>
__device__ __forceinline__ void divide_direct(F* x, long long rows, F divisor) {
  using V = typename Vec16<F>::V;
  constexpr int kW = Vec16<F>::kW;
  const long long tid = threadIdx.x;
  const Split16<F> sp = split16(x, rows);
  const long long edge = sp.lead + (rows - sp.tail0);
  for (long long i = tid; i < edge; i += kColThreads) {
    const long long r = i < sp.lead ? i : sp.tail0 + (i - sp.lead);
    x[r] = x[r] / divisor;
  }
  V* xv = reinterpret_cast<V*>(x + sp.lead);
  constexpr int kU = 4;
  for (long long q0 = tid; q0 < sp.body; q0 += kU * kColThreads) {
    V held[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long q = q0 + static_cast<long long>(u) * kColThreads;
      if (q < sp.body) held[u] = xv[q];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long q = q0 + static_cast<long long>(u) * kColThreads;
      if (q >= sp.body) continue;
#pragma unroll
      for (int e = 0; e < kW; ++e) elem<F>(held[u], e) = elem<F>(held[u], e) / divisor;
      xv[q] = held[u];
    }
  }
}

// The largest modulus over rows [0, rows) of x, read by every thread (16-byte loads
// where aligned).  kFlag: non-finite moduli are flagged and left out (column_norms);
// otherwise every modulus competes and NaN never wins (the reflector's norm).
template <bool kFlag, typename F>
__device__ __forceinline__ void peak_direct(const F* x, long long rows, F* peak, bool* flagged) {
  using V = typename Vec16<F>::V;
  constexpr int kW = Vec16<F>::kW;
  const long long tid = threadIdx.x;
  const Split16<F> sp = split16(x, rows);
  auto visit = [&](F value) {
    if (kFlag) {
      track(value, peak, flagged);
    } else {
      const F m = modulus(value);
      *peak = m > *peak ? m : *peak;
    }
  };
  const long long edge = sp.lead + (rows - sp.tail0);
  for (long long i = tid; i < edge; i += kColThreads) visit(x[i < sp.lead ? i : sp.tail0 + (i - sp.lead)]);
  const V* xv = reinterpret_cast<const V*>(x + sp.lead);
  constexpr int kU = 4;
  for (long long q0 = tid; q0 < sp.body; q0 += kU * kColThreads) {
    V held[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long q = q0 + static_cast<long long>(u) * kColThreads;
      if (q < sp.body) held[u] = xv[q];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (q0 + static_cast<long long>(u) * kColThreads >= sp.body) continue;
#pragma unroll
      for (int e = 0; e < kW; ++e) visit(elem<F>(held[u], e));
    }
  }
}

// Block-wide maximum and any-flag, returned to every thread.
template <typename F>
__device__ __forceinline__ void block_peak(ColSmem<F>& sm, F peak, bool flagged, F* scale, bool* bad) {
  const F wm = butterfly(peak, MaxOp());
  const bool wb = __any_sync(kAllLanes, flagged);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm.red[warp] = wm;
    sm.bad[warp] = wb ? 1 : 0;
  }
  __syncthreads();
  F mx = F(0);
  int bb = 0;
#pragma unroll
  for (int q = 0; q < kColWarps; ++q) {
    mx = sm.red[q] > mx ? sm.red[q] : mx;
    bb |= sm.bad[q];
  }
  __syncthreads();
  *scale = mx;
  *bad = bb != 0;
}

// a / b for 0 <= a <= b, b > 0 fixed per column, equal to the IEEE quotient, without a
// division per element.  With r = RN(1/b) (within half an ulp of 1/b):
//   q0 = RN(a r);  q1 = RN(q0 + (a - b q0) r);  q2 = RN(q1 + (a - b q1) r).
// The remainders are exact (one fma each).  q0 is within 1.5 ulp of a/b, so
// q0 + (a - b q0) r = a/b + (a/b - q0)(b r - 1) is within 2^-51 ulp of a/b, and q1, its
// nearest double, is within one ulp of a/b.  Markstein's theorem (y within half an
// ulp of 1/b, q within one ulp of a/b, remainder exact => RN(q + (a - b q) y) =
// RN(a/b)) then makes q2 the IEEE quotient.  The theorem needs every quantity normal
// and exact: b in [2^-900, 2^900] (checked once per column; otherwise every element
// divides) and a = 0 or a >= max(b 2^-900, 2^-960) (q >= 2^-900, remainders above
// 2^-1012); smaller a divide.  F32: the same with 2^-60, 2^60, b 2^-60 and 2^-90.
template <typename F>
struct ScaledQuotient {
  F b, r, threshold;
  bool fast;
};

static __device__ __noinline__ double ieee_quotient(double a, double b) { return a / b; }
static __device__ __noinline__ float ieee_quotient(float a, float b) { return a / b; }

__device__ __forceinline__ ScaledQuotient<double> make_quotient(double b) {
  ScaledQuotient<double> q;
  q.b = b;
  q.r = 1.0 / b;
  q.fast = b >= 0x1p-900 && b <= 0x1p900;
  q.threshold = fmax(b * 0x1p-900, 0x1p-960);
  return q;
}
__device__ __forceinline__ ScaledQuotient<float> make_quotient(float b) {
  ScaledQuotient<float> q;
  q.b = b;
  q.r = 1.0f / b;
  q.fast = b >= 0x1p-60f && b <= 0x1p60f;
  q.threshold = fmaxf(b * 0x1p-60f, 0x1p-90f);
  return q;
}

// The fast quotient (exact when quotient_safe holds) and its precondition, kept apart
// so that a thread's quotients interleave without a call between them.
__device__ __forceinline__ double quotient_fast(const ScaledQuotient<double>& s, double a) {
  const double q0 = __dmul_rn(a, s.r);
  const double q1 = __fma_rn(__fma_rn(-s.b, q0, a), s.r, q0);
  return __fma_rn(__fma_rn(-s.b, q1, a), s.r, q1);
}
__device__ __forceinline__ float quotient_fast(const ScaledQuotient<float>& s, float a) {
  const float q0 = __fmul_rn(a, s.r);
  const float q1 = __fmaf_rn(__fmaf_rn(-s.b, q0, a), s.r, q0);
  return __fmaf_rn(__fmaf_rn(-s.b, q1, a), s.r, q1);
}
template <typename F>
__device__ __forceinline__ bool quotient_safe(const ScaledQuotient<F>& s, F a) {
  return s.fast && (a == F(0) || a >= s.threshold);
}

// The reference's chain of (|x| / scale)^2 over rows [0, rows) of x (scale > 0), the
// block's only norm phase.  The helper warps load x straight from global memory (after an
// update it is L2-hot), turn it into |x| / scale and store it into buffer g %
// kNormBufs; the chain warp folds each buffer in the reference's lane order and frees
// it.  A helper issues the loads of its next segment before it waits for a free buffer,
// so the loads run while the chain folds.  Returns the butterfly-summed chain to every
// thread (0 in a block that stopped).
//
// Measured at config-5 size (65536 rows), this phase takes 20-28 us per block against
// 10.4 us for the chain alone: the helpers' loads and quotients share the SM with the
// chain, and the 134 MB matrix, about the size of L2, is streamed by every phase.
// Staging by bulk copies or by cp.async (64 KB in flight per block) measured the same or
// slower.
// kFromL2: the helpers read x from L2 (ld.global.cg), bypassing this SM's L1: rows of x
// written by other blocks of a cluster, whose cache lines this block may hold from its own
// loads of neighbouring rows.
template <typename F, bool kFromL2 = false>
__device__ __forceinline__ F scaled_norm(ColSmem<F>& sm, const F* x, long long rows, F scale, long long* status) {
  using S = ColSmem<F>;
  constexpr int kSeg = S::kNormSeg;
  constexpr int kPer = kSeg / kColHelpers;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long nseg = (rows + kSeg - 1) / kSeg;
  F* bufs = &sm.raw[0][0];
  if (warp >= kColHelperWarp0) {
    const ScaledQuotient<F> quo = make_quotient(scale);
    const int h = tid - 32 * kColHelperWarp0;
    F held[kPer];
    auto load = [&](long long g) {
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const long long i = g * kSeg + h + static_cast<long long>(kColHelpers) * q;
        held[q] = i < rows ? (kFromL2 ? __ldcg(x + i) : x[i]) : F(0);
      }
    };
    if (nseg > 0) load(0);
    for (long long g = 0; g < nseg; ++g) {
      F qv[kPer];
      bool unsafe = false;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const F a = modulus(held[q]);
        qv[q] = quotient_fast(quo, a);
        unsafe |= !quotient_safe(quo, a);
      }
      if (unsafe) {
        // Operands outside the fast quotient's range: IEEE division for those.
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
          const F a = modulus(held[q]);
          if (!quotient_safe(quo, a)) qv[q] = ieee_quotient(a, quo.b);
        }
      }
      if (g + 1 < nseg) load(g + 1);
      const int b = static_cast<int>(g % kNormBufs);
      if (__any_sync(kAllLanes, aborted(sm))) break;
      if (g >= kNormBufs &&
          !__all_sync(kAllLanes, bar_wait(&sm.freed[b], static_cast<unsigned>(((g - kNormBufs) / kNormBufs) & 1)))) {
        if (lane == 0) fail(sm, status);
        break;
      }
      F* buf = bufs + static_cast<long long>(b) * kSeg;
#pragma unroll
      for (int q = 0; q < kPer; ++q) buf[h + kColHelpers * q] = qv[q];
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.ready[b]);
    }
  } else if (warp == 0) {
    F acc = F(0);
    // As in ring_dot: a helper that stops leaves a buffer unfilled, and the chain's
    // bounded wait on it runs out.
    const long long count = __any_sync(kAllLanes, aborted(sm)) ? 0 : nseg;
    for (long long g = 0; g < count; ++g) {
      const int b = static_cast<int>(g % kNormBufs);
      if (!__all_sync(kAllLanes, bar_wait(&sm.ready[b], static_cast<unsigned>((g / kNormBufs) & 1)))) {
        if (lane == 0) fail(sm, status);
        break;
      }
      const F* buf = bufs + static_cast<long long>(b) * kSeg;
      const long long e0 = g * kSeg;
      if (e0 + kSeg <= rows) {
        acc = fold_squares<F, kSeg / 32>(buf, lane, acc);
      } else {
        const int len = static_cast<int>(rows - e0);
        for (int i = lane; i < len; i += 32) acc = fma_rn(buf[i], buf[i], acc);
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.freed[b]);
    }
    acc = butterfly(acc, AddOp());
    if (lane == 0) sm.dot = acc;
  }
  __syncthreads();
  return aborted(sm) ? F(0) : sm.dot;
}

}  // namespace rrqr
}  // namespace t4a
