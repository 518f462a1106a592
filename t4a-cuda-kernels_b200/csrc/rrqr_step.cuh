// Fused RRQR step kernels (F32/F64, one column-major matrix: row stride 1).
//
// One step of the reference loop -- column_norms, select_pivot, swap_columns,
// reflector, apply_reflector over the trailing columns (reference bench
// examples/bench_kernels.rs:2390-2623) -- in two launches with the same arithmetic:
//
//  pivot   one warp of the previous column pass's last block (every block publishes
//          its norm and draws a ticket; the one that draws the last sees them all):
//          the reference's pivot choice from the norms, and the reflector's scalars
//          (x0, alpha, denominator, coefficient) from the pivot column's norm, which
//          equals the reflector's own norm whenever the column is finite (the same
//          walk and the same operations); otherwise the norm is walked again.
//  swap    flat over rows: column swap, permutation swap, the reflector's scaling of
//          the new column `step` and its alpha, in one pass.
//  column  one block per trailing column: the reference's 32-lane dot chain times the
//          coefficient, the update t -= v * dot (the reference's fma), and the next
//          step's scaled sum-of-squares norm chain of the updated column, whose
//          maximum the update found (a maximum is exact in any order).
// Step 0's norms run the column pass's norm chain after a walk for the maximum.
//
// Q formation (column_q) reuses the column pass's dot and update phases
// (col_dot_update): reflector `step` of the factorized matrix applied to one column of
// Q per block, the same arithmetic as apply_reflector over Q's columns.
#pragma once

#include "rrqr_core.cuh"

namespace t4a {
namespace rrqr {

// Per-step scalars handed from the pivot pass to the swap pass.
template <typename F>
struct StepRecord {
  long long pivot;
  F alpha;
  F denominator;
  int scale;  // 0: norm == 0 (the reference leaves the column as swapped)
};

template <typename F>
struct FusedArgs {
  F* w;               // matrix, column-major
  long long m, n;     // rows, columns
  long long ld;       // column stride
  long long* perm;    // n
  F* coeff;           // reflector coefficients, one per step
  long long* pivots;  // pivot of each step
  long long* status;  // sticky non-finite flag
  F* norms;           // n
  long long span;     // elements from w to the end of the matrix
  StepRecord<F>* rec;
  unsigned* done;     // blocks of the running column pass that have written their norm
};

// pivot pass: one warp.
template <typename F>
__device__ __forceinline__ void fused_pivot(const FusedArgs<F>& a, long long step) {
  const int lane = threadIdx.x & 31;
  F local_max = F(0);
  long long local_original = kNone, local_column = kNone;
  bool invalid = false;
  for (long long column = step + lane; column < a.n; column += kPlane) {
    const F norm = a.norms[column];
    const long long original = a.perm[column];
    if (norm < F(0)) {
      invalid = true;
    } else if (norm > local_max || (norm == local_max && original < local_original)) {
      local_max = norm;
      local_original = original;
      local_column = column;
    }
  }
  const F maximum = plane_max(local_max);
  const long long original = plane_min(local_max == maximum ? local_original : kNone);
  const long long selected = plane_min(local_max == maximum && local_original == original ? local_column : kNone);
  const bool any_invalid = __any_sync(kFull, invalid);
  const long long pivot = selected == kNone ? step : selected;
  // Reflector of the column that the swap brings to `step` (reference rrqr.cu:290-332).
  F norm = a.norms[pivot];
  if (!(norm >= F(0))) {
    // Non-finite column: the reflector's own walk (it does not skip non-finite values).
    norm = column_norm<F, F, false, 1>(a.w, pivot * a.ld, 1, step, a.m, lane, nullptr);
  }
  const F x0 = a.w[pivot * a.ld + step];
  if (lane == 0) {
    a.pivots[step] = pivot;
    if (any_invalid) *a.status = 1;
    StepRecord<F> r;
    r.pivot = pivot;
    if (norm == F(0)) {
      r.scale = 0;
      r.alpha = F(0);
      r.denominator = F(1);
      a.coeff[step] = F(0);
    } else {
      const F phase = x0 < F(0) ? F(-1) : F(1);
      r.alpha = -phase * norm;
      r.denominator = x0 - r.alpha;
      r.scale = 1;
      a.coeff[step] = F(1) + mag(x0) / norm;
    }
    *a.rec = r;
  }
}

// swap pass: rows [0, m), flat.
template <typename F>
__device__ __forceinline__ void fused_swap(const FusedArgs<F>& a, long long step, long long row) {
  const StepRecord<F> r = *a.rec;
  F* cs = a.w + step * a.ld;
  F* cp = a.w + r.pivot * a.ld;
  const F left = cs[row];
  const F right = cp[row];
  F moved = r.pivot == step ? left : right;  // the value that lands in column `step`
  if (r.scale) {
    if (row == step) {
      moved = r.alpha;
    } else if (row > step) {
      moved = moved / r.denominator;
    }
  }
  cs[row] = moved;
  if (r.pivot != step) {
    cp[row] = left;
    if (row == 0) {
      const long long s = a.perm[step];
      a.perm[step] = a.perm[r.pivot];
      a.perm[r.pivot] = s;
    }
  }
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

__device__ __noinline__ double ieee_quotient(double a, double b) { return a / b; }
__device__ __noinline__ float ieee_quotient(float a, float b) { return a / b; }

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

// ---- column pass: one block per column ----------------------------------------------
// For trailing column j of step s the block runs, in order:
//   dot     the reference's 32-lane chain (lane l folds rows s + l, s + l + 32, ...)
//           of v_i t_ij over rows [s, m), v_s = 1, plane-summed, times coeff[s];
//   update  t_ij = fma(-v_i, dot, t_ij) over rows [s, m), last rows first, with the
//           maximum magnitude and the non-finite flag of rows (s, m);
//   norm    (when step s + 1 runs) the reference's scaled sum-of-squares chain of the
//           updated rows [s + 1, m) with that maximum, into norms[j].
// The update re-reads what the dot just streamed and the norm re-reads what the update
// just wrote (last written first), so both mostly hit L2.  Step 0's norms run the norm
// chain after a walk for the maximum (the "first" pass, one block per column).
//
// Roles: warp 0 runs the chains.  Lane 0 of warps 1-3 (the producers) stream segments
// into a ring of kColStages shared-memory stages with bulk copies (cp.async.bulk),
// completing on the stage's `full` mbarrier; ring position p belongs to producer
// p mod 3, which reuses a stage once its consumer has released it on the stage's
// `empty` mbarrier (warp 0 for chain segments, the helper warps 4-11 for update
// segments).  One warp's bulk copies are served one after another (about 55 GB/s of
// 16 KB copies from L2, more for larger ones), so three producers keep three streams going per block.  The
// update's segments (v and t, last first) follow the dot's in the same ring, so their
// copies start while the dot chain finishes; the helpers compute and store them.  For
// the norm, the helpers turn each landed segment into scaled magnitudes in place and
// signal the stage's `ready` mbarrier.  Every wait is bounded: one that runs out stops
// the block and sets bit 1 of the status word.
//
// Stage placement: element e of a segment sits at slot sh + e, where sh * sizeof(F)
// is the operand's address modulo 16 at its first row (segments are multiples of 16
// bytes), so the 16-byte-aligned bytes covering a segment copy to slot 0.  Those
// bytes may include neighbouring rows or columns of the matrix; only where they would
// leave the matrix's span are edge elements loaded one by one instead.
constexpr int kColHelpers = 256;
constexpr int kColProducers = 3;                     // divides kColStages
constexpr int kColHelperWarp0 = 1 + kColProducers;  // first helper warp
constexpr int kColThreads = 32 * kColHelperWarp0 + kColHelpers;
constexpr int kColWarps = kColThreads / 32;
// Three 32 KB stages (96 KB, two blocks per SM).  A bulk copy costs its issuing warp
// about the same time whatever its size, so fewer and larger stages beat a deeper ring
// of small ones.
constexpr int kColStages = 3;
constexpr int kColStageBytes = 32768;
constexpr unsigned kColWaitLimit = 1u << 20;  // try_wait rounds before giving up
constexpr unsigned kColSuspendNs = 1000;

template <typename F>
struct ColSmem {
  static constexpr int kPad = 16 / static_cast<int>(sizeof(F));
  static constexpr int kSeg1 = kColStageBytes / static_cast<int>(sizeof(F));  // norm: elements per segment
  static constexpr int kSeg2 = kSeg1 / 2;                                      // dot: per operand and segment
  static constexpr int kRegion2 = kSeg2 + kPad;                                // dot: slots of one operand
  static constexpr int kStage = kSeg1 + 2 * kPad;
  F raw[kColStages][kStage];
  unsigned long long full[kColStages];
  unsigned long long empty[kColStages];
  unsigned long long ready[kColStages];
  unsigned long long dot_ready;
  F red[kColWarps];
  int bad[kColWarps];
  F dot;
  int abort;
  int last;  // this block drew the column pass's last ticket
};

__device__ __forceinline__ unsigned col_smem(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

// Bounded wait for phase `parity` of an mbarrier; false when the limit ran out.
__device__ __forceinline__ bool col_wait(const unsigned long long* bar, unsigned parity) {
  const unsigned addr = col_smem(bar);
  for (unsigned it = 0; it < kColWaitLimit; ++it) {
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

__device__ __forceinline__ void col_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(col_smem(bar)) : "memory");
}
// `empty` expects one arrival per helper warp: the chain warp arrives for all of them.
__device__ __forceinline__ void col_release_all(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(col_smem(bar)), "n"(kColHelpers / 32) : "memory");
}

// Orders this thread's generic-proxy writes before later bulk copies (async proxy).
__device__ __forceinline__ void col_fence_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void col_fence_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ int ring_stage(long long p) { return static_cast<int>(p % kColStages); }
__device__ __forceinline__ unsigned ring_parity(long long p) { return static_cast<unsigned>((p / kColStages) & 1); }

template <typename F>
__device__ __forceinline__ int slot_shift(const F* p) {
  return static_cast<int>((reinterpret_cast<unsigned long long>(p) & 15) / sizeof(F));
}

// One operand streamed by segments: rows [0, rows) from `base`.
template <typename F>
struct ColStream {
  const F* base;
  long long rows;
  int seg;     // elements per segment
  int sh;      // slot of element 0 (address of base modulo 16, in elements)
  int region;  // first slot of this operand within a stage
  const F* lo;  // the operand's buffer: aligned copies never leave [lo, hi)
  const F* hi;
};

// Producer index of this thread (lane 0 of warps 1 .. kColProducers), or -1.
__device__ __forceinline__ int col_producer() {
  const int warp = threadIdx.x >> 5;
  return (threadIdx.x & 31) == 0 && warp >= 1 && warp <= kColProducers ? warp - 1 : -1;
}
// First ring position >= p0 that producer k owns.
__device__ __forceinline__ long long col_first_position(long long p0, int k) {
  return p0 + ((k - p0 % kColProducers) % kColProducers + kColProducers) % kColProducers;
}

template <typename F>
__device__ __forceinline__ void col_fail(ColSmem<F>& sm, long long* status) {
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  atomicOr(reinterpret_cast<unsigned long long*>(status), 2ull);
}
template <typename F>
__device__ __forceinline__ bool col_aborted(ColSmem<F>& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort) != 0;
}

// Producer: ring position p holds segment g of every operand.  Waits (bounded) until
// warp 0 has released the stage's previous use, then issues the bulk copies.
template <typename F, int Ops>
__device__ __forceinline__ bool col_issue(ColSmem<F>& sm, const ColStream<F>* ops, long long p, long long g) {
  constexpr unsigned long long es = sizeof(F);
  const int st = ring_stage(p);
  if (p >= kColStages && !col_wait(&sm.empty[st], ring_parity(p - kColStages))) return false;
  unsigned long long c0[Ops], c1[Ops], g0[Ops];
  unsigned tx = 0;
  bool edges = false;
#pragma unroll
  for (int o = 0; o < Ops; ++o) {
    const unsigned long long w0 = (reinterpret_cast<unsigned long long>(ops[o].lo) + 15) & ~15ull;
    const unsigned long long w1 = reinterpret_cast<unsigned long long>(ops[o].hi) & ~15ull;
    const long long e0 = g * ops[o].seg;
    const long long e1 = ops[o].rows < e0 + ops[o].seg ? ops[o].rows : e0 + ops[o].seg;
    g0[o] = reinterpret_cast<unsigned long long>(ops[o].base + e0);
    const unsigned long long g1 = reinterpret_cast<unsigned long long>(ops[o].base + e1);
    c0[o] = (g0[o] & ~15ull) > w0 ? (g0[o] & ~15ull) : w0;
    c1[o] = ((g1 + 15) & ~15ull) < w1 ? ((g1 + 15) & ~15ull) : w1;
    if (c1[o] < c0[o]) c1[o] = c0[o];
    // Elements outside [c0, c1): only where the aligned bytes would leave the span.
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
  if (edges) col_fence_shared();
  const unsigned bar = col_smem(&sm.full[st]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
#pragma unroll
  for (int o = 0; o < Ops; ++o) {
    if (c1[o] > c0[o]) {
      const unsigned dst = col_smem(sm.raw[st] + ops[o].region + ops[o].sh) +
                           static_cast<unsigned>(static_cast<long long>(c0[o]) - static_cast<long long>(g0[o]));
      asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                   "l"(c0[o]), "r"(static_cast<unsigned>(c1[o] - c0[o])), "r"(bar)
                   : "memory");
    }
  }
  return true;
}

// Chain folds over one full segment (N elements per lane).  Each load is issued
// kFoldAhead elements before its fma, which covers the shared-memory latency with the
// dependent fma chain (8 cycles per FP64 fma) in a few registers.
constexpr int kFoldAhead = 6;
template <typename F, int N>
__device__ __forceinline__ F fold_dot(const F* bv, const F* bt, int lane, F acc) {
  F xv[kFoldAhead], xt[kFoldAhead];
#pragma unroll
  for (int k = 0; k < kFoldAhead; ++k) {
    xv[k] = bv[lane + 32 * k];
    xt[k] = bt[lane + 32 * k];
  }
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const F v = xv[k % kFoldAhead], t = xt[k % kFoldAhead];
    if (k + kFoldAhead < N) {
      xv[k % kFoldAhead] = bv[lane + 32 * (k + kFoldAhead)];
      xt[k % kFoldAhead] = bt[lane + 32 * (k + kFoldAhead)];
    }
    acc = fused(v, t, acc);
  }
  return acc;
}
template <typename F, int N>
__device__ __forceinline__ F fold_squares(const F* b, int lane, F acc) {
  F x[kFoldAhead];
#pragma unroll
  for (int k = 0; k < kFoldAhead; ++k) x[k] = b[lane + 32 * k];
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const F v = x[k % kFoldAhead];
    if (k + kFoldAhead < N) x[k % kFoldAhead] = b[lane + 32 * (k + kFoldAhead)];
    acc = fused(v, v, acc);
  }
  return acc;
}

// Block-wide maximum and any-flag, broadcast to every thread.
template <typename F>
__device__ __forceinline__ void col_block_max(ColSmem<F>& sm, F local_max, bool invalid, F* scale, bool* bad) {
  const F wm = plane_max(local_max);
  const bool wb = __any_sync(kFull, invalid);
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

template <typename F>
__device__ __forceinline__ void track_max(F value, F* local_max, bool* invalid) {
  const F m = mag(value);
  const bool nf = not_finite(m);
  *invalid = *invalid || nf;
  *local_max = (!nf && m > *local_max) ? m : *local_max;
}

// The norm chain over rows [0, rows) of `base` (ring positions from p0); returns the
// chain warp's lane sums (zero elsewhere).  `issued` counts the producer's positions.
template <typename F>
__device__ __forceinline__ F col_norm_chain(ColSmem<F>& sm, const FusedArgs<F>& a, const F* base, long long rows,
                                            F scale, long long p0, long long* issued) {
  using S = ColSmem<F>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long nseg = (rows + S::kSeg1 - 1) / S::kSeg1;
  ColStream<F> op;
  op.base = base;
  op.rows = rows;
  op.seg = S::kSeg1;
  op.sh = slot_shift(base);
  op.region = 0;
  op.lo = a.w;
  op.hi = a.w + a.span;
  F acc = F(0);
  const int k = col_producer();
  if (k >= 0) {
    for (long long p = col_first_position(p0, k); p < p0 + nseg && !col_aborted(sm); p += kColProducers) {
      if (!col_issue<F, 1>(sm, &op, p, p - p0)) {
        col_fail(sm, a.status);
        break;
      }
      *issued = p + 1;
    }
  } else if (warp >= kColHelperWarp0) {
    // Helpers: scaled magnitudes in place, then the stage's `ready` arrival.  `ready`
    // is used by the norm chain only: its phase for position p counts the earlier
    // norm positions on the same stage.
    const ScaledQuotient<F> quo = make_quotient(scale);
    const int h = tid - 32 * kColHelperWarp0;
    for (long long g = 0; g < nseg; ++g) {
      if (__any_sync(kFull, col_aborted(sm))) break;
      const long long p = p0 + g;
      const int st = ring_stage(p);
      if (!__all_sync(kFull, col_wait(&sm.full[st], ring_parity(p)))) {
        if (lane == 0) col_fail(sm, a.status);
        break;
      }
      const long long e0 = g * S::kSeg1;
      const int len = static_cast<int>(rows - e0 < S::kSeg1 ? rows - e0 : S::kSeg1);
      F* b = sm.raw[st] + op.sh;
      constexpr int kPer = S::kSeg1 / kColHelpers;
      F qv[kPer];
      bool unsafe = false;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int i = h + kColHelpers * q;
        const F x = i < len ? mag(b[i]) : F(0);
        qv[q] = quotient_fast(quo, x);
        unsafe |= !quotient_safe(quo, x);
      }
      if (unsafe) {
        // Operands outside the fast quotient's range: IEEE division for those.
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
          const int i = h + kColHelpers * q;
          const F x = i < len ? mag(b[i]) : F(0);
          if (!quotient_safe(quo, x)) qv[q] = ieee_quotient(x, quo.b);
        }
      }
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int i = h + kColHelpers * q;
        if (i < len) b[i] = qv[q];
      }
      col_fence_shared();
      __syncwarp();
      if (lane == 0) col_arrive(&sm.ready[st]);
    }
  } else if (warp == 0) {
    for (long long g = 0; g < nseg; ++g) {
      if (__any_sync(kFull, col_aborted(sm))) break;
      const long long p = p0 + g;
      const int st = ring_stage(p);
      const long long before = p0 > st ? (p0 - st + kColStages - 1) / kColStages : 0;  // earlier uses, not norm
      const unsigned parity = static_cast<unsigned>((p / kColStages - before) & 1);
      if (!__all_sync(kFull, col_wait(&sm.ready[st], parity))) {
        if (lane == 0) col_fail(sm, a.status);
        break;
      }
      const F* b = sm.raw[st] + op.sh;
      const long long e0 = g * S::kSeg1;
      if (e0 + S::kSeg1 <= rows) {
        acc = fold_squares<F, S::kSeg1 / 32>(b, lane, acc);
      } else {
        const int len = static_cast<int>(rows - e0);
        for (int i = lane; i < len; i += 32) acc = fused(b[i], b[i], acc);
      }
      __syncwarp();
      if (lane == 0) col_release_all(&sm.empty[st]);
    }
  }
  return acc;
}

template <typename F>
__device__ __forceinline__ void col_init(ColSmem<F>& sm) {
  if (threadIdx.x == 0) {
    for (int q = 0; q < kColStages; ++q) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(col_smem(&sm.full[q])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(col_smem(&sm.empty[q])), "n"(kColHelpers / 32)
                   : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(col_smem(&sm.ready[q])), "n"(kColHelpers / 32)
                   : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(col_smem(&sm.dot_ready)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.abort = 0;
  }
  __syncthreads();
}

// Producer k waits (bounded) for the last position it issued on each of its stages, so
// that no bulk copy is in flight when the block exits.
template <typename F>
__device__ __forceinline__ void col_drain(ColSmem<F>& sm, long long issued, int k, long long* status) {
  const long long first = issued > kColStages ? issued - kColStages : 0;
  for (long long p = col_first_position(first, k); p < issued; p += kColProducers)
    if (!col_wait(&sm.full[ring_stage(p)], ring_parity(p)))
      atomicOr(reinterpret_cast<unsigned long long*>(status), 2ull);
}

template <typename F>
__device__ __forceinline__ void col_write_norm(ColSmem<F>& sm, const FusedArgs<F>& a, long long j, F acc, F scale,
                                               bool bad) {
  if ((threadIdx.x >> 5) == 0) {
    const F norm = scale * sqrt(plane_sum(acc));
    if ((threadIdx.x & 31) == 0) a.norms[j] = (bad || not_finite(norm) || col_aborted(sm)) ? F(-1) : norm;
  }
}

// After this block's norm is written (by thread 0): publish it and draw a ticket; the
// block that draws the last one sees every norm of the pass and selects the pivot of
// `pivot_step` with its warp 0, then rearms the counter for the next pass.
template <typename F>
__device__ __forceinline__ void col_pivot_if_last(const FusedArgs<F>& a, long long pivot_step, ColSmem<F>& sm) {
  if (threadIdx.x == 0) {
    __threadfence();
    sm.last = atomicAdd(a.done, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    if (threadIdx.x < 32) fused_pivot(a, pivot_step);
    if (threadIdx.x == 0) *a.done = 0;
  }
}

// First pass: column j = blockIdx.x, its maximum by a walk, then its norm (step 0).
template <typename F>
__device__ __forceinline__ void column_first(const FusedArgs<F>& a, ColSmem<F>& sm) {
  const long long j = blockIdx.x;
  if (j >= a.n) return;
  const F* col = a.w + j * a.ld;
  col_init(sm);
  F local_max = F(0);
  bool invalid = false;
  for (long long row = threadIdx.x; row < a.m; row += kColThreads) track_max(col[row], &local_max, &invalid);
  F scale;
  bool bad;
  col_block_max(sm, local_max, invalid, &scale, &bad);
  long long issued = 0;
  F acc = F(0);
  if (!bad && scale > F(0)) acc = col_norm_chain(sm, a, col, a.m, scale, 0, &issued);
  __syncthreads();
  if (col_producer() >= 0) col_drain(sm, issued, col_producer(), a.status);
  col_write_norm(sm, a, j, acc, scale, bad);
  col_pivot_if_last(a, 0, sm);
}

// The dot and update phases of a column pass: t -= v * (coeff[step] * dot(v, t)) over
// rows [step, m) of the target column `tcol`, the reflector read from `vcol` (its row
// `step` is the implicit 1).  v lies in [vlo, vhi), t in [tlo, thi).  Returns the
// positions this thread issued as a producer (for col_drain); the helpers' maximum of
// the updated rows below `step` goes to local_max / invalid.
template <typename F>
__device__ __forceinline__ long long col_dot_update(const FusedArgs<F>& a, long long step, const F* vcol, F* tcol,
                                                    const F* vlo, const F* vhi, const F* tlo, const F* thi,
                                                    ColSmem<F>& sm, F* local_max_out, bool* invalid_out) {
  using S = ColSmem<F>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long rows = a.m - step;
  long long issued = 0;
  // Ring positions [0, nseg): the dot's segments; [nseg, 2 nseg): the update's, last
  // segment first; then the norm's.
  const long long nseg = (rows + S::kSeg2 - 1) / S::kSeg2;
  ColStream<F> ops[2];
  ops[0].base = vcol + step;
  ops[1].base = tcol + step;
#pragma unroll
  for (int o = 0; o < 2; ++o) {
    ops[o].rows = rows;
    ops[o].seg = S::kSeg2;
    ops[o].sh = slot_shift(ops[o].base);
    ops[o].region = o * S::kRegion2;
  }
  ops[0].lo = vlo;
  ops[0].hi = vhi;
  ops[1].lo = tlo;
  ops[1].hi = thi;
  F local_max = F(0);
  bool invalid = false;
  const int k = col_producer();
  if (k >= 0) {
    for (long long p = k; p < 2 * nseg && !col_aborted(sm); p += kColProducers) {
      const long long g = p < nseg ? p : 2 * nseg - 1 - p;
      if (!col_issue<F, 2>(sm, ops, p, g)) {
        col_fail(sm, a.status);
        break;
      }
      issued = p + 1;
    }
  } else if (warp == 0) {
    F acc = F(0);
    for (long long g = 0; g < nseg; ++g) {
      if (__any_sync(kFull, col_aborted(sm))) break;
      const int st = ring_stage(g);
      if (!__all_sync(kFull, col_wait(&sm.full[st], ring_parity(g)))) {
        if (lane == 0) col_fail(sm, a.status);
        break;
      }
      const F* bv = sm.raw[st] + ops[0].sh;
      const F* bt = sm.raw[st] + S::kRegion2 + ops[1].sh;
      const long long e0 = g * S::kSeg2;
      if (g == 0) {
        // Row `step` of the reflector is an implicit 1.
        const int len = static_cast<int>(rows < S::kSeg2 ? rows : S::kSeg2);
        for (int i = lane; i < len; i += 32) acc = fused(i == 0 ? F(1) : bv[i], bt[i], acc);
      } else if (e0 + S::kSeg2 <= rows) {
        acc = fold_dot<F, S::kSeg2 / 32>(bv, bt, lane, acc);
      } else {
        const int len = static_cast<int>(rows - e0);
        for (int i = lane; i < len; i += 32) acc = fused(bv[i], bt[i], acc);
      }
      __syncwarp();
      if (lane == 0) col_release_all(&sm.empty[st]);
    }
    const F d = plane_sum(acc) * a.coeff[step];
    if (lane == 0) {
      sm.dot = d;
      col_arrive(&sm.dot_ready);
    }
  } else if (warp >= kColHelperWarp0) {
    // update: t = fma(-v, dot, t) from the staged segments, stored straight to memory
    const int h = tid - 32 * kColHelperWarp0;
    const bool ok = __all_sync(kFull, col_wait(&sm.dot_ready, 0));
    if (!ok && lane == 0) col_fail(sm, a.status);
    const F d = sm.dot;
    for (long long k = 0; ok && k < nseg; ++k) {
      if (__any_sync(kFull, col_aborted(sm))) break;
      const long long p = nseg + k, g = nseg - 1 - k;
      const int st = ring_stage(p);
      if (!__all_sync(kFull, col_wait(&sm.full[st], ring_parity(p)))) {
        if (lane == 0) col_fail(sm, a.status);
        break;
      }
      const F* bv = sm.raw[st] + ops[0].sh;
      const F* bt = sm.raw[st] + S::kRegion2 + ops[1].sh;
      const long long e0 = g * S::kSeg2;
      const int len = static_cast<int>(rows - e0 < S::kSeg2 ? rows - e0 : S::kSeg2);
      F* out = tcol + step + e0;
#pragma unroll
      for (int q = 0; q < S::kSeg2 / kColHelpers; ++q) {
        const int i = h + kColHelpers * q;
        if (i < len) {
          const bool lead = e0 + i == 0;
          const F nt = fused(-(lead ? F(1) : bv[i]), d, bt[i]);
          out[i] = nt;
          if (!lead) track_max(nt, &local_max, &invalid);
        }
      }
      __syncwarp();
      if (lane == 0) col_arrive(&sm.empty[st]);
    }
    col_fence_global();
  }
  *local_max_out = local_max;
  *invalid_out = invalid;
  return issued;
}

// Step pass: trailing column j = step + 1 + blockIdx.x.
template <typename F>
__device__ __forceinline__ void column_step(const FusedArgs<F>& a, long long step, bool next_norm, ColSmem<F>& sm) {
  const long long j = step + 1 + blockIdx.x;
  if (j >= a.n) return;
  const int k = col_producer();
  F* tcol = a.w + j * a.ld;
  const long long rows = a.m - step;
  const long long nseg = (rows + ColSmem<F>::kSeg2 - 1) / ColSmem<F>::kSeg2;
  col_init(sm);
  F local_max;
  bool invalid;
  long long issued = col_dot_update(a, step, a.w + step * a.ld, tcol, a.w, a.w + a.span, a.w, a.w + a.span, sm,
                                    &local_max, &invalid);
  F scale;
  bool bad;
  col_block_max(sm, local_max, invalid, &scale, &bad);
  // the next step's norm of rows [step + 1, m)
  F acc = F(0);
  if (next_norm && !col_aborted(sm) && !bad && scale > F(0))
    acc = col_norm_chain(sm, a, tcol + step + 1, rows - 1, scale, 2 * nseg, &issued);
  __syncthreads();
  if (k >= 0) col_drain(sm, issued, k, a.status);
  if (next_norm) {
    col_write_norm(sm, a, j, acc, scale, bad);
    col_pivot_if_last(a, step + 1, sm);
  }
}

// Q formation pass: the dot and update phases of reflector `step` (a column of a.w,
// coefficient a.coeff[step]) applied to column j = blockIdx.x of Q (q, column stride
// qld, q_span elements); the same arithmetic as apply_reflector over Q's columns.
template <typename F>
__device__ __forceinline__ void column_q(const FusedArgs<F>& a, long long step, F* q, long long qld, long long qcols,
                                         long long q_span, ColSmem<F>& sm) {
  const long long j = blockIdx.x;
  if (j >= qcols) return;
  const int k = col_producer();
  col_init(sm);
  F local_max;
  bool invalid;
  const long long issued = col_dot_update(a, step, a.w + step * a.ld, q + j * qld, a.w, a.w + a.span, q, q + q_span,
                                          sm, &local_max, &invalid);
  __syncthreads();
  if (k >= 0) col_drain(sm, issued, k, a.status);
}

}  // namespace rrqr
}  // namespace t4a
