// The row-sharded RRQR step, shared by the two multi-GPU drivers: rrqr_dist.cu (the
// exchanges as NCCL all-gathers) and rrqr_p2p.cu (the exchanges fused into the step
// kernels as stores into every peer's memory over NVLink).  Both run the same
// arithmetic, so they give the same bits.
//
// Rank r holds rows [row0, row0 + mr) of every column, column-major.  Per step s every
// rank combines the norm parts of the trailing columns in rank order, chooses the pivot
// (the reference's rule) and the reflector's scalars, swaps its rows of columns s and
// pivot and scales its rows below s of the new column s (the owner of row s writes
// alpha); then per trailing column the chain of v t over its rows >= s (the reference's
// lane order within the rank's block; v_s = 1 on the owner); then, from the dot parts
// summed in rank order, the update t -= v d of its rows and the next step's norm parts
// of rows >= s + 1: the largest finite modulus, the chain of (|t| / that)^2, a
// non-finite flag, the same pair over every modulus when a value is non-finite (the
// reflector's form), and the value at row s + 1 with an owner flag.  Norm parts combine
// as norm = S sqrt(sum_r w_r ssq_r), S = max_r scale_r, w_r = 1 when scale_r == S and
// (scale_r / S)^2 otherwise, with separately rounded products and sums.  With one rank
// every combination is exact, so a world of one reproduces the single-GPU driver bit for
// bit; with several, norms and dots round differently from the single-GPU order, and
// pivots agree wherever norms are well separated (the rank-revealing prefix).
#pragma once

#include "rrqr_step.cuh"

namespace t4a {
namespace rrqr {

// One rank's norm parts of one column (eight elements, so a vector of them moves as F).
template <typename F>
struct NormPart {
  F scale;   // largest finite modulus of the rank's rows
  F ssq;     // chain of (|x| / scale)^2, butterfly-summed
  F rscale;  // the reflector's form (every modulus competes): equal to scale / ssq for a
  F rssq;    // finite column
  F xrow;    // value at the step's leading row (owner only)
  F bad;     // 1: a non-finite modulus
  F own;     // 1: this rank holds the leading row
  F pad;
};

template <typename F>
struct DistRecord {
  long long pivot;
  F alpha;
  F divisor;
  int scale;  // 0: norm == 0 (no scaling, coefficient 0)
};

template <typename F>
struct DistArgs {
  F* w;              // local rows, column-major
  long long mr;      // local rows
  long long n;       // columns
  long long ld;      // column stride
  long long row0;    // global index of local row 0
  int world;
  long long* perm;   // n (replicated)
  F* coeff;          // one per step (replicated)
  long long* pivots;
  long long* status;
  NormPart<F>* nsend;  // trailing columns' parts of this rank (NCCL driver)
  NormPart<F>* nrecv;  // every rank's parts: [world][stride], see combined_norm
  F* dsend;            // (NCCL driver)
  F* drecv;            // every rank's dot parts
  DistRecord<F>* rec;
};

// First local row at global row >= s, and whether this rank holds global row s.
template <typename F>
__device__ __forceinline__ long long local_from(const DistArgs<F>& a, long long s) {
  const long long lo = s - a.row0;
  return lo < 0 ? 0 : (lo > a.mr ? a.mr : lo);
}
template <typename F>
__device__ __forceinline__ bool holds(const DistArgs<F>& a, long long s) {
  return s >= a.row0 && s < a.row0 + a.mr;
}

// Separately rounded products and sums (no contraction into fma), so that the combine
// is the same arithmetic on every rank and in the CPU restatement.
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// Combined norm of one column from rank r's part at nrecv[r * stride + idx]: the
// column_norms form (-1 for a non-finite column) or the reflector's form.
template <typename F, bool kReflector>
__device__ __forceinline__ F combined_norm(const DistArgs<F>& a, long long stride, long long idx) {
  F scale = F(0);
  bool bad = false;
  for (int r = 0; r < a.world; ++r) {
    const NormPart<F>& p = a.nrecv[r * stride + idx];
    const F sc = kReflector ? p.rscale : p.scale;
    bad = bad || p.bad != F(0);
    scale = sc > scale ? sc : scale;
  }
  if (!kReflector && bad) return F(-1);
  F ssq = F(0);
  for (int r = 0; r < a.world; ++r) {
    const NormPart<F>& p = a.nrecv[r * stride + idx];
    const F sc = kReflector ? p.rscale : p.scale;
    if (sc > F(0)) {
      const F ratio = sc == scale ? F(1) : sc / scale;
      ssq = add_rn(ssq, mul_rn(mul_rn(ratio, ratio), kReflector ? p.rssq : p.ssq));
    }
  }
  const F norm = mul_rn(scale, sqrt(ssq));
  return !kReflector && nonfinite(norm) ? F(-1) : norm;
}

template <typename F>
__device__ __forceinline__ F leading_value(const DistArgs<F>& a, long long stride, long long idx) {
  F x = F(0);
  for (int r = 0; r < a.world; ++r) {
    const NormPart<F>& p = a.nrecv[r * stride + idx];
    if (p.own != F(0)) x = p.xrow;
  }
  return x;
}

// The dot of one column: rank r's part at drecv[r * stride + idx], summed in rank order
// from rank 0's part (so one rank's part passes unchanged), times the coefficient.
template <typename F>
__device__ __forceinline__ F combined_dot(const DistArgs<F>& a, long long stride, long long idx, F coeff) {
  F d = a.drecv[idx];
  for (int r = 1; r < a.world; ++r) d = add_rn(d, a.drecv[r * stride + idx]);
  return mul_rn(d, coeff);
}

// The norm parts of column `col` over this rank's rows [lo, mr) (global rows >= s),
// handed to emit(part) by thread 0.  have_peak: the largest modulus and flag of those
// rows are already known (from the update).
template <typename F, typename Emit>
__device__ __forceinline__ void norm_parts(const DistArgs<F>& a, ColSmem<F>& sm, const F* col, long long lo, long long s,
                                           F peak, bool flagged, bool have_peak, Emit emit) {
  const long long rows = a.mr - lo;
  F scale;
  bool bad;
  if (!have_peak) {
    peak = F(0);
    flagged = false;
    if (rows > 0) peak_direct<true>(col + lo, rows, &peak, &flagged);
  }
  block_peak(sm, peak, flagged, &scale, &bad);
  F ssq = F(0);
  if (!bad && scale > F(0) && rows > 0) ssq = scaled_norm(sm, col + lo, rows, scale, a.status);
  F rscale = scale, rssq = ssq;
  if (bad && threadIdx.x < 32) {
    const ScaledSum<F> r = chain_parts<false, 1>(Strip<const F>{col + lo, 1}, 0, rows, nullptr);
    rscale = r.scale;
    rssq = r.ssq;
  }
  if (threadIdx.x == 0) {
    NormPart<F> p;
    p.scale = scale;
    p.ssq = ssq;
    p.rscale = rscale;
    p.rssq = rssq;
    p.own = holds(a, s) ? F(1) : F(0);
    p.xrow = holds(a, s) ? col[s - a.row0] : F(0);
    p.bad = bad ? F(1) : F(0);
    p.pad = F(0);
    emit(p);
  }
}

// One warp: the pivot of step s and the reflector's scalars from the combined norms of
// columns s .. n-1 (norm_of(c): the column_norms form of column c's combined norm; rank
// r's part of column c at nrecv[r * stride + c - first]); with `writer`, lane 0 records
// the step (record, pivot, coefficient, flag).  Returns the record (the caller shares it
// through shared memory).
// kBatch: choose_pivot's batch (1 when norm_of combines the ranks' parts itself).
template <typename F, int kBatch = 8, typename NormOf>
__device__ __forceinline__ DistRecord<F> shard_pivot(const DistArgs<F>& a, long long s, long long stride,
                                                     long long first, bool writer, NormOf norm_of) {
  bool flagged = false;
  const long long pivot =
      choose_pivot<F, kBatch>(s, a.n, norm_of, [&](long long c) { return a.perm[c]; }, &flagged);
  F norm = norm_of(pivot);
  if (!(norm >= F(0))) norm = combined_norm<F, true>(a, stride, pivot - first);
  const F x0 = leading_value(a, stride, pivot - first);
  DistRecord<F> r;
  r.pivot = pivot;
  F c = F(0);
  if (norm == F(0)) {
    r.scale = 0;
    r.alpha = F(0);
    r.divisor = F(1);
  } else {
    const Householder<F> h = householder(x0, norm);
    r.scale = 1;
    r.alpha = h.alpha;
    r.divisor = h.divisor;
    c = h.coeff;
  }
  if (writer && lane_id() == 0) {
    *a.rec = r;
    a.pivots[s] = pivot;
    a.coeff[s] = c;
    if (flagged) *a.status |= 1;
  }
  return r;
}

// This rank's rows of the swap of columns s and r.pivot, with the reflector's scaling
// of the new column s (grid-stride over the local rows).
template <typename F>
__device__ __forceinline__ void shard_swap(const DistArgs<F>& a, long long s, const DistRecord<F>& r) {
  F* cs = a.w + s * a.ld;
  F* cp = a.w + r.pivot * a.ld;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.mr;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long g = a.row0 + i;
    const F left = cs[i];
    F moved = r.pivot == s ? left : cp[i];
    if (r.scale) {
      if (g == s) {
        moved = r.alpha;
      } else if (g > s) {
        moved = moved / r.divisor;
      }
    }
    cs[i] = moved;
    if (r.pivot != s) cp[i] = left;
  }
}

// The permutation's swap of step s (one thread).
template <typename F>
__device__ __forceinline__ void shard_perm_swap(const DistArgs<F>& a, long long s, long long pivot) {
  if (pivot != s) {
    const long long x = a.perm[s];
    a.perm[s] = a.perm[pivot];
    a.perm[pivot] = x;
  }
}

}  // namespace rrqr
}  // namespace t4a
