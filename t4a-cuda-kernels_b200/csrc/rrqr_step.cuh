// Fused RRQR steps, Q formation and the column-engine forms of the primitives (F32/F64
// columns with unit row stride), built on the column engine (rrqr_engine.cuh).
//
// One step of the reference loop -- column_norms, select_pivot, swap_columns,
// reflector, apply_reflector over the trailing columns (reference bench
// examples/bench_kernels.rs:2390-2623) -- runs in two launches with the same arithmetic:
//  pivot   one warp of the previous column pass's last block (every block publishes
//          its norm and draws a ticket; the block that draws the last one sees them
//          all): the reference's pivot choice, and the reflector's scalars from the
//          pivot column's norm, which equals the reflector's own norm whenever the
//          column is finite (the same walk and the same operations); otherwise the
//          reflector's walk runs again;
//  swap    flat over rows: column swap, permutation swap, the reflector's scaling of
//          the new column `step` and its alpha, in one pass;
//  column  one block per trailing column: ring_dot, update_direct (with the maximum of
//          the updated rows), then the next step's scaled_norm of the updated column.
// Step 0's norms are a block per column: peak_direct, then scaled_norm.
//
// Q formation (column_q) applies reflector `step` of the factorized matrix to one
// column of Q per block with ring_dot and update_direct -- apply_reflector's arithmetic.
#pragma once

#include "rrqr_engine.cuh"

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
  long long* status;  // bit 0: a non-finite norm (sticky); bit 1: a bounded wait ran out
  F* norms;           // n
  StepRecord<F>* rec;
  unsigned* done;     // blocks of the running column pass that have written their norm
};

// Pivot pass: one warp (lane 0 writes).
template <typename F>
__device__ __forceinline__ void fused_pivot(const FusedArgs<F>& a, long long step) {
  bool flagged = false;
  const long long pivot = choose_pivot<F>(
      step, a.n, [&](long long c) { return a.norms[c]; }, [&](long long c) { return a.perm[c]; }, &flagged);
  F norm = a.norms[pivot];
  if (!(norm >= F(0))) {
    // A non-finite column: the reflector's own walk, in which every modulus competes.
    norm = chain_norm<false, 1>(Strip<const F>{a.w + pivot * a.ld, 1}, step, a.m, nullptr);
  }
  const F x0 = a.w[pivot * a.ld + step];
  if (lane_id() == 0) {
    a.pivots[step] = pivot;
    if (flagged) *a.status |= 1;
    StepRecord<F> r;
    r.pivot = pivot;
    if (norm == F(0)) {
      r.scale = 0;
      r.alpha = F(0);
      r.denominator = F(1);
      a.coeff[step] = F(0);
    } else {
      const Householder<F> h = householder(x0, norm);
      r.scale = 1;
      r.alpha = h.alpha;
      r.denominator = h.divisor;
      a.coeff[step] = h.coeff;
    }
    *a.rec = r;
  }
}

// Swap pass, row `row` of [0, m).
template <typename F>
__device__ __forceinline__ void fused_swap(const FusedArgs<F>& a, long long step, long long row) {
  const StepRecord<F> r = *a.rec;
  F* cs = a.w + step * a.ld;
  F* cp = a.w + r.pivot * a.ld;
  const F left = cs[row];
  F moved = r.pivot == step ? left : cp[row];  // the value that lands in column `step`
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

// After this block's norm is written (by thread 0): publish it and draw a ticket; the
// block that draws the last one sees every norm of the pass and selects the pivot of
// `pivot_step` with its warp 0, then rearms the counter for the next pass.
// `tickets`: the blocks of the pass that draw one (every block; a clustered pass: the
// leaders).
template <typename F>
__device__ __forceinline__ void pivot_if_last(const FusedArgs<F>& a, long long pivot_step, ColSmem<F>& sm,
                                              unsigned tickets) {
  if (threadIdx.x == 0) {
    __threadfence();
    sm.last = atomicAdd(a.done, 1u) == tickets - 1 ? 1 : 0;
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    if (threadIdx.x < 32) fused_pivot(a, pivot_step);
    if (threadIdx.x == 0) *a.done = 0;
  }
}

// The column_norms result of rows [0, rows) of x (scale from peak_direct<true>): the
// norm, or -1 when a modulus or the norm is not finite or the block stopped.
template <typename F>
__device__ __forceinline__ F engine_column_norm(ColSmem<F>& sm, const F* x, long long rows, long long* status) {
  F peak = F(0);
  bool flagged = false;
  peak_direct<true>(x, rows, &peak, &flagged);
  F scale;
  bool bad;
  block_peak(sm, peak, flagged, &scale, &bad);
  F total = F(0);
  if (!bad && scale > F(0)) total = scaled_norm(sm, x, rows, scale, status);
  const F norm = scale * sqrt(total);
  return (bad || nonfinite(norm) || aborted(sm)) ? F(-1) : norm;
}

// First pass: column j = blockIdx.x, its norm over all rows (step 0), then the ticket.
template <typename F>
__device__ __forceinline__ void column_first(const FusedArgs<F>& a, ColSmem<F>& sm) {
  const long long j = blockIdx.x;
  if (j >= a.n) return;
  engine_init(sm);
  const F norm = engine_column_norm(sm, a.w + j * a.ld, a.m, a.status);
  if (threadIdx.x == 0) a.norms[j] = norm;
  pivot_if_last(a, 0, sm, gridDim.x);
}

// Step pass: trailing column j = step + 1 + blockIdx.x.
template <typename F>
__device__ __forceinline__ void column_step(const FusedArgs<F>& a, long long step, bool next_norm, ColSmem<F>& sm) {
  const long long j = step + 1 + blockIdx.x;
  if (j >= a.n) return;
  engine_init(sm);
  Producer pr = producer_start();
  const F* v = a.w + step * a.ld + step;
  F* t = a.w + j * a.ld + step;
  const long long rows = a.m - step;
  const F d = ring_dot(sm, pr, 0, v, t, rows, a.coeff[step], a.status);
  F peak = F(0);
  bool flagged = false;
  if (!aborted(sm)) update_direct<true>(v, t, rows, d, &peak, &flagged);
  F scale;
  bool bad;
  block_peak(sm, peak, flagged, &scale, &bad);
  // the next step's norm of rows [step + 1, m)
  F total = F(0);
  if (next_norm && !aborted(sm) && !bad && scale > F(0))
    total = scaled_norm(sm, t + 1, rows - 1, scale, a.status);
  drain(sm, pr, a.status);
  if (next_norm) {
    const F norm = scale * sqrt(total);
    if (threadIdx.x == 0) a.norms[j] = (bad || nonfinite(norm) || aborted(sm)) ? F(-1) : norm;
    pivot_if_last(a, step + 1, sm, gridDim.x);
  }
}

// Clustered step pass, for steps with few trailing columns: a cluster of `csize` blocks
// per trailing column j = step + 1 + blockIdx.x / csize.  The leader (rank 0) runs the
// dot chain as column_step does; after a cluster barrier every block reads the
// coefficient from the leader's shared memory and updates its own slice of the rows
// (slices of a multiple of 32 rows, so every slice starts at the same 16-byte phase),
// then writes its block peak and flag into the leader's shared memory; after a second
// barrier the leader takes their maximum and runs the norm and the ticket as
// column_step does.  The update is elementwise and the maximum exact, so the bits are
// column_step's.  The leader's norm reads the column from L2: other blocks wrote rows
// of cache lines that its own update may have brought into its L1.
template <typename F>
__device__ __forceinline__ void column_step_cluster(const FusedArgs<F>& a, long long step, bool next_norm,
                                                    ColSmem<F>& sm, unsigned csize) {
  const long long j = step + 1 + blockIdx.x / csize;
  if (j >= a.n) return;  // the same for every block of the cluster
  const unsigned rank = cluster_rank();
  engine_init(sm);
  Producer pr = producer_start();
  const F* v = a.w + step * a.ld + step;
  F* t = a.w + j * a.ld + step;
  const long long rows = a.m - step;
  if (rank == 0) ring_dot(sm, pr, 0, v, t, rows, a.coeff[step], a.status);
  cluster_barrier();
  const F d = cluster_load(&sm.dot, 0);
  const bool stopped = cluster_load(&sm.abort, 0) != 0;
  const long long slice = ((rows + csize - 1) / csize + 31) / 32 * 32;
  const long long lo = static_cast<long long>(rank) * slice < rows ? static_cast<long long>(rank) * slice : rows;
  const long long hi = lo + slice < rows ? lo + slice : rows;
  F peak = F(0);
  bool flagged = false;
  if (!stopped && hi > lo) update_direct<true>(v + lo, t + lo, hi - lo, d, &peak, &flagged, rank == 0);
  F scale;
  bool bad;
  block_peak(sm, peak, flagged, &scale, &bad);
  if (threadIdx.x == 0) {
    cluster_store(&sm.cpeak[rank], 0, scale);
    cluster_store(&sm.cbad[rank], 0, bad ? 1 : 0);
  }
  cluster_barrier();
  if (rank != 0) return;
  scale = F(0);
  bad = false;
  for (unsigned q = 0; q < csize; ++q) {
    scale = sm.cpeak[q] > scale ? sm.cpeak[q] : scale;
    bad = bad || sm.cbad[q] != 0;
  }
  F total = F(0);
  if (next_norm && !aborted(sm) && !bad && scale > F(0))
    total = scaled_norm<F, true>(sm, t + 1, rows - 1, scale, a.status);
  drain(sm, pr, a.status);
  if (next_norm) {
    const F norm = scale * sqrt(total);
    if (threadIdx.x == 0) a.norms[j] = (bad || nonfinite(norm) || aborted(sm)) ? F(-1) : norm;
    pivot_if_last(a, step + 1, sm, gridDim.x / csize);
  }
}

// Q formation pass: reflector `step` (column `step` of w, coefficient coeff[step])
// applied to column j = blockIdx.x of Q (column stride qld).
template <typename F>
__device__ __forceinline__ void column_q(const FusedArgs<F>& a, long long step, F* q, long long qld, long long qcols,
                                         ColSmem<F>& sm) {
  const long long j = blockIdx.x;
  if (j >= qcols) return;
  engine_init(sm);
  Producer pr = producer_start();
  const F* v = a.w + step * a.ld + step;
  F* t = q + j * qld + step;
  const long long rows = a.m - step;
  const F d = ring_dot(sm, pr, 0, v, t, rows, a.coeff[step], a.status);
  if (!aborted(sm)) update_direct<false>(v, t, rows, d, static_cast<F*>(nullptr), static_cast<bool*>(nullptr));
  drain(sm, pr, a.status);
}

// ---- the primitives on the column engine (one block per task) -----------------------

// column_norms of one column: rows [step, rows) of x (x at row 0, unit stride).
template <typename F>
__device__ __forceinline__ void engine_norms_task(const F* x, long long step, long long rows, F* out,
                                                  long long* status, ColSmem<F>& sm) {
  engine_init(sm);
  const F norm = engine_column_norm(sm, x + step, rows - step, status);
  if (threadIdx.x == 0) *out = norm;
}

// reflector of one column: x at row 0, unit stride; rows [step, rows).  A block that
// stops leaves the column and the coefficient untouched.
template <typename F>
__device__ __forceinline__ void engine_reflect_task(F* x, long long step, long long rows, F* coeff, long long* status,
                                                    ColSmem<F>& sm) {
  engine_init(sm);
  F* col = x + step;
  const long long n = rows - step;
  F peak = F(0);
  bool flagged = false;
  peak_direct<false>(col, n, &peak, &flagged);
  F scale;
  bool bad;
  block_peak(sm, peak, flagged, &scale, &bad);
  F total = F(0);
  if (scale > F(0)) total = scaled_norm(sm, col, n, scale, status);
  const F norm = scale * sqrt(total);
  const F x0 = col[0];
  __syncthreads();  // x0 is read by every thread before row `step` is written
  if (aborted(sm)) return;
  if (norm == F(0)) {
    if (threadIdx.x == 0) *coeff = F(0);
    return;
  }
  const Householder<F> h = householder(x0, norm);
  divide_direct(col + 1, n - 1, h.divisor);
  if (threadIdx.x == 0) {
    col[0] = h.alpha;
    *coeff = h.coeff;
  }
}

// apply_reflector onto one target column: v and t at row `step`, rows - step rows.
template <typename F>
__device__ __forceinline__ void engine_apply_task(const F* v, F* t, long long n, F coeff, long long* status,
                                                  ColSmem<F>& sm) {
  engine_init(sm);
  Producer pr = producer_start();
  const F d = ring_dot(sm, pr, 0, v, t, n, coeff, status);
  if (!aborted(sm)) update_direct<false>(v, t, n, d, static_cast<F*>(nullptr), static_cast<bool*>(nullptr));
  drain(sm, pr, status);
}

}  // namespace rrqr
}  // namespace t4a
