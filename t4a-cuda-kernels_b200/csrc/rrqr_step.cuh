// Fused RRQR step kernels (F32/F64, one column-major matrix: row stride 1).
//
// One step of the reference loop -- column_norms, select_pivot, swap_columns,
// reflector, apply_reflector over the trailing columns (reference bench
// examples/bench_kernels.rs:2390-2623) -- in four passes with the same arithmetic:
//
//  pivot   one warp: the reference's pivot choice from the norms; the reflector's
//          scalars (x0, alpha, denominator, coefficient) from the pivot column's norm,
//          which equals the reflector's own norm whenever the column is finite (the
//          same walk and the same operations); otherwise the norm is walked again.
//  swap    flat over rows: column swap, permutation swap, the reflector's scaling of
//          the new column `step` and its alpha, in one pass.
//  dot     one warp per trailing column: the reference's 32-lane dot chain times the
//          coefficient, into `dots`.
//  update  flat over trailing elements: t -= v * dot (the reference's fma), and for
//          rows > step the next step's column maximum and non-finite flag (a maximum
//          is exact in any order), so the next step's norms need one walk only.
//  norms   one warp per column: the reference's scaled sum-of-squares chain with the
//          maximum from `update` (step 0 walks for the maximum as well).
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
  F* dots;            // n
  unsigned long long* colmax;  // n: bits of the next step's column maximum
  int* colbad;                 // n: next step's non-finite flag
  StepRecord<F>* rec;
};

// Maximum as ordered bits: positive finite doubles/floats order like their bits.
__device__ __forceinline__ unsigned long long max_bits(double v) { return __double_as_longlong(v); }
__device__ __forceinline__ unsigned long long max_bits(float v) { return __float_as_uint(v); }
template <typename F>
__device__ __forceinline__ F from_bits(unsigned long long b) {
  if constexpr (sizeof(F) == 8) {
    return __longlong_as_double(static_cast<long long>(b));
  } else {
    return __uint_as_float(static_cast<unsigned>(b));
  }
}

// norms pass: columns [step, n), one warp each.  `walk_max`: step 0 (no update pass
// has produced the maximum yet).
template <typename F>
__device__ __forceinline__ void fused_norms(const FusedArgs<F>& a, long long step, bool walk_max) {
  const long long j = step + warp_task();
  if (j >= a.n) return;
  const int lane = threadIdx.x & 31;
  const F* col = a.w + j * a.ld;
  F scale;
  bool bad;
  if (walk_max) {
    F local_max = F(0);
    bool invalid = false;
#pragma unroll 8
    for (long long row = step + lane; row < a.m; row += kPlane) {
      const F value = mag(col[row]);
      if (not_finite(value)) {
        invalid = true;
      } else if (value > local_max) {
        local_max = value;
      }
    }
    scale = plane_max(local_max);
    bad = __any_sync(kFull, invalid);
  } else {
    scale = from_bits<F>(a.colmax[j]);
    bad = a.colbad[j] != 0;
  }
  F local_sum = F(0);
  if (!bad && scale > F(0)) {
#pragma unroll 8
    for (long long row = step + lane; row < a.m; row += kPlane) {
      const F scaled = mag(col[row]) / scale;
      local_sum = fused(scaled, scaled, local_sum);
    }
  }
  const F norm = scale * sqrt(plane_sum(local_sum));
  if (lane == 0) a.norms[j] = (bad || not_finite(norm)) ? F(-1) : norm;
}

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
    norm = column_norm<F, F, false>(a.w, pivot * a.ld, 1, step, a.m, lane, nullptr);
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

// dot pass: trailing columns (step, n), one warp each.
template <typename F>
__device__ __forceinline__ void fused_dot(const FusedArgs<F>& a, long long step) {
  const long long j = step + 1 + warp_task();
  if (j >= a.n) return;
  const int lane = threadIdx.x & 31;
  const F* v = a.w + step * a.ld;
  const F* t = a.w + j * a.ld;
  F dot = F(0);
#pragma unroll 8
  for (long long row = step + lane; row < a.m; row += kPlane) {
    const F vv = row == step ? F(1) : v[row];
    dot = fused(vv, t[row], dot);
  }
  dot = plane_sum(dot) * a.coeff[step];
  if (lane == 0) {
    a.dots[j] = dot;
    a.colmax[j] = 0;
    a.colbad[j] = 0;
  }
}

// update pass: block (row tile, column j), kUpdateRows rows of column j per block.
constexpr int kUpdateThreads = 256;
constexpr int kUpdatePerThread = 8;
constexpr int kUpdateRows = kUpdateThreads * kUpdatePerThread;

template <typename F>
__device__ __forceinline__ void fused_update(const FusedArgs<F>& a, long long step, long long j, long long tile) {
  __shared__ unsigned long long wmax[kUpdateThreads / 32];
  __shared__ int wbad[kUpdateThreads / 32];
  const F* v = a.w + step * a.ld;
  F* t = a.w + j * a.ld;
  const F d = a.dots[j];
  const long long r0 = step + tile * kUpdateRows + threadIdx.x;
  F local_max = F(0);
  bool invalid = false;
#pragma unroll
  for (int q = 0; q < kUpdatePerThread; ++q) {
    const long long row = r0 + static_cast<long long>(q) * kUpdateThreads;
    if (row < a.m) {
      const F vv = row == step ? F(1) : v[row];
      const F nt = fused(-vv, d, t[row]);
      t[row] = nt;
      if (row > step) {
        const F value = mag(nt);
        if (not_finite(value)) {
          invalid = true;
        } else if (value > local_max) {
          local_max = value;
        }
      }
    }
  }
  const F m = plane_max(local_max);
  const bool bad = __any_sync(kFull, invalid);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    wmax[warp] = m > F(0) ? max_bits(m) : 0ull;
    wbad[warp] = bad ? 1 : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long bm = 0;
    int bb = 0;
    for (int q = 0; q < kUpdateThreads / 32; ++q) {
      bm = wmax[q] > bm ? wmax[q] : bm;
      bb |= wbad[q];
    }
    if (bm != 0) atomicMax(&a.colmax[j], bm);
    if (bb) atomicOr(&a.colbad[j], 1);
  }
}

}  // namespace rrqr
}  // namespace t4a
