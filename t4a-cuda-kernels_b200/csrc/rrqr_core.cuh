// Rank-revealing QR: the general device bodies of the primitives (any layout, every
// dtype of the ABI), sm_100a.
//
// Numerical contract.  The reference's RRQR kernels (cuda/src/rrqr.cu) reduce every
// column over 32 lanes: lane l visits rows first + l + 32 k for k = 0, 1, ... in order,
// and the 32 lane results meet in an xor butterfly over distances 1, 2, 4, 8, 16.  Pivot
// indices are only reproducible when every norm, dot and update rounds exactly as there,
// so the bodies below keep that visiting order and the operations of each visit (the
// reference's contracted multiply-adds spelled as fma).  Everything else is this
// library's: one warp per task, loads issued in batches ahead of the fold, the pivot as a
// lexicographic best-of reduction, and layout decoding shared with the general-rank
// (`_any`) layouts through templates.
//
//   column_norms    (reference rrqr.cu:144-190)  scaled 2-norm, -1 for a non-finite column
//   select_pivot    (:197-239)  largest norm; ties: smaller original column, then column
//   swap_columns    (:244-284)  exchange of column step and the pivot, and of their perm
//   reflector       (:290-380)  Householder vector and coefficient of column step
//   apply_reflector (:386-448)  t -= v (coeff <v, t>) for one target column
//   extract_r       (:452-470)  upper triangle
//   prefix_rank     (:476-509)  first diagonal entry below max(atol, rtol |r00|)
//   identity_shifted (reference linalg_aux.cu:200-211)
#pragma once

#include "common.cuh"

namespace t4a {
namespace rrqr {

constexpr int kLanes = 32;
constexpr unsigned kAllLanes = 0xffffffffu;
constexpr long long kNoIndex = 0x7fffffffffffffffll;

// ---- element traits ---------------------------------------------------------------

template <typename T> struct Scalar {
  using Real = T;
  static constexpr bool kComplex = false;
};
template <> struct Scalar<c32> {
  using Real = float;
  static constexpr bool kComplex = true;
};
template <> struct Scalar<c64> {
  using Real = double;
  static constexpr bool kComplex = true;
};
template <typename T> using RealOf = typename Scalar<T>::Real;

// |v| as the reference forms it: a real value by its sign test (so -0 stays -0), a
// complex one by hypot.
__device__ __forceinline__ float modulus(float v) { return v < 0.0f ? -v : v; }
__device__ __forceinline__ double modulus(double v) { return v < 0.0 ? -v : v; }
__device__ __forceinline__ float modulus(c32 v) { return hypotf(v.re, v.im); }
__device__ __forceinline__ double modulus(c64 v) { return hypot(v.re, v.im); }

template <typename R>
__device__ __forceinline__ bool nonfinite(R v) {
  return v - v != R(0);
}

__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename T> __device__ __forceinline__ T zero_of() { return T(0); }
template <> __device__ __forceinline__ c32 zero_of<c32>() { return c32{0.0f, 0.0f}; }
template <> __device__ __forceinline__ c64 zero_of<c64>() { return c64{0.0, 0.0}; }
template <typename T> __device__ __forceinline__ T one_of() { return T(1); }
template <> __device__ __forceinline__ c32 one_of<c32>() { return c32{1.0f, 0.0f}; }
template <> __device__ __forceinline__ c64 one_of<c64>() { return c64{1.0, 0.0}; }

// ---- warp butterflies (xor distances 1, 2, 4, 8, 16) -----------------------------------

struct AddOp {
  template <typename V> __device__ __forceinline__ V operator()(V mine, V other) const { return mine + other; }
};
// The partner's value wins only when strictly larger (a NaN never replaces a value).
struct MaxOp {
  template <typename V> __device__ __forceinline__ V operator()(V mine, V other) const {
    return other > mine ? other : mine;
  }
};
struct MinOp {
  template <typename V> __device__ __forceinline__ V operator()(V mine, V other) const {
    return other < mine ? other : mine;
  }
};

template <typename V, typename Op>
__device__ __forceinline__ V butterfly(V v, Op op) {
#pragma unroll
  for (int d = 1; d < kLanes; d <<= 1) v = op(v, __shfl_xor_sync(kAllLanes, v, d));
  return v;
}

__device__ __forceinline__ int lane_id() { return static_cast<int>(threadIdx.x & 31); }

// ---- layouts ----------------------------------------------------------------------

// Offset of batch `b` over the axes first .. rank-1 of a layout (axis `first` fastest).
// L is t4a_cuda_layout or the general-rank t4a_cuda_layout_any (arrays in device
// memory); both expose rank / extents / strides / offset.
template <typename L>
__device__ __forceinline__ long long batch_base(const L& l, int first, long long b) {
  long long off = 0;
  for (int ax = first; ax < l.rank; ++ax) {
    const long long e = l.extents[ax];
    const long long q = b / e;
    off += (b - q * e) * l.strides[ax];
    b = q;
  }
  return off;
}

template <typename L>
__device__ __forceinline__ long long batches_from(const L& l, int first) {
  long long n = 1;
  for (int ax = first; ax < l.rank; ++ax) n *= l.extents[ax];
  return n;
}

// Warp-task index: the warps of the grid numbered block-major.
__device__ __forceinline__ long long warp_task() {
  return static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
}

// ---- the lane chain ----------------------------------------------------------------

// One strided column: element r is p[r * stride].
template <typename T>
struct Strip {
  T* p;
  long long stride;
};

// Lane `lane` visits rows first + lane + 32 k (k ascending) below `rows`, loading
// kDepth of them before handing each to `visit(value, row)` in order.  Only the loads
// run ahead; the fold that `visit` performs keeps the reference's order.
template <int kDepth, typename T, typename Visit>
__device__ __forceinline__ void lane_chain(Strip<const T> s, long long first, long long rows, int lane, Visit visit) {
  for (long long r0 = first + lane; r0 < rows; r0 += static_cast<long long>(kDepth) * kLanes) {
    T held[kDepth];
#pragma unroll
    for (int b = 0; b < kDepth; ++b) {
      const long long r = r0 + static_cast<long long>(b) * kLanes;
      if (r < rows) held[b] = s.p[r * s.stride];
    }
#pragma unroll
    for (int b = 0; b < kDepth; ++b) {
      const long long r = r0 + static_cast<long long>(b) * kLanes;
      if (r < rows) visit(held[b], r);
    }
  }
}

// Rows held per lane ahead of the fold: 16 for real values, 8 for complex ones (16-byte
// elements would otherwise hold 64 registers per lane).
template <typename T> struct ChainDepth { static constexpr int value = Scalar<T>::kComplex ? 8 : 16; };

// The two halves of a max-scaled norm before they meet: the scale and the butterfly sum
// of the chain of (|x| / scale)^2 (the norm is scale * sqrt(ssq)).
template <typename R>
struct ScaledSum {
  R scale;
  R ssq;
};

// The reference's max-scaled 2-norm of rows [first, rows): scale = the largest finite
// modulus, then scale * sqrt(sum over the chain of (|x| / scale)^2).  With kFlag, a
// non-finite modulus is excluded from the scale and reported in *flagged (any lane);
// without it every modulus competes for the scale, as in the reflector.  chain_parts
// returns the scale and the summed chain, chain_norm the norm.
template <bool kFlag, int kDepth, typename T>
__device__ __forceinline__ ScaledSum<RealOf<T>> chain_parts(Strip<const T> s, long long first, long long rows,
                                                           bool* flagged) {
  using R = RealOf<T>;
  const int lane = lane_id();
  R peak = R(0);
  bool seen = false;
  lane_chain<kDepth>(s, first, rows, lane, [&](const T& x, long long) {
    const R m = modulus(x);
    if (kFlag && nonfinite(m)) {
      seen = true;
    } else if (m > peak) {
      peak = m;
    }
  });
  const R scale = butterfly(peak, MaxOp());
  R ssq = R(0);
  if (scale > R(0)) {
    lane_chain<kDepth>(s, first, rows, lane, [&](const T& x, long long) {
      const R q = modulus(x) / scale;
      ssq = fma_rn(q, q, ssq);
    });
  }
  if (kFlag) *flagged = __any_sync(kAllLanes, seen);
  return ScaledSum<R>{scale, butterfly(ssq, AddOp())};
}

template <bool kFlag, int kDepth, typename T>
__device__ __forceinline__ RealOf<T> chain_norm(Strip<const T> s, long long first, long long rows, bool* flagged) {
  const ScaledSum<RealOf<T>> p = chain_parts<kFlag, kDepth>(s, first, rows, flagged);
  return p.scale * sqrt(p.ssq);
}

// ---- column_norms ------------------------------------------------------------------

// Task = (batch, column >= step), batch-major over the trailing columns.  Writes the
// column's norm, or -1 when a modulus or the norm itself is not finite.
template <typename T, typename L>
__device__ __forceinline__ void norms_task(const T* w, RealOf<T>* norms, const L& wl, const L& nl, long long step,
                                           long long task) {
  using R = RealOf<T>;
  const long long width = wl.extents[1] - step;
  const long long b = task / width;
  const long long col = step + (task - b * width);
  Strip<const T> s{w + wl.offset + col * wl.strides[1] + batch_base(wl, 2, b), wl.strides[0]};
  bool flagged = false;
  const R norm = chain_norm<true, ChainDepth<T>::value>(s, step, wl.extents[0], &flagged);
  if (lane_id() == 0)
    norms[nl.offset + col * nl.strides[0] + batch_base(nl, 1, b)] = (flagged || nonfinite(norm)) ? R(-1) : norm;
}

// ---- select_pivot ------------------------------------------------------------------

// A pivot candidate and the reference's order on them: the larger norm wins; equal
// norms go to the smaller original column, then to the smaller column index.  A lane's
// scan in ascending column order followed by this butterfly picks the same column as
// the reference's three successive plane reductions (maximum norm, then minimum
// original among its holders, then minimum column among those), since the order is
// total.
template <typename R>
struct Candidate {
  R norm;
  long long original;
  long long column;
};

template <typename R>
__device__ __forceinline__ bool outranks(const Candidate<R>& a, const Candidate<R>& b) {
  if (a.norm != b.norm) return a.norm > b.norm;
  if (a.original != b.original) return a.original < b.original;
  return a.column < b.column;
}

template <typename R>
__device__ __forceinline__ Candidate<R> best_over_warp(Candidate<R> c) {
#pragma unroll
  for (int d = 1; d < kLanes; d <<= 1) {
    Candidate<R> o;
    o.norm = __shfl_xor_sync(kAllLanes, c.norm, d);
    o.original = __shfl_xor_sync(kAllLanes, c.original, d);
    o.column = __shfl_xor_sync(kAllLanes, c.column, d);
    if (outranks(o, c)) c = o;
  }
  return c;
}

// The pivot among `columns` candidates from `step` on: norm(c) and original(c) give a
// column's norm and original index.  Negative norms (the non-finite sentinel) are not
// candidates and set *flagged; NaN norms are skipped.  The empty candidate holds norm 0,
// so a zero-norm column still beats it; with no candidate the pivot is `step`.
// Each lane visits its columns in ascending order, kBatch at a time: their norms and
// original indices are all loaded before any is compared, so the loads overlap (a
// caller whose norm_at computes rather than loads takes kBatch 1).
template <typename R, int kBatch = 8, typename NormAt, typename OriginalAt>
__device__ __forceinline__ long long choose_pivot(long long step, long long columns, NormAt norm_at,
                                                  OriginalAt original_at, bool* flagged) {
  Candidate<R> best{R(0), kNoIndex, kNoIndex};
  bool negative = false;
  for (long long c0 = step + lane_id(); c0 < columns; c0 += static_cast<long long>(kLanes) * kBatch) {
    R norms[kBatch];
    long long originals[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const long long c = c0 + static_cast<long long>(k) * kLanes;
      if (c < columns) {
        norms[k] = norm_at(c);
        originals[k] = original_at(c);
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const long long c = c0 + static_cast<long long>(k) * kLanes;
      if (c >= columns) continue;
      if (norms[k] < R(0)) {
        negative = true;
        continue;
      }
      const Candidate<R> cand{norms[k], originals[k], c};
      if (cand.norm > best.norm || (cand.norm == best.norm && cand.original < best.original)) best = cand;
    }
  }
  best = best_over_warp(best);
  *flagged = __any_sync(kAllLanes, negative);
  return best.column == kNoIndex ? step : best.column;
}

template <typename R, typename L>
__device__ __forceinline__ void pivot_task(const R* norms, const long long* perm, long long* pivots,
                                           long long* status, const L& nl, const L& pl, long long step,
                                           long long b) {
  const R* nb = norms + nl.offset + batch_base(nl, 1, b);
  const long long* pb = perm + pl.offset + batch_base(pl, 1, b);
  const long long ns = nl.strides[0], ps = pl.strides[0];
  bool flagged = false;
  const long long pivot = choose_pivot<R>(
      step, nl.extents[0], [&](long long c) { return nb[c * ns]; }, [&](long long c) { return pb[c * ps]; },
      &flagged);
  if (lane_id() == 0) {
    pivots[b] = pivot;
    if (flagged) status[b] = 1;
  }
}

// ---- swap_columns ------------------------------------------------------------------

// Element `pos` = (row, batch), row fastest: exchanges rows of columns step and
// pivots[batch]; the batch's row-0 element also exchanges the two permutation entries.
template <typename T, typename L>
__device__ __forceinline__ void swap_element(T* w, long long* perm, const long long* pivots, const L& wl,
                                             const L& pl, long long step, long long pos) {
  const long long rows = wl.extents[0];
  const long long b = pos / rows;
  const long long row = pos - b * rows;
  const long long pivot = pivots[b];
  if (pivot == step) return;
  T* base = w + wl.offset + row * wl.strides[0] + batch_base(wl, 2, b);
  T* a = base + step * wl.strides[1];
  T* c = base + pivot * wl.strides[1];
  const T held = *a;
  *a = *c;
  *c = held;
  if (row == 0) {
    long long* p = perm + pl.offset + batch_base(pl, 1, b);
    const long long x = p[step * pl.strides[0]];
    p[step * pl.strides[0]] = p[pivot * pl.strides[0]];
    p[pivot * pl.strides[0]] = x;
  }
}

// ---- reflector ---------------------------------------------------------------------

// The reference's complex quotient n / d = (n conj(d)) / |d|^2 with |d|^2 unscaled
// (not the library division of <complex>): the same expressions, so the same rounding.
__device__ __forceinline__ c32 quotient(c32 n, c32 d) {
  const float dd = d.re * d.re + d.im * d.im;
  return c32{(n.re * d.re + n.im * d.im) / dd, (n.im * d.re - n.re * d.im) / dd};
}
__device__ __forceinline__ c64 quotient(c64 n, c64 d) {
  const double dd = d.re * d.re + d.im * d.im;
  return c64{(n.re * d.re + n.im * d.im) / dd, (n.im * d.re - n.re * d.im) / dd};
}
__device__ __forceinline__ float quotient(float n, float d) { return n / d; }
__device__ __forceinline__ double quotient(double n, double d) { return n / d; }

// Householder scalars of a column with leading entry x0 and norm `norm` > 0:
// alpha = -phase(x0) norm (phase = sign for reals, x0/|x0| for complex values, 1 at 0),
// the divisor x0 - alpha of the tail, and the coefficient 1 + |x0| / norm.
template <typename T>
struct Householder {
  T alpha;
  T divisor;
  T coeff;
};

__device__ __forceinline__ Householder<float> householder(float x0, float norm) {
  const float alpha = -(x0 < 0.0f ? -1.0f : 1.0f) * norm;
  return {alpha, x0 - alpha, 1.0f + modulus(x0) / norm};
}
__device__ __forceinline__ Householder<double> householder(double x0, double norm) {
  const double alpha = -(x0 < 0.0 ? -1.0 : 1.0) * norm;
  return {alpha, x0 - alpha, 1.0 + modulus(x0) / norm};
}
template <typename C, typename R>
__device__ __forceinline__ Householder<C> householder_complex(C x0, R norm) {
  const R mag = modulus(x0);
  const R pre = mag == R(0) ? R(1) : x0.re / mag;
  const R pim = mag == R(0) ? R(0) : x0.im / mag;
  const C alpha{-pre * norm, -pim * norm};
  return {alpha, C{x0.re - alpha.re, x0.im - alpha.im}, C{R(1) + mag / norm, R(0)}};
}
__device__ __forceinline__ Householder<c32> householder(c32 x0, float norm) { return householder_complex(x0, norm); }
__device__ __forceinline__ Householder<c64> householder(c64 x0, double norm) { return householder_complex(x0, norm); }

// One warp builds the reflector of column `col` (element r at col[r * rs]) in place:
// the tail rows step+1 .. divided by the divisor, row `step` set to alpha; coefficient
// 0 (and the column untouched) when the norm is 0.  x0 is read by every lane before any
// store, as the reference broadcasts it first.
template <typename T>
__device__ __forceinline__ void reflect_column(T* col, long long rs, T* coeff, long long step, long long rows) {
  using R = RealOf<T>;
  const R norm = chain_norm<false, ChainDepth<T>::value>(Strip<const T>{col, rs}, step, rows, nullptr);
  const T x0 = col[step * rs];
  __syncwarp();
  if (norm == R(0)) {
    if (lane_id() == 0) *coeff = zero_of<T>();
    return;
  }
  const Householder<T> h = householder(x0, norm);
  for (long long r = step + 1 + lane_id(); r < rows; r += kLanes) col[r * rs] = quotient(col[r * rs], h.divisor);
  if (lane_id() == 0) {
    col[step * rs] = h.alpha;
    *coeff = h.coeff;
  }
}

// ---- apply_reflector ---------------------------------------------------------------

// <v, t> over rows [step, rows) with v_step = 1, times the coefficient; then
// t_r -= v_r d.  Reals: the chain is fma(v, t, acc) and the update fma(-v, d, t), the
// reference's contractions.  Complex: conj(v) t accumulated per component, the
// coefficient applied as a complex product, t -= v d.
template <typename R>
__device__ __forceinline__ void reflect_target(Strip<const R> v, Strip<R> t, R coeff, long long step,
                                               long long rows) {
  const int lane = lane_id();
  constexpr int kDepth = ChainDepth<R>::value;
  R acc = R(0);
  for (long long r0 = step + lane; r0 < rows; r0 += static_cast<long long>(kDepth) * kLanes) {
    R vv[kDepth], tt[kDepth];
#pragma unroll
    for (int b = 0; b < kDepth; ++b) {
      const long long r = r0 + static_cast<long long>(b) * kLanes;
      if (r < rows) {
        vv[b] = r == step ? R(1) : v.p[r * v.stride];
        tt[b] = t.p[r * t.stride];
      }
    }
#pragma unroll
    for (int b = 0; b < kDepth; ++b)
      if (r0 + static_cast<long long>(b) * kLanes < rows) acc = fma_rn(vv[b], tt[b], acc);
  }
  const R d = butterfly(acc, AddOp()) * coeff;
  for (long long r0 = step + lane; r0 < rows; r0 += static_cast<long long>(kDepth) * kLanes) {
    R vv[kDepth], tt[kDepth];
#pragma unroll
    for (int b = 0; b < kDepth; ++b) {
      const long long r = r0 + static_cast<long long>(b) * kLanes;
      if (r < rows) {
        vv[b] = r == step ? R(1) : v.p[r * v.stride];
        tt[b] = t.p[r * t.stride];
      }
    }
#pragma unroll
    for (int b = 0; b < kDepth; ++b) {
      const long long r = r0 + static_cast<long long>(b) * kLanes;
      if (r < rows) t.p[r * t.stride] = fma_rn(-vv[b], d, tt[b]);
    }
  }
}

template <typename C>
__device__ __forceinline__ void reflect_target_complex(Strip<const C> v, Strip<C> t, C coeff, long long step,
                                                       long long rows) {
  using R = RealOf<C>;
  R sre = R(0), sim = R(0);
  lane_chain<ChainDepth<C>::value>(v, step, rows, lane_id(), [&](const C& vr, long long r) {
    const C vx = r == step ? one_of<C>() : vr;
    const C x = t.p[r * t.stride];
    sre += vx.re * x.re + vx.im * x.im;
    sim += vx.re * x.im - vx.im * x.re;
  });
  const R are = butterfly(sre, AddOp()), aim = butterfly(sim, AddOp());
  const C d{are * coeff.re - aim * coeff.im, are * coeff.im + aim * coeff.re};
  for (long long r = step + lane_id(); r < rows; r += kLanes) {
    const C vx = r == step ? one_of<C>() : v.p[r * v.stride];
    C& x = t.p[r * t.stride];
    const C p{vx.re * d.re - vx.im * d.im, vx.re * d.im + vx.im * d.re};
    x = C{x.re - p.re, x.im - p.im};
  }
}

template <typename T>
__device__ __forceinline__ void reflect_onto(Strip<const T> v, Strip<T> t, T coeff, long long step, long long rows) {
  if constexpr (Scalar<T>::kComplex) {
    reflect_target_complex<T>(v, t, coeff, step, rows);
  } else {
    reflect_target<T>(v, t, coeff, step, rows);
  }
}

// ---- prefix_rank -------------------------------------------------------------------

// rank = the first diagonal index d with !(|r_dd| > max(atol, rtol |r_00|)) (so a NaN
// fails), or k when there is none; *flagged when a diagonal modulus is not finite.  The
// threshold uses the comparison, not fmax, so a NaN tolerance propagates as in the
// reference.
template <typename T>
__device__ __forceinline__ long long leading_rank(const T* r, long long diag_stride, long long k, RealOf<T> rtol,
                                                  RealOf<T> atol, bool* flagged) {
  using R = RealOf<T>;
  const R rel = rtol * modulus(r[0]);
  const R bound = atol > rel ? atol : rel;
  long long first = kNoIndex;
  bool bad = false;
  for (long long d = lane_id(); d < k; d += kLanes) {
    const R m = modulus(r[d * diag_stride]);
    bad = bad || nonfinite(m);
    if (!(m > bound) && first == kNoIndex) first = d;
  }
  first = butterfly(first, MinOp());
  *flagged = __any_sync(kAllLanes, bad);
  return first == kNoIndex ? k : first;
}

// ---- flat element kernels ----------------------------------------------------------

// Coordinates (row, column, batch) of flat element `f` of a matrix layout.
template <typename L>
__device__ __forceinline__ void matrix_coords(const L& l, long long f, long long* row, long long* col, long long* b) {
  const long long e0 = l.extents[0], e1 = l.extents[1];
  const long long q = f / e0;
  *row = f - q * e0;
  *b = q / e1;
  *col = q - *b * e1;
}

template <typename L>
__device__ __forceinline__ long long matrix_at(const L& l, long long row, long long col, long long b) {
  return l.offset + row * l.strides[0] + col * l.strides[1] + batch_base(l, 2, b);
}

// R element `f`: the work matrix's entry on and above the diagonal, zero below.
template <typename T, typename L>
__device__ __forceinline__ void upper_element(const T* w, T* r, const L& wl, const L& rl, long long f) {
  long long row, col, b;
  matrix_coords(rl, f, &row, &col, &b);
  r[matrix_at(rl, row, col, b)] = row <= col ? w[matrix_at(wl, row, col, b)] : zero_of<T>();
}

// Identity shifted down by `start` rows: element (i, j) is 1 where i == start + j
// (the starting point of Q formation).
template <typename T, typename L>
__device__ __forceinline__ void shifted_identity_element(T* out, const L& l, long long start, long long f) {
  long long row, col, b;
  matrix_coords(l, f, &row, &col, &b);
  out[matrix_at(l, row, col, b)] = row == start + col ? one_of<T>() : zero_of<T>();
}

}  // namespace rrqr
}  // namespace t4a
