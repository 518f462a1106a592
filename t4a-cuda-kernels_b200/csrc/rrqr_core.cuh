// Rank-revealing QR primitives: reference-exact device bodies (sm_100a).
//
// Every reduction of the reference is a 32-lane plane: lane l folds rows
// start + l + 32k in order and the plane finishes with an ascending xor tree
// (reference cuda/src/rrqr.cu:55-82).  Column norms are max-scaled two-pass 2-norms
// (:144-190), pivots break ties by the original column and then the column index
// (:197-239), the reflector is Householder with alpha = -sign(x0)*norm (:290-380),
// and the update is a dot product followed by a rank-one correction (:386-448).
// The bodies here keep that arithmetic operation for operation (the reference's
// contracted multiply-adds written as fma), so norms, reflectors, updates and pivots
// are bit-identical for F32 and F64.  The work mapping is this library's: a task is
// one warp (not one block), so a block may carry several tasks.
#pragma once

#include "common.cuh"

namespace t4a {
namespace rrqr {

constexpr int kPlane = 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr long long kNone = 0x7fffffffffffffffll;

template <typename T> struct RealOf { using F = T; };
template <> struct RealOf<c32> { using F = float; };
template <> struct RealOf<c64> { using F = double; };

// Magnitudes exactly as the reference forms them (a negative zero stays negative).
__device__ __forceinline__ float mag(float v) { return v < 0.0f ? -v : v; }
__device__ __forceinline__ double mag(double v) { return v < 0.0 ? -v : v; }
__device__ __forceinline__ float mag(c32 v) { return hypotf(v.re, v.im); }
__device__ __forceinline__ double mag(c64 v) { return hypot(v.re, v.im); }

__device__ __forceinline__ float fused(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fused(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename F>
__device__ __forceinline__ F plane_sum(F v) {
#pragma unroll
  for (int o = 1; o < kPlane; o <<= 1) v = v + __shfl_xor_sync(kFull, v, o);
  return v;
}

template <typename F>
__device__ __forceinline__ F plane_max(F v) {
#pragma unroll
  for (int o = 1; o < kPlane; o <<= 1) {
    const F other = __shfl_xor_sync(kFull, v, o);
    v = other > v ? other : v;
  }
  return v;
}

__device__ __forceinline__ long long plane_min(long long v) {
#pragma unroll
  for (int o = 1; o < kPlane; o <<= 1) {
    const long long other = __shfl_xor_sync(kFull, v, o);
    v = other < v ? other : v;
  }
  return v;
}

template <typename F>
__device__ __forceinline__ bool not_finite(F v) {
  return v - v != F(0);
}

// Offset of batch `batch` over the layout's axes first..rank-1 (axis `first` fastest).
// L is t4a_cuda_layout or the general-rank t4a_cuda_layout_any (arrays in device
// memory); every body below reads either through the same field names.
template <typename L>
__device__ __forceinline__ long long batch_offset(long long batch, const L& l, int first) {
  long long off = 0;
  for (int ax = first; ax < l.rank; ++ax) {
    const long long e = l.extents[ax];
    off += (batch % e) * l.strides[ax];
    batch /= e;
  }
  return off;
}

template <typename L>
__device__ __forceinline__ long long batch_count(const L& l, int first) {
  long long n = 1;
  for (int ax = first; ax < l.rank; ++ax) n *= l.extents[ax];
  return n;
}

// Warp task ids: warp w of block b is task b * (warps per block) + w.
__device__ __forceinline__ long long warp_task() {
  return static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
}

// Max-scaled 2-norm of rows [step, rows) of one column (all lanes return it);
// `bad` = a non-finite magnitude was seen (the reflector's walk ignores it).
template <typename T, typename F, bool kCheck, int kNormBatch = 16>
__device__ __forceinline__ F column_norm(const T* w, long long base, long long rs, long long step, long long rows,
                                         int lane, bool* bad) {
  // Both walks take batches of kNormBatch rows per lane, every load of a batch issued
  // before any is used, so a lane keeps that many global loads in flight; the sum of
  // squares still folds rows step + lane + 32 k in ascending order.  (The fused pivot's
  // rarely taken re-walk uses batches of 1, which keeps its kernels' registers.)
  F local_max = F(0);
  bool invalid = false;
  for (long long row0 = step + lane; row0 < rows; row0 += kNormBatch * kPlane) {
    T xb[kNormBatch];
#pragma unroll
    for (int b = 0; b < kNormBatch; ++b) {
      const long long row = row0 + static_cast<long long>(b) * kPlane;
      if (row < rows) xb[b] = w[base + row * rs];
    }
#pragma unroll
    for (int b = 0; b < kNormBatch; ++b) {
      if (row0 + static_cast<long long>(b) * kPlane < rows) {
        const F value = mag(xb[b]);
        if (kCheck && not_finite(value)) {
          invalid = true;
        } else if (value > local_max) {
          local_max = value;
        }
      }
    }
  }
  const F scale = plane_max(local_max);
  F local_sum = F(0);
  if (scale > F(0)) {
    for (long long row0 = step + lane; row0 < rows; row0 += kNormBatch * kPlane) {
      T xb[kNormBatch];
#pragma unroll
      for (int b = 0; b < kNormBatch; ++b) {
        const long long row = row0 + static_cast<long long>(b) * kPlane;
        if (row < rows) xb[b] = w[base + row * rs];
      }
#pragma unroll
      for (int b = 0; b < kNormBatch; ++b) {
        if (row0 + static_cast<long long>(b) * kPlane < rows) {
          const F scaled = mag(xb[b]) / scale;
          local_sum = fused(scaled, scaled, local_sum);
        }
      }
    }
  }
  if (kCheck) *bad = __any_sync(kFull, invalid);
  return scale * sqrt(plane_sum(local_sum));
}

// column_norms (reference rrqr.cu:144-190): one warp per (batch, column >= step).
template <typename T, typename L>
__device__ __forceinline__ void column_norms_task(const T* w, typename RealOf<T>::F* norms, const L& wl, const L& nl,
                                                  long long step, long long task) {
  using F = typename RealOf<T>::F;
  const long long trailing = wl.extents[1] - step;
  const long long batch = task / trailing;
  const long long column = step + task % trailing;
  const int lane = threadIdx.x & 31;
  const long long base = wl.offset + column * wl.strides[1] + batch_offset(batch, wl, 2);
  bool bad = false;
  const F norm = column_norm<T, F, true>(w, base, wl.strides[0], step, wl.extents[0], lane, &bad);
  if (lane == 0) norms[nl.offset + column * nl.strides[0] + batch_offset(batch, nl, 1)] =
      (bad || not_finite(norm)) ? F(-1) : norm;
}

// select_pivot (reference rrqr.cu:197-239): one warp per batch.
template <typename F, typename L>
__device__ __forceinline__ void select_pivot_task(const F* norms, const long long* perm, long long* pivots,
                                                  long long* status, const L& nl, const L& pl, long long step,
                                                  long long batch) {
  const long long columns = nl.extents[0];
  const int lane = threadIdx.x & 31;
  const long long nb = nl.offset + batch_offset(batch, nl, 1);
  const long long pb = pl.offset + batch_offset(batch, pl, 1);
  F local_max = F(0);
  long long local_original = kNone, local_column = kNone;
  bool invalid = false;
  for (long long column = step + lane; column < columns; column += kPlane) {
    const F norm = norms[nb + column * nl.strides[0]];
    const long long original = perm[pb + column * pl.strides[0]];
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
  if (lane == 0) {
    pivots[batch] = selected == kNone ? step : selected;
    if (any_invalid) status[batch] = 1;
  }
}

// swap_columns (reference rrqr.cu:244-284): element (row, batch) of a flat walk.
template <typename T, typename L>
__device__ __forceinline__ void swap_columns_elem(T* w, long long* perm, const long long* pivots, const L& wl,
                                                  const L& pl, long long step, long long pos) {
  const long long rows = wl.extents[0];
  const long long row = pos % rows;
  const long long batch = pos / rows;
  const long long pivot = pivots[batch];
  if (pivot == step) return;
  const long long base = wl.offset + row * wl.strides[0] + batch_offset(batch, wl, 2);
  const long long left = base + step * wl.strides[1];
  const long long right = base + pivot * wl.strides[1];
  const T v = w[left];
  w[left] = w[right];
  w[right] = v;
  if (row == 0) {
    const long long pbase = pl.offset + batch_offset(batch, pl, 1);
    const long long first = pbase + step * pl.strides[0];
    const long long second = pbase + pivot * pl.strides[0];
    const long long s = perm[first];
    perm[first] = perm[second];
    perm[second] = s;
  }
}

template <typename T>
__device__ __forceinline__ T complex_div(T n, T d) {
  return n / d;
}
template <>
__device__ __forceinline__ c32 complex_div<c32>(c32 n, c32 d) {
  const float norm = d.re * d.re + d.im * d.im;
  return {(n.re * d.re + n.im * d.im) / norm, (n.im * d.re - n.re * d.im) / norm};
}
template <>
__device__ __forceinline__ c64 complex_div<c64>(c64 n, c64 d) {
  const double norm = d.re * d.re + d.im * d.im;
  return {(n.re * d.re + n.im * d.im) / norm, (n.im * d.re - n.re * d.im) / norm};
}

template <typename T> struct IsComplex { static constexpr bool value = false; };
template <> struct IsComplex<c32> { static constexpr bool value = true; };
template <> struct IsComplex<c64> { static constexpr bool value = true; };

// reflector (reference rrqr.cu:290-380): one warp per batch.
template <typename F>
__device__ __forceinline__ void reflector_real(F* w, F* coeff, long long base, long long rs, long long ci,
                                               long long step, long long rows) {
  const int lane = threadIdx.x & 31;
  const F norm = column_norm<F, F, false>(w, base, rs, step, rows, lane, nullptr);
  F x0 = lane == 0 ? w[base + step * rs] : F(0);
  x0 = __shfl_sync(kFull, x0, 0);
  if (norm == F(0)) {
    if (lane == 0) coeff[ci] = F(0);
    return;
  }
  const F phase = x0 < F(0) ? F(-1) : F(1);
  const F alpha = -phase * norm;
  const F denominator = x0 - alpha;
  for (long long row = step + 1 + lane; row < rows; row += kPlane) w[base + row * rs] /= denominator;
  if (lane == 0) {
    w[base + step * rs] = alpha;
    coeff[ci] = F(1) + mag(x0) / norm;
  }
}

template <typename C>
__device__ __forceinline__ void reflector_complex(C* w, C* coeff, long long base, long long rs, long long ci,
                                               long long step, long long rows) {
  using F = typename RealOf<C>::F;
  const int lane = threadIdx.x & 31;
  const F norm = column_norm<C, F, false>(w, base, rs, step, rows, lane, nullptr);
  C x0;
  x0.re = lane == 0 ? w[base + step * rs].re : F(0);
  x0.im = lane == 0 ? w[base + step * rs].im : F(0);
  x0.re = __shfl_sync(kFull, x0.re, 0);
  x0.im = __shfl_sync(kFull, x0.im, 0);
  if (norm == F(0)) {
    if (lane == 0) coeff[ci] = C{F(0), F(0)};
    return;
  }
  const F x0_abs = mag(x0);
  C phase;
  if (x0_abs == F(0)) {
    phase = C{F(1), F(0)};
  } else {
    phase = C{x0.re / x0_abs, x0.im / x0_abs};
  }
  const C alpha{-phase.re * norm, -phase.im * norm};
  const C denominator{x0.re - alpha.re, x0.im - alpha.im};
  for (long long row = step + 1 + lane; row < rows; row += kPlane)
    w[base + row * rs] = complex_div<C>(w[base + row * rs], denominator);
  if (lane == 0) {
    w[base + step * rs] = alpha;
    coeff[ci] = C{F(1) + x0_abs / norm, F(0)};
  }
}

template <typename T>
__device__ __forceinline__ void reflector_task(T* w, T* coeff, long long base, long long rs, long long ci,
                                               long long step, long long rows) {
  if constexpr (IsComplex<T>::value) {
    reflector_complex<T>(w, coeff, base, rs, ci, step, rows);
  } else {
    reflector_real<T>(w, coeff, base, rs, ci, step, rows);
  }
}

// apply_reflector (reference rrqr.cu:386-448): one warp per (batch, target column).
template <typename F>
__device__ __forceinline__ void apply_real(const F* packed, F* target, const F* coeff, long long pb, long long tb,
                                           long long ci, long long step, long long rows, long long prs,
                                           long long trs) {
  // Batches of kApplyBatch rows per lane: every load of a batch is issued before the
  // batch is folded, so a lane keeps that many global loads in flight instead of
  // waiting on each; the fold order (rows step + lane + 32 k, ascending) is unchanged.
  constexpr int kApplyBatch = 16;
  const int lane = threadIdx.x & 31;
  F dot = F(0);
  for (long long row0 = step + lane; row0 < rows; row0 += kApplyBatch * kPlane) {
    F vb[kApplyBatch], xb[kApplyBatch];
#pragma unroll
    for (int b = 0; b < kApplyBatch; ++b) {
      const long long row = row0 + static_cast<long long>(b) * kPlane;
      if (row < rows) {
        vb[b] = row == step ? F(1) : packed[pb + row * prs];
        xb[b] = target[tb + row * trs];
      }
    }
#pragma unroll
    for (int b = 0; b < kApplyBatch; ++b)
      if (row0 + static_cast<long long>(b) * kPlane < rows) dot = fused(vb[b], xb[b], dot);
  }
  dot = plane_sum(dot) * coeff[ci];
  for (long long row0 = step + lane; row0 < rows; row0 += kApplyBatch * kPlane) {
    F vb[kApplyBatch], xb[kApplyBatch];
#pragma unroll
    for (int b = 0; b < kApplyBatch; ++b) {
      const long long row = row0 + static_cast<long long>(b) * kPlane;
      if (row < rows) {
        vb[b] = row == step ? F(1) : packed[pb + row * prs];
        xb[b] = target[tb + row * trs];
      }
    }
#pragma unroll
    for (int b = 0; b < kApplyBatch; ++b) {
      const long long row = row0 + static_cast<long long>(b) * kPlane;
      if (row < rows) target[tb + row * trs] = fused(-vb[b], dot, xb[b]);
    }
  }
}

template <typename C>
__device__ __forceinline__ void apply_complex(const C* packed, C* target, const C* coeff, long long pb, long long tb,
                                           long long ci, long long step, long long rows, long long prs,
                                           long long trs) {
  using F = typename RealOf<C>::F;
  const int lane = threadIdx.x & 31;
  F dre = F(0), dim = F(0);
  for (long long row = step + lane; row < rows; row += kPlane) {
    const C v = row == step ? C{F(1), F(0)} : packed[pb + row * prs];
    const C x = target[tb + row * trs];
    // conj(v) * x
    dre += v.re * x.re + v.im * x.im;
    dim += v.re * x.im - v.im * x.re;
  }
  const C c = coeff[ci];
  const F sre = plane_sum(dre), sim = plane_sum(dim);
  const C dot{sre * c.re - sim * c.im, sre * c.im + sim * c.re};
  for (long long row = step + lane; row < rows; row += kPlane) {
    const C v = row == step ? C{F(1), F(0)} : packed[pb + row * prs];
    C& t = target[tb + row * trs];
    const C p{v.re * dot.re - v.im * dot.im, v.re * dot.im + v.im * dot.re};
    t = C{t.re - p.re, t.im - p.im};
  }
}

template <typename T>
__device__ __forceinline__ void apply_task(const T* packed, T* target, const T* coeff, long long pb, long long tb,
                                           long long ci, long long step, long long rows, long long prs,
                                           long long trs) {
  if constexpr (IsComplex<T>::value) {
    apply_complex<T>(packed, target, coeff, pb, tb, ci, step, rows, prs, trs);
  } else {
    apply_real<T>(packed, target, coeff, pb, tb, ci, step, rows, prs, trs);
  }
}

// prefix_rank (reference rrqr.cu:476-509): one warp per batch.
template <typename T, typename L>
__device__ __forceinline__ void prefix_rank_task(const T* r, long long* rank, long long* status, const L& rl,
                                                 typename RealOf<T>::F rtol,
                                                 typename RealOf<T>::F atol, long long batch) {
  using F = typename RealOf<T>::F;
  const long long k = rl.extents[0];
  const int lane = threadIdx.x & 31;
  const long long base = rl.offset + batch_offset(batch, rl, 2);
  const F leading = mag(r[base]);
  const F relative = rtol * leading;
  const F threshold = atol > relative ? atol : relative;
  long long first_failure = kNone;
  bool invalid = false;
  for (long long d = lane; d < k; d += kPlane) {
    const F value = mag(r[base + d * rl.strides[0] + d * rl.strides[1]]);
    if (not_finite(value)) invalid = true;
    if (!(value > threshold) && d < first_failure) first_failure = d;
  }
  const long long failure = plane_min(first_failure);
  const bool any_invalid = __any_sync(kFull, invalid);
  if (lane == 0) {
    rank[batch] = failure == kNone ? k : failure;
    if (any_invalid) status[batch] = 1;
  }
}

// extract_r (reference rrqr.cu:449-470): element `flat` of R.
template <typename T, typename L>
__device__ __forceinline__ void extract_r_elem(const T* w, T* r, const L& wl, const L& rl, long long flat) {
  const long long row = flat % rl.extents[0];
  const long long column = (flat / rl.extents[0]) % rl.extents[1];
  const long long batch = flat / (rl.extents[0] * rl.extents[1]);
  T value;
  memset(&value, 0, sizeof(T));
  if (row <= column)
    value = w[wl.offset + row * wl.strides[0] + column * wl.strides[1] + batch_offset(batch, wl, 2)];
  r[rl.offset + row * rl.strides[0] + column * rl.strides[1] + batch_offset(batch, rl, 2)] = value;
}

template <typename T> __device__ __forceinline__ T unit_of() { return T(1); }
template <> __device__ __forceinline__ c32 unit_of<c32>() { return {1.0f, 0.0f}; }
template <> __device__ __forceinline__ c64 unit_of<c64>() { return {1.0, 0.0}; }

// out(i, j, batch) = 1 where i == start + j, else 0 (reference linalg_aux.cu:200-211):
// the identity that Q formation starts from, shifted down by `start` rows.
template <typename T, typename L>
__device__ __forceinline__ void identity_shifted_elem(T* out, const L& l, long long start, long long flat) {
  const long long row = flat % l.extents[0];
  const long long column = (flat / l.extents[0]) % l.extents[1];
  const long long batch = flat / (l.extents[0] * l.extents[1]);
  T value;
  memset(&value, 0, sizeof(T));
  if (row == start + column) value = unit_of<T>();
  out[l.offset + row * l.strides[0] + column * l.strides[1] + batch_offset(batch, l, 2)] = value;
}

}  // namespace rrqr
}  // namespace t4a
