// Entry bodies of the RRQR kernels, shared by the exported module symbols
// (rrqr_abi.cu) and this library's launchers (rrqr_fast.cu).  Each takes the kernel's
// argument list with layouts of type L (t4a_cuda_layout, or the general-rank
// t4a_cuda_layout_any whose arrays live in device memory), decodes the dtype tag once
// and counts its tasks from the layouts on the device.  Warp entries run one task per
// warp (warps past the task count return); flat entries are grid-stride walks.
#pragma once

#include "rrqr_core.cuh"

namespace t4a {
namespace rrqr {
namespace entry {

__device__ __forceinline__ long long flat_begin() {
  return static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ long long flat_stride() { return static_cast<long long>(gridDim.x) * blockDim.x; }

// Calls fn(T{}) with T the element type of `dtype` among the floating tags (F32, F64,
// C32, C64), or among every numeric tag when kIntegers; unknown tags do nothing (the
// ABI's "no work").
template <bool kIntegers, typename Fn>
__device__ __forceinline__ void by_dtype(int dtype, Fn fn) {
  switch (dtype) {
    case T4A_CUDA_F32: fn(float{}); break;
    case T4A_CUDA_F64: fn(double{}); break;
    case T4A_CUDA_C32: fn(c32{}); break;
    case T4A_CUDA_C64: fn(c64{}); break;
    case T4A_CUDA_I32:
      if constexpr (kIntegers) fn(0);
      break;
    case T4A_CUDA_I64:
      if constexpr (kIntegers) fn(0ll);
      break;
    default: break;
  }
}

template <typename L>
__device__ __forceinline__ void column_norms_entry(const void* work, void* norms, int dtype, const L& wl,
                                                   const L& nl, long long step) {
  const long long task = warp_task();
  if (task >= batches_from(wl, 2) * (wl.extents[1] - step)) return;
  by_dtype<false>(dtype, [&](auto tag) {
    using T = decltype(tag);
    norms_task<T>(static_cast<const T*>(work), static_cast<RealOf<T>*>(norms), wl, nl, step, task);
  });
}

template <typename L>
__device__ __forceinline__ void select_pivot_entry(const void* norms, const void* permutation, void* pivots,
                                                   void* status, int dtype, const L& nl, const L& pl,
                                                   long long step) {
  const long long b = warp_task();
  if (b >= batches_from(nl, 1)) return;
  auto* piv = static_cast<long long*>(pivots);
  auto* st = static_cast<long long*>(status);
  const auto* perm = static_cast<const long long*>(permutation);
  if (dtype == T4A_CUDA_F32) pivot_task<float>(static_cast<const float*>(norms), perm, piv, st, nl, pl, step, b);
  if (dtype == T4A_CUDA_F64) pivot_task<double>(static_cast<const double*>(norms), perm, piv, st, nl, pl, step, b);
}

template <typename L>
__device__ __forceinline__ void swap_entry(void* work, void* permutation, const void* pivots, int dtype,
                                           const L& wl, const L& pl, long long step) {
  by_dtype<true>(dtype, [&](auto tag) {
    using T = decltype(tag);
    const long long len = wl.extents[0] * batches_from(wl, 2);
    for (long long p = flat_begin(); p < len; p += flat_stride())
      swap_element<T>(static_cast<T*>(work), static_cast<long long*>(permutation),
                      static_cast<const long long*>(pivots), wl, pl, step, p);
  });
}

template <typename L>
__device__ __forceinline__ void reflector_entry(void* work, void* coeff, int dtype, const L& wl, const L& cl,
                                                long long step) {
  const long long b = warp_task();
  if (b >= batches_from(wl, 2)) return;
  by_dtype<false>(dtype, [&](auto tag) {
    using T = decltype(tag);
    T* col = static_cast<T*>(work) + wl.offset + step * wl.strides[1] + batch_base(wl, 2, b);
    T* c = static_cast<T*>(coeff) + cl.offset + step * cl.strides[0] + batch_base(cl, 1, b);
    reflect_column<T>(col, wl.strides[0], c, step, wl.extents[0]);
  });
}

template <typename L>
__device__ __forceinline__ void apply_entry(const void* packed, void* target, const void* coeff, int dtype,
                                            const L& pl, const L& tl, const L& cl, long long step,
                                            long long first_column, long long column_count) {
  const long long task = warp_task();
  if (column_count <= 0 || task >= batches_from(pl, 2) * column_count) return;
  const long long b = task / column_count;
  const long long column = first_column + (task - b * column_count);
  by_dtype<false>(dtype, [&](auto tag) {
    using T = decltype(tag);
    Strip<const T> v{static_cast<const T*>(packed) + pl.offset + step * pl.strides[1] + batch_base(pl, 2, b),
                     pl.strides[0]};
    Strip<T> t{static_cast<T*>(target) + tl.offset + column * tl.strides[1] + batch_base(tl, 2, b), tl.strides[0]};
    const T c = static_cast<const T*>(coeff)[cl.offset + step * cl.strides[0] + batch_base(cl, 1, b)];
    reflect_onto<T>(v, t, c, step, pl.extents[0]);
  });
}

template <typename L>
__device__ __forceinline__ void extract_entry(const void* work, void* r, int dtype, const L& wl, const L& rl) {
  by_dtype<false>(dtype, [&](auto tag) {
    using T = decltype(tag);
    const long long len = rl.extents[0] * rl.extents[1] * batches_from(rl, 2);
    for (long long f = flat_begin(); f < len; f += flat_stride())
      upper_element<T>(static_cast<const T*>(work), static_cast<T*>(r), wl, rl, f);
  });
}

template <typename L>
__device__ __forceinline__ void prefix_rank_entry(const void* r, void* rank, void* status, int dtype, const L& rl,
                                                  double rtol, double atol) {
  const long long b = warp_task();
  if (b >= batches_from(rl, 2)) return;
  by_dtype<false>(dtype, [&](auto tag) {
    using T = decltype(tag);
    using R = RealOf<T>;
    bool flagged = false;
    const T* base = static_cast<const T*>(r) + rl.offset + batch_base(rl, 2, b);
    const long long k = leading_rank<T>(base, rl.strides[0] + rl.strides[1], rl.extents[0], static_cast<R>(rtol),
                                        static_cast<R>(atol), &flagged);
    if (lane_id() == 0) {
      static_cast<long long*>(rank)[b] = k;
      if (flagged) static_cast<long long*>(status)[b] = 1;
    }
  });
}

template <typename L>
__device__ __forceinline__ void identity_entry(void* out, int dtype, const L& l, long long start) {
  if (l.rank < 2) return;
  by_dtype<true>(dtype, [&](auto tag) {
    using T = decltype(tag);
    const long long len = l.extents[0] * l.extents[1] * batches_from(l, 2);
    for (long long f = flat_begin(); f < len; f += flat_stride())
      shifted_identity_element<T>(static_cast<T*>(out), l, start, f);
  });
}

}  // namespace entry
}  // namespace rrqr
}  // namespace t4a
