// Entry bodies of the RRQR kernels, shared by the exported module symbols
// (rrqr_abi.cu) and this library's general-rank launchers (rrqr_fast.cu): each takes
// the kernel's argument list with layouts of type L (t4a_cuda_layout, or the
// general-rank t4a_cuda_layout_any whose arrays live in device memory) and counts its
// tasks from the layouts on the device.  Plane entries run one task per warp (tasks
// beyond the count return); flat entries are grid-stride walks.
#pragma once

#include "rrqr_core.cuh"

namespace t4a {
namespace rrqr {
namespace entry {

__device__ __forceinline__ long long flat_begin() {
  return static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ long long flat_stride() { return static_cast<long long>(gridDim.x) * blockDim.x; }

template <typename L>
__device__ __forceinline__ void column_norms_entry(const void* work, void* norms, int dtype, const L& wl,
                                                   const L& nl, long long step) {
  const long long tasks = batch_count(wl, 2) * (wl.extents[1] - step);
  const long long task = warp_task();
  if (task >= tasks) return;
  switch (dtype) {
    case T4A_CUDA_F32:
      column_norms_task<float>(static_cast<const float*>(work), static_cast<float*>(norms), wl, nl, step, task);
      break;
    case T4A_CUDA_F64:
      column_norms_task<double>(static_cast<const double*>(work), static_cast<double*>(norms), wl, nl, step, task);
      break;
    case T4A_CUDA_C32:
      column_norms_task<c32>(static_cast<const c32*>(work), static_cast<float*>(norms), wl, nl, step, task);
      break;
    case T4A_CUDA_C64:
      column_norms_task<c64>(static_cast<const c64*>(work), static_cast<double*>(norms), wl, nl, step, task);
      break;
    default: break;
  }
}

template <typename L>
__device__ __forceinline__ void select_pivot_entry(const void* norms, const void* permutation, void* pivots,
                                                   void* status, int dtype, const L& nl, const L& pl,
                                                   long long step) {
  const long long batch = warp_task();
  if (batch >= batch_count(nl, 1)) return;
  auto* piv = static_cast<long long*>(pivots);
  auto* st = static_cast<long long*>(status);
  const auto* perm = static_cast<const long long*>(permutation);
  switch (dtype) {
    case T4A_CUDA_F32:
      select_pivot_task<float>(static_cast<const float*>(norms), perm, piv, st, nl, pl, step, batch);
      break;
    case T4A_CUDA_F64:
      select_pivot_task<double>(static_cast<const double*>(norms), perm, piv, st, nl, pl, step, batch);
      break;
    default: break;
  }
}

template <typename T, typename L>
__device__ __forceinline__ void swap_walk(void* work, void* permutation, const void* pivots, const L& wl,
                                          const L& pl, long long step) {
  const long long len = wl.extents[0] * batch_count(wl, 2);
  for (long long p = flat_begin(); p < len; p += flat_stride())
    swap_columns_elem<T>(static_cast<T*>(work), static_cast<long long*>(permutation),
                         static_cast<const long long*>(pivots), wl, pl, step, p);
}

template <typename L>
__device__ __forceinline__ void swap_entry(void* work, void* permutation, const void* pivots, int dtype,
                                           const L& wl, const L& pl, long long step) {
  switch (dtype) {
    case T4A_CUDA_F32: swap_walk<float>(work, permutation, pivots, wl, pl, step); break;
    case T4A_CUDA_F64: swap_walk<double>(work, permutation, pivots, wl, pl, step); break;
    case T4A_CUDA_I32: swap_walk<int>(work, permutation, pivots, wl, pl, step); break;
    case T4A_CUDA_I64: swap_walk<long long>(work, permutation, pivots, wl, pl, step); break;
    case T4A_CUDA_C32: swap_walk<c32>(work, permutation, pivots, wl, pl, step); break;
    case T4A_CUDA_C64: swap_walk<c64>(work, permutation, pivots, wl, pl, step); break;
    default: break;
  }
}

template <typename T, typename L>
__device__ __forceinline__ void reflector_one(void* work, void* coeff, const L& wl, const L& cl, long long step,
                                              long long batch) {
  const long long base = wl.offset + step * wl.strides[1] + batch_offset(batch, wl, 2);
  const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
  reflector_task(static_cast<T*>(work), static_cast<T*>(coeff), base, wl.strides[0], ci, step, wl.extents[0]);
}

template <typename L>
__device__ __forceinline__ void reflector_entry(void* work, void* coeff, int dtype, const L& wl, const L& cl,
                                                long long step) {
  const long long batch = warp_task();
  if (batch >= batch_count(wl, 2)) return;
  switch (dtype) {
    case T4A_CUDA_F32: reflector_one<float>(work, coeff, wl, cl, step, batch); break;
    case T4A_CUDA_F64: reflector_one<double>(work, coeff, wl, cl, step, batch); break;
    case T4A_CUDA_C32: reflector_one<c32>(work, coeff, wl, cl, step, batch); break;
    case T4A_CUDA_C64: reflector_one<c64>(work, coeff, wl, cl, step, batch); break;
    default: break;
  }
}

template <typename T, typename L>
__device__ __forceinline__ void apply_one(const void* packed, void* target, const void* coeff, const L& pl,
                                          const L& tl, const L& cl, long long step, long long first_column,
                                          long long column_count, long long task) {
  const long long batch = task / column_count;
  const long long column = first_column + task % column_count;
  const long long pb = pl.offset + step * pl.strides[1] + batch_offset(batch, pl, 2);
  const long long tb = tl.offset + column * tl.strides[1] + batch_offset(batch, tl, 2);
  const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
  apply_task(static_cast<const T*>(packed), static_cast<T*>(target), static_cast<const T*>(coeff), pb, tb, ci, step,
             pl.extents[0], pl.strides[0], tl.strides[0]);
}

template <typename L>
__device__ __forceinline__ void apply_entry(const void* packed, void* target, const void* coeff, int dtype,
                                            const L& pl, const L& tl, const L& cl, long long step,
                                            long long first_column, long long column_count) {
  const long long task = warp_task();
  if (column_count <= 0 || task >= batch_count(pl, 2) * column_count) return;
  switch (dtype) {
    case T4A_CUDA_F32:
      apply_one<float>(packed, target, coeff, pl, tl, cl, step, first_column, column_count, task);
      break;
    case T4A_CUDA_F64:
      apply_one<double>(packed, target, coeff, pl, tl, cl, step, first_column, column_count, task);
      break;
    case T4A_CUDA_C32:
      apply_one<c32>(packed, target, coeff, pl, tl, cl, step, first_column, column_count, task);
      break;
    case T4A_CUDA_C64:
      apply_one<c64>(packed, target, coeff, pl, tl, cl, step, first_column, column_count, task);
      break;
    default: break;
  }
}

template <typename T, typename L>
__device__ __forceinline__ void extract_walk(const void* work, void* r, const L& wl, const L& rl) {
  long long len = 1;
  for (int ax = 0; ax < rl.rank; ++ax) len *= rl.extents[ax];
  for (long long f = flat_begin(); f < len; f += flat_stride())
    extract_r_elem<T>(static_cast<const T*>(work), static_cast<T*>(r), wl, rl, f);
}

template <typename L>
__device__ __forceinline__ void extract_entry(const void* work, void* r, int dtype, const L& wl, const L& rl) {
  switch (dtype) {
    case T4A_CUDA_F32: extract_walk<float>(work, r, wl, rl); break;
    case T4A_CUDA_F64: extract_walk<double>(work, r, wl, rl); break;
    case T4A_CUDA_C32: extract_walk<c32>(work, r, wl, rl); break;
    case T4A_CUDA_C64: extract_walk<c64>(work, r, wl, rl); break;
    default: break;
  }
}

template <typename L>
__device__ __forceinline__ void prefix_rank_entry(const void* r, void* rank, void* status, int dtype, const L& rl,
                                                  double rtol, double atol) {
  const long long batch = warp_task();
  if (batch >= batch_count(rl, 2)) return;
  auto* rk = static_cast<long long*>(rank);
  auto* st = static_cast<long long*>(status);
  switch (dtype) {
    case T4A_CUDA_F32:
      prefix_rank_task<float>(static_cast<const float*>(r), rk, st, rl, static_cast<float>(rtol),
                              static_cast<float>(atol), batch);
      break;
    case T4A_CUDA_F64:
      prefix_rank_task<double>(static_cast<const double*>(r), rk, st, rl, rtol, atol, batch);
      break;
    case T4A_CUDA_C32:
      prefix_rank_task<c32>(static_cast<const c32*>(r), rk, st, rl, static_cast<float>(rtol),
                            static_cast<float>(atol), batch);
      break;
    case T4A_CUDA_C64:
      prefix_rank_task<c64>(static_cast<const c64*>(r), rk, st, rl, rtol, atol, batch);
      break;
    default: break;
  }
}

template <typename T, typename L>
__device__ __forceinline__ void identity_walk(void* out, const L& l, long long start) {
  long long len = 1;
  for (int ax = 0; ax < l.rank; ++ax) len *= l.extents[ax];
  for (long long f = flat_begin(); f < len; f += flat_stride())
    identity_shifted_elem<T>(static_cast<T*>(out), l, start, f);
}

template <typename L>
__device__ __forceinline__ void identity_entry(void* out, int dtype, const L& l, long long start) {
  if (l.rank < 2) return;
  switch (dtype) {
    case T4A_CUDA_F32: identity_walk<float>(out, l, start); break;
    case T4A_CUDA_F64: identity_walk<double>(out, l, start); break;
    case T4A_CUDA_I32: identity_walk<int>(out, l, start); break;
    case T4A_CUDA_I64: identity_walk<long long>(out, l, start); break;
    case T4A_CUDA_C32: identity_walk<c32>(out, l, start); break;
    case T4A_CUDA_C64: identity_walk<c64>(out, l, start); break;
    default: break;
  }
}

}  // namespace entry
}  // namespace rrqr
}  // namespace t4a
