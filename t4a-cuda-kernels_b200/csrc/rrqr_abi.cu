// Exported RRQR symbols of the kernel ABI, for callers that load the module and
// launch by name (reference signatures cuda/src/rrqr.cu:513-705).  Plane entries run
// one task per warp, so both the reference's geometry (one 32-lane block per task)
// and this library's (several warps per block) are correct; flat entries are
// grid-stride walks.
#include "rrqr_core.cuh"

using namespace t4a;
using namespace t4a::rrqr;

namespace {

__device__ __forceinline__ long long flat_begin() {
  return static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ long long flat_stride() { return static_cast<long long>(gridDim.x) * blockDim.x; }

}  // namespace

extern "C" __global__ void t4a_cuda_initialize_permutation(void* permutation, long long n, long long len) {
  if (n <= 0) return;
  for (long long p = flat_begin(); p < len; p += flat_stride()) static_cast<long long*>(permutation)[p] = p % n;
}

extern "C" __global__ void t4a_cuda_column_norms(const void* work, void* norms, int dtype, t4a_cuda_layout work_layout,
                                                 t4a_cuda_layout norms_layout, long long step) {
  const long long tasks = batch_count(work_layout, 2) * (work_layout.extents[1] - step);
  const long long task = warp_task();
  if (task >= tasks) return;
  switch (dtype) {
    case T4A_CUDA_F32:
      column_norms_task<float>(static_cast<const float*>(work), static_cast<float*>(norms), work_layout,
                               norms_layout, step, task);
      break;
    case T4A_CUDA_F64:
      column_norms_task<double>(static_cast<const double*>(work), static_cast<double*>(norms), work_layout,
                                norms_layout, step, task);
      break;
    case T4A_CUDA_C32:
      column_norms_task<c32>(static_cast<const c32*>(work), static_cast<float*>(norms), work_layout, norms_layout,
                             step, task);
      break;
    case T4A_CUDA_C64:
      column_norms_task<c64>(static_cast<const c64*>(work), static_cast<double*>(norms), work_layout, norms_layout,
                             step, task);
      break;
    default: break;
  }
}

extern "C" __global__ void t4a_cuda_select_pivot(const void* norms, const void* permutation, void* pivots,
                                                 void* status, int dtype, t4a_cuda_layout norms_layout,
                                                 t4a_cuda_layout permutation_layout, long long step) {
  const long long batch = warp_task();
  if (batch >= batch_count(norms_layout, 1)) return;
  auto* piv = static_cast<long long*>(pivots);
  auto* st = static_cast<long long*>(status);
  const auto* perm = static_cast<const long long*>(permutation);
  switch (dtype) {
    case T4A_CUDA_F32:
      select_pivot_task<float>(static_cast<const float*>(norms), perm, piv, st, norms_layout, permutation_layout,
                               step, batch);
      break;
    case T4A_CUDA_F64:
      select_pivot_task<double>(static_cast<const double*>(norms), perm, piv, st, norms_layout, permutation_layout,
                                step, batch);
      break;
    default: break;
  }
}

template <typename T>
__device__ __forceinline__ void swap_walk(void* work, void* permutation, const void* pivots,
                                          const t4a_cuda_layout& wl, const t4a_cuda_layout& pl, long long step) {
  const long long len = wl.extents[0] * batch_count(wl, 2);
  for (long long p = flat_begin(); p < len; p += flat_stride())
    swap_columns_elem<T>(static_cast<T*>(work), static_cast<long long*>(permutation),
                         static_cast<const long long*>(pivots), wl, pl, step, p);
}

extern "C" __global__ void t4a_cuda_swap_columns(void* work, void* permutation, const void* pivots, int dtype,
                                                 t4a_cuda_layout work_layout, t4a_cuda_layout permutation_layout,
                                                 long long step) {
  switch (dtype) {
    case T4A_CUDA_F32: swap_walk<float>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    case T4A_CUDA_F64: swap_walk<double>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    case T4A_CUDA_I32: swap_walk<int>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    case T4A_CUDA_I64: swap_walk<long long>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    case T4A_CUDA_C32: swap_walk<c32>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    case T4A_CUDA_C64: swap_walk<c64>(work, permutation, pivots, work_layout, permutation_layout, step); break;
    default: break;
  }
}

template <typename T>
__device__ __forceinline__ void reflector_entry(void* work, void* coeff, const t4a_cuda_layout& wl,
                                                const t4a_cuda_layout& cl, long long step, long long batch) {
  const long long base = wl.offset + step * wl.strides[1] + batch_offset(batch, wl, 2);
  const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
  reflector_task(static_cast<T*>(work), static_cast<T*>(coeff), base, wl.strides[0], ci, step, wl.extents[0]);
}

extern "C" __global__ void t4a_cuda_reflector(void* work, void* coeff, int dtype, t4a_cuda_layout work_layout,
                                              t4a_cuda_layout coeff_layout, long long step) {
  const long long batch = warp_task();
  if (batch >= batch_count(work_layout, 2)) return;
  switch (dtype) {
    case T4A_CUDA_F32: reflector_entry<float>(work, coeff, work_layout, coeff_layout, step, batch); break;
    case T4A_CUDA_F64: reflector_entry<double>(work, coeff, work_layout, coeff_layout, step, batch); break;
    case T4A_CUDA_C32: reflector_entry<c32>(work, coeff, work_layout, coeff_layout, step, batch); break;
    case T4A_CUDA_C64: reflector_entry<c64>(work, coeff, work_layout, coeff_layout, step, batch); break;
    default: break;
  }
}

template <typename T>
__device__ __forceinline__ void apply_entry(const void* packed, void* target, const void* coeff,
                                            const t4a_cuda_layout& pl, const t4a_cuda_layout& tl,
                                            const t4a_cuda_layout& cl, long long step, long long first_column,
                                            long long column_count, long long task) {
  const long long batch = task / column_count;
  const long long column = first_column + task % column_count;
  const long long pb = pl.offset + step * pl.strides[1] + batch_offset(batch, pl, 2);
  const long long tb = tl.offset + column * tl.strides[1] + batch_offset(batch, tl, 2);
  const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
  apply_task(static_cast<const T*>(packed), static_cast<T*>(target), static_cast<const T*>(coeff), pb, tb, ci, step,
             pl.extents[0], pl.strides[0], tl.strides[0]);
}

extern "C" __global__ void t4a_cuda_apply_reflector(const void* packed, void* target, const void* coeff, int dtype,
                                                    t4a_cuda_layout packed_layout, t4a_cuda_layout target_layout,
                                                    t4a_cuda_layout coeff_layout, long long step,
                                                    long long first_column, long long column_count) {
  const long long task = warp_task();
  if (column_count <= 0 || task >= batch_count(packed_layout, 2) * column_count) return;
  switch (dtype) {
    case T4A_CUDA_F32:
      apply_entry<float>(packed, target, coeff, packed_layout, target_layout, coeff_layout, step, first_column,
                         column_count, task);
      break;
    case T4A_CUDA_F64:
      apply_entry<double>(packed, target, coeff, packed_layout, target_layout, coeff_layout, step, first_column,
                          column_count, task);
      break;
    case T4A_CUDA_C32:
      apply_entry<c32>(packed, target, coeff, packed_layout, target_layout, coeff_layout, step, first_column,
                       column_count, task);
      break;
    case T4A_CUDA_C64:
      apply_entry<c64>(packed, target, coeff, packed_layout, target_layout, coeff_layout, step, first_column,
                       column_count, task);
      break;
    default: break;
  }
}

template <typename T>
__device__ __forceinline__ void extract_walk(const void* work, void* r, const t4a_cuda_layout& wl,
                                             const t4a_cuda_layout& rl) {
  long long len = 1;
  for (int ax = 0; ax < rl.rank; ++ax) len *= rl.extents[ax];
  for (long long f = flat_begin(); f < len; f += flat_stride())
    extract_r_elem<T>(static_cast<const T*>(work), static_cast<T*>(r), wl, rl, f);
}

extern "C" __global__ void t4a_cuda_extract_r(const void* work, void* r, int dtype, t4a_cuda_layout work_layout,
                                              t4a_cuda_layout r_layout) {
  switch (dtype) {
    case T4A_CUDA_F32: extract_walk<float>(work, r, work_layout, r_layout); break;
    case T4A_CUDA_F64: extract_walk<double>(work, r, work_layout, r_layout); break;
    case T4A_CUDA_C32: extract_walk<c32>(work, r, work_layout, r_layout); break;
    case T4A_CUDA_C64: extract_walk<c64>(work, r, work_layout, r_layout); break;
    default: break;
  }
}

extern "C" __global__ void t4a_cuda_prefix_rank(const void* r, void* rank, void* status, int dtype,
                                                t4a_cuda_layout r_layout, double rtol, double atol) {
  const long long batch = warp_task();
  if (batch >= batch_count(r_layout, 2)) return;
  auto* rk = static_cast<long long*>(rank);
  auto* st = static_cast<long long*>(status);
  switch (dtype) {
    case T4A_CUDA_F32:
      prefix_rank_task<float>(static_cast<const float*>(r), rk, st, r_layout, static_cast<float>(rtol),
                              static_cast<float>(atol), batch);
      break;
    case T4A_CUDA_F64:
      prefix_rank_task<double>(static_cast<const double*>(r), rk, st, r_layout, rtol, atol, batch);
      break;
    case T4A_CUDA_C32:
      prefix_rank_task<c32>(static_cast<const c32*>(r), rk, st, r_layout, static_cast<float>(rtol),
                            static_cast<float>(atol), batch);
      break;
    case T4A_CUDA_C64:
      prefix_rank_task<c64>(static_cast<const c64*>(r), rk, st, r_layout, rtol, atol, batch);
      break;
    default: break;
  }
}
