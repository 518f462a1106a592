// Exported RRQR symbols of the kernel ABI, for callers that load the module and
// launch by name: the by-value entries (reference signatures cuda/src/rrqr.cu:513-705)
// and their general-rank `_any` twins (:930-1108), whose layouts keep extents and
// strides in device memory.  Both sets run the same entry bodies (rrqr_entries.cuh),
// templated on the layout type.  Plane entries run one task per warp, so both the reference's
// geometry (one 32-lane block per task) and this library's (several warps per block)
// are correct; flat entries are grid-stride walks.
#include "rrqr_entries.cuh"

using namespace t4a;
using namespace t4a::rrqr;
using namespace t4a::rrqr::entry;

// ---- by-value layouts (rank <= 8) ---------------------------------------------

extern "C" __global__ void t4a_cuda_initialize_permutation(void* permutation, long long n, long long len) {
  if (n <= 0) return;
  for (long long p = flat_begin(); p < len; p += flat_stride()) static_cast<long long*>(permutation)[p] = p % n;
}

extern "C" __global__ void t4a_cuda_column_norms(const void* work, void* norms, int dtype, t4a_cuda_layout work_layout,
                                                 t4a_cuda_layout norms_layout, long long step) {
  column_norms_entry(work, norms, dtype, work_layout, norms_layout, step);
}

extern "C" __global__ void t4a_cuda_select_pivot(const void* norms, const void* permutation, void* pivots,
                                                 void* status, int dtype, t4a_cuda_layout norms_layout,
                                                 t4a_cuda_layout permutation_layout, long long step) {
  select_pivot_entry(norms, permutation, pivots, status, dtype, norms_layout, permutation_layout, step);
}

extern "C" __global__ void t4a_cuda_swap_columns(void* work, void* permutation, const void* pivots, int dtype,
                                                 t4a_cuda_layout work_layout, t4a_cuda_layout permutation_layout,
                                                 long long step) {
  swap_entry(work, permutation, pivots, dtype, work_layout, permutation_layout, step);
}

extern "C" __global__ void t4a_cuda_reflector(void* work, void* coeff, int dtype, t4a_cuda_layout work_layout,
                                              t4a_cuda_layout coeff_layout, long long step) {
  reflector_entry(work, coeff, dtype, work_layout, coeff_layout, step);
}

extern "C" __global__ void t4a_cuda_apply_reflector(const void* packed, void* target, const void* coeff, int dtype,
                                                    t4a_cuda_layout packed_layout, t4a_cuda_layout target_layout,
                                                    t4a_cuda_layout coeff_layout, long long step,
                                                    long long first_column, long long column_count) {
  apply_entry(packed, target, coeff, dtype, packed_layout, target_layout, coeff_layout, step, first_column,
              column_count);
}

extern "C" __global__ void t4a_cuda_extract_r(const void* work, void* r, int dtype, t4a_cuda_layout work_layout,
                                              t4a_cuda_layout r_layout) {
  extract_entry(work, r, dtype, work_layout, r_layout);
}

extern "C" __global__ void t4a_cuda_prefix_rank(const void* r, void* rank, void* status, int dtype,
                                                t4a_cuda_layout r_layout, double rtol, double atol) {
  prefix_rank_entry(r, rank, status, dtype, r_layout, rtol, atol);
}

// ---- general-rank layouts (`_any`) --------------------------------------------

extern "C" __global__ void t4a_cuda_column_norms_any(const void* work, void* norms, int dtype,
                                                     t4a_cuda_layout_any work_layout,
                                                     t4a_cuda_layout_any norms_layout, long long step) {
  column_norms_entry(work, norms, dtype, work_layout, norms_layout, step);
}

extern "C" __global__ void t4a_cuda_select_pivot_any(const void* norms, const void* permutation, void* pivots,
                                                     void* status, int dtype, t4a_cuda_layout_any norms_layout,
                                                     t4a_cuda_layout_any permutation_layout, long long step) {
  select_pivot_entry(norms, permutation, pivots, status, dtype, norms_layout, permutation_layout, step);
}

extern "C" __global__ void t4a_cuda_swap_columns_any(void* work, void* permutation, const void* pivots, int dtype,
                                                     t4a_cuda_layout_any work_layout,
                                                     t4a_cuda_layout_any permutation_layout, long long step) {
  swap_entry(work, permutation, pivots, dtype, work_layout, permutation_layout, step);
}

extern "C" __global__ void t4a_cuda_reflector_any(void* work, void* coeff, int dtype, t4a_cuda_layout_any work_layout,
                                                  t4a_cuda_layout_any coeff_layout, long long step) {
  reflector_entry(work, coeff, dtype, work_layout, coeff_layout, step);
}

extern "C" __global__ void t4a_cuda_apply_reflector_any(const void* packed, void* target, const void* coeff, int dtype,
                                                        t4a_cuda_layout_any packed_layout,
                                                        t4a_cuda_layout_any target_layout,
                                                        t4a_cuda_layout_any coeff_layout, long long step,
                                                        long long first_column, long long column_count) {
  apply_entry(packed, target, coeff, dtype, packed_layout, target_layout, coeff_layout, step, first_column,
              column_count);
}

extern "C" __global__ void t4a_cuda_extract_r_any(const void* work, void* r, int dtype, t4a_cuda_layout_any work_layout,
                                                  t4a_cuda_layout_any r_layout) {
  extract_entry(work, r, dtype, work_layout, r_layout);
}

extern "C" __global__ void t4a_cuda_prefix_rank_any(const void* r, void* rank, void* status, int dtype,
                                                    t4a_cuda_layout_any r_layout, double rtol, double atol) {
  prefix_rank_entry(r, rank, status, dtype, r_layout, rtol, atol);
}
