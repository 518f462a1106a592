// Exported movement symbols of the kernel ABI, for callers that load the module and
// launch by name (reference signatures cuda/src/movement.cu:514-656).  Each block
// builds the permutation plan from its arguments (uniform, a few hundred
// instructions), then runs the plan's path (movement_core.cuh).  The paths need the
// dynamic shared memory the planner reports; with less they fall back to the
// element-per-thread walk, so the reference's own geometry is still correct.
#include "movement_core.cuh"

namespace t4a {
namespace {

__device__ __forceinline__ int move_esize(int dtype) {
  switch (dtype) {
    case T4A_CUDA_F32:
    case T4A_CUDA_I32: return 4;
    case T4A_CUDA_F64:
    case T4A_CUDA_I64:
    case T4A_CUDA_C32: return 8;
    case T4A_CUDA_BOOL: return 1;
    case T4A_CUDA_C64: return 16;
    default: return 0;
  }
}

__device__ __forceinline__ void run_plan(const PermPlan& p, void* dst, const void* src) {
  const bool smem_ok = move_dynamic_smem() >= static_cast<unsigned>(perm_smem_bytes(p, block_threads()));
  switch (p.esize) {
    case 1: perm_run<1>(p, dst, src, smem_ok); break;
    case 4: perm_run<4>(p, dst, src, smem_ok); break;
    case 8: perm_run<8>(p, dst, src, smem_ok); break;
    case 16: perm_run<16>(p, dst, src, smem_ok); break;
    default: break;
  }
}

__device__ __forceinline__ void compact_strides(const t4a_cuda_layout& l, long long* st) {
  long long s = 1;
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    st[d] = s;
    if (d < l.rank) s *= l.extents[d];
  }
}

}  // namespace
}  // namespace t4a

using namespace t4a;

// dst[f] = src[decode(f, src_layout)]: gather into a compact destination.
extern "C" __global__ void __launch_bounds__(256) t4a_cuda_materialize_strided(
    void* dst, const void* src, int dtype, t4a_cuda_layout src_layout, long long len) {
  const int es = move_esize(dtype);
  if (es == 0 || len <= 0) return;
  long long ds[kMaxRank];
  compact_strides(src_layout, ds);
  const PermPlan p = make_perm_plan(src_layout.rank, src_layout.extents, src_layout.strides, ds,
                                    src_layout.offset, 0, es);
  run_plan(p, dst, src);
}

// dst[decode(f, dst_layout)] = src[f]: scatter a compact source into a view.
extern "C" __global__ void __launch_bounds__(256) t4a_cuda_contiguous_to_view(
    void* dst, const void* src, int dtype, t4a_cuda_layout dst_layout, long long len) {
  const int es = move_esize(dtype);
  if (es == 0 || len <= 0) return;
  long long ss[kMaxRank];
  compact_strides(dst_layout, ss);
  const PermPlan p = make_perm_plan(dst_layout.rank, dst_layout.extents, ss, dst_layout.strides, 0,
                                    dst_layout.offset, es);
  run_plan(p, dst, src);
}

// Both layouts share the source's extents.
extern "C" __global__ void __launch_bounds__(256) t4a_cuda_strided_to_strided(
    void* dst, const void* src, int dtype, t4a_cuda_layout src_layout, t4a_cuda_layout dst_layout,
    long long len) {
  const int es = move_esize(dtype);
  if (es == 0 || len <= 0) return;
  const PermPlan p = make_perm_plan(src_layout.rank, src_layout.extents, src_layout.strides,
                                    dst_layout.strides, src_layout.offset, dst_layout.offset, es);
  run_plan(p, dst, src);
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_copy_exact(void* dst, const void* src, int dtype,
                                                                     long long len) {
  const int es = move_esize(dtype);
  if (es == 0 || len <= 0) return;
  const long long one = 1;
  const PermPlan p = make_perm_plan(1, &len, &one, &one, 0, 0, es);
  run_plan(p, dst, src);
}

// dst[b*S + i + j*M] = src[src_offset + b*S + i*N + j], M = dst_fast_extent,
// N = src_fast_extent, S = batch_stride; the batch count is gridDim.z, as in the
// reference's launch contract (docs/abi/c-kernel-abi.md "Tiled transpose").  The
// configuration only shaped the reference's tile; any valid one is accepted here.
extern "C" __global__ void __launch_bounds__(256) t4a_cuda_tiled_transpose(
    void* dst, const void* src, int dtype, long long src_offset, long long batch_stride,
    long long dst_fast_extent, long long src_fast_extent, t4a_cuda_transpose_config config) {
  (void)config;
  const int es = move_esize(dtype);
  if (es == 0) return;
  const long long ext[3] = {dst_fast_extent, src_fast_extent, 1};
  const long long ss[3] = {src_fast_extent, 1, batch_stride};
  const long long ds[3] = {1, dst_fast_extent, batch_stride};
  const long long b = blockIdx.z;
  const PermPlan p = make_perm_plan(2, ext, ss, ds, src_offset + b * batch_stride, b * batch_stride, es);
  run_plan(p, dst, src);
}

// Compact destination <- rank-mapped source; an input axis of extent one broadcasts.
extern "C" __global__ void __launch_bounds__(256) t4a_cuda_broadcast_in_dim(
    void* out, const void* in, int dtype, t4a_cuda_layout out_layout, t4a_cuda_layout in_layout,
    t4a_cuda_axis_values dims, long long out_len) {
  const int es = move_esize(dtype);
  if (es == 0 || out_len <= 0) return;
  long long ss[kMaxRank], ds[kMaxRank];
  compact_strides(out_layout, ds);
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) ss[d] = 0;
#pragma unroll
  for (int s = 0; s < kMaxRank; ++s) {
    if (s < dims.rank && in_layout.extents[s] != 1) {
#pragma unroll
      for (int d = 0; d < kMaxRank; ++d)
        if (d == dims.values[s]) ss[d] += in_layout.strides[s];
    }
  }
  const PermPlan p = make_perm_plan(out_layout.rank, out_layout.extents, ss, ds, in_layout.offset, 0, es);
  run_plan(p, out, in);
}


extern "C" __global__ void __launch_bounds__(256) t4a_cuda_fill_zero(void* out, int dtype, long long len) {
  switch (move_esize(dtype)) {
    case 1: zero_fill<1>(out, nullptr, len); break;
    case 4: zero_fill<4>(out, nullptr, len); break;
    case 8: zero_fill<8>(out, nullptr, len); break;
    case 16: zero_fill<16>(out, nullptr, len); break;
    default: break;
  }
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_fill_zero_view(void* out, int dtype,
                                                                         t4a_cuda_layout layout, long long len) {
  switch (move_esize(dtype)) {
    case 1: zero_fill<1>(out, &layout, len); break;
    case 4: zero_fill<4>(out, &layout, len); break;
    case 8: zero_fill<8>(out, &layout, len); break;
    case 16: zero_fill<16>(out, &layout, len); break;
    default: break;
  }
}

// General-rank twins (reference cuda/src/movement.cu:612-665): element-wise walks over
// layouts whose arrays live in device memory (movement_any.cuh).
#include "movement_any.cuh"

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_fill_zero_view_any(void* out, int dtype,
                                                                            t4a_cuda_layout_any layout,
                                                                            long long len) {
#define T4A_CALL(E, A) t4a::any::fill_zero_view<E, A>(out, layout, len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(out), T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_materialize_strided_any(
    void* dst, const void* src, int dtype, t4a_cuda_layout_any src_layout, long long len) {
#define T4A_CALL(E, A) t4a::any::materialize<E, A>(dst, src, src_layout, len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_contiguous_to_view_any(
    void* dst, const void* src, int dtype, t4a_cuda_layout_any dst_layout, long long len) {
#define T4A_CALL(E, A) t4a::any::to_view<E, A>(dst, src, dst_layout, len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_strided_to_strided_any(
    void* dst, const void* src, int dtype, t4a_cuda_layout_any src_layout, t4a_cuda_layout_any dst_layout,
    long long len) {
#define T4A_CALL(E, A) t4a::any::strided_copy<E, A>(dst, src, src_layout, dst_layout, len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_broadcast_in_dim_any(
    void* out, const void* in, int dtype, t4a_cuda_layout_any out_layout, t4a_cuda_layout_any in_layout,
    t4a_cuda_axis_values_any dims, long long out_len) {
#define T4A_CALL(E, A) t4a::any::broadcast<E, A>(out, in, out_layout, in_layout, dims, out_len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(out) | T4A_ANY_BITS(in), T4A_CALL)
#undef T4A_CALL
}
