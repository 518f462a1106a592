// Movement planning (reference src/lib.rs:1465-1737, :1498-1535) and the host
// launchers of the movement entries.  The launchers rebuild the permutation plan on
// the host and launch one kernel per path, compiled for that path alone.
#include <cuda_runtime.h>

#include "movement_any.cuh"
#include "movement_core.cuh"
#include "plan_common.h"
#include "runtime.h"

namespace t4a {
namespace {

template <int B, int V, bool A16, bool AFF>
__global__ void __launch_bounds__(256) k_rows(PermPlan p, void* dst, const void* src) {
  using E = typename Elem<B>::T;
  perm_rows<E, V, A16, AFF>(p, static_cast<E*>(dst), static_cast<const E*>(src));
}

template <int B, bool VS, bool VD, bool AFF>
__global__ void __launch_bounds__(256, 4) k_tiles(PermPlan p, void* dst, const void* src) {
  using E = typename Elem<B>::T;
  perm_tiles<E, VS, VD, AFF>(p, static_cast<E*>(dst), static_cast<const E*>(src));
}

// Launch a rows/tiles kernel variant with the plan's affine choice.
template <int B, int V, bool A16>
void launch_rows(bool aff, dim3 grid, dim3 block, unsigned smem, cudaStream_t s, const PermPlan& p, void* dst,
                 const void* src) {
  if (aff) {
    k_rows<B, V, A16, true><<<grid, block, smem, s>>>(p, dst, src);
  } else {
    k_rows<B, V, A16, false><<<grid, block, smem, s>>>(p, dst, src);
  }
}

template <int B, bool VS, bool VD>
void launch_tiles(bool aff, dim3 grid, dim3 block, unsigned smem, cudaStream_t s, const PermPlan& p, void* dst,
                  const void* src) {
  if (aff) {
    k_tiles<B, VS, VD, true><<<grid, block, smem, s>>>(p, dst, src);
  } else {
    k_tiles<B, VS, VD, false><<<grid, block, smem, s>>>(p, dst, src);
  }
}

template <int B>
__global__ void __launch_bounds__(256) k_generic(PermPlan p, void* dst, const void* src) {
  using E = typename Elem<B>::T;
  perm_generic<E>(p, static_cast<E*>(dst), static_cast<const E*>(src));
}

template <int B>
__global__ void __launch_bounds__(256) k_zero(void* out, t4a_cuda_layout l, long long len, bool view) {
  zero_fill<B>(out, view ? &l : nullptr, len);
}

int host_esize(int dtype) { return plan::dtype_size(dtype); }

constexpr int kMoveVariant = 32;  // t4a_launch.variant = kMoveVariant + PermKind

// Geometry of a plan's path.
int perm_geometry(const PermPlan& p, t4a_launch* launch) {
  using namespace plan;
  if (p.kind == kPermEmpty) {
    *launch = empty_launch();
    return T4A_OK;
  }
  // Rows and tiles are per-warp units (8 warps per block); generic is per thread.
  unsigned long long units = 0;
  constexpr unsigned long long kWarpsPerBlock = kPermThreads / 32;
  if (p.kind == kPermRows) {
    const PermRowsShape shape = perm_rows_shape(p, perm_rows_vec(p));
    units = ceil_div(ceil_div(p.rest.len, shape.rows) * ceil_div(p.run.len, shape.seg), kWarpsPerBlock);
  } else if (p.kind == kPermTiles) {
    units = ceil_div(static_cast<unsigned long long>(p.rest.len) * ceil_div(p.run.len, warp_tile_d(p.esize)) *
                         ceil_div(p.srun.len, warp_tile_s(p.esize)),
                     kWarpsPerBlock);
  } else {
    units = ceil_div(p.len, kPermThreads);
  }
  if (units > kMaxGridX) units = kMaxGridX;  // every path is grid-stride
  *launch = make_launch(units, kPermThreads, 1, perm_smem_bytes(p), kMoveVariant + p.kind);
  return T4A_OK;
}

__global__ void __launch_bounds__(256) k_generic_words8(PermPlan p, void* dst, const void* src) {
  perm_generic<Words8>(p, static_cast<Words8*>(dst), static_cast<const Words8*>(src));
}

template <int B>
int launch_plan_sized(const PermPlan& p, void* dst, const void* src, dim3 grid, unsigned smem, cudaStream_t s) {
  if constexpr (B == 8) {
    if (off8(dst, src)) {
      k_generic_words8<<<grid, dim3(kPermThreads), 0, s>>>(p, dst, src);
      return runtime::check_launch();
    }
  }
  constexpr int VV = B >= 16 ? 1 : 16 / B;
  const bool src_al = (reinterpret_cast<unsigned long long>(src) & 15ull) == 0;
  const bool dst_al = (reinterpret_cast<unsigned long long>(dst) & 15ull) == 0;
  const dim3 block(kPermThreads);
  const bool rows_vec = VV > 1 && src_al && dst_al && perm_vec(p, 0) == VV && perm_vec(p, 1) == VV;
  const bool aff = perm_affine(p, rows_vec ? VV : 1);
  if (p.kind == kPermRows) {
    if constexpr (VV > 1) {
      if (rows_vec) {
        launch_rows<B, VV, true>(aff, grid, block, smem, s, p, dst, src);
        return runtime::check_launch();
      }
    }
    if (B == 16 && src_al && dst_al) {
      launch_rows<B, 1, true>(aff, grid, block, smem, s, p, dst, src);
    } else {
      launch_rows<B, 1, false>(aff, grid, block, smem, s, p, dst, src);
    }
  } else if (p.kind == kPermTiles) {
    const bool vs = src_al && (VV == 1 || perm_vec(p, 0) == VV);
    const bool vd = dst_al && (VV == 1 || perm_vec(p, 1) == VV);
    if (vs && vd) {
      launch_tiles<B, true, true>(aff, grid, block, smem, s, p, dst, src);
    } else if (vs) {
      launch_tiles<B, true, false>(aff, grid, block, smem, s, p, dst, src);
    } else if (vd) {
      launch_tiles<B, false, true>(aff, grid, block, smem, s, p, dst, src);
    } else {
      launch_tiles<B, false, false>(aff, grid, block, smem, s, p, dst, src);
    }
  } else if (p.kind == kPermGeneric) {
    k_generic<B><<<grid, block, 0, s>>>(p, dst, src);
  }
  return runtime::check_launch();
}

int launch_plan(const PermPlan& p, void* dst, const void* src, void* stream) {
  if (p.kind == kPermEmpty) return T4A_OK;
  t4a_launch l;
  perm_geometry(p, &l);
  const dim3 grid(l.grid[0]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (p.esize) {
    case 1: return launch_plan_sized<1>(p, dst, src, grid, l.shared_bytes, s);
    case 4: return launch_plan_sized<4>(p, dst, src, grid, l.shared_bytes, s);
    case 8: return launch_plan_sized<8>(p, dst, src, grid, l.shared_bytes, s);
    case 16: return launch_plan_sized<16>(p, dst, src, grid, l.shared_bytes, s);
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
}

void compact_strides_host(const t4a_cuda_layout& l, long long* st) {
  long long s = 1;
  for (int d = 0; d < T4A_CUDA_MAX_RANK; ++d) {
    st[d] = s;
    if (d < l.rank) s *= l.extents[d];
  }
}

PermPlan materialize_plan(int dtype, const t4a_cuda_layout& src) {
  long long ds[T4A_CUDA_MAX_RANK];
  compact_strides_host(src, ds);
  return make_perm_plan(src.rank, src.extents, src.strides, ds, src.offset, 0, host_esize(dtype));
}

PermPlan view_plan(int dtype, const t4a_cuda_layout& dst) {
  long long ss[T4A_CUDA_MAX_RANK];
  compact_strides_host(dst, ss);
  return make_perm_plan(dst.rank, dst.extents, ss, dst.strides, 0, dst.offset, host_esize(dtype));
}

PermPlan strided_plan(int dtype, const t4a_cuda_layout& src, const t4a_cuda_layout& dst) {
  return make_perm_plan(src.rank, src.extents, src.strides, dst.strides, src.offset, dst.offset, host_esize(dtype));
}

PermPlan transpose_plan(int dtype, long long src_offset, long long batch_stride, long long m, long long n,
                        long long batches) {
  const long long ext[3] = {m, n, batches};
  const long long ss[3] = {n, 1, batch_stride};
  const long long ds[3] = {1, m, batch_stride};
  return make_perm_plan(3, ext, ss, ds, src_offset, 0, host_esize(dtype));
}

PermPlan broadcast_plan(int dtype, const t4a_cuda_layout& out, const t4a_cuda_layout& in, const long long* dims,
                        int ndims) {
  long long ss[T4A_CUDA_MAX_RANK] = {0}, ds[T4A_CUDA_MAX_RANK];
  compact_strides_host(out, ds);
  for (int s = 0; s < ndims; ++s)
    if (in.extents[s] != 1) ss[dims[s]] += in.strides[s];
  return make_perm_plan(out.rank, out.extents, ss, ds, in.offset, 0, host_esize(dtype));
}

int check_dtype_move(int dtype) { return host_esize(dtype) ? T4A_OK : T4A_ERR_UNSUPPORTED_DTYPE; }

// General-rank twins: the same bodies as the exported `_any` symbols.
template <int E, int A>
__global__ void __launch_bounds__(256) k_zero_any(void* out, t4a_cuda_layout_any l, long long len) {
  any::fill_zero_view<E, A>(out, l, len);
}
template <int E, int A>
__global__ void __launch_bounds__(256) k_materialize_any(void* dst, const void* src, t4a_cuda_layout_any l,
                                                         long long len) {
  any::materialize<E, A>(dst, src, l, len);
}
template <int E, int A>
__global__ void __launch_bounds__(256) k_to_view_any(void* dst, const void* src, t4a_cuda_layout_any l, long long len) {
  any::to_view<E, A>(dst, src, l, len);
}
template <int E, int A>
__global__ void __launch_bounds__(256) k_strided_any(void* dst, const void* src, t4a_cuda_layout_any sl,
                                                     t4a_cuda_layout_any dl, long long len) {
  any::strided_copy<E, A>(dst, src, sl, dl, len);
}
template <int E, int A>
__global__ void __launch_bounds__(256) k_broadcast_any(void* out, const void* in, t4a_cuda_layout_any ol,
                                                       t4a_cuda_layout_any il, t4a_cuda_axis_values_any dims,
                                                       long long len) {
  any::broadcast<E, A>(out, in, ol, il, dims, len);
}

// Host checks of a general-rank layout that need no device access.
int check_layout_any(const t4a_cuda_layout_any& l) {
  if (l.rank < 0 || l.reserved != 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (l.rank > 0 && (l.extents == nullptr || l.strides == nullptr)) return T4A_ERR_NULL_ARGUMENT;
  return T4A_OK;
}

// Common prologue of the `_any` launchers: launch shape, count and dtype.
int any_prologue(const t4a_launch* launch, long long len, int dtype, dim3* grid, dim3* block, bool* empty) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (host_esize(dtype) == 0) return T4A_ERR_UNSUPPORTED_DTYPE;
  *empty = len == 0 || launch->grid[0] == 0 || launch->block[0] == 0;
  *grid = dim3(launch->grid[0], launch->grid[1] ? launch->grid[1] : 1, launch->grid[2] ? launch->grid[2] : 1);
  *block = dim3(launch->block[0], launch->block[1] ? launch->block[1] : 1, launch->block[2] ? launch->block[2] : 1);
  return T4A_OK;
}

}  // namespace
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;

extern "C" {

// plan_materialize_strided (src/lib.rs:1630).
int t4a_plan_materialize_strided(int dtype, const t4a_cuda_layout* src, long long src_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  T4A_TRY(check_layout(src));
  long long len;
  T4A_TRY(element_count(*src, &len));
  T4A_TRY(check_span(*src, src_len, host_esize(dtype)));
  return perm_geometry(materialize_plan(dtype, *src), launch);
}

// plan_contiguous_to_view (src/lib.rs:1645).
int t4a_plan_contiguous_to_view(int dtype, const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  T4A_TRY(check_layout(dst));
  long long len;
  T4A_TRY(element_count(*dst, &len));
  T4A_TRY(require_destination(*dst));
  T4A_TRY(check_span(*dst, dst_len, host_esize(dtype)));
  return perm_geometry(view_plan(dtype, *dst), launch);
}

// plan_strided_to_strided (src/lib.rs:1660).
int t4a_plan_strided_to_strided(int dtype, const t4a_cuda_layout* src, long long src_len,
                                const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  T4A_TRY(check_layout(src));
  T4A_TRY(check_layout(dst));
  if (src->rank != dst->rank) return T4A_ERR_COUNT_MISMATCH;
  for (int d = 0; d < src->rank; ++d)
    if (src->extents[d] != dst->extents[d]) return T4A_ERR_COUNT_MISMATCH;
  long long len;
  T4A_TRY(element_count(*src, &len));
  T4A_TRY(require_destination(*dst));
  T4A_TRY(check_span(*src, src_len, host_esize(dtype)));
  T4A_TRY(check_span(*dst, dst_len, host_esize(dtype)));
  return perm_geometry(strided_plan(dtype, *src, *dst), launch);
}

// plan_copy_exact (src/lib.rs:1624).
int t4a_plan_copy_exact(int dtype, long long len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  const long long one = 1;
  return perm_geometry(make_perm_plan(1, &len, &one, &one, 0, 0, host_esize(dtype)), launch);
}

// plan_fill_zero (src/lib.rs:1601) / plan_fill_zero_view (:1609).
int t4a_plan_fill_zero(int dtype, long long len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (len == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  unsigned long long grid;
  T4A_TRY(grid_of(len, kFlatBlock, &grid));
  *launch = make_launch(grid, kFlatBlock, 1, 0, 0);
  return T4A_OK;
}

int t4a_plan_fill_zero_view(int dtype, const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  T4A_TRY(check_layout(dst));
  long long len;
  T4A_TRY(element_count(*dst, &len));
  T4A_TRY(require_destination(*dst));
  T4A_TRY(check_span(*dst, dst_len, host_esize(dtype)));
  return t4a_plan_fill_zero(dtype, len, launch);
}

// plan_tiled_transpose (src/lib.rs:1685): the grid's z dimension is the batch count.
int t4a_plan_tiled_transpose(int dtype, t4a_cuda_transpose_config config, long long src_offset,
                             long long batch_stride, long long dst_fast_extent, long long src_fast_extent,
                             long long batches, long long src_len, long long dst_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  const int t = config.tile, r = config.block_rows, pad = config.padding, v = config.vector_width;
  if (!(t == 8 || t == 16 || t == 32) || !(r == 4 || r == 8 || r == 16) || pad < 0 || pad > 1 ||
      !(v == 1 || v == 2 || v == 4) || t % v != 0)
    return T4A_ERR_INVALID_TRANSPOSE_CONFIG;
  if (dst_fast_extent < 0 || src_fast_extent < 0 || batches < 0 || src_offset < 0) return T4A_ERR_NEGATIVE_COUNT;
  long long matrix, span, end;
  if (mul_overflows(dst_fast_extent, src_fast_extent, &matrix)) return T4A_ERR_OVERFLOW;
  if (batch_stride != matrix) return T4A_ERR_INVALID_TRANSPOSE_CONFIG;
  if (mul_overflows(matrix, batches, &span)) return T4A_ERR_OVERFLOW;
  if (add_overflows(src_offset, span, &end)) return T4A_ERR_OVERFLOW;
  if (end > src_len || span > dst_len) return T4A_ERR_OFFSET_OUT_OF_SPAN;
  if (static_cast<long long>(t) * (t + pad) * host_esize(dtype) > 48 * 1024) return T4A_ERR_LAUNCH_LIMIT;
  if (ceil_div(dst_fast_extent, t) > kMaxGridX || ceil_div(src_fast_extent, t) > kMaxGridYZ ||
      static_cast<unsigned long long>(batches) > kMaxGridYZ)
    return T4A_ERR_LAUNCH_LIMIT;
  if (matrix == 0 || batches == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  const PermPlan p = transpose_plan(dtype, src_offset, batch_stride, dst_fast_extent, src_fast_extent, 1);
  T4A_TRY(perm_geometry(p, launch));
  launch->grid[2] = static_cast<unsigned>(batches);
  return T4A_OK;
}

// plan_broadcast_in_dim (src/lib.rs:1498).
int t4a_plan_broadcast_in_dim(int dtype, const t4a_cuda_layout* out, long long out_len, const t4a_cuda_layout* in,
                              long long in_len, const long long* dims, int ndims, t4a_launch* launch) {
  if (launch == nullptr || (ndims > 0 && dims == nullptr)) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  T4A_TRY(check_layout(out));
  T4A_TRY(check_layout(in));
  T4A_TRY(require_compact(*out));
  T4A_TRY(require_destination(*out));
  if (ndims != in->rank) return T4A_ERR_RANK_LENGTH;
  bool seen[T4A_CUDA_MAX_RANK] = {false};
  for (int s = 0; s < ndims; ++s) {
    if (dims[s] < 0 || dims[s] >= out->rank) return T4A_ERR_INVALID_AXIS;
    if (seen[dims[s]]) return T4A_ERR_DUPLICATE_AXIS;
    seen[dims[s]] = true;
    if (in->extents[s] != out->extents[dims[s]] && in->extents[s] != 1) return T4A_ERR_SHAPE_MISMATCH;
  }
  long long len;
  T4A_TRY(element_count(*out, &len));
  T4A_TRY(check_span(*in, in_len, host_esize(dtype)));
  T4A_TRY(check_span(*out, out_len, host_esize(dtype)));
  return perm_geometry(broadcast_plan(dtype, *out, *in, dims, ndims), launch);
}

// ---- launchers: the argument lists of the kernel symbols ----------------------

int t4a_launch_materialize_strided(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                   t4a_cuda_layout src_layout, long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  (void)len;
  T4A_TRY(check_dtype_move(dtype));
  return launch_plan(materialize_plan(dtype, src_layout), dst, src, stream);
}

int t4a_launch_contiguous_to_view(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                  t4a_cuda_layout dst_layout, long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  (void)len;
  T4A_TRY(check_dtype_move(dtype));
  return launch_plan(view_plan(dtype, dst_layout), dst, src, stream);
}

int t4a_launch_strided_to_strided(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                  t4a_cuda_layout src_layout, t4a_cuda_layout dst_layout, long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  (void)len;
  T4A_TRY(check_dtype_move(dtype));
  return launch_plan(strided_plan(dtype, src_layout, dst_layout), dst, src, stream);
}

int t4a_launch_copy_exact(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                          long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_dtype_move(dtype));
  const long long one = 1;
  return launch_plan(make_perm_plan(1, &len, &one, &one, 0, 0, host_esize(dtype)), dst, src, stream);
}

int t4a_launch_tiled_transpose(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                               long long src_offset, long long batch_stride, long long dst_fast_extent,
                               long long src_fast_extent, t4a_cuda_transpose_config config) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  (void)config;
  T4A_TRY(check_dtype_move(dtype));
  if (launch->grid[0] == 0 || launch->grid[2] == 0) return T4A_OK;
  const long long batches = launch->grid[2];
  return launch_plan(transpose_plan(dtype, src_offset, batch_stride, dst_fast_extent, src_fast_extent, batches),
                     dst, src, stream);
}

int t4a_launch_broadcast_in_dim(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype,
                                t4a_cuda_layout out_layout, t4a_cuda_layout in_layout, t4a_cuda_axis_values dims,
                                long long out_len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  (void)out_len;
  T4A_TRY(check_dtype_move(dtype));
  return launch_plan(broadcast_plan(dtype, out_layout, in_layout, dims.values, dims.rank), out, in, stream);
}

int t4a_launch_fill_zero(const t4a_launch* launch, void* stream, void* out, int dtype, long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch->grid[0] == 0) return T4A_OK;
  t4a_cuda_layout none;
  std::memset(&none, 0, sizeof(none));
  const dim3 grid(launch->grid[0]), block(launch->block[0]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (host_esize(dtype)) {
    case 1: k_zero<1><<<grid, block, 0, s>>>(out, none, len, false); break;
    case 4: k_zero<4><<<grid, block, 0, s>>>(out, none, len, false); break;
    case 8: k_zero<8><<<grid, block, 0, s>>>(out, none, len, false); break;
    case 16: k_zero<16><<<grid, block, 0, s>>>(out, none, len, false); break;
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
  return runtime::check_launch();
}

int t4a_launch_fill_zero_view(const t4a_launch* launch, void* stream, void* out, int dtype, t4a_cuda_layout layout,
                              long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch->grid[0] == 0) return T4A_OK;
  const dim3 grid(launch->grid[0]), block(launch->block[0]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (host_esize(dtype)) {
    case 1: k_zero<1><<<grid, block, 0, s>>>(out, layout, len, true); break;
    case 4: k_zero<4><<<grid, block, 0, s>>>(out, layout, len, true); break;
    case 8: k_zero<8><<<grid, block, 0, s>>>(out, layout, len, true); break;
    case 16: k_zero<16><<<grid, block, 0, s>>>(out, layout, len, true); break;
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
  return runtime::check_launch();
}

int t4a_movement_any_geometry(long long len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (len == 0) {
    *launch = plan::empty_launch();
    return T4A_OK;
  }
  const unsigned long long grid = plan::ceil_div(static_cast<unsigned long long>(len), 256);
  const unsigned long long cap = 148ull * 64;
  *launch = plan::make_launch(grid < cap ? grid : cap, 256, 1, 0, 0);
  return T4A_OK;
}

// Launches KERNEL<E, A> for the dtype's element size E and the widest access A that
// the buffers' bases (BITS, their OR) allow.
#define T4A_ANY_LAUNCH(BITS, KERNEL, ...)                                           \
  switch (host_esize(dtype)) {                                                      \
    case 1: KERNEL<1, 1><<<grid, block, 0, s>>>(__VA_ARGS__); break;                \
    case 4: KERNEL<4, 4><<<grid, block, 0, s>>>(__VA_ARGS__); break;                \
    case 8:                                                                         \
      if (((BITS) & 7ull) == 0) KERNEL<8, 8><<<grid, block, 0, s>>>(__VA_ARGS__);   \
      else KERNEL<8, 4><<<grid, block, 0, s>>>(__VA_ARGS__);                        \
      break;                                                                        \
    case 16:                                                                        \
      if (((BITS) & 15ull) == 0) KERNEL<16, 16><<<grid, block, 0, s>>>(__VA_ARGS__); \
      else if (((BITS) & 7ull) == 0) KERNEL<16, 8><<<grid, block, 0, s>>>(__VA_ARGS__); \
      else KERNEL<16, 4><<<grid, block, 0, s>>>(__VA_ARGS__);                       \
      break;                                                                        \
    default: return T4A_ERR_UNSUPPORTED_DTYPE;                                      \
  }

int t4a_launch_fill_zero_view_any(const t4a_launch* launch, void* stream, void* out, int dtype,
                                  t4a_cuda_layout_any layout, long long len) {
  dim3 grid, block;
  bool empty;
  T4A_TRY(any_prologue(launch, len, dtype, &grid, &block, &empty));
  T4A_TRY(check_layout_any(layout));
  if (empty) return T4A_OK;
  if (out == nullptr) return T4A_ERR_NULL_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T4A_ANY_LAUNCH(T4A_ANY_BITS(out), k_zero_any, out, layout, len)
  return runtime::check_launch();
}

int t4a_launch_materialize_strided_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                       t4a_cuda_layout_any src_layout, long long len) {
  dim3 grid, block;
  bool empty;
  T4A_TRY(any_prologue(launch, len, dtype, &grid, &block, &empty));
  T4A_TRY(check_layout_any(src_layout));
  if (empty) return T4A_OK;
  if (dst == nullptr || src == nullptr) return T4A_ERR_NULL_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T4A_ANY_LAUNCH(T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), k_materialize_any, dst, src, src_layout, len)
  return runtime::check_launch();
}

int t4a_launch_contiguous_to_view_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                      t4a_cuda_layout_any dst_layout, long long len) {
  dim3 grid, block;
  bool empty;
  T4A_TRY(any_prologue(launch, len, dtype, &grid, &block, &empty));
  T4A_TRY(check_layout_any(dst_layout));
  if (empty) return T4A_OK;
  if (dst == nullptr || src == nullptr) return T4A_ERR_NULL_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T4A_ANY_LAUNCH(T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), k_to_view_any, dst, src, dst_layout, len)
  return runtime::check_launch();
}

int t4a_launch_strided_to_strided_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                      t4a_cuda_layout_any src_layout, t4a_cuda_layout_any dst_layout,
                                      long long len) {
  dim3 grid, block;
  bool empty;
  T4A_TRY(any_prologue(launch, len, dtype, &grid, &block, &empty));
  T4A_TRY(check_layout_any(src_layout));
  T4A_TRY(check_layout_any(dst_layout));
  if (src_layout.rank != dst_layout.rank) return T4A_ERR_RANK_LENGTH;
  if (empty) return T4A_OK;
  if (dst == nullptr || src == nullptr) return T4A_ERR_NULL_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T4A_ANY_LAUNCH(T4A_ANY_BITS(dst) | T4A_ANY_BITS(src), k_strided_any, dst, src, src_layout, dst_layout, len)
  return runtime::check_launch();
}

int t4a_launch_broadcast_in_dim_any(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype,
                                    t4a_cuda_layout_any out_layout, t4a_cuda_layout_any in_layout,
                                    t4a_cuda_axis_values_any dims, long long out_len) {
  dim3 grid, block;
  bool empty;
  T4A_TRY(any_prologue(launch, out_len, dtype, &grid, &block, &empty));
  T4A_TRY(check_layout_any(out_layout));
  T4A_TRY(check_layout_any(in_layout));
  if (dims.rank != in_layout.rank || dims.reserved != 0) return T4A_ERR_RANK_LENGTH;
  if (dims.rank > 0 && dims.values == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (empty) return T4A_OK;
  if (out == nullptr || in == nullptr) return T4A_ERR_NULL_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T4A_ANY_LAUNCH(T4A_ANY_BITS(out) | T4A_ANY_BITS(in), k_broadcast_any, out, in, out_layout, in_layout, dims, out_len)
  return runtime::check_launch();
}
#undef T4A_ANY_LAUNCH

// One call: validate and copy between two layouts of the same extents.
int t4a_copy_strided(void* stream, int dtype, void* dst, const t4a_cuda_layout* dst_layout, long long dst_len,
                     const void* src, const t4a_cuda_layout* src_layout, long long src_len) {
  if (dst == nullptr || src == nullptr) return T4A_ERR_NULL_ARGUMENT;
  t4a_launch launch;
  T4A_TRY(t4a_plan_strided_to_strided(dtype, src_layout, src_len, dst_layout, dst_len, &launch));
  long long len;
  T4A_TRY(element_count(*src_layout, &len));
  return t4a_launch_strided_to_strided(&launch, stream, dst, src, dtype, *src_layout, *dst_layout, len);
}

}  // extern "C"
