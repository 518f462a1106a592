// General-rank gather and additive scatter, the `_any` twins of the gather and
// scatter_add entries (reference cuda/src/gather_scatter.cu:280-452, symbols :587,
// :619): layouts and dimension maps live in device memory, so any rank is accepted.
//
// Element-wise grid-stride walks (any launch geometry is correct):
//   gather       out[view_out(f)] = operand[offset + sum over output axes of the
//                window coordinates, plus the clamped starts read from the indices]
//   scatter_add  out[start(f) + window(f)] += updates[view_updates(f)], skipped when
//                the window does not fit the destination
// with the reference's semantics: the first window position naming an axis wins, a
// batch position skips the index-vector axis, every start component reads one
// element of the index vector (the same element when the index tensor has none), and
// clamped starts follow clamp_start.  Unlike the fast entries no window plan is built:
// the per-axis roles are looked up in the maps as each coordinate is decoded, so the
// state per thread is O(1) whatever the rank.
//
// Before any thread reads the maps, one thread per block checks that they address
// existing axes, that the index tensor's rank matches, and that the element count
// fits the walked layout's extents; a block that finds them malformed does nothing.
#pragma once

#include "gather_scatter_plan.h"
#include "movement_any.cuh"

namespace t4a {
namespace any {

// Flat position over every grid and block dimension (so 2-D and 3-D geometries visit
// each position once, which the atomics of scatter_add need).
__device__ __forceinline__ long long grid_first() {
  const long long block = blockIdx.x + static_cast<long long>(gridDim.x) * (blockIdx.y + static_cast<long long>(gridDim.y) * blockIdx.z);
  return block * block_threads() + flat_tid();
}
__device__ __forceinline__ long long grid_step() {
  return static_cast<long long>(gridDim.x) * gridDim.y * gridDim.z * block_threads();
}

__device__ __forceinline__ bool layout_ok(const t4a_cuda_layout_any& l) {
  return l.rank >= 0 && (l.rank == 0 || (l.extents != nullptr && l.strides != nullptr));
}

// n values in [0, rank), pairwise distinct when `distinct`.
__device__ __forceinline__ bool axes_ok(const long long* axes, int n, int rank, bool distinct) {
  if (n < 0 || (n > 0 && axes == nullptr)) return false;
  for (int i = 0; i < n; ++i) {
    if (axes[i] < 0 || axes[i] >= rank) return false;
    if (distinct)
      for (int j = 0; j < i; ++j)
        if (axes[j] == axes[i]) return false;
  }
  return true;
}

// len > 0 elements decode over positive extents whose product is at least len.
__device__ __forceinline__ bool count_fits(const t4a_cuda_layout_any& l, long long len) {
  constexpr long long kMax = 0x7fffffffffffffffll;
  long long n = 1;
  for (int d = 0; d < l.rank; ++d) {
    const long long e = l.extents[d];
    if (e <= 0) return false;
    n = n > kMax / e ? kMax : n * e;
  }
  return len <= n;
}

__device__ __forceinline__ bool index_rank_ok(int walked_rank, int window_rank, int index_vector_dim,
                                              const t4a_cuda_layout_any& il) {
  return index_vector_dim >= 0 && index_vector_dim <= il.rank &&
         walked_rank - window_rank + (index_vector_dim < il.rank ? 1 : 0) == il.rank;
}

__device__ __forceinline__ bool gather_ok(const t4a_cuda_layout_any& ol, const t4a_cuda_layout_any& al,
                                          const t4a_cuda_layout_any& il, const t4a_cuda_gather_plan_any& g,
                                          long long len) {
  return layout_ok(ol) && layout_ok(al) && layout_ok(il) && g.operand_rank == al.rank && g.out_rank == ol.rank &&
         axes_ok(g.window_dims, g.window_rank, al.rank, false) &&
         axes_ok(g.offset_dims, g.window_rank, ol.rank, true) &&
         axes_ok(g.start_index_map, g.start_map_len, al.rank, false) &&
         (g.start_map_len == 0 || g.slice_sizes != nullptr) &&
         index_rank_ok(ol.rank, g.window_rank, g.index_vector_dim, il) && count_fits(ol, len);
}

__device__ __forceinline__ bool scatter_ok(const t4a_cuda_layout_any& ol, const t4a_cuda_layout_any& il,
                                           const t4a_cuda_layout_any& ul, const t4a_cuda_scatter_plan_any& g,
                                           long long len) {
  return layout_ok(ol) && layout_ok(il) && layout_ok(ul) && g.operand_rank == ol.rank &&
         g.updates_rank == ul.rank && axes_ok(g.window_dims, g.window_rank, ol.rank, false) &&
         axes_ok(g.update_window_dims, g.window_rank, ul.rank, true) &&
         axes_ok(g.scatter_dims, g.scatter_map_len, ol.rank, false) &&
         index_rank_ok(ul.rank, g.window_rank, g.index_vector_dim, il) && count_fits(ul, len);
}

__device__ __forceinline__ int first_position(const long long* dims, int n, int axis) {
  for (int q = 0; q < n; ++q)
    if (dims[q] == axis) return q;
  return -1;
}

// Index-tensor axis of batch position `pos`: the index-vector axis is stepped over.
__device__ __forceinline__ int batch_axis(int pos, bool vector_present, int index_vector_dim) {
  return pos + ((vector_present && pos >= index_vector_dim) ? 1 : 0);
}

template <typename C, typename I>
__device__ __forceinline__ void gather_walk(C* __restrict__ out, const C* __restrict__ operand,
                                            const I* __restrict__ idx, const t4a_cuda_layout_any& ol,
                                            const t4a_cuda_layout_any& al, const t4a_cuda_layout_any& il,
                                            const t4a_cuda_gather_plan_any& g, long long len) {
  const bool vec = g.index_vector_dim < il.rank;
  const long long cstride = vec ? il.strides[g.index_vector_dim] : 0;
  for (long long f = grid_first(); f < len; f += grid_step()) {
    long long rest = f, src = al.offset, dst = ol.offset, ib = il.offset;
    int pos = 0;
    for (int ax = 0; ax < ol.rank; ++ax) {
      const long long e = ol.extents[ax];
      const long long c = rest % e;
      rest /= e;
      dst += c * ol.strides[ax];
      const int q = first_position(g.offset_dims, g.window_rank, ax);
      if (q >= 0) {
        src += c * al.strides[g.window_dims[q]];
      } else {
        ib += c * il.strides[batch_axis(pos, vec, g.index_vector_dim)];
        ++pos;
      }
    }
    for (int k = 0; k < g.start_map_len; ++k) {
      const int ax = static_cast<int>(g.start_index_map[k]);
      src += clamp_start<I>(idx[ib + k * cstride], al.extents[ax], g.slice_sizes[ax]) * al.strides[ax];
    }
    out[dst] = operand[src];
  }
}

// F: component type, K: components per element (2 for complex: the real and the
// imaginary part are added separately, as the reference does).
template <typename F, int K, typename I>
__device__ __forceinline__ void scatter_walk(F* __restrict__ out, const F* __restrict__ updates,
                                             const I* __restrict__ idx, const t4a_cuda_layout_any& ol,
                                             const t4a_cuda_layout_any& il, const t4a_cuda_layout_any& ul,
                                             const t4a_cuda_scatter_plan_any& g, long long len) {
  const bool vec = g.index_vector_dim < il.rank;
  const long long cstride = vec ? il.strides[g.index_vector_dim] : 0;
  for (long long f = grid_first(); f < len; f += grid_step()) {
    long long rest = f, src = ul.offset, window = 0, ib = il.offset;
    int pos = 0;
    for (int ax = 0; ax < ul.rank; ++ax) {
      const long long e = ul.extents[ax];
      const long long c = rest % e;
      rest /= e;
      src += c * ul.strides[ax];
      const int q = first_position(g.update_window_dims, g.window_rank, ax);
      if (q >= 0) {
        window += c * ol.strides[g.window_dims[q]];
      } else {
        ib += c * il.strides[batch_axis(pos, vec, g.index_vector_dim)];
        ++pos;
      }
    }
    // Per destination axis: the window's extent there (the last window position naming
    // the axis, else 1) and the sum of the clamped starts scattered onto it.
    long long dst = ol.offset;
    bool fits = true;
    for (int ax = 0; ax < ol.rank && fits; ++ax) {
      long long shape = 1;
      for (int q = 0; q < g.window_rank; ++q)
        if (g.window_dims[q] == ax) shape = ul.extents[g.update_window_dims[q]];
      long long base = 0;
      for (int k = 0; k < g.scatter_map_len; ++k)
        if (g.scatter_dims[k] == ax) base += clamp_start<I>(idx[ib + k * cstride], ol.extents[ax], shape);
      fits = base + shape <= ol.extents[ax];
      dst += base * ol.strides[ax];
    }
    if (!fits) continue;
    dst += window;
#pragma unroll
    for (int r = 0; r < K; ++r) atomicAdd(out + dst * K + r, updates[src * K + r]);
  }
}

template <typename I>
__device__ __forceinline__ void gather_typed(void* out, const void* operand, const void* indices, int dtype,
                                             const t4a_cuda_layout_any& ol, const t4a_cuda_layout_any& al,
                                             const t4a_cuda_layout_any& il, const t4a_cuda_gather_plan_any& g,
                                             long long len) {
  const I* idx = static_cast<const I*>(indices);
#define T4A_CALL(E, A) \
  gather_walk<Elem<E, A>, I>(static_cast<Elem<E, A>*>(out), static_cast<const Elem<E, A>*>(operand), idx, ol, al, il, g, len)
  T4A_ANY_ESIZE_SWITCH(dtype, T4A_ANY_BITS(out) | T4A_ANY_BITS(operand), T4A_CALL)
#undef T4A_CALL
}

template <typename I>
__device__ __forceinline__ void scatter_typed(void* out, const void* indices, const void* updates, int dtype,
                                              const t4a_cuda_layout_any& ol, const t4a_cuda_layout_any& il,
                                              const t4a_cuda_layout_any& ul, const t4a_cuda_scatter_plan_any& g,
                                              long long len) {
  const I* idx = static_cast<const I*>(indices);
  switch (dtype) {
    case T4A_CUDA_F32:
      scatter_walk<float, 1, I>(static_cast<float*>(out), static_cast<const float*>(updates), idx, ol, il, ul, g, len);
      break;
    case T4A_CUDA_F64:
      scatter_walk<double, 1, I>(static_cast<double*>(out), static_cast<const double*>(updates), idx, ol, il, ul, g,
                                 len);
      break;
    case T4A_CUDA_C32:
      scatter_walk<float, 2, I>(static_cast<float*>(out), static_cast<const float*>(updates), idx, ol, il, ul, g, len);
      break;
    case T4A_CUDA_C64:
      scatter_walk<double, 2, I>(static_cast<double*>(out), static_cast<const double*>(updates), idx, ol, il, ul, g,
                                 len);
      break;
    default: break;
  }
}

// The whole entry bodies: the block-wide map check, then the walk for the index and
// data types.
__device__ __forceinline__ void gather_entry(void* out, const void* operand, const void* indices, int dtype,
                                             int index_dtype, const t4a_cuda_layout_any& ol,
                                             const t4a_cuda_layout_any& al, const t4a_cuda_layout_any& il,
                                             const t4a_cuda_gather_plan_any& g, long long len) {
  __shared__ int ok;
  if (len <= 0) return;
  if (flat_tid() == 0) ok = gather_ok(ol, al, il, g, len);
  __syncthreads();
  if (!ok) return;
  switch (index_dtype) {
    case T4A_CUDA_F32: gather_typed<float>(out, operand, indices, dtype, ol, al, il, g, len); break;
    case T4A_CUDA_F64: gather_typed<double>(out, operand, indices, dtype, ol, al, il, g, len); break;
    case T4A_CUDA_I32: gather_typed<int>(out, operand, indices, dtype, ol, al, il, g, len); break;
    case T4A_CUDA_I64: gather_typed<long long>(out, operand, indices, dtype, ol, al, il, g, len); break;
    default: break;
  }
}

__device__ __forceinline__ void scatter_entry(void* out, const void* indices, const void* updates, int dtype,
                                              int index_dtype, const t4a_cuda_layout_any& ol,
                                              const t4a_cuda_layout_any& il, const t4a_cuda_layout_any& ul,
                                              const t4a_cuda_scatter_plan_any& g, long long len) {
  __shared__ int ok;
  if (len <= 0) return;
  if (flat_tid() == 0) ok = scatter_ok(ol, il, ul, g, len);
  __syncthreads();
  if (!ok) return;
  switch (index_dtype) {
    case T4A_CUDA_F32: scatter_typed<float>(out, indices, updates, dtype, ol, il, ul, g, len); break;
    case T4A_CUDA_F64: scatter_typed<double>(out, indices, updates, dtype, ol, il, ul, g, len); break;
    case T4A_CUDA_I32: scatter_typed<int>(out, indices, updates, dtype, ol, il, ul, g, len); break;
    case T4A_CUDA_I64: scatter_typed<long long>(out, indices, updates, dtype, ol, il, ul, g, len); break;
    default: break;
  }
}

}  // namespace any
}  // namespace t4a
