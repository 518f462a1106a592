// General-rank movement bodies, the `_any` twins of the movement entries (reference
// cuda/src/movement.cu:612-665): layouts whose extents and strides live in device
// memory, any rank.  Element-wise walks (grid-stride, so any geometry is correct):
//   fill_zero_view       out[view(f)] = 0
//   materialize_strided  dst[f] = src[view(f)]
//   contiguous_to_view   dst[view(f)] = src[f]
//   strided_to_strided   dst[dst_view(f)] = src[src_view(f)], both decoded over the
//                        source's extents
//   broadcast_in_dim     out[f] = in[sum over input axes a of c_dims[a](f) * stride_a],
//                        the coordinate taken as 0 on an input axis of extent 1
// where view(f) decodes the flat index f (axis 0 fastest) over the layout's extents
// into offset + sum of coordinate * stride.  Elements move as raw bytes of the
// dtype's size, in accesses as wide as the buffers' bases allow (complex64 and
// complex128 are only 4- and 8-byte aligned in the ABI).
#pragma once

#include "common.cuh"

namespace t4a {
namespace any {

template <int E, int A>
struct alignas(A) Elem {
  unsigned char b[E];
};

__device__ __forceinline__ long long view_of(long long f, int rank, const long long* extents,
                                             const long long* strides, long long offset) {
  for (int d = 0; d < rank; ++d) {
    const long long e = extents[d];
    offset += (f % e) * strides[d];
    f /= e;
  }
  return offset;
}

__device__ __forceinline__ long long compact_coordinate(long long f, const long long* extents, int axis) {
  for (int d = 0; d < axis; ++d) f /= extents[d];
  return f % extents[axis];
}

__device__ __forceinline__ long long flat_first() {
  return static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ long long flat_step() { return static_cast<long long>(gridDim.x) * blockDim.x; }

template <int E, int A>
__device__ __forceinline__ void fill_zero_view(void* out, const t4a_cuda_layout_any& l, long long len) {
  Elem<E, A> z;
#pragma unroll
  for (int i = 0; i < E; ++i) z.b[i] = 0;
  for (long long f = flat_first(); f < len; f += flat_step())
    static_cast<Elem<E, A>*>(out)[view_of(f, l.rank, l.extents, l.strides, l.offset)] = z;
}

template <int E, int A>
__device__ __forceinline__ void materialize(void* dst, const void* src, const t4a_cuda_layout_any& l, long long len) {
  for (long long f = flat_first(); f < len; f += flat_step())
    static_cast<Elem<E, A>*>(dst)[f] = static_cast<const Elem<E, A>*>(src)[view_of(f, l.rank, l.extents, l.strides, l.offset)];
}

template <int E, int A>
__device__ __forceinline__ void to_view(void* dst, const void* src, const t4a_cuda_layout_any& l, long long len) {
  for (long long f = flat_first(); f < len; f += flat_step())
    static_cast<Elem<E, A>*>(dst)[view_of(f, l.rank, l.extents, l.strides, l.offset)] = static_cast<const Elem<E, A>*>(src)[f];
}

template <int E, int A>
__device__ __forceinline__ void strided_copy(void* dst, const void* src, const t4a_cuda_layout_any& sl,
                                             const t4a_cuda_layout_any& dl, long long len) {
  for (long long f = flat_first(); f < len; f += flat_step()) {
    const long long si = view_of(f, sl.rank, sl.extents, sl.strides, sl.offset);
    const long long di = view_of(f, sl.rank, sl.extents, dl.strides, dl.offset);
    static_cast<Elem<E, A>*>(dst)[di] = static_cast<const Elem<E, A>*>(src)[si];
  }
}

template <int E, int A>
__device__ __forceinline__ void broadcast(void* out, const void* in, const t4a_cuda_layout_any& ol,
                                          const t4a_cuda_layout_any& il, const t4a_cuda_axis_values_any& dims,
                                          long long len) {
  for (long long f = flat_first(); f < len; f += flat_step()) {
    long long index = il.offset;
    for (int a = 0; a < dims.rank; ++a) {
      if (il.extents[a] != 1)
        index += compact_coordinate(f, ol.extents, static_cast<int>(dims.values[a])) * il.strides[a];
    }
    static_cast<Elem<E, A>*>(out)[f] = static_cast<const Elem<E, A>*>(in)[index];
  }
}

__device__ __forceinline__ int elem_bytes(int dtype) {
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

}  // namespace any
}  // namespace t4a

// Calls CALL(E, A) for the dtype's element size E and the widest access A <= E that
// every element reaches, given BITS = the OR of the buffers' base addresses (unknown
// dtypes do nothing).
#define T4A_ANY_ESIZE_SWITCH(DTYPE, BITS, CALL)                        \
  switch (t4a::any::elem_bytes(DTYPE)) {                               \
    case 1: CALL(1, 1); break;                                         \
    case 4: CALL(4, 4); break;                                         \
    case 8:                                                            \
      if (((BITS) & 7ull) == 0) CALL(8, 8); else CALL(8, 4);           \
      break;                                                           \
    case 16:                                                           \
      if (((BITS) & 15ull) == 0) CALL(16, 16);                         \
      else if (((BITS) & 7ull) == 0) CALL(16, 8);                      \
      else CALL(16, 4);                                                \
      break;                                                           \
    default: break;                                                    \
  }

#define T4A_ANY_BITS(P) reinterpret_cast<unsigned long long>(P)
