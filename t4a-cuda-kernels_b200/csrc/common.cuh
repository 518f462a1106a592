// Device helpers shared by the t4a_b200 kernels (sm_100a).
//
// Element arithmetic follows the kernel ABI's contract (reference
// docs/abi/c-kernel-abi.md "Arithmetic semantics", cuda/include/t4a/abi.cuh:590-818):
// IEEE float arithmetic without fast math or flush-to-zero, wrapping integer
// arithmetic, NaN-propagating extrema, squares rounded once through fma, and
// the complex product in its contracted form.
#pragma once

#include <cstdint>

#include "../../include/t4a_b200/abi.h"

namespace t4a {

constexpr int kMaxRank = T4A_CUDA_MAX_RANK;
constexpr int kWarp = 32;

using c32 = t4a_cuda_c32;
using c64 = t4a_cuda_c64;

// ---- element arithmetic ----------------------------------------------------
template <typename T>
struct Num {
  static __device__ __forceinline__ T add(T a, T b) { return a + b; }
  static __device__ __forceinline__ T mul(T a, T b) { return a * b; }
};

template <>
struct Num<int> {
  static __device__ __forceinline__ int add(int a, int b) {
    return static_cast<int>(static_cast<unsigned>(a) + static_cast<unsigned>(b));
  }
  static __device__ __forceinline__ int mul(int a, int b) {
    return static_cast<int>(static_cast<unsigned>(a) * static_cast<unsigned>(b));
  }
};

template <>
struct Num<long long> {
  static __device__ __forceinline__ long long add(long long a, long long b) {
    return static_cast<long long>(static_cast<unsigned long long>(a) + static_cast<unsigned long long>(b));
  }
  static __device__ __forceinline__ long long mul(long long a, long long b) {
    return static_cast<long long>(static_cast<unsigned long long>(a) * static_cast<unsigned long long>(b));
  }
};

// Complex products: re = fma(a.re, b.re, -(a.im*b.im)), im = fma(a.im, b.re, a.re*b.im).
// Written with explicit fma so the rounding does not depend on the compiler's
// contraction choices; this is the form whose results match the reference golden.
template <>
struct Num<c32> {
  static __device__ __forceinline__ c32 add(c32 a, c32 b) { return {a.re + b.re, a.im + b.im}; }
  static __device__ __forceinline__ c32 mul(c32 a, c32 b) {
    return {__fmaf_rn(a.re, b.re, -__fmul_rn(a.im, b.im)), __fmaf_rn(a.im, b.re, __fmul_rn(a.re, b.im))};
  }
};

template <>
struct Num<c64> {
  static __device__ __forceinline__ c64 add(c64 a, c64 b) { return {a.re + b.re, a.im + b.im}; }
  static __device__ __forceinline__ c64 mul(c64 a, c64 b) {
    return {__fma_rn(a.re, b.re, -__dmul_rn(a.im, b.im)), __fma_rn(a.im, b.re, __dmul_rn(a.re, b.im))};
  }
};

__device__ __forceinline__ float square(float x) { return __fmaf_rn(x, x, 0.0f); }
__device__ __forceinline__ double square(double x) { return __fma_rn(x, x, 0.0); }
template <typename T>
__device__ __forceinline__ T square(T x) { return Num<T>::mul(x, x); }

// NaN-propagating extrema: the ordered extremum (-0.0 below +0.0), NaN when either
// operand is NaN.  F32 uses the one-instruction max.NaN / min.NaN (a canonical NaN);
// F64, which has no such form, returns the NaN operand (the left one first).  Only
// "is NaN" is part of the ABI's contract, not the payload.
__device__ __forceinline__ float nan_max(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ double nan_max(double a, double b) {
  const double m = fmax(a, b);
  const double r = b != b ? b : m;
  return a != a ? a : r;
}
__device__ __forceinline__ float nan_min(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ double nan_min(double a, double b) {
  const double m = fmin(a, b);
  const double r = b != b ? b : m;
  return a != a ? a : r;
}
template <typename T>
__device__ __forceinline__ T nan_max(T a, T b) { return a > b ? a : b; }
template <typename T>
__device__ __forceinline__ T nan_min(T a, T b) { return a < b ? a : b; }

// ---- fold objects ----------------------------------------------------------
// seed: the accumulator's first value from the axis' first element;
// fold: accumulator folds one element; combine: two accumulators meet.
struct OpSum {
  static constexpr bool kRegroup = true;
  template <typename T> __device__ __forceinline__ T seed(T x) const { return x; }
  template <typename T> __device__ __forceinline__ T fold(T a, T x) const { return Num<T>::add(a, x); }
  template <typename T> __device__ __forceinline__ T combine(T a, T b) const { return Num<T>::add(a, b); }
};
struct OpProd {
  static constexpr bool kRegroup = false;
  template <typename T> __device__ __forceinline__ T seed(T x) const { return x; }
  template <typename T> __device__ __forceinline__ T fold(T a, T x) const { return Num<T>::mul(a, x); }
  template <typename T> __device__ __forceinline__ T combine(T a, T b) const { return Num<T>::mul(a, b); }
};
struct OpSumSq {
  static constexpr bool kRegroup = true;
  template <typename T> __device__ __forceinline__ T seed(T x) const { return square(x); }
  template <typename T> __device__ __forceinline__ T fold(T a, T x) const { return Num<T>::add(a, square(x)); }
  template <typename T> __device__ __forceinline__ T combine(T a, T b) const { return Num<T>::add(a, b); }
};
struct OpMax {
  static constexpr bool kRegroup = true;
  template <typename T> __device__ __forceinline__ T seed(T x) const { return x; }
  template <typename T> __device__ __forceinline__ T fold(T a, T x) const { return nan_max(a, x); }
  template <typename T> __device__ __forceinline__ T combine(T a, T b) const { return nan_max(a, b); }
};
struct OpMin {
  static constexpr bool kRegroup = true;
  template <typename T> __device__ __forceinline__ T seed(T x) const { return x; }
  template <typename T> __device__ __forceinline__ T fold(T a, T x) const { return nan_min(a, x); }
  template <typename T> __device__ __forceinline__ T combine(T a, T b) const { return nan_min(a, b); }
};

// ---- warp shuffles for every element type ---------------------------------
template <typename T>
__device__ __forceinline__ T shfl_xor(T v, int offset, unsigned mask) { return __shfl_xor_sync(mask, v, offset); }
template <>
__device__ __forceinline__ c32 shfl_xor<c32>(c32 v, int offset, unsigned mask) {
  return {__shfl_xor_sync(mask, v.re, offset), __shfl_xor_sync(mask, v.im, offset)};
}
template <>
__device__ __forceinline__ c64 shfl_xor<c64>(c64 v, int offset, unsigned mask) {
  return {__shfl_xor_sync(mask, v.re, offset), __shfl_xor_sync(mask, v.im, offset)};
}

// Lanes of this thread's warp that exist in the block (a block narrower than a warp
// leaves the upper lanes empty).
__device__ __forceinline__ unsigned warp_mask_of_block() {
  const int threads = blockDim.x * blockDim.y * blockDim.z;
  return threads >= 32 ? 0xffffffffu : ((1u << threads) - 1u);
}

// Ascending xor tree over aligned groups of `width` lanes (width <= 32): lane 0 of
// each group ends with the balanced tree of the group's values in lane order.
template <typename Op, typename T>
__device__ __forceinline__ T lane_tree(T v, int width, Op op) {
  const unsigned mask = warp_mask_of_block();
  for (int offset = 1; offset < width; offset <<= 1) v = op.combine(v, shfl_xor(v, offset, mask));
  return v;
}

// ---- 16-byte vectors ---------------------------------------------------------
template <typename T>
struct VecOf {
  static constexpr int kLanes = 16 / static_cast<int>(sizeof(T));
};
template <>
struct VecOf<c32> {
  static constexpr int kLanes = 1;  // component-aligned only
};

// A V-element vector; V > 1 only when V * sizeof(T) == 16, and then it is one
// 16-byte load (the caller proves the alignment).  V == 1 keeps the element's own
// alignment, so a component-aligned complex element is never loaded as 16 bytes.
template <typename T, int V>
struct alignas(V > 1 ? 16 : alignof(T)) Vec {
  T v[V];
};

template <typename T, int V>
__device__ __forceinline__ Vec<T, V> load_vec(const T* p) {
  if constexpr (V > 1 && V * sizeof(T) == 16) {
    return *reinterpret_cast<const Vec<T, V>*>(p);
  } else {
    Vec<T, V> r;
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = p[i];
    return r;
  }
}

// ---- layout helpers ----------------------------------------------------------
// Offset of flat index `flat` decoded over `extents` (axis 0 fastest) with `strides`.
__device__ __forceinline__ long long decode_offset(long long flat, const t4a_cuda_layout& l,
                                                   const long long* strides, long long offset) {
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d < l.rank) {
      const long long e = l.extents[d];
      offset += (flat % e) * strides[d];
      flat /= e;
    }
  }
  return offset;
}

__device__ __forceinline__ long long layout_count(const t4a_cuda_layout& l) {
  long long n = 1;
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d)
    if (d < l.rank) n *= l.extents[d];
  return n;
}

__device__ __forceinline__ int block_threads() { return blockDim.x * blockDim.y * blockDim.z; }
__device__ __forceinline__ int flat_tid() {
  return threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z);
}

}  // namespace t4a
