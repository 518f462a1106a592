// t4a_oracle: CPU restatement of the t4a-cuda-kernels hot path.
//
// TEST INFRASTRUCTURE ONLY: the checker and the timed CPU baseline.  Nothing in
// the shipped library links or calls this file.
//
// Built with -ffp-contract=off, so every multiply-add below rounds exactly as it
// is written; where the reference kernels fuse a multiply into an add, this file
// calls fma() explicitly.  Citations are into the reference project
// (tensor4all/t4a-cuda-kernels).

#include "t4a_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// Threading helper for the CPU baseline: a static partition of [0, n).
// ---------------------------------------------------------------------------
void parallel_for(long long n, int threads, const std::function<void(long long, long long)>& body) {
  if (threads <= 1 || n < 2) {
    body(0, n);
    return;
  }
  const long long parts = std::min<long long>(threads, n);
  std::vector<std::thread> pool;
  pool.reserve(parts);
  for (long long p = 0; p < parts; ++p) {
    const long long lo = n * p / parts;
    const long long hi = n * (p + 1) / parts;
    pool.emplace_back([&body, lo, hi]() { body(lo, hi); });
  }
  for (auto& thread : pool) thread.join();
}

// ---------------------------------------------------------------------------
// Device arithmetic conventions (reference tests/gpu_reduce.rs:2602-2800):
// IEEE round-to-nearest; an f32 NaN result is the canonical 0x7fffffff; an f64
// NaN result keeps a NaN operand's payload (quieted, left operand first) or is
// 0xfff8000000000000 when neither operand is NaN.  Extrema select an operand,
// NaN first (left, then right), and order -0.0 below +0.0.
// ---------------------------------------------------------------------------
inline float f32_nan_fix(float lhs, float rhs, float value) {
  (void)lhs;
  (void)rhs;
  if (value != value) {
    uint32_t bits = 0x7fffffffu;
    std::memcpy(&value, &bits, 4);
  }
  return value;
}

inline double f64_nan_fix(double lhs, double rhs, double value) {
  if (value == value) return value;
  uint64_t bits;
  if (lhs != lhs) {
    std::memcpy(&bits, &lhs, 8);
    bits |= 0x0008000000000000ull;
  } else if (rhs != rhs) {
    std::memcpy(&bits, &rhs, 8);
    bits |= 0x0008000000000000ull;
  } else {
    bits = 0xfff8000000000000ull;
  }
  std::memcpy(&value, &bits, 8);
  return value;
}

template <typename F>
inline F extremum(F lhs, F rhs, bool max) {
  if (lhs != lhs) return lhs;
  if (rhs != rhs) return rhs;
  if (lhs == F(0) && rhs == F(0)) {
    const bool positive = !std::signbit(lhs) || !std::signbit(rhs);
    const bool negative = std::signbit(lhs) || std::signbit(rhs);
    if (max) return positive ? F(0.0) : F(-0.0);
    return negative ? F(-0.0) : F(0.0);
  }
  if (max) return rhs > lhs ? rhs : lhs;
  return rhs < lhs ? rhs : lhs;
}

// Element arithmetic per type.  `add`, `mul`, `sq`, `max`, `min`.
template <typename T>
struct Arith;

template <>
struct Arith<float> {
  static float add(float a, float b) { return f32_nan_fix(a, b, a + b); }
  static float mul(float a, float b) { return f32_nan_fix(a, b, a * b); }
  static float sq(float a) { return f32_nan_fix(a, a, std::fmaf(a, a, 0.0f)); }
  static float max(float a, float b) { return extremum(a, b, true); }
  static float min(float a, float b) { return extremum(a, b, false); }
};

template <>
struct Arith<double> {
  static double add(double a, double b) { return f64_nan_fix(a, b, a + b); }
  static double mul(double a, double b) { return f64_nan_fix(a, b, a * b); }
  static double sq(double a) { return f64_nan_fix(a, a, std::fma(a, a, 0.0)); }
  static double max(double a, double b) { return extremum(a, b, true); }
  static double min(double a, double b) { return extremum(a, b, false); }
};

template <typename I, typename U>
struct IntArith {
  static I add(I a, I b) { return static_cast<I>(static_cast<U>(a) + static_cast<U>(b)); }
  static I mul(I a, I b) { return static_cast<I>(static_cast<U>(a) * static_cast<U>(b)); }
  static I sq(I a) { return mul(a, a); }
  static I max(I a, I b) { return a > b ? a : b; }
  static I min(I a, I b) { return a < b ? a : b; }
};
template <>
struct Arith<int32_t> : IntArith<int32_t, uint32_t> {};
template <>
struct Arith<int64_t> : IntArith<int64_t, uint64_t> {};

// Complex products round like the device's contracted form: the real part is
// fma(a.re, b.re, -(a.im * b.im)) and the imaginary part fma(a.im, b.re, a.re * b.im)
// (mode 3 below).  Of the five candidate forms this is the one that reproduces every
// complex PROD case of the reference golden bit for bit.
template <typename F>
struct Complex {
  F re;
  F im;
};

template <typename F>
inline F fused(F a, F b, F c);
template <>
inline float fused<float>(float a, float b, float c) { return std::fmaf(a, b, c); }
template <>
inline double fused<double>(double a, double b, double c) { return std::fma(a, b, c); }

template <typename F>
inline F fix(F a, F b, F v);
template <>
inline float fix<float>(float a, float b, float v) { return f32_nan_fix(a, b, v); }
template <>
inline double fix<double>(double a, double b, double v) { return f64_nan_fix(a, b, v); }

int g_complex_contraction = 3;  // 0: none, 1..4: which product of re/im is fused

template <typename F>
struct Arith<Complex<F>> {
  using C = Complex<F>;
  static C add(C a, C b) { return {fix(a.re, b.re, a.re + b.re), fix(a.im, b.im, a.im + b.im)}; }
  static C mul(C a, C b) {
    F re, im;
    if (g_complex_contraction == 0) {
      re = a.re * b.re - a.im * b.im;
      im = a.re * b.im + a.im * b.re;
    } else if (g_complex_contraction == 1) {
      re = fused(a.re, b.re, -(a.im * b.im));
      im = fused(a.re, b.im, a.im * b.re);
    } else if (g_complex_contraction == 2) {
      re = fused(-a.im, b.im, a.re * b.re);
      im = fused(a.im, b.re, a.re * b.im);
    } else if (g_complex_contraction == 3) {
      re = fused(a.re, b.re, -(a.im * b.im));
      im = fused(a.im, b.re, a.re * b.im);
    } else {
      re = fused(-a.im, b.im, a.re * b.re);
      im = fused(a.re, b.im, a.im * b.re);
    }
    // NaN results: the component conventions of the element type.
    if (re != re) re = fix(a.re, b.re, re);
    if (im != im) im = fix(a.re, b.im, im);
    return {re, im};
  }
  static C sq(C a) { return mul(a, a); }
  static C max(C a, C) { return a; }
  static C min(C a, C) { return a; }
};

using c32 = Complex<float>;
using c64 = Complex<double>;

// ---------------------------------------------------------------------------
// Reductions: fold objects (reference cuda/src/reduce.cu:30-108).
// ---------------------------------------------------------------------------
enum { OP_SUM = 0, OP_PROD = 1, OP_SUMSQ = 2, OP_MAX = 3, OP_MIN = 4 };

template <typename T>
struct Fold {
  int op;
  T seed(T x) const { return op == OP_SUMSQ ? Arith<T>::sq(x) : x; }
  T fold(T acc, T x) const {
    switch (op) {
      case OP_SUM: return Arith<T>::add(acc, x);
      case OP_PROD: return Arith<T>::mul(acc, x);
      case OP_SUMSQ: return Arith<T>::add(acc, Arith<T>::sq(x));
      case OP_MAX: return Arith<T>::max(acc, x);
      default: return Arith<T>::min(acc, x);
    }
  }
  T combine(T a, T b) const { return op == OP_SUMSQ ? Arith<T>::add(a, b) : fold(a, b); }
};

template <typename T>
constexpr int vector_lanes() {
  return 0;
}
template <>
constexpr int vector_lanes<float>() { return 4; }
template <>
constexpr int vector_lanes<double>() { return 2; }
template <>
constexpr int vector_lanes<int32_t>() { return 4; }
template <>
constexpr int vector_lanes<int64_t>() { return 2; }

// Lane 0's value of the ascending xor tree over `n` lanes: each level combines
// the lower half (left operand) with the upper half (reduce.cu:148-157).
template <typename T>
T xor_tree(const Fold<T>& f, const T* lanes, int n) {
  if (n == 1) return lanes[0];
  const int half = n / 2;
  return f.combine(xor_tree(f, lanes, half), xor_tree(f, lanes + half, half));
}

// Serial lane walk: lane t seeds from element t and folds t + k*W
// (reduce.cu:350-365 for pass 1, :259-308 for the plane walk).
template <typename T>
T serial_lane(const Fold<T>& f, const T* in, long long base, long long stride, long long start,
              long long end, int width, int lane) {
  long long index = start + lane;
  T acc = f.seed(in[base + index * stride]);
  for (index += width; index < end; index += width) acc = f.fold(acc, in[base + index * stride]);
  return acc;
}

// The revision-13 group walk over a contiguous chunk (reduce.cu:462-525).
template <typename T>
T vector_lane(const Fold<T>& f, const T* chunk, long long len, int width, int lane) {
  constexpr int V = vector_lanes<T>();
  const long long groups = len / V;
  const long long w = width;
  auto group = [&](long long g) -> T {
    const T* x = chunk + g * V;
    if (V == 4) {
      return f.combine(f.combine(f.seed(x[0]), f.seed(x[1])), f.combine(f.seed(x[2]), f.seed(x[3])));
    }
    return f.combine(f.seed(x[0]), f.seed(x[1]));
  };
  T acc = group(lane);
  for (int b = 1; b < 4; ++b) {
    if (lane + b * w < groups) acc = f.combine(acc, group(lane + b * w));
  }
  long long index = lane + 4 * w;
  for (; index + 3 * w < groups; index += 4 * w) {
    const T low = f.combine(group(index), group(index + w));
    const T high = f.combine(group(index + 2 * w), group(index + 3 * w));
    acc = f.combine(acc, f.combine(low, high));
  }
  for (int b = 0; b < 3; ++b) {
    if (index + b * w < groups) acc = f.combine(acc, group(index + b * w));
  }
  const long long tail_start = groups * V;
  if (lane < len - tail_start) acc = f.fold(acc, chunk[tail_start + lane]);
  return acc;
}

// One pass-1 cube: fold of chunk [start, end) of the axis at `base`
// (reduce.cu:528-555 walk choice, :587-633 body).
template <typename T>
T pass1_cube(const Fold<T>& f, const T* in, long long base, long long stride, long long start,
             long long end, int width) {
  T lanes[32];
  constexpr int V = vector_lanes<T>();
  const bool vector = V != 0 && f.op != OP_PROD && stride == 1 && (end - start) / V >= width;
  for (int lane = 0; lane < width; ++lane) {
    lanes[lane] = vector ? vector_lane(f, in + base + start, end - start, width, lane)
                         : serial_lane(f, in, base, stride, start, end, width, lane);
  }
  return xor_tree(f, lanes, width);
}

// A plane reduction of `len` elements with `width` lanes (direct plane strategy and
// the combine pass; reduce.cu:313-340, wide fold :170-194 is the same balanced tree).
template <typename T>
T plane_line(const Fold<T>& f, const T* in, long long base, long long stride, long long len,
             int width) {
  std::vector<T> lanes(width);
  for (int lane = 0; lane < width; ++lane) lanes[lane] = serial_lane(f, in, base, stride, 0, len, width, lane);
  return xor_tree(f, lanes.data(), width);
}

// Unit strategy: one serial fold over the whole axis (reduce.cu:198-224).
template <typename T>
T unit_line(const Fold<T>& f, const T* in, long long base, long long stride, long long len) {
  T acc = f.seed(in[base]);
  for (long long i = 1; i < len; ++i) acc = f.fold(acc, in[base + i * stride]);
  return acc;
}

bool op_supports(int op, int dtype) {
  switch (op) {
    case OP_SUM:
    case OP_PROD:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_I32 ||
             dtype == T4A_CUDA_I64 || dtype == T4A_CUDA_C32 || dtype == T4A_CUDA_C64;
    case OP_SUMSQ:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64;
    case OP_MAX:
    case OP_MIN:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_I32 ||
             dtype == T4A_CUDA_I64;
    default:
      return false;
  }
}

long long element_count(const t4a_cuda_layout& l) {
  long long n = 1;
  for (int d = 0; d < l.rank; ++d) n *= l.extents[d];
  return n;
}

template <typename T>
int reduce_typed(int op, T* out, const t4a_cuda_layout& out_l, const T* in,
                 const t4a_cuda_layout& in_l, int axis, int width, T* partials_out,
                 const t4a_oracle_reduce_topology& topo, int threads) {
  const long long outputs = element_count(out_l);
  const long long len = in_l.extents[axis];
  const long long stride = in_l.strides[axis];
  const Fold<T> f{op};
  const Fold<T> fc{topo.kind == 1 ? topo.combine_op : op};
  // Compact partials strides (input extents with the axis set to `splits`).
  long long pstrides[T4A_CUDA_MAX_RANK] = {0};
  if (topo.kind == 1) {
    long long s = 1;
    for (int d = 0; d < in_l.rank; ++d) {
      pstrides[d] = s;
      s *= d == axis ? topo.splits : in_l.extents[d];
    }
  }
  std::vector<T> scratch;
  T* partials = partials_out;
  if (topo.kind == 1 && partials == nullptr) {
    scratch.resize(static_cast<size_t>(outputs * topo.splits));
    partials = scratch.data();
  }
  parallel_for(outputs, threads, [&](long long lo, long long hi) {
    for (long long o = lo; o < hi; ++o) {
      long long rest = o, base = in_l.offset, out_off = out_l.offset, pbase = 0;
      for (int d = 0; d < out_l.rank; ++d) {
        const long long c = rest % out_l.extents[d];
        rest /= out_l.extents[d];
        base += c * in_l.strides[d];
        out_off += c * out_l.strides[d];
        pbase += c * pstrides[d];
      }
      T result;
      if (topo.kind == 0) {
        result = topo.direct_strategy == T4A_CUDA_REDUCE_UNIT ? unit_line(f, in, base, stride, len)
                                                              : plane_line(f, in, base, stride, len, width);
      } else {
        const long long splits = topo.splits, chunk = topo.chunk_len;
        for (long long s = 0; s < splits; ++s) {
          const long long start = s * chunk;
          const long long end = s + 1 == splits ? len : start + chunk;
          partials[pbase + s * pstrides[axis]] = pass1_cube(f, in, base, stride, start, end, width);
        }
        result = topo.combine_strategy == T4A_CUDA_REDUCE_UNIT
                     ? unit_line(fc, partials, pbase, pstrides[axis], splits)
                     : plane_line(fc, partials, pbase, pstrides[axis], splits, topo.combine_width);
      }
      out[out_off] = result;
    }
  });
  return 0;
}

}  // namespace

extern "C" {

// Restated planner choices: split_policy (src/lib.rs:3152-3166), strategy_for
// (:3235-3241), combine_geometry and combine_block_width (:3435-3455).
int t4a_oracle_reduce_topology_for(int op, long long len, int width, t4a_oracle_reduce_topology* t) {
  if (width != 8 && width != 16 && width != 32) return -1;
  std::memset(t, 0, sizeof(*t));
  long long splits = len / (static_cast<long long>(width) * 8);
  splits = std::min<long long>(std::max<long long>(splits, 1), 4096);
  if (len < 1 || splits <= 1) {
    t->kind = 0;
    t->direct_strategy = len <= width ? T4A_CUDA_REDUCE_UNIT : T4A_CUDA_REDUCE_PLANE;
    return 0;
  }
  t->kind = 1;
  t->splits = splits;
  t->chunk_len = len / splits;
  t->combine_op = op == OP_SUMSQ ? OP_SUM : op;
  if (t->combine_op == OP_PROD || splits < 64) {
    t->combine_strategy = splits <= width ? T4A_CUDA_REDUCE_UNIT : T4A_CUDA_REDUCE_PLANE;
    t->combine_width = width;
  } else {
    const long long target = splits / 8;
    int w = 64;
    while (w < target && w < 512) w *= 2;
    t->combine_strategy = T4A_CUDA_REDUCE_PLANE;
    t->combine_width = std::min(w, 512);
  }
  return 0;
}

static int reduce_dispatch(int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                           const void* in, const t4a_cuda_layout* in_layout, int axis, int width,
                           void* partials, t4a_oracle_reduce_topology* topo_out, int threads) {
  if (!op_supports(op, dtype) || axis < 0 || axis >= in_layout->rank) return -1;
  t4a_oracle_reduce_topology topo;
  if (t4a_oracle_reduce_topology_for(op, in_layout->extents[axis], width, &topo) != 0) return -1;
  if (topo_out) *topo_out = topo;
  switch (dtype) {
    case T4A_CUDA_F32:
      return reduce_typed(op, (float*)out, *out_layout, (const float*)in, *in_layout, axis, width,
                          (float*)partials, topo, threads);
    case T4A_CUDA_F64:
      return reduce_typed(op, (double*)out, *out_layout, (const double*)in, *in_layout, axis, width,
                          (double*)partials, topo, threads);
    case T4A_CUDA_I32:
      return reduce_typed(op, (int32_t*)out, *out_layout, (const int32_t*)in, *in_layout, axis,
                          width, (int32_t*)partials, topo, threads);
    case T4A_CUDA_I64:
      return reduce_typed(op, (int64_t*)out, *out_layout, (const int64_t*)in, *in_layout, axis,
                          width, (int64_t*)partials, topo, threads);
    case T4A_CUDA_C32:
      return reduce_typed(op, (c32*)out, *out_layout, (const c32*)in, *in_layout, axis, width,
                          (c32*)partials, topo, threads);
    case T4A_CUDA_C64:
      return reduce_typed(op, (c64*)out, *out_layout, (const c64*)in, *in_layout, axis, width,
                          (c64*)partials, topo, threads);
    default:
      return -1;
  }
}

int t4a_oracle_reduce(int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                      const void* in, const t4a_cuda_layout* in_layout, int axis, int width,
                      void* partials, t4a_oracle_reduce_topology* topo_out) {
  return reduce_dispatch(dtype, op, out, out_layout, in, in_layout, axis, width, partials, topo_out, 1);
}

int t4a_oracle_reduce_threaded(int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                               const void* in, const t4a_cuda_layout* in_layout, int axis,
                               int width, int threads) {
  return reduce_dispatch(dtype, op, out, out_layout, in, in_layout, axis, width, nullptr, nullptr,
                         threads);
}

// Test hook: which contraction form the complex product uses (see Arith<Complex>).
int t4a_oracle_set_complex_contraction(int mode) {
  const int old = g_complex_contraction;
  g_complex_contraction = mode;
  return old;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Movement (reference cuda/src/movement.cu:98-145 bodies, :213-262 transpose tile,
// :412-438 broadcast).  Element moves are byte copies, so dtype only sets the size.
// ---------------------------------------------------------------------------
namespace {

int dtype_size(int dtype) {
  switch (dtype) {
    case T4A_CUDA_F32: return 4;
    case T4A_CUDA_F64: return 8;
    case T4A_CUDA_I32: return 4;
    case T4A_CUDA_I64: return 8;
    case T4A_CUDA_BOOL: return 1;
    case T4A_CUDA_C32: return 8;
    case T4A_CUDA_C64: return 16;
    default: return 0;
  }
}

inline long long decode(long long flat, const t4a_cuda_layout& l, const long long* strides, long long offset) {
  for (int d = 0; d < l.rank; ++d) {
    const long long c = flat % l.extents[d];
    flat /= l.extents[d];
    offset += c * strides[d];
  }
  return offset;
}

}  // namespace

extern "C" {

int t4a_oracle_strided_to_strided(int dtype, void* dst, const void* src, const t4a_cuda_layout* s,
                                  const t4a_cuda_layout* d, int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*s);
  parallel_for(len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) {
      const long long si = decode(f, *s, s->strides, s->offset);
      const long long di = decode(f, *s, d->strides, d->offset);
      std::memcpy((char*)dst + di * es, (const char*)src + si * es, es);
    }
  });
  return 0;
}

int t4a_oracle_materialize_strided(int dtype, void* dst, const void* src, const t4a_cuda_layout* s,
                                   int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*s);
  parallel_for(len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) {
      const long long si = decode(f, *s, s->strides, s->offset);
      std::memcpy((char*)dst + f * es, (const char*)src + si * es, es);
    }
  });
  return 0;
}

int t4a_oracle_contiguous_to_view(int dtype, void* dst, const void* src, const t4a_cuda_layout* d,
                                  int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*d);
  parallel_for(len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) {
      const long long di = decode(f, *d, d->strides, d->offset);
      std::memcpy((char*)dst + di * es, (const char*)src + f * es, es);
    }
  });
  return 0;
}

// dst[b*S + i + j*M] = src[src_offset + b*S + i*N + j], M = dst_fast_extent,
// N = src_fast_extent (docs/abi/c-kernel-abi.md "Tiled transpose").
int t4a_oracle_tiled_transpose(int dtype, void* dst, const void* src, long long src_offset,
                               long long batch_stride, long long m, long long n, long long batches,
                               int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  parallel_for(batches * m, threads, [&](long long lo, long long hi) {
    for (long long bi = lo; bi < hi; ++bi) {
      const long long b = bi / m, i = bi % m;
      for (long long j = 0; j < n; ++j) {
        std::memcpy((char*)dst + (b * batch_stride + i + j * m) * es,
                    (const char*)src + (src_offset + b * batch_stride + i * n + j) * es, es);
      }
    }
  });
  return 0;
}

int t4a_oracle_broadcast_in_dim(int dtype, void* out, const void* in, const t4a_cuda_layout* o,
                                const t4a_cuda_layout* i, const t4a_cuda_axis_values* dims,
                                int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*o);
  parallel_for(len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) {
      long long coords[T4A_CUDA_MAX_RANK] = {0};
      long long rest = f;
      for (int d = 0; d < o->rank; ++d) {
        coords[d] = rest % o->extents[d];
        rest /= o->extents[d];
      }
      long long index = i->offset;
      for (int s = 0; s < dims->rank; ++s) {
        const long long c = i->extents[s] == 1 ? 0 : coords[dims->values[s]];
        index += c * i->strides[s];
      }
      std::memcpy((char*)out + f * es, (const char*)in + index * es, es);
    }
  });
  return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Gather and additive scatter (reference cuda/src/gather_scatter.cu:22-32 clamp,
// :52-127 gather, :131-276 scatter).
// ---------------------------------------------------------------------------
namespace {

template <typename I>
long long clamp_start(I start, long long dim, long long window) {
  const long long max_start = dim > window ? dim - window : 0;
  if (!(start > static_cast<I>(0))) return 0;
  // A float start at or above 2^64 (+inf included) converts to the largest u64 on
  // the device (cvt.rzi saturates); C++ leaves that conversion undefined.
  if (static_cast<double>(start) >= 18446744073709551616.0) return max_start;
  const unsigned long long raw = static_cast<unsigned long long>(start);
  return raw < static_cast<unsigned long long>(max_start) ? static_cast<long long>(raw) : max_start;
}

template <typename I>
long long read_start(const void* indices, long long at, long long dim, long long window) {
  return clamp_start<I>(static_cast<const I*>(indices)[at], dim, window);
}

long long start_of(int index_dtype, const void* indices, long long at, long long dim, long long window) {
  switch (index_dtype) {
    case T4A_CUDA_F32: return read_start<float>(indices, at, dim, window);
    case T4A_CUDA_F64: return read_start<double>(indices, at, dim, window);
    case T4A_CUDA_I32: return read_start<int32_t>(indices, at, dim, window);
    default: return read_start<int64_t>(indices, at, dim, window);
  }
}

int index_batch_axis(int position, bool vector_present, int index_vector_dim) {
  return position + ((vector_present && position >= index_vector_dim) ? 1 : 0);
}

}  // namespace

extern "C" {

int t4a_oracle_gather(int dtype, int index_dtype, void* out, const void* operand, const void* indices,
                      const t4a_cuda_layout* ol, const t4a_cuda_layout* opl,
                      const t4a_cuda_layout* il, const t4a_cuda_gather_plan* plan, int threads) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*ol);
  const bool vector_present = plan->index_vector_dim < il->rank;
  const long long component_stride = vector_present ? il->strides[plan->index_vector_dim] : 0;
  parallel_for(len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) {
      long long in_index = opl->offset, out_index = ol->offset, ibase = il->offset, rest = f;
      int batch_position = 0;
      for (int a = 0; a < ol->rank; ++a) {
        const long long c = rest % ol->extents[a];
        rest /= ol->extents[a];
        out_index += c * ol->strides[a];
        int window_pos = -1;
        for (int p = 0; p < plan->window_rank; ++p) {
          if (plan->offset_dims[p] == a) {
            window_pos = p;
            break;
          }
        }
        if (window_pos >= 0) {
          in_index += c * opl->strides[plan->window_dims[window_pos]];
        } else {
          const int tensor_axis = index_batch_axis(batch_position, vector_present, plan->index_vector_dim);
          ibase += c * il->strides[tensor_axis];
          ++batch_position;
        }
      }
      for (int comp = 0; comp < plan->start_map_len; ++comp) {
        const int axis = static_cast<int>(plan->start_index_map[comp]);
        in_index += start_of(index_dtype, indices, ibase + comp * component_stride, opl->extents[axis],
                             plan->slice_sizes[axis]) *
                    opl->strides[axis];
      }
      std::memcpy((char*)out + out_index * es, (const char*)operand + in_index * es, es);
    }
  });
  return 0;
}

int t4a_oracle_scatter_add(int dtype, int index_dtype, void* out, const void* indices,
                           const void* updates, const t4a_cuda_layout* ol,
                           const t4a_cuda_layout* il, const t4a_cuda_layout* ul,
                           const t4a_cuda_scatter_plan* plan, int threads) {
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64 && dtype != T4A_CUDA_C32 && dtype != T4A_CUDA_C64)
    return -1;
  const long long len = element_count(*ul);
  const bool vector_present = plan->index_vector_dim < il->rank;
  const long long component_stride = vector_present ? il->strides[plan->index_vector_dim] : 0;
  auto window_shape = [&](int axis) -> long long {
    long long shape = 1;
    for (int p = 0; p < plan->window_rank; ++p) {
      if (plan->window_dims[p] == axis) shape = ul->extents[plan->update_window_dims[p]];
    }
    return shape;
  };
  // Destination of update element f, or -1 when its window does not fit.
  auto destination = [&](long long f) -> long long {
    long long base[T4A_CUDA_MAX_RANK] = {0};
    long long window_offset = 0, ibase = il->offset, rest = f;
    int batch_position = 0;
    for (int a = 0; a < ul->rank; ++a) {
      const long long c = rest % ul->extents[a];
      rest /= ul->extents[a];
      int window_pos = -1;
      for (int p = 0; p < plan->window_rank; ++p) {
        if (plan->update_window_dims[p] == a) {
          window_pos = p;
          break;
        }
      }
      if (window_pos >= 0) {
        window_offset += c * ol->strides[plan->window_dims[window_pos]];
      } else {
        const int tensor_axis = index_batch_axis(batch_position, vector_present, plan->index_vector_dim);
        ibase += c * il->strides[tensor_axis];
        ++batch_position;
      }
    }
    for (int comp = 0; comp < plan->scatter_map_len; ++comp) {
      const int axis = static_cast<int>(plan->scatter_dims[comp]);
      base[axis] += start_of(index_dtype, indices, ibase + comp * component_stride, ol->extents[axis],
                             window_shape(axis));
    }
    long long offset = ol->offset;
    for (int a = 0; a < ol->rank; ++a) {
      if (base[a] + window_shape(a) > ol->extents[a]) return -1;
      offset += base[a] * ol->strides[a];
    }
    return offset + window_offset;
  };
  // Serial in update order; `threads` > 1 partitions destinations, so each thread
  // scans every update and applies only those landing in its own range, which keeps
  // the per-destination order serial.
  const long long out_span = [&]() {
    long long hi = ol->offset;
    for (int a = 0; a < ol->rank; ++a) hi += (ol->extents[a] - 1) * std::max<long long>(ol->strides[a], 0);
    return hi + 1;
  }();
  std::vector<long long> dest(len);
  const long long upd_len = len;
  parallel_for(upd_len, threads, [&](long long lo, long long hi) {
    for (long long f = lo; f < hi; ++f) dest[f] = destination(f);
  });
  parallel_for(out_span, threads, [&](long long lo, long long hi) {
    for (long long f = 0; f < upd_len; ++f) {
      const long long dst = dest[f];
      if (dst < lo || dst >= hi) continue;
      const long long src = decode(f, *ul, ul->strides, ul->offset);
      switch (dtype) {
        case T4A_CUDA_F32: ((float*)out)[dst] += ((const float*)updates)[src]; break;
        case T4A_CUDA_F64: ((double*)out)[dst] += ((const double*)updates)[src]; break;
        case T4A_CUDA_C32:
          ((float*)out)[2 * dst] += ((const float*)updates)[2 * src];
          ((float*)out)[2 * dst + 1] += ((const float*)updates)[2 * src + 1];
          break;
        default:
          ((double*)out)[2 * dst] += ((const double*)updates)[2 * src];
          ((double*)out)[2 * dst + 1] += ((const double*)updates)[2 * src + 1];
          break;
      }
    }
  });
  return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// RRQR primitives (reference cuda/src/rrqr.cu).  Every plane sum is the 32-lane
// walk (lane l folds rows start + l + 32k in order) followed by the ascending xor
// tree, and the multiply-adds the reference kernels contract are fma() here, so
// F64 norms, reflectors, trailing updates and pivots are reproduced bit for bit.
// ---------------------------------------------------------------------------
namespace {

constexpr int kPlane = 32;
constexpr long long kNone = 0x7fffffffffffffffLL;

inline double magnitude(double v) { return v < 0.0 ? -v : v; }
inline float magnitude(float v) { return v < 0.0f ? -v : v; }
inline double magnitude(c64 v) { return std::hypot(v.re, v.im); }
inline float magnitude(c32 v) { return std::hypot(v.re, v.im); }

template <typename F>
F tree_sum(const F* lanes, int n) {
  if (n == 1) return lanes[0];
  return tree_sum(lanes, n / 2) + tree_sum(lanes + n / 2, n / 2);
}

template <typename F>
F tree_max(const F* lanes, int n) {
  if (n == 1) return lanes[0];
  const F a = tree_max(lanes, n / 2), b = tree_max(lanes + n / 2, n / 2);
  return b > a ? b : a;
}

long long batch_offset(long long batch, const t4a_cuda_layout& l, int first_axis) {
  long long offset = 0, rest = batch;
  for (int a = first_axis; a < l.rank; ++a) {
    offset += (rest % l.extents[a]) * l.strides[a];
    rest /= l.extents[a];
  }
  return offset;
}

long long batch_count(const t4a_cuda_layout& l, int first_axis) {
  long long n = 1;
  for (int a = first_axis; a < l.rank; ++a) n *= l.extents[a];
  return n;
}

// Max-scaled 2-norm of rows [step, rows) of one column (rrqr.cu:144-190, :285-310).
// `invalid` non-NULL selects the column_norms form, whose maximum skips a
// non-finite magnitude and flags it; the reflector form (NULL) folds it.
template <typename T, typename F>
F scaled_norm(const T* x, long long base, long long row_stride, long long step, long long rows,
              bool* invalid) {
  F local_max[kPlane], local_sum[kPlane];
  bool bad = false;
  for (int lane = 0; lane < kPlane; ++lane) {
    F m = F(0);
    for (long long row = step + lane; row < rows; row += kPlane) {
      const F value = magnitude(x[base + row * row_stride]);
      if (invalid != nullptr && value - value != F(0)) {
        bad = true;
      } else if (value > m) {
        m = value;
      }
    }
    local_max[lane] = m;
  }
  const F scale = tree_max(local_max, kPlane);
  for (int lane = 0; lane < kPlane; ++lane) {
    F s = F(0);
    if (scale > F(0)) {
      for (long long row = step + lane; row < rows; row += kPlane) {
        const F scaled = magnitude(x[base + row * row_stride]) / scale;
        s = fused(scaled, scaled, s);
      }
    }
    local_sum[lane] = s;
  }
  if (invalid) *invalid = bad;
  return scale * std::sqrt(tree_sum(local_sum, kPlane));
}

template <typename T, typename F>
void column_norms_t(const T* work, F* norms, const t4a_cuda_layout& w, const t4a_cuda_layout& nl,
                    long long step, int threads) {
  const long long rows = w.extents[0], cols = w.extents[1], trailing = cols - step;
  const long long tasks = batch_count(w, 2) * trailing;
  parallel_for(tasks, threads, [&](long long lo, long long hi) {
    for (long long task = lo; task < hi; ++task) {
      const long long batch = task / trailing, column = step + task % trailing;
      const long long base = w.offset + column * w.strides[1] + batch_offset(batch, w, 2);
      bool invalid = false;
      const F norm = scaled_norm<T, F>(work, base, w.strides[0], step, rows, &invalid);
      const bool bad = invalid || norm - norm != F(0);
      norms[nl.offset + column * nl.strides[0] + batch_offset(batch, nl, 1)] = bad ? F(-1) : norm;
    }
  });
}

template <typename F>
void select_pivot_t(const F* norms, const long long* perm, long long* pivots, long long* status,
                    const t4a_cuda_layout& nl, const t4a_cuda_layout& pl, long long step) {
  const long long batches = batch_count(nl, 1), columns = nl.extents[0];
  for (long long batch = 0; batch < batches; ++batch) {
    const long long nbase = nl.offset + batch_offset(batch, nl, 1);
    const long long pbase = pl.offset + batch_offset(batch, pl, 1);
    F lmax[kPlane];
    long long lorig[kPlane], lcol[kPlane];
    bool invalid = false;
    for (int lane = 0; lane < kPlane; ++lane) {
      F m = F(0);
      long long orig = kNone, col = kNone;
      for (long long column = step + lane; column < columns; column += kPlane) {
        const F norm = norms[nbase + column * nl.strides[0]];
        const long long original = perm[pbase + column * pl.strides[0]];
        if (norm < F(0)) {
          invalid = true;
        } else if (norm > m || (norm == m && original < orig)) {
          m = norm;
          orig = original;
          col = column;
        }
      }
      lmax[lane] = m;
      lorig[lane] = orig;
      lcol[lane] = col;
    }
    const F maximum = tree_max(lmax, kPlane);
    long long original = kNone;
    for (int lane = 0; lane < kPlane; ++lane)
      if (lmax[lane] == maximum) original = std::min(original, lorig[lane]);
    long long selected = kNone;
    for (int lane = 0; lane < kPlane; ++lane)
      if (lmax[lane] == maximum && lorig[lane] == original) selected = std::min(selected, lcol[lane]);
    pivots[batch] = selected == kNone ? step : selected;
    if (invalid) status[batch] = 1;
  }
}

template <typename T>
void swap_columns_t(T* work, long long* perm, const long long* pivots, const t4a_cuda_layout& w,
                    const t4a_cuda_layout& pl, long long step) {
  const long long rows = w.extents[0], batches = batch_count(w, 2);
  for (long long batch = 0; batch < batches; ++batch) {
    const long long pivot = pivots[batch];
    if (pivot == step) continue;
    for (long long row = 0; row < rows; ++row) {
      const long long base = w.offset + row * w.strides[0] + batch_offset(batch, w, 2);
      std::swap(work[base + step * w.strides[1]], work[base + pivot * w.strides[1]]);
    }
    const long long pbase = pl.offset + batch_offset(batch, pl, 1);
    std::swap(perm[pbase + step * pl.strides[0]], perm[pbase + pivot * pl.strides[0]]);
  }
}

// Householder reflector of column `step` in place (rrqr.cu:312-335 real).
template <typename F>
void reflector_real_t(F* work, F* coeff, const t4a_cuda_layout& w, const t4a_cuda_layout& cl, long long step) {
  const long long batches = batch_count(w, 2), rows = w.extents[0];
  for (long long batch = 0; batch < batches; ++batch) {
    const long long base = w.offset + step * w.strides[1] + batch_offset(batch, w, 2);
    const long long rs = w.strides[0];
    const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
    const F norm = scaled_norm<F, F>(work, base, rs, step, rows, nullptr);
    const F x0 = work[base + step * rs];
    if (norm == F(0)) {
      coeff[ci] = F(0);
      continue;
    }
    const F phase = x0 < F(0) ? F(-1) : F(1);
    const F alpha = -phase * norm;
    const F denominator = x0 - alpha;
    for (long long row = step + 1; row < rows; ++row) work[base + row * rs] /= denominator;
    work[base + step * rs] = alpha;
    coeff[ci] = F(1) + magnitude(x0) / norm;
  }
}

template <typename F>
Complex<F> cdiv(Complex<F> n, Complex<F> d) {
  const F norm = d.re * d.re + d.im * d.im;
  return {(n.re * d.re + n.im * d.im) / norm, (n.im * d.re - n.re * d.im) / norm};
}

template <typename F>
void reflector_complex_t(Complex<F>* work, Complex<F>* coeff, const t4a_cuda_layout& w,
                         const t4a_cuda_layout& cl, long long step) {
  using C = Complex<F>;
  const long long batches = batch_count(w, 2), rows = w.extents[0];
  for (long long batch = 0; batch < batches; ++batch) {
    const long long base = w.offset + step * w.strides[1] + batch_offset(batch, w, 2);
    const long long rs = w.strides[0];
    const long long ci = cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1);
    const F norm = scaled_norm<C, F>(work, base, rs, step, rows, nullptr);
    const C x0 = work[base + step * rs];
    if (norm == F(0)) {
      coeff[ci] = C{F(0), F(0)};
      continue;
    }
    const F x0_abs = magnitude(x0);
    const C phase = x0_abs == F(0) ? C{F(1), F(0)} : C{x0.re / x0_abs, x0.im / x0_abs};
    const C alpha{-phase.re * norm, -phase.im * norm};
    const C denominator{x0.re - alpha.re, x0.im - alpha.im};
    for (long long row = step + 1; row < rows; ++row) work[base + row * rs] = cdiv(work[base + row * rs], denominator);
    work[base + step * rs] = alpha;
    coeff[ci] = C{F(1) + x0_abs / norm, F(0)};
  }
}

// Apply reflector `step` to target columns (rrqr.cu:386-401 real).
template <typename F>
void apply_real_t(const F* packed, F* target, const F* coeff, const t4a_cuda_layout& pl,
                  const t4a_cuda_layout& tl, const t4a_cuda_layout& cl, long long step,
                  long long first_column, long long column_count, int threads) {
  const long long batches = batch_count(pl, 2), rows = pl.extents[0];
  parallel_for(batches * column_count, threads, [&](long long lo, long long hi) {
    for (long long task = lo; task < hi; ++task) {
      const long long batch = task / column_count, column = first_column + task % column_count;
      const long long pb = pl.offset + step * pl.strides[1] + batch_offset(batch, pl, 2);
      const long long tb = tl.offset + column * tl.strides[1] + batch_offset(batch, tl, 2);
      const F c = coeff[cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1)];
      F lanes[kPlane];
      for (int lane = 0; lane < kPlane; ++lane) {
        F dot = F(0);
        for (long long row = step + lane; row < rows; row += kPlane) {
          const F v = row == step ? F(1) : packed[pb + row * pl.strides[0]];
          dot = fused(v, target[tb + row * tl.strides[0]], dot);
        }
        lanes[lane] = dot;
      }
      const F dot = tree_sum(lanes, kPlane) * c;
      for (long long row = step; row < rows; ++row) {
        const F v = row == step ? F(1) : packed[pb + row * pl.strides[0]];
        F& t = target[tb + row * tl.strides[0]];
        t = fused(-v, dot, t);
      }
    }
  });
}

template <typename F>
void apply_complex_t(const Complex<F>* packed, Complex<F>* target, const Complex<F>* coeff,
                     const t4a_cuda_layout& pl, const t4a_cuda_layout& tl, const t4a_cuda_layout& cl,
                     long long step, long long first_column, long long column_count, int threads) {
  using C = Complex<F>;
  const long long batches = batch_count(pl, 2), rows = pl.extents[0];
  parallel_for(batches * column_count, threads, [&](long long lo, long long hi) {
    for (long long task = lo; task < hi; ++task) {
      const long long batch = task / column_count, column = first_column + task % column_count;
      const long long pb = pl.offset + step * pl.strides[1] + batch_offset(batch, pl, 2);
      const long long tb = tl.offset + column * tl.strides[1] + batch_offset(batch, tl, 2);
      const C c = coeff[cl.offset + step * cl.strides[0] + batch_offset(batch, cl, 1)];
      F re_l[kPlane], im_l[kPlane];
      for (int lane = 0; lane < kPlane; ++lane) {
        F re = F(0), im = F(0);
        for (long long row = step + lane; row < rows; row += kPlane) {
          const C v = row == step ? C{F(1), F(0)} : packed[pb + row * pl.strides[0]];
          const C x = target[tb + row * tl.strides[0]];
          re += v.re * x.re + v.im * x.im;
          im += v.re * x.im - v.im * x.re;
        }
        re_l[lane] = re;
        im_l[lane] = im;
      }
      const F sr = tree_sum(re_l, kPlane), si = tree_sum(im_l, kPlane);
      const C dot{sr * c.re - si * c.im, sr * c.im + si * c.re};
      for (long long row = step; row < rows; ++row) {
        const C v = row == step ? C{F(1), F(0)} : packed[pb + row * pl.strides[0]];
        C& t = target[tb + row * tl.strides[0]];
        const C p = Arith<C>::mul(v, dot);
        t = C{t.re - p.re, t.im - p.im};
      }
    }
  });
}

}  // namespace

extern "C" {

int t4a_oracle_initialize_permutation(long long* perm, long long n, long long len) {
  if (n <= 0) return -1;
  for (long long p = 0; p < len; ++p) perm[p] = p % n;
  return 0;
}

int t4a_oracle_column_norms(int dtype, const void* work, void* norms, const t4a_cuda_layout* w,
                            const t4a_cuda_layout* nl, long long step, int threads) {
  switch (dtype) {
    case T4A_CUDA_F32: column_norms_t<float, float>((const float*)work, (float*)norms, *w, *nl, step, threads); return 0;
    case T4A_CUDA_F64: column_norms_t<double, double>((const double*)work, (double*)norms, *w, *nl, step, threads); return 0;
    case T4A_CUDA_C32: column_norms_t<c32, float>((const c32*)work, (float*)norms, *w, *nl, step, threads); return 0;
    case T4A_CUDA_C64: column_norms_t<c64, double>((const c64*)work, (double*)norms, *w, *nl, step, threads); return 0;
    default: return -1;
  }
}

int t4a_oracle_select_pivot(int dtype, const void* norms, const long long* perm, long long* pivots,
                            long long* status, const t4a_cuda_layout* nl, const t4a_cuda_layout* pl,
                            long long step) {
  switch (dtype) {
    case T4A_CUDA_F32: select_pivot_t<float>((const float*)norms, perm, pivots, status, *nl, *pl, step); return 0;
    case T4A_CUDA_F64: select_pivot_t<double>((const double*)norms, perm, pivots, status, *nl, *pl, step); return 0;
    default: return -1;
  }
}

int t4a_oracle_swap_columns(int dtype, void* work, long long* perm, const long long* pivots,
                            const t4a_cuda_layout* w, const t4a_cuda_layout* pl, long long step) {
  switch (dtype_size(dtype)) {
    case 4: swap_columns_t<int32_t>((int32_t*)work, perm, pivots, *w, *pl, step); return 0;
    case 8: swap_columns_t<int64_t>((int64_t*)work, perm, pivots, *w, *pl, step); return 0;
    case 16: swap_columns_t<c64>((c64*)work, perm, pivots, *w, *pl, step); return 0;
    default: return -1;
  }
}

int t4a_oracle_reflector(int dtype, void* work, void* coeff, const t4a_cuda_layout* w,
                         const t4a_cuda_layout* cl, long long step) {
  switch (dtype) {
    case T4A_CUDA_F32: reflector_real_t<float>((float*)work, (float*)coeff, *w, *cl, step); return 0;
    case T4A_CUDA_F64: reflector_real_t<double>((double*)work, (double*)coeff, *w, *cl, step); return 0;
    case T4A_CUDA_C32: reflector_complex_t<float>((c32*)work, (c32*)coeff, *w, *cl, step); return 0;
    case T4A_CUDA_C64: reflector_complex_t<double>((c64*)work, (c64*)coeff, *w, *cl, step); return 0;
    default: return -1;
  }
}

int t4a_oracle_apply_reflector(int dtype, const void* packed, void* target, const void* coeff,
                               const t4a_cuda_layout* pl, const t4a_cuda_layout* tl,
                               const t4a_cuda_layout* cl, long long step, long long first_column,
                               long long column_count, int threads) {
  switch (dtype) {
    case T4A_CUDA_F32: apply_real_t<float>((const float*)packed, (float*)target, (const float*)coeff, *pl, *tl, *cl, step, first_column, column_count, threads); return 0;
    case T4A_CUDA_F64: apply_real_t<double>((const double*)packed, (double*)target, (const double*)coeff, *pl, *tl, *cl, step, first_column, column_count, threads); return 0;
    case T4A_CUDA_C32: apply_complex_t<float>((const c32*)packed, (c32*)target, (const c32*)coeff, *pl, *tl, *cl, step, first_column, column_count, threads); return 0;
    case T4A_CUDA_C64: apply_complex_t<double>((const c64*)packed, (c64*)target, (const c64*)coeff, *pl, *tl, *cl, step, first_column, column_count, threads); return 0;
    default: return -1;
  }
}

// Restates linalg_aux.cu:200-211: the element at flat position f (axis 0 fastest) holds
// one exactly when its row equals start + its column.
int t4a_oracle_identity_shifted(int dtype, void* out, const t4a_cuda_layout* l, long long start) {
  const int es = dtype_size(dtype);
  if (!es || l->rank < 2 || dtype == T4A_CUDA_BOOL) return -1;
  const long long len = element_count(*l);
  for (long long f = 0; f < len; ++f) {
    const long long row = f % l->extents[0];
    const long long col = (f / l->extents[0]) % l->extents[1];
    const long long batch = f / (l->extents[0] * l->extents[1]);
    char* dst = (char*)out + (l->offset + row * l->strides[0] + col * l->strides[1] + batch_offset(batch, *l, 2)) * es;
    std::memset(dst, 0, es);
    if (row != start + col) continue;
    switch (dtype) {
      case T4A_CUDA_F32: case T4A_CUDA_C32: { const float one = 1.0f; std::memcpy(dst, &one, 4); break; }
      case T4A_CUDA_F64: case T4A_CUDA_C64: { const double one = 1.0; std::memcpy(dst, &one, 8); break; }
      case T4A_CUDA_I32: { const int one = 1; std::memcpy(dst, &one, 4); break; }
      case T4A_CUDA_I64: { const long long one = 1; std::memcpy(dst, &one, 8); break; }
      default: return -1;
    }
  }
  return 0;
}

int t4a_oracle_extract_r(int dtype, const void* work, void* r, const t4a_cuda_layout* w,
                         const t4a_cuda_layout* rl) {
  const int es = dtype_size(dtype);
  if (!es) return -1;
  const long long len = element_count(*rl);
  for (long long f = 0; f < len; ++f) {
    const long long row = f % rl->extents[0];
    const long long col = (f / rl->extents[0]) % rl->extents[1];
    const long long batch = f / (rl->extents[0] * rl->extents[1]);
    char* dst = (char*)r + (rl->offset + row * rl->strides[0] + col * rl->strides[1] + batch_offset(batch, *rl, 2)) * es;
    if (row <= col) {
      std::memcpy(dst, (const char*)work + (w->offset + row * w->strides[0] + col * w->strides[1] + batch_offset(batch, *w, 2)) * es, es);
    } else {
      std::memset(dst, 0, es);
    }
  }
  return 0;
}

}  // extern "C"

namespace {
template <typename T, typename F>
void prefix_rank_t(const T* r, long long* rank, long long* status, const t4a_cuda_layout& rl, F rtol, F atol) {
  const long long batches = batch_count(rl, 2), k = rl.extents[0];
  for (long long batch = 0; batch < batches; ++batch) {
    const long long base = rl.offset + batch_offset(batch, rl, 2);
    const F leading = magnitude(r[base]);
    const F relative = rtol * leading;
    const F threshold = atol > relative ? atol : relative;
    long long failure = kNone;
    bool invalid = false;
    for (long long d = 0; d < k; ++d) {
      const F value = magnitude(r[base + d * rl.strides[0] + d * rl.strides[1]]);
      if (value - value != F(0)) invalid = true;
      if (!(value > threshold) && d < failure) failure = d;
    }
    rank[batch] = failure == kNone ? k : failure;
    if (invalid) status[batch] = 1;
  }
}
}  // namespace

extern "C" {

int t4a_oracle_prefix_rank(int dtype, const void* r, long long* rank, long long* status,
                           const t4a_cuda_layout* rl, double rtol, double atol) {
  switch (dtype) {
    case T4A_CUDA_F32: prefix_rank_t<float, float>((const float*)r, rank, status, *rl, (float)rtol, (float)atol); return 0;
    case T4A_CUDA_F64: prefix_rank_t<double, double>((const double*)r, rank, status, *rl, rtol, atol); return 0;
    case T4A_CUDA_C32: prefix_rank_t<c32, float>((const c32*)r, rank, status, *rl, (float)rtol, (float)atol); return 0;
    case T4A_CUDA_C64: prefix_rank_t<c64, double>((const c64*)r, rank, status, *rl, rtol, atol); return 0;
    default: return -1;
  }
}

long long t4a_oracle_rrqr_f64(double* work, long long m, long long n, long long steps, long long* perm,
                              double* coeff, double rtol, double atol, int threads) {
  t4a_cuda_layout w{};
  w.rank = 2;
  w.extents[0] = m;
  w.extents[1] = n;
  w.strides[0] = 1;
  w.strides[1] = m;
  t4a_cuda_layout vec{};
  vec.rank = 1;
  vec.extents[0] = n;
  vec.strides[0] = 1;
  t4a_cuda_layout cl = vec;
  cl.extents[0] = steps;
  std::vector<double> norms(n);
  long long pivot = 0, status = 0;
  t4a_oracle_initialize_permutation(perm, n, n);
  for (long long step = 0; step < steps; ++step) {
    column_norms_t<double, double>(work, norms.data(), w, vec, step, threads);
    select_pivot_t<double>(norms.data(), perm, &pivot, &status, vec, vec, step);
    swap_columns_t<double>(work, perm, &pivot, w, vec, step);
    reflector_real_t<double>(work, coeff, w, cl, step);
    if (n - step - 1 > 0) apply_real_t<double>(work, work, coeff, w, w, cl, step, step + 1, n - step - 1, threads);
  }
  // R = triu(work[:steps, :]); rank from its diagonal.
  t4a_cuda_layout rl{};
  rl.rank = 2;
  rl.extents[0] = steps;
  rl.extents[1] = n;
  rl.strides[0] = 1;
  rl.strides[1] = steps;
  std::vector<double> r(steps * n);
  t4a_oracle_extract_r(T4A_CUDA_F64, work, r.data(), &w, &rl);
  long long rank = 0, rstatus = 0;
  prefix_rank_t<double, double>(r.data(), &rank, &rstatus, rl, rtol, atol);
  return rank;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Row-sharded RRQR (the restatement of t4a_dist_rrqr, which has no reference
// counterpart: the reference has no multi-device code).  A rank holds rows
// [row0, row0 + mr) of every column, column-major with column stride ld.  Every chain
// runs the reference's lane order over the rank's own rows (lane l visits the rows
// first + l + 32 k of the rank's range), every plane sum is the ascending xor tree, and
// the parts meet in rank order with separately rounded products and sums.  The four
// functions are one rank's share of a step; t4a_oracle_rrqr_rows_sharded_f64 runs the
// ranks of one matrix in turn, exchanging their parts as the all-gathers would.
// ---------------------------------------------------------------------------
namespace {

constexpr int kPartElems = 8;  // scale, ssq, rscale, rssq, xrow, bad, own, pad

long long dist_local_from(long long s, long long row0, long long mr) {
  const long long lo = s - row0;
  return lo < 0 ? 0 : (lo > mr ? mr : lo);
}

// Lane chains over rows [lo, mr) of one column: max-scaled parts (flagged or not).
void dist_scaled_parts(const double* col, long long lo, long long mr, bool flagged, double* scale_out,
                       double* ssq_out, bool* bad_out) {
  double lmax[kPlane], lsum[kPlane];
  bool bad = false;
  for (int lane = 0; lane < kPlane; ++lane) {
    double m = 0.0;
    for (long long r = lo + lane; r < mr; r += kPlane) {
      const double v = magnitude(col[r]);
      if (flagged && v - v != 0.0) {
        bad = true;
      } else if (v > m) {
        m = v;
      }
    }
    lmax[lane] = m;
  }
  const double scale = tree_max(lmax, kPlane);
  for (int lane = 0; lane < kPlane; ++lane) {
    double s = 0.0;
    if (scale > 0.0 && !(flagged && bad))
      for (long long r = lo + lane; r < mr; r += kPlane) {
        const double q = magnitude(col[r]) / scale;
        s = std::fma(q, q, s);
      }
    lsum[lane] = s;
  }
  *scale_out = scale;
  *ssq_out = (flagged && bad) ? 0.0 : tree_sum(lsum, kPlane);
  if (bad_out) *bad_out = bad;
}

double dist_combined(const double* parts, int world, long long count, long long idx, bool reflector) {
  double scale = 0.0;
  bool bad = false;
  for (int r = 0; r < world; ++r) {
    const double* p = parts + (r * count + idx) * kPartElems;
    const double sc = reflector ? p[2] : p[0];
    bad = bad || p[5] != 0.0;
    scale = sc > scale ? sc : scale;
  }
  if (!reflector && bad) return -1.0;
  double ssq = 0.0;
  for (int r = 0; r < world; ++r) {
    const double* p = parts + (r * count + idx) * kPartElems;
    const double sc = reflector ? p[2] : p[0];
    if (sc > 0.0) {
      const double ratio = sc == scale ? 1.0 : sc / scale;
      const double w = ratio * ratio;
      const double term = w * (reflector ? p[3] : p[1]);
      ssq = ssq + term;
    }
  }
  const double norm = scale * std::sqrt(ssq);
  return !reflector && norm - norm != 0.0 ? -1.0 : norm;
}

}  // namespace

extern "C" {

// Norm parts of columns first_col .. n-1 over this rank's rows at global rows >= s.
int t4a_oracle_dist_norm_parts(const double* local, long long mr, long long n, long long ld, long long row0,
                               long long s, long long first_col, double* parts) {
  const long long lo = dist_local_from(s, row0, mr);
  const bool holds = s >= row0 && s < row0 + mr;
  for (long long j = first_col; j < n; ++j) {
    const double* col = local + j * ld;
    double* p = parts + (j - first_col) * kPartElems;
    bool bad = false;
    dist_scaled_parts(col, lo, mr, true, &p[0], &p[1], &bad);
    if (bad) {
      dist_scaled_parts(col, lo, mr, false, &p[2], &p[3], nullptr);
    } else {
      p[2] = p[0];
      p[3] = p[1];
    }
    p[4] = holds ? col[s - row0] : 0.0;
    p[5] = bad ? 1.0 : 0.0;
    p[6] = holds ? 1.0 : 0.0;
    p[7] = 0.0;
  }
  return 0;
}

// Step s's pivot, reflector scalars, column swap and scaling of this rank's rows, from
// every rank's parts of columns s .. n-1 (world blocks of n - s parts).  perm, coeff,
// pivots and status are this rank's replicated copies.
int t4a_oracle_dist_select_swap(double* local, long long mr, long long n, long long ld, long long row0, long long s,
                                const double* parts, int world, long long* perm, double* coeff, long long* pivots,
                                long long* status) {
  const long long count = n - s;
  std::vector<double> norms(n, 0.0);
  for (long long c = s; c < n; ++c) norms[c] = dist_combined(parts, world, count, c - s, false);
  t4a_cuda_layout vec{};
  vec.rank = 1;
  vec.extents[0] = n;
  vec.strides[0] = 1;
  long long pivot = 0;
  select_pivot_t<double>(norms.data(), perm, &pivot, status, vec, vec, s);
  double norm = norms[pivot];
  if (!(norm >= 0.0)) norm = dist_combined(parts, world, count, pivot - s, true);
  double x0 = 0.0;
  for (int r = 0; r < world; ++r) {
    const double* p = parts + (r * count + (pivot - s)) * kPartElems;
    if (p[6] != 0.0) x0 = p[4];
  }
  pivots[s] = pivot;
  const bool scale = norm != 0.0;
  double alpha = 0.0, divisor = 1.0;
  if (scale) {
    const double phase = x0 < 0.0 ? -1.0 : 1.0;
    alpha = -phase * norm;
    divisor = x0 - alpha;
    coeff[s] = 1.0 + magnitude(x0) / norm;
  } else {
    coeff[s] = 0.0;
  }
  for (long long i = 0; i < mr; ++i) {
    const long long g = row0 + i;
    const double left = local[s * ld + i];
    double moved = pivot == s ? left : local[pivot * ld + i];
    if (scale) {
      if (g == s) {
        moved = alpha;
      } else if (g > s) {
        moved = moved / divisor;
      }
    }
    local[s * ld + i] = moved;
    if (pivot != s) local[pivot * ld + i] = left;
  }
  if (pivot != s) std::swap(perm[s], perm[pivot]);
  return 0;
}

// Dot parts of step s: chains of v t over this rank's rows >= s (v_s = 1 on its owner),
// for columns s+1 .. n-1.
int t4a_oracle_dist_dot_parts(const double* local, long long mr, long long n, long long ld, long long row0,
                              long long s, double* dots) {
  const long long lo = dist_local_from(s, row0, mr);
  const bool holds = s >= row0 && s < row0 + mr;
  const double* v = local + s * ld;
  for (long long j = s + 1; j < n; ++j) {
    const double* t = local + j * ld;
    double lanes[kPlane];
    for (int lane = 0; lane < kPlane; ++lane) {
      double acc = 0.0;
      for (long long r = lo + lane; r < mr; r += kPlane) acc = std::fma(r == lo && holds ? 1.0 : v[r], t[r], acc);
      lanes[lane] = acc;
    }
    dots[j - s - 1] = tree_sum(lanes, kPlane);
  }
  return 0;
}

// Update of step s on this rank's rows: d = (rank-ordered sum of every rank's dot part)
// * coeff[s], t -= v d.
int t4a_oracle_dist_update(double* local, long long mr, long long n, long long ld, long long row0, long long s,
                           const double* dots, int world, const double* coeff) {
  const long long lo = dist_local_from(s, row0, mr);
  const bool holds = s >= row0 && s < row0 + mr;
  const long long count = n - s - 1;
  const double* v = local + s * ld;
  for (long long j = s + 1; j < n; ++j) {
    double d = dots[j - s - 1];
    for (int r = 1; r < world; ++r) d = d + dots[r * count + (j - s - 1)];
    d = d * coeff[s];
    double* t = local + j * ld;
    for (long long r = lo; r < mr; ++r) t[r] = std::fma(-(r == lo && holds ? 1.0 : v[r]), d, t[r]);
  }
  return 0;
}

// The whole row-sharded factorization of one column-major [m, n] matrix, its rows split
// into `world` balanced blocks (the first m % world hold one row more), the ranks run in
// turn.  perm (n), coeff (steps), pivots (steps) are the replicated results; returns the
// status word (bit 0: a non-finite norm).
long long t4a_oracle_rrqr_rows_sharded_f64(double* work, long long m, long long n, long long steps, int world,
                                           long long* perm, double* coeff, long long* pivots) {
  std::vector<long long> row0(world), mr(world);
  for (int r = 0; r < world; ++r) {
    const long long base = m / world, extra = m % world;
    row0[r] = r * base + std::min<long long>(r, extra);
    mr[r] = base + (r < extra ? 1 : 0);
  }
  // Each rank's block as its own column-major buffer.
  std::vector<std::vector<double>> blocks(world);
  for (int r = 0; r < world; ++r) {
    blocks[r].resize(mr[r] * n);
    for (long long j = 0; j < n; ++j)
      for (long long i = 0; i < mr[r]; ++i) blocks[r][j * mr[r] + i] = work[j * m + row0[r] + i];
  }
  std::vector<std::vector<long long>> perms(world, std::vector<long long>(n));
  std::vector<std::vector<double>> coeffs(world, std::vector<double>(std::max<long long>(steps, 1)));
  std::vector<std::vector<long long>> pivs(world, std::vector<long long>(std::max<long long>(steps, 1)));
  std::vector<long long> status(world, 0);
  for (int r = 0; r < world; ++r)
    for (long long c = 0; c < n; ++c) perms[r][c] = c;
  std::vector<double> parts(world * n * kPartElems), dots(world * n);
  for (int r = 0; r < world; ++r)
    t4a_oracle_dist_norm_parts(blocks[r].data(), mr[r], n, mr[r], row0[r], 0, 0, parts.data() + r * n * kPartElems);
  for (long long s = 0; s < steps; ++s) {
    for (int r = 0; r < world; ++r)
      t4a_oracle_dist_select_swap(blocks[r].data(), mr[r], n, mr[r], row0[r], s, parts.data(), world,
                                  perms[r].data(), coeffs[r].data(), pivs[r].data(), &status[r]);
    const long long count = n - s - 1;
    if (count <= 0) continue;
    for (int r = 0; r < world; ++r)
      t4a_oracle_dist_dot_parts(blocks[r].data(), mr[r], n, mr[r], row0[r], s, dots.data() + r * count);
    for (int r = 0; r < world; ++r)
      t4a_oracle_dist_update(blocks[r].data(), mr[r], n, mr[r], row0[r], s, dots.data(), world, coeffs[r].data());
    if (s + 1 < steps)
      for (int r = 0; r < world; ++r)
        t4a_oracle_dist_norm_parts(blocks[r].data(), mr[r], n, mr[r], row0[r], s + 1, s + 1,
                                   parts.data() + r * count * kPartElems);
  }
  for (int r = 0; r < world; ++r)
    for (long long j = 0; j < n; ++j)
      for (long long i = 0; i < mr[r]; ++i) work[j * m + row0[r] + i] = blocks[r][j * mr[r] + i];
  for (long long c = 0; c < n; ++c) perm[c] = perms[0][c];
  for (long long s = 0; s < steps; ++s) {
    coeff[s] = coeffs[0][s];
    pivots[s] = pivs[0][s];
  }
  return status[0];
}

}  // extern "C"
