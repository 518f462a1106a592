// Host-side validation shared by the t4a_plan_* planners: a restatement of the
// reference's LayoutRef checks and small require_* rules (src/lib.rs:332-450,
// :949-1027, :1457-1482, :2065-2090, :3604-3620, :4051-4066).
#pragma once

#include <climits>
#include <cstdint>
#include <cstring>

#include "../../include/t4a_b200.h"

namespace t4a {
namespace plan {

constexpr unsigned kFlatBlock = 256;
constexpr unsigned kPlaneBlock = 32;
constexpr unsigned kMaxGridX = 0x7fffffffu;
constexpr unsigned kMaxGridYZ = 65535u;

#define T4A_TRY(expr)            \
  do {                           \
    const int t4a_rc_ = (expr);  \
    if (t4a_rc_ != T4A_OK) return t4a_rc_; \
  } while (0)

inline bool mul_overflows(long long a, long long b, long long* out) { return __builtin_mul_overflow(a, b, out); }
inline bool add_overflows(long long a, long long b, long long* out) { return __builtin_add_overflow(a, b, out); }

inline int dtype_size(int dtype) {
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

// A layout is well formed: rank 0..8 and no negative extent (Layout::new).
inline int check_layout(const t4a_cuda_layout* l) {
  if (l == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (l->rank < 0 || l->rank > T4A_CUDA_MAX_RANK) return T4A_ERR_RANK_OUT_OF_RANGE;
  for (int d = 0; d < l->rank; ++d)
    if (l->extents[d] < 0) return T4A_ERR_NEGATIVE_EXTENT;
  return T4A_OK;
}

inline int element_count(const t4a_cuda_layout& l, long long* count) {
  long long n = 1;
  for (int d = 0; d < l.rank; ++d)
    if (mul_overflows(n, l.extents[d], &n)) return T4A_ERR_OVERFLOW;
  *count = n;
  return T4A_OK;
}

inline int reachable(const t4a_cuda_layout& l, bool maximum, long long* out) {
  long long total = l.offset;
  for (int d = 0; d < l.rank; ++d) {
    long long step;
    if (mul_overflows(l.extents[d] - 1, l.strides[d], &step)) return T4A_ERR_OVERFLOW;
    step = maximum ? (step > 0 ? step : 0) : (step < 0 ? step : 0);
    if (add_overflows(total, step, &total)) return T4A_ERR_OVERFLOW;
  }
  *out = total;
  return T4A_OK;
}

// LayoutRef::check_span: every reachable element index lies in [0, len).
inline int check_span(const t4a_cuda_layout& l, long long len, int element_size) {
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  long long count;
  T4A_TRY(element_count(l, &count));
  if (count == 0) return T4A_OK;
  long long lo, hi;
  T4A_TRY(reachable(l, false, &lo));
  T4A_TRY(reachable(l, true, &hi));
  if (lo < 0 || hi >= len) return T4A_ERR_OFFSET_OUT_OF_SPAN;
  long long bytes;
  if (mul_overflows(hi, element_size, &bytes)) return T4A_ERR_OVERFLOW;
  return T4A_OK;
}

inline bool is_compact(const t4a_cuda_layout& l) {
  if (l.offset != 0) return false;
  long long stride = 1;
  for (int d = 0; d < l.rank; ++d) {
    if (l.strides[d] != stride) return false;
    if (mul_overflows(stride, l.extents[d], &stride)) return false;
  }
  return true;
}

inline int require_compact(const t4a_cuda_layout& l) { return is_compact(l) ? T4A_OK : T4A_ERR_NOT_COMPACT; }

// require_destination: no broadcast axis with more than one element.
inline int require_destination(const t4a_cuda_layout& l) {
  for (int d = 0; d < l.rank; ++d)
    if (l.extents[d] > 1 && l.strides[d] == 0) return T4A_ERR_BROADCAST_DESTINATION;
  return T4A_OK;
}

inline int require_axis(long long axis, int rank) { return axis >= 0 && axis < rank ? T4A_OK : T4A_ERR_INVALID_AXIS; }

inline int require_matrix(const t4a_cuda_layout& l) { return l.rank >= 2 ? T4A_OK : T4A_ERR_RANK_OUT_OF_RANGE; }

inline int extent_product(const long long* extents, int n, long long* out) {
  long long p = 1;
  for (int i = 0; i < n; ++i)
    if (mul_overflows(p, extents[i], &p)) return T4A_ERR_OVERFLOW;
  *out = p;
  return T4A_OK;
}

inline t4a_launch empty_launch() {
  t4a_launch l;
  std::memset(&l, 0, sizeof(l));
  l.block[0] = kFlatBlock;
  l.block[1] = 1;
  l.block[2] = 1;
  return l;
}

inline t4a_launch make_launch(unsigned long long grid, unsigned bx, unsigned by, unsigned smem, int variant) {
  t4a_launch l;
  std::memset(&l, 0, sizeof(l));
  l.grid[0] = static_cast<unsigned>(grid);
  l.grid[1] = grid == 0 ? 0 : 1;
  l.grid[2] = grid == 0 ? 0 : 1;
  l.block[0] = bx;
  l.block[1] = by;
  l.block[2] = 1;
  l.shared_bytes = smem;
  l.variant = variant;
  return l;
}

inline unsigned long long ceil_div(unsigned long long a, unsigned long long b) { return (a + b - 1) / b; }

inline int grid_of(unsigned long long units, unsigned long long per_block, unsigned long long* grid) {
  const unsigned long long g = ceil_div(units, per_block);
  if (g > kMaxGridX) return T4A_ERR_LAUNCH_LIMIT;
  *grid = g;
  return T4A_OK;
}

}  // namespace plan
}  // namespace t4a
