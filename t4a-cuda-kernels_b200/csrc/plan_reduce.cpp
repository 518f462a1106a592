// Reduction planning: the reference's validation and Auto policy (src/lib.rs:3033-3557)
// with this library's launch geometry.
//
// Numerical topology is set by the plan alone: the split count and chunk length
// (split_policy), the pass-1 plane width W, and the combine pass's strategy and width
// (combine_geometry).  These are kept exactly as the reference computes them, so a
// reduction planned here folds the same elements in the same order as the reference.
// Only the geometry (grid, block, dynamic shared memory, path) is this library's.
#include "plan_common.h"
#include "reduce_paths.h"

namespace t4a {
namespace plan {
namespace {

constexpr long long kMinChunkPlanes = 8;
constexpr long long kMaxSplits = 4096;
constexpr long long kWideCombineMinSplits = 64;
constexpr long long kCombineFoldsPerLane = 8;

bool op_supports(int op, int dtype) {
  switch (op) {
    case T4A_CUDA_REDUCE_SUM:
    case T4A_CUDA_REDUCE_PROD:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_I32 ||
             dtype == T4A_CUDA_I64 || dtype == T4A_CUDA_C32 || dtype == T4A_CUDA_C64;
    case T4A_CUDA_REDUCE_SUM_SQUARES:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64;
    case T4A_CUDA_REDUCE_MAX:
    case T4A_CUDA_REDUCE_MIN:
      return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_I32 ||
             dtype == T4A_CUDA_I64;
    default:
      return false;
  }
}

int combine_op_of(int op) { return op == T4A_CUDA_REDUCE_SUM_SQUARES ? T4A_CUDA_REDUCE_SUM : op; }

bool plane_width_ok(unsigned w) { return w == 8 || w == 16 || w == 32; }
bool combine_width_ok(unsigned w) { return w == 64 || w == 128 || w == 256 || w == 512; }

int strategy_for(long long len, unsigned w) {
  return len <= static_cast<long long>(w) ? T4A_CUDA_REDUCE_UNIT : T4A_CUDA_REDUCE_PLANE;
}

// reduce_problem (src/lib.rs:3193-3233).
int reduce_problem(int dtype, int op, const t4a_cuda_layout* out, long long out_len,
                   const t4a_cuda_layout* in, long long in_len, unsigned axis, long long* reduce_len,
                   long long* output_len) {
  T4A_TRY(check_layout(out));
  T4A_TRY(check_layout(in));
  if (!op_supports(op, dtype)) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_axis(axis, in->rank));
  if (out->rank != in->rank) return T4A_ERR_RANK_LENGTH;
  for (int d = 0; d < in->rank; ++d)
    if (d != static_cast<int>(axis) && out->extents[d] != in->extents[d]) return T4A_ERR_SHAPE_MISMATCH;
  if (out->extents[axis] != 1) return T4A_ERR_SHAPE_MISMATCH;
  *reduce_len = in->extents[axis];
  if (*reduce_len < 1) return T4A_ERR_NEGATIVE_COUNT;
  T4A_TRY(element_count(*out, output_len));
  T4A_TRY(require_destination(*out));
  T4A_TRY(check_span(*in, in_len, dtype_size(dtype)));
  T4A_TRY(check_span(*out, out_len, dtype_size(dtype)));
  return T4A_OK;
}

// Geometry of a pass over `src` (the input, or the partials for the combine pass):
// which kernel path serves it and its grid/block/shared memory.
int pass_geometry(int dtype, int strategy, unsigned w, const t4a_cuda_layout& src, unsigned axis,
                  long long outputs, long long splits, bool partials_pass, t4a_launch* launch) {
  if (outputs == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  const int esize = dtype_size(dtype);
  unsigned long long grid = 0;
  const unsigned by = kTileThreads / (w <= 32 ? w : kTileThreads);
  if (partials_pass || (strategy == T4A_CUDA_REDUCE_PLANE && w <= 32)) {
    const int vec = strided_vec_lanes(dtype);
    if (strided_path_applies(src, static_cast<int>(axis), static_cast<int>(w), vec)) {
      const InnerRun run = inner_run(src, static_cast<int>(axis));
      const unsigned long long slots =
          static_cast<unsigned long long>(run.ext / vec) * outer_count(src, static_cast<int>(axis), run.r);
      T4A_TRY(grid_of(slots, kSlotsPerTile, &grid));
      grid *= static_cast<unsigned long long>(splits);
      if (grid > kMaxGridX) return T4A_ERR_LAUNCH_LIMIT;
      *launch = make_launch(grid, 32, kTileThreads / 32, kStridedSmem, kPathStrided);
      return T4A_OK;
    }
    T4A_TRY(grid_of(static_cast<unsigned long long>(outputs) * splits, kTileThreads / w, &grid));
    *launch = make_launch(grid, w, by, 0, kPathCubes);
    return T4A_OK;
  }
  if (strategy == T4A_CUDA_REDUCE_PLANE) {  // wider than a warp
    T4A_TRY(grid_of(outputs, 1, &grid));
    *launch = make_launch(grid, w, 1, 0, kPathWide);
    return T4A_OK;
  }
  const int rows = unit_rows_per_tile(src, static_cast<int>(axis), esize);
  if (rows > 0) {
    T4A_TRY(grid_of(outputs, rows, &grid));
    *launch = make_launch(grid, w, by, unit_rows_smem(src, rows, esize), kPathUnitRows);
    return T4A_OK;
  }
  T4A_TRY(grid_of(outputs, kTileThreads, &grid));
  *launch = make_launch(grid, w, by, 0, kPathUnit);
  return T4A_OK;
}

int partials_layout_for(const t4a_cuda_layout& in, unsigned axis, long long splits, t4a_cuda_layout* out) {
  std::memset(out, 0, sizeof(*out));
  out->rank = in.rank;
  long long stride = 1;
  for (int d = 0; d < in.rank; ++d) {
    out->extents[d] = d == static_cast<int>(axis) ? splits : in.extents[d];
    out->strides[d] = stride;
    if (mul_overflows(stride, out->extents[d], &stride)) return T4A_ERR_OVERFLOW;
  }
  return T4A_OK;
}

}  // namespace
}  // namespace plan
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;

extern "C" {

int t4a_split_policy(long long len, unsigned w, int* has_split, t4a_split* split) {
  if (has_split == nullptr || split == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (!plane_width_ok(w)) return T4A_ERR_INVALID_PLANE_WIDTH;
  *has_split = 0;
  split->splits = 1;
  split->chunk_len = len;
  if (len < 1) return T4A_OK;
  long long splits = len / (static_cast<long long>(w) * kMinChunkPlanes);
  splits = splits < 1 ? 1 : (splits > kMaxSplits ? kMaxSplits : splits);
  if (splits <= 1) return T4A_OK;
  *has_split = 1;
  split->splits = splits;
  split->chunk_len = len / splits;
  return T4A_OK;
}

int t4a_plan_reduce(int dtype, int op, int strategy, const t4a_cuda_layout* out, long long out_len,
                    const t4a_cuda_layout* in, long long in_len, unsigned axis, unsigned w,
                    t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  // check_reduce_width (src/lib.rs:3291).
  if (strategy == T4A_CUDA_REDUCE_UNIT) {
    if (!plane_width_ok(w)) return T4A_ERR_INVALID_PLANE_WIDTH;
  } else if (strategy == T4A_CUDA_REDUCE_PLANE) {
    if (!plane_width_ok(w) && !combine_width_ok(w)) return T4A_ERR_INVALID_PLANE_WIDTH;
  } else {
    return T4A_ERR_UNSUPPORTED_OP;
  }
  long long len, outputs;
  T4A_TRY(reduce_problem(dtype, op, out, out_len, in, in_len, axis, &len, &outputs));
  // check_strategy (src/lib.rs:3299).
  if (strategy == T4A_CUDA_REDUCE_UNIT && len > static_cast<long long>(w)) return T4A_ERR_STRATEGY_MISMATCH;
  if (strategy == T4A_CUDA_REDUCE_PLANE && len < static_cast<long long>(w)) return T4A_ERR_STRATEGY_MISMATCH;
  // launch_for's grid limits (src/lib.rs:3243-3289).
  if (strategy == T4A_CUDA_REDUCE_UNIT) {
    if (ceil_div(static_cast<unsigned long long>(outputs), w) > kMaxGridX) return T4A_ERR_LAUNCH_LIMIT;
  } else if (static_cast<unsigned long long>(outputs) > kMaxGridX) {
    return T4A_ERR_LAUNCH_LIMIT;
  }
  return pass_geometry(dtype, strategy, w, *in, axis, outputs, 1, false, launch);
}

int t4a_plan_reduce_partials(int dtype, int op, const t4a_cuda_layout* partials, long long partials_len,
                             const t4a_cuda_layout* in, long long in_len, unsigned axis, t4a_split split,
                             unsigned w, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(partials));
  T4A_TRY(check_layout(in));
  if (!plane_width_ok(w)) return T4A_ERR_INVALID_PLANE_WIDTH;
  if (!op_supports(op, dtype)) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_axis(axis, in->rank));
  if (partials->rank != in->rank) return T4A_ERR_RANK_LENGTH;
  for (int d = 0; d < in->rank; ++d)
    if (d != static_cast<int>(axis) && partials->extents[d] != in->extents[d]) return T4A_ERR_SHAPE_MISMATCH;
  const long long len = in->extents[axis];
  if (len < 1) return T4A_ERR_NEGATIVE_COUNT;
  if (split.splits < 2 || split.chunk_len < static_cast<long long>(w) || split.chunk_len != len / split.splits ||
      split.splits > kMaxSplits)
    return T4A_ERR_INVALID_SPLIT;
  if (partials->extents[axis] != split.splits) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_destination(*partials));
  T4A_TRY(check_span(*in, in_len, dtype_size(dtype)));
  T4A_TRY(check_span(*partials, partials_len, dtype_size(dtype)));
  long long outputs = 1;
  for (int d = 0; d < partials->rank; ++d)
    if (d != static_cast<int>(axis) && mul_overflows(outputs, partials->extents[d], &outputs)) return T4A_ERR_OVERFLOW;
  unsigned long long cubes;
  if (__builtin_mul_overflow(static_cast<unsigned long long>(outputs), static_cast<unsigned long long>(split.splits), &cubes))
    return T4A_ERR_OVERFLOW;
  if (cubes > kMaxGridX) return T4A_ERR_LAUNCH_LIMIT;
  return pass_geometry(dtype, T4A_CUDA_REDUCE_PLANE, w, *in, axis, outputs, split.splits, true, launch);
}

int t4a_reduction_partials_layout(const t4a_cuda_layout* in, unsigned axis, long long splits,
                                  t4a_cuda_layout* partials) {
  if (partials == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(in));
  T4A_TRY(require_axis(axis, in->rank));
  return partials_layout_for(*in, axis, splits, partials);
}

int t4a_plan_reduction(int dtype, int op, const t4a_cuda_layout* out, long long out_len,
                       const t4a_cuda_layout* in, long long in_len, unsigned axis, unsigned w,
                       t4a_reduction_plan* plan) {
  if (plan == nullptr) return T4A_ERR_NULL_ARGUMENT;
  std::memset(plan, 0, sizeof(*plan));
  if (!plane_width_ok(w)) return T4A_ERR_INVALID_PLANE_WIDTH;
  long long len, outputs;
  T4A_TRY(reduce_problem(dtype, op, out, out_len, in, in_len, axis, &len, &outputs));
  const int strategy = strategy_for(len, w);
  int has_split;
  t4a_split split;
  T4A_TRY(t4a_split_policy(len, w, &has_split, &split));
  if (!has_split) {
    plan->is_split = 0;
    plan->strategy = strategy;
    return t4a_plan_reduce(dtype, op, strategy, out, out_len, in, in_len, axis, w, &plan->launch);
  }
  t4a_cuda_layout partials;
  T4A_TRY(partials_layout_for(*in, axis, split.splits, &partials));
  long long partials_len;
  T4A_TRY(element_count(partials, &partials_len));
  plan->is_split = 1;
  plan->split = split;
  T4A_TRY(t4a_plan_reduce_partials(dtype, op, &partials, partials_len, in, in_len, axis, split, w, &plan->pass1));
  // combine_geometry (src/lib.rs:3447) and combine_block_width (:3435).
  const int cop = combine_op_of(op);
  int cstrategy;
  unsigned cwidth;
  if (cop == T4A_CUDA_REDUCE_PROD || split.splits < kWideCombineMinSplits) {
    cstrategy = strategy_for(split.splits, w);
    cwidth = w;
  } else {
    const long long target = split.splits / kCombineFoldsPerLane;
    unsigned width = static_cast<unsigned>(kWideCombineMinSplits);
    while (static_cast<long long>(width) < target && width < 512) width *= 2;
    cstrategy = T4A_CUDA_REDUCE_PLANE;
    cwidth = width < 512 ? width : 512;
  }
  plan->combine_strategy = cstrategy;
  plan->combine_op = cop;
  return t4a_plan_reduce(dtype, cop, cstrategy, out, out_len, &partials, partials_len, axis, cwidth, &plan->pass2);
}

int t4a_abi_revision(void) { return T4A_CUDA_ABI_REVISION; }

const char* t4a_status_string(int status) {
  switch (status) {
    case T4A_OK: return "ok";
    case T4A_ERR_RANK_OUT_OF_RANGE: return "rank exceeds the supported maximum";
    case T4A_ERR_RANK_LENGTH: return "extent/stride count does not match the rank";
    case T4A_ERR_NEGATIVE_EXTENT: return "negative extent";
    case T4A_ERR_NEGATIVE_COUNT: return "negative element count";
    case T4A_ERR_OVERFLOW: return "size or address arithmetic overflowed";
    case T4A_ERR_COUNT_MISMATCH: return "element count differs from the extent product";
    case T4A_ERR_OFFSET_OUT_OF_SPAN: return "layout reaches outside the supplied allocation";
    case T4A_ERR_BROADCAST_DESTINATION: return "destination axis with extent > 1 has stride 0";
    case T4A_ERR_UNSUPPORTED_DTYPE: return "entry does not support this dtype";
    case T4A_ERR_NOT_ELEMENTWISE: return "entry is not a flat element-wise entry";
    case T4A_ERR_LAUNCH_LIMIT: return "launch geometry exceeds the device limits";
    case T4A_ERR_INVALID_TRANSPOSE_CONFIG: return "invalid or unsupported transpose configuration";
    case T4A_ERR_INVALID_AXIS: return "axis outside the operand rank";
    case T4A_ERR_DUPLICATE_AXIS: return "the same axis appears twice";
    case T4A_ERR_NOT_COMPACT: return "operand must be compact";
    case T4A_ERR_SHAPE_MISMATCH: return "operand extents do not match the operation";
    case T4A_ERR_INVALID_STEP: return "slice step must be at least one";
    case T4A_ERR_INVALID_PADDING: return "interior padding must be non-negative";
    case T4A_ERR_DOMAIN_TOO_LARGE: return "validation domain exceeds the 32-bit status word";
    case T4A_ERR_INVALID_STRIDE: return "sampling stride must be at least one";
    case T4A_ERR_STRATEGY_MISMATCH: return "reduction strategy does not fit the axis length";
    case T4A_ERR_INVALID_PLANE_WIDTH: return "plane width must be 8, 16 or 32";
    case T4A_ERR_INVALID_SPLIT: return "inconsistent split tuple";
    case T4A_ERR_INDEX_VECTOR_MISMATCH: return "index vector size differs from the map length";
    case T4A_ERR_UNSUPPORTED_OP: return "operation is not supported for this dtype or operand side";
    case T4A_ERR_CUDA: return "a CUDA runtime call failed";
    case T4A_ERR_WORKSPACE: return "workspace missing or too small";
    case T4A_ERR_NULL_ARGUMENT: return "a required pointer argument is NULL";
    default: return "unknown status";
  }
}

}  // extern "C"
