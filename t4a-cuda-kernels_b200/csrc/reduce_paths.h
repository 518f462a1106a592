// Layout analysis of the single-axis reductions, shared by the host planner and the
// kernels, so both sides agree on which path serves a launch.
#pragma once

#include "../../include/t4a_b200/abi.h"

#if defined(__CUDACC__)
#define T4A_HD __host__ __device__ __forceinline__
#else
#define T4A_HD inline
#endif

namespace t4a {

// Threads per block of every reduction path except the wide combine plane.
constexpr int kTileThreads = 256;
// Strided-axis tile: kSlotsPerTile vector slots (contiguous outputs) x kLaneGroups
// groups of W/kLaneGroups lanes.
constexpr int kSlotsPerTile = 32;
constexpr int kLaneGroups = 8;
// Shared memory of the strided path: one 16-byte vector per thread.
constexpr int kStridedSmem = kTileThreads * 16;
// Byte budget of one shared-memory tile of the UNIT rows path.
constexpr int kUnitRowsBytes = 32768;

// Path tags carried in t4a_launch.variant (values >= 16, so they never collide with
// the reference's RankVariant 0/1).
enum ReducePath {
  kPathCubes = 16,      // one W-lane plane per (output, split)
  kPathStrided = 17,    // strided axis, tiles of contiguous outputs
  kPathUnitRows = 18,   // UNIT, short contiguous axis staged through shared memory
  kPathUnit = 19,       // UNIT, one thread per output
  kPathWide = 20,       // PLANE wider than a warp, one block per output
};

// The unit-stride run of non-reduce axes [0, r) of the input: strides 1, e0, e0*e1 ...
struct InnerRun {
  int r;
  long long ext;
};

T4A_HD InnerRun inner_run(const t4a_cuda_layout& in, int axis) {
  InnerRun run{0, 1};
  if (axis == 0 || in.rank < 1 || in.strides[0] != 1) return run;
  long long expect = 1;
  for (int d = 0; d < T4A_CUDA_MAX_RANK; ++d) {
    if (d < axis && d < in.rank && run.r == d && in.strides[d] == expect) {
      run.r = d + 1;
      expect *= in.extents[d];
      run.ext = expect;
    }
  }
  return run;
}

// Number of outputs outside the inner run (the product of the other non-axis extents).
T4A_HD long long outer_count(const t4a_cuda_layout& in, int axis, int inner_r) {
  long long n = 1;
  for (int d = 0; d < T4A_CUDA_MAX_RANK; ++d)
    if (d < in.rank && d >= inner_r && d != axis) n *= in.extents[d];
  return n;
}

// Whether 16-byte vectors of `vec` elements over the inner run start aligned for any
// 16-byte-aligned base pointer: the offset, the run length and every stride outside
// the run are multiples of `vec`.
T4A_HD bool strided_vectors_fit(const t4a_cuda_layout& in, const InnerRun& run, int vec) {
  if (vec <= 1) return true;  // element loads (complex types) need no extra alignment
  if (in.offset % vec != 0 || run.ext % vec != 0) return false;
  for (int d = 0; d < T4A_CUDA_MAX_RANK; ++d)
    if (d < in.rank && d >= run.r && in.strides[d] % vec != 0) return false;
  return true;
}

// The strided path serves W == 32 planes over a strided axis whose outputs have a
// unit-stride run that splits into whole vectors of `vec` elements (16 bytes, or one
// element for the complex types).
T4A_HD bool strided_path_applies(const t4a_cuda_layout& in, int axis, int W, int vec) {
  if (W != 32 || axis < 0 || axis >= in.rank) return false;
  const long long s = in.strides[axis];
  if (s == 0 || s == 1) return false;
  const InnerRun run = inner_run(in, axis);
  return run.r > 0 && strided_vectors_fit(in, run, vec);
}

T4A_HD bool compact_beyond_axis0(const t4a_cuda_layout& l) {
  if (l.rank < 1 || l.strides[0] != 1) return false;
  long long expect = l.extents[0];
  for (int d = 1; d < T4A_CUDA_MAX_RANK; ++d) {
    if (d < l.rank) {
      if (l.extents[d] != 1 && l.strides[d] != expect) return false;
      expect *= l.extents[d];
    }
  }
  return true;
}

// Rows (outputs) per tile of the UNIT rows path, 0 when it does not apply.
T4A_HD int unit_rows_per_tile(const t4a_cuda_layout& in, int axis, int elem_bytes) {
  if (axis != 0 || in.rank < 1) return 0;
  const long long len = in.extents[0];
  if (len < 1 || len > 32 || !compact_beyond_axis0(in)) return 0;
  const long long pitch = len | 1;
  long long rows = kUnitRowsBytes / (pitch * elem_bytes);
  if (rows > kTileThreads) rows = kTileThreads;
  return rows >= 32 ? static_cast<int>(rows) : 0;
}

T4A_HD int unit_rows_smem(const t4a_cuda_layout& in, int rows, int elem_bytes) {
  return rows * static_cast<int>(in.extents[0] | 1) * elem_bytes;
}

// Vector lanes of the strided path for an element size: 16-byte vectors for the 4- and
// 8-byte reals and integers, single elements for the complex types.
T4A_HD int strided_vec_lanes(int dtype) {
  switch (dtype) {
    case T4A_CUDA_F32:
    case T4A_CUDA_I32: return 4;
    case T4A_CUDA_F64:
    case T4A_CUDA_I64: return 2;
    default: return 1;
  }
}

}  // namespace t4a
