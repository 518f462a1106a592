// Index-space analysis of XLA-style gather and additive scatter, shared by the host
// planner and the kernels.
//
// Both entries move windows: gather copies, for every batch position b, the window of
// the operand at the clamped start(b) to the output's window at b; scatter adds the
// window of `updates` at b into the destination window at start(b) (skipped when it
// does not fit).  The plan splits the window axes into a run that is contiguous on both
// sides (copied or added with 16-byte vectors) and the remaining window axes, and lists
// the batch axes with their output (gather) or updates (scatter) strides and their
// index-tensor strides.  Semantics: reference cuda/src/gather_scatter.cu:22-32 (clamp),
// :52-127 (gather), :131-276 (scatter).
#pragma once

#include "../../include/t4a_b200/abi.h"

#if defined(__CUDACC__)
#define T4A_HD __host__ __device__ __forceinline__
#else
#define T4A_HD inline
#endif

namespace t4a {

// A group of axes walked as one mixed-radix counter (axis 0 fastest), with two
// strides per axis.
struct IdxGroup {
  int n;
  long long ext[T4A_CUDA_MAX_RANK];
  long long a[T4A_CUDA_MAX_RANK];
  long long b[T4A_CUDA_MAX_RANK];
  long long len;
};

struct WindowPlan {
  int esize;
  // Window: `run` elements contiguous on both sides (stride 1), then the other window
  // axes (a = side-A stride, b = side-B stride).
  long long run;
  IdxGroup wrest;
  // Batch axes (a = stride in the index tensor, b = side-B stride).  Side A is the
  // operand for gather and the destination for scatter; side B is the output for
  // gather and the updates for scatter.
  IdxGroup batch;
  long long a_offset;      // operand (gather) / destination (scatter) layout offset
  long long b_offset;      // output (gather) / updates (scatter) layout offset
  long long idx_offset;    // index tensor layout offset
  long long comp_stride;   // index-vector axis stride (0 when absent)
  int ncomp;               // start components
  long long comp_dim[T4A_CUDA_MAX_RANK];     // operand extent of the component's axis
  long long comp_window[T4A_CUDA_MAX_RANK];  // window extent on that axis
  long long comp_stride_a[T4A_CUDA_MAX_RANK];  // side-A stride of that axis
  // Scatter only: per side-A axis, the window extent, for the fit check.
  int a_rank;
  long long a_ext[T4A_CUDA_MAX_RANK];
  long long a_window[T4A_CUDA_MAX_RANK];
};

T4A_HD void idx_clear(IdxGroup& g) {
  g.n = 0;
  g.len = 1;
  for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) g.ext[i] = g.a[i] = g.b[i] = 0;
}

T4A_HD void idx_push(IdxGroup& g, long long e, long long a, long long b) {
  g.ext[g.n] = e;
  g.a[g.n] = a;
  g.b[g.n] = b;
  ++g.n;
  g.len *= e;
}

// Window axes (extents w[], side-A strides sa[], side-B strides sb[]) -> run + rest.
// The run is the chain of axes with strides 1, e0, e0*e1, ... on both sides.
T4A_HD void split_window(int n, const long long* w, const long long* sa, const long long* sb, WindowPlan& p) {
  bool used[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
  long long run = 1;
  for (bool grew = true; grew;) {
    grew = false;
    for (int i = 0; i < n; ++i) {
      if (!used[i] && w[i] > 1 && sa[i] == run && sb[i] == run) {
        used[i] = true;
        run *= w[i];
        grew = true;
        break;
      }
    }
  }
  p.run = run;
  idx_clear(p.wrest);
  for (int i = 0; i < n; ++i)
    if (!used[i] && w[i] != 1) idx_push(p.wrest, w[i], sa[i], sb[i]);
}

// The maps address only existing axes (the planner guarantees more; the exported
// kernels check this much before indexing the layouts with them).
T4A_HD bool axes_in_range(const long long* axes, int n, int rank) {
  if (n < 0 || n > T4A_CUDA_MAX_RANK) return false;
  for (int i = 0; i < n; ++i)
    if (axes[i] < 0 || axes[i] >= rank) return false;
  return true;
}

T4A_HD bool layouts_ok(const t4a_cuda_layout& a, const t4a_cuda_layout& b, const t4a_cuda_layout& c) {
  return a.rank >= 0 && a.rank <= T4A_CUDA_MAX_RANK && b.rank >= 0 && b.rank <= T4A_CUDA_MAX_RANK && c.rank >= 0 &&
         c.rank <= T4A_CUDA_MAX_RANK;
}

T4A_HD bool gather_maps_ok(const t4a_cuda_layout& out, const t4a_cuda_layout& operand,
                           const t4a_cuda_layout& indices, const t4a_cuda_gather_plan& g) {
  return layouts_ok(out, operand, indices) && axes_in_range(g.window_dims, g.window_rank, operand.rank) &&
         axes_in_range(g.offset_dims, g.window_rank, out.rank) &&
         axes_in_range(g.start_index_map, g.start_map_len, operand.rank) && g.index_vector_dim >= 0 &&
         g.index_vector_dim <= indices.rank && out.rank - g.window_rank + (g.index_vector_dim < indices.rank) ==
                                                    indices.rank;
}

T4A_HD bool scatter_maps_ok(const t4a_cuda_layout& out, const t4a_cuda_layout& indices,
                            const t4a_cuda_layout& updates, const t4a_cuda_scatter_plan& g) {
  return layouts_ok(out, indices, updates) && axes_in_range(g.window_dims, g.window_rank, out.rank) &&
         axes_in_range(g.update_window_dims, g.window_rank, updates.rank) &&
         axes_in_range(g.scatter_dims, g.scatter_map_len, out.rank) && g.index_vector_dim >= 0 &&
         g.index_vector_dim <= indices.rank &&
         updates.rank - g.window_rank + (g.index_vector_dim < indices.rank) == indices.rank;
}

// Gather: side A = operand, side B = output.
T4A_HD WindowPlan make_gather_plan(const t4a_cuda_layout& out, const t4a_cuda_layout& operand,
                                   const t4a_cuda_layout& indices, const t4a_cuda_gather_plan& g, int esize) {
  WindowPlan p;
  p.esize = esize;
  p.a_offset = operand.offset;
  p.b_offset = out.offset;
  p.idx_offset = indices.offset;
  const bool vector_present = g.index_vector_dim < indices.rank;
  p.comp_stride = vector_present ? indices.strides[g.index_vector_dim] : 0;
  long long w[T4A_CUDA_MAX_RANK], sa[T4A_CUDA_MAX_RANK], sb[T4A_CUDA_MAX_RANK];
  for (int q = 0; q < g.window_rank; ++q) {
    const int oa = static_cast<int>(g.window_dims[q]);
    const int ob = static_cast<int>(g.offset_dims[q]);
    w[q] = out.extents[ob];
    sa[q] = operand.strides[oa];
    sb[q] = out.strides[ob];
  }
  split_window(g.window_rank, w, sa, sb, p);
  idx_clear(p.batch);
  int pos = 0;
  for (int ax = 0; ax < out.rank; ++ax) {
    bool is_window = false;
    for (int q = 0; q < g.window_rank; ++q)
      if (g.offset_dims[q] == ax) is_window = true;
    if (is_window) continue;
    const int tensor_axis = pos + ((vector_present && pos >= g.index_vector_dim) ? 1 : 0);
    idx_push(p.batch, out.extents[ax], indices.strides[tensor_axis], out.strides[ax]);
    ++pos;
  }
  p.ncomp = g.start_map_len;
  for (int c = 0; c < g.start_map_len; ++c) {
    const int ax = static_cast<int>(g.start_index_map[c]);
    p.comp_dim[c] = operand.extents[ax];
    p.comp_window[c] = g.slice_sizes[ax];
    p.comp_stride_a[c] = operand.strides[ax];
  }
  p.a_rank = 0;
  return p;
}

// Scatter: side A = destination, side B = updates.
T4A_HD WindowPlan make_scatter_plan(const t4a_cuda_layout& out, const t4a_cuda_layout& indices,
                                    const t4a_cuda_layout& updates, const t4a_cuda_scatter_plan& g, int esize) {
  WindowPlan p;
  p.esize = esize;
  p.a_offset = out.offset;
  p.b_offset = updates.offset;
  p.idx_offset = indices.offset;
  const bool vector_present = g.index_vector_dim < indices.rank;
  p.comp_stride = vector_present ? indices.strides[g.index_vector_dim] : 0;
  long long w[T4A_CUDA_MAX_RANK], sa[T4A_CUDA_MAX_RANK], sb[T4A_CUDA_MAX_RANK];
  for (int q = 0; q < g.window_rank; ++q) {
    const int oa = static_cast<int>(g.window_dims[q]);
    const int ub = static_cast<int>(g.update_window_dims[q]);
    w[q] = updates.extents[ub];
    sa[q] = out.strides[oa];
    sb[q] = updates.strides[ub];
  }
  split_window(g.window_rank, w, sa, sb, p);
  idx_clear(p.batch);
  int pos = 0;
  for (int ax = 0; ax < updates.rank; ++ax) {
    bool is_window = false;
    for (int q = 0; q < g.window_rank; ++q)
      if (g.update_window_dims[q] == ax) is_window = true;
    if (is_window) continue;
    const int tensor_axis = pos + ((vector_present && pos >= g.index_vector_dim) ? 1 : 0);
    idx_push(p.batch, updates.extents[ax], indices.strides[tensor_axis], updates.strides[ax]);
    ++pos;
  }
  // Window extent per destination axis (one on axes without a window position).
  p.a_rank = out.rank;
  for (int ax = 0; ax < T4A_CUDA_MAX_RANK; ++ax) {
    p.a_ext[ax] = ax < out.rank ? out.extents[ax] : 1;
    p.a_window[ax] = 1;
  }
  for (int q = 0; q < g.window_rank; ++q)
    p.a_window[g.window_dims[q]] = updates.extents[g.update_window_dims[q]];
  p.ncomp = g.scatter_map_len;
  for (int c = 0; c < g.scatter_map_len; ++c) {
    const int ax = static_cast<int>(g.scatter_dims[c]);
    p.comp_dim[c] = out.extents[ax];
    p.comp_window[c] = p.a_window[ax];
    p.comp_stride_a[c] = out.strides[ax];
  }
  return p;
}

// Every update window fits the destination.  Clamping keeps each start at most
// max(extent - window, 0), so a window fits exactly when no axis' window is wider than
// its extent: the per-update fit check of the reference (gather_scatter.cu:203-218)
// is the same for every update.
T4A_HD bool scatter_windows_fit(const WindowPlan& p) {
  for (int ax = 0; ax < T4A_CUDA_MAX_RANK; ++ax)
    if (ax < p.a_rank && p.a_window[ax] > p.a_ext[ax]) return false;
  return true;
}

// Widest power-of-two access (<= 16 bytes) that every run start on both sides is
// aligned to, given the two base pointers.
T4A_HD int window_vec_bytes(const WindowPlan& p, unsigned long long base_a, unsigned long long base_b) {
  const long long es = p.esize;
  unsigned long long bits = base_a | base_b | static_cast<unsigned long long>(p.run * es) |
                            static_cast<unsigned long long>(p.a_offset * es) |
                            static_cast<unsigned long long>(p.b_offset * es);
  for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) {
    if (i < p.wrest.n)
      bits |= static_cast<unsigned long long>(p.wrest.a[i] * es) | static_cast<unsigned long long>(p.wrest.b[i] * es);
    if (i < p.batch.n) bits |= static_cast<unsigned long long>(p.batch.b[i] * es);
    if (i < p.ncomp) bits |= static_cast<unsigned long long>(p.comp_stride_a[i] * es);
  }
  int v = 16;
  while (v > 1 && (bits & static_cast<unsigned long long>(v - 1)) != 0) v >>= 1;
  return v;
}

// Largest element offset a layout reaches (negative strides contribute nothing).
T4A_HD long long layout_max_offset(const t4a_cuda_layout& l) {
  long long hi = l.offset;
  for (int d = 0; d < T4A_CUDA_MAX_RANK; ++d)
    if (d < l.rank && l.extents[d] > 0 && l.strides[d] > 0) hi += (l.extents[d] - 1) * l.strides[d];
  return hi;
}

// Clamped start (reference clamp_window_start): start <= 0 (or NaN) -> 0, else the
// truncated start, at most max(dim - window, 0).
template <typename I>
T4A_HD long long clamp_start(I start, long long dim, long long window) {
  const long long max_start = dim > window ? dim - window : 0;
  if (!(start > static_cast<I>(0))) return 0;
  const unsigned long long raw = static_cast<unsigned long long>(start);
  return raw < static_cast<unsigned long long>(max_start) ? static_cast<long long>(raw) : max_start;
}

}  // namespace t4a
