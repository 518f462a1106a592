// Gather / scatter_add planning (reference src/lib.rs:2779-3029, CGatherPlan and
// CScatterPlan at :4192-4303) and the host launchers.  The launchers rebuild the
// window plan on the host, pick the vector width from the plan and the pointers,
// and launch a kernel compiled for that width and index type.
#include <cuda_runtime.h>

#include <atomic>

#include "gather_scatter_core.cuh"
#include "plan_common.h"
#include "runtime.h"

namespace t4a {
namespace {

template <typename I, int V>
__global__ void __launch_bounds__(kGatherThreads) k_gather(WindowPlan p, void* out, const void* operand,
                                                           const void* indices, long long units, long long nvec,
                                                           Pieces pc, int lshift) {
  __shared__ GatherSlot slots[kGatherThreads];
  gather_units<I, V>(p, static_cast<unsigned char*>(out), static_cast<const unsigned char*>(operand),
                     static_cast<const I*>(indices), units, nvec, pc, lshift, slots);
}

// One-kernel scatter: each block groups a chunk in shared memory and folds it.
template <typename F, typename I, int V>
__global__ void __launch_bounds__(kScatterThreads, 2) k_scatter(WindowPlan p, void* out, const void* indices,
                                                                const void* updates, long long units,
                                                                long long nvec) {
  __shared__ ScatterSmem sm;
  scatter_units<F, I, V>(p, static_cast<unsigned char*>(out), static_cast<const unsigned char*>(updates),
                         static_cast<const I*>(indices), units, nvec, sm);
}

// Two-kernel scatter, pass 1: grouped list of every chunk; clears the status word.
template <typename I, int V>
__global__ void __launch_bounds__(kGroupThreads, 2) k_scatter_group(WindowPlan p, const void* indices,
                                                                    long long units, long long nvec,
                                                                    GroupedPiece* list, int* status) {
  __shared__ GroupTable<kGroupChunk> t;
  if (blockIdx.x == 0 && threadIdx.x == 0) *status = 0;
  scatter_group_pass<I, V>(p, static_cast<const I*>(indices), units, nvec, list, t);
}

constexpr int kFoldThreads = 256;
constexpr size_t kScatterStatusBytes = 16;  // leading status word of the workspace
constexpr int kFoldBlocksPerSm = 3;

// Two-kernel scatter, pass 2 for 16-byte vectors: bulk copies in, bulk reductions out.
template <typename F>
__global__ void __launch_bounds__(kFoldThreads, kFoldBlocksPerSm) k_scatter_fold_bulk(const GroupedPiece* list,
                                                                                     long long total, long long nvec,
                                                                                     void* out, const void* updates,
                                                                                     int* status) {
  extern __shared__ __align__(16) unsigned char stage[];
  scatter_fold_bulk<F>(list, total, nvec, static_cast<unsigned char*>(out), static_cast<const unsigned char*>(updates),
                       stage, status);
}

// Two-kernel scatter, pass 2: streaming fold of the list (no block barrier).
template <typename F, int V>
__global__ void __launch_bounds__(kFoldThreads, kFoldBlocksPerSm) k_scatter_fold(const GroupedPiece* list,
                                                                                long long total, long long nvec,
                                                                                void* out, const void* updates) {
  extern __shared__ __align__(16) unsigned char stage[];
  scatter_fold_pass<F, V>(list, total, nvec, static_cast<unsigned char*>(out),
                          static_cast<const unsigned char*>(updates), stage);
}

// The owned-part scatter (t4a_scatter_add_range, t4a_scatter_add_cyclic): pass 1 lists
// only the pieces whose destination lies in the part this caller holds (OwnedPart),
// with offsets within that part, reserving each chunk's slice of the list on the counter
// at `reserve`; pass 2 folds the list's *count entries into `out`, which holds the part.
template <typename I, int V>
__global__ void __launch_bounds__(kGroupThreads, 2) k_scatter_group_range(WindowPlan p, const void* indices,
                                                                          long long units, long long nvec,
                                                                          GroupedPiece* list, int* status,
                                                                          OwnedPart own, unsigned long long* reserve) {
  __shared__ GroupTable<kGroupChunk> t;
  if (blockIdx.x == 0 && threadIdx.x == 0) *status = 0;
  scatter_group_pass<I, V, true>(p, static_cast<const I*>(indices), units, nvec, list, t, own, reserve);
}

template <typename F>
__global__ void __launch_bounds__(kFoldThreads, kFoldBlocksPerSm) k_scatter_fold_bulk_counted(
    const GroupedPiece* list, const unsigned long long* count, long long nvec, void* out, const void* updates,
    int* status) {
  extern __shared__ __align__(16) unsigned char stage[];
  scatter_fold_bulk<F>(list, static_cast<long long>(*count), nvec, static_cast<unsigned char*>(out),
                       static_cast<const unsigned char*>(updates), stage, status);
}

template <typename F, int V>
__global__ void __launch_bounds__(kFoldThreads, kFoldBlocksPerSm) k_scatter_fold_counted(
    const GroupedPiece* list, const unsigned long long* count, long long nvec, void* out, const void* updates) {
  extern __shared__ __align__(16) unsigned char stage[];
  scatter_fold_pass<F, V>(list, static_cast<long long>(*count), nvec, static_cast<unsigned char*>(out),
                          static_cast<const unsigned char*>(updates), stage);
}

constexpr int kGatherVariant = 48;
constexpr int kScatterVariant = 49;
constexpr unsigned long long kResidentBlocks = 148ull * 8;  // grid cap: a few waves of resident blocks
constexpr unsigned long long kScatterBlocksPerSm = 2;

int index_size(int index_dtype) {
  switch (index_dtype) {
    case T4A_CUDA_F32:
    case T4A_CUDA_I32: return 4;
    case T4A_CUDA_F64:
    case T4A_CUDA_I64: return 8;
    default: return 0;
  }
}

int require_index_dtype(int index_dtype) { return index_size(index_dtype) ? T4A_OK : T4A_ERR_UNSUPPORTED_DTYPE; }

// require_unique_axes (src/lib.rs:2815).
int require_unique_axes(const long long* axes, int n, long long rank) {
  for (int i = 0; i < n; ++i) {
    if (axes[i] < 0 || axes[i] >= rank) return T4A_ERR_INVALID_AXIS;
    for (int j = 0; j < i; ++j)
      if (axes[j] == axes[i]) return T4A_ERR_DUPLICATE_AXIS;
  }
  return T4A_OK;
}

// index_vector_size (src/lib.rs:2838): the vector axis' extent, 1 when absent.
int index_vector_size(const t4a_cuda_layout& indices, int index_vector_dim, long long* size) {
  if (index_vector_dim < 0 || index_vector_dim > indices.rank) return T4A_ERR_INVALID_AXIS;
  *size = index_vector_dim == indices.rank ? 1 : indices.extents[index_vector_dim];
  return T4A_OK;
}

// Index batch extents: the index extents without the vector axis.
int index_batch_extents(const t4a_cuda_layout& indices, int index_vector_dim, long long* out) {
  int n = 0;
  for (int ax = 0; ax < indices.rank; ++ax)
    if (ax != index_vector_dim) out[n++] = indices.extents[ax];
  return n;
}

// The by-value mirror's counts are within the ABI's fixed arrays (CGatherPlan::new,
// CScatterPlan::new, src/lib.rs:4208, :4274).
int check_counts(int a, int b, int c) {
  if (a < 0 || b < 0 || c < 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (a > T4A_CUDA_MAX_RANK || b > T4A_CUDA_MAX_RANK || c > T4A_CUDA_MAX_RANK) return T4A_ERR_RANK_OUT_OF_RANGE;
  return T4A_OK;
}

// plan_gather validation (src/lib.rs:2867-2965).
int validate_gather(int dtype, int index_dtype, const t4a_cuda_layout& out, long long out_len,
                    const t4a_cuda_layout& operand, long long operand_len, const t4a_cuda_layout& indices,
                    long long indices_len, const t4a_cuda_gather_plan& g) {
  using namespace plan;
  if (dtype_size(dtype) == 0) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_index_dtype(index_dtype));
  T4A_TRY(require_compact(indices));
  T4A_TRY(check_counts(g.operand_rank, g.window_rank, g.start_map_len));
  const int operand_rank = operand.rank;
  if (g.operand_rank != operand_rank) return T4A_ERR_RANK_LENGTH;
  for (int ax = 0; ax < operand_rank; ++ax)
    if (g.slice_sizes[ax] < 0) return T4A_ERR_NEGATIVE_EXTENT;
  T4A_TRY(require_unique_axes(g.start_index_map, g.start_map_len, operand_rank));
  T4A_TRY(require_unique_axes(g.window_dims, g.window_rank, operand_rank));
  long long vsize = 0;
  T4A_TRY(index_vector_size(indices, g.index_vector_dim, &vsize));
  if (vsize != g.start_map_len) return T4A_ERR_INDEX_VECTOR_MISMATCH;
  for (int ax = 0; ax < operand_rank; ++ax) {
    bool window = false;
    for (int q = 0; q < g.window_rank; ++q)
      if (g.window_dims[q] == ax) window = true;
    if (window) {
      if (g.slice_sizes[ax] > operand.extents[ax]) return T4A_ERR_SHAPE_MISMATCH;
    } else if (g.slice_sizes[ax] != 1) {
      return T4A_ERR_SHAPE_MISMATCH;
    }
  }
  long long batch[T4A_CUDA_MAX_RANK];
  const int nbatch = index_batch_extents(indices, g.index_vector_dim, batch);
  const int out_rank = nbatch + g.window_rank;
  for (int q = 0; q < g.window_rank; ++q)
    if (g.offset_dims[q] < 0 || g.offset_dims[q] >= out_rank) return T4A_ERR_INVALID_AXIS;
  T4A_TRY(require_unique_axes(g.offset_dims, g.window_rank, out_rank));
  if (out_rank > T4A_CUDA_MAX_RANK) return T4A_ERR_SHAPE_MISMATCH;
  long long derived[T4A_CUDA_MAX_RANK] = {0};
  bool filled[T4A_CUDA_MAX_RANK] = {false};
  for (int q = 0; q < g.window_rank; ++q) {
    derived[g.offset_dims[q]] = g.slice_sizes[g.window_dims[q]];
    filled[g.offset_dims[q]] = true;
  }
  int b = 0;
  for (int ax = 0; ax < out_rank; ++ax) {
    if (!filled[ax]) {
      if (b >= nbatch) return T4A_ERR_SHAPE_MISMATCH;
      derived[ax] = batch[b++];
    }
  }
  if (b != nbatch) return T4A_ERR_SHAPE_MISMATCH;
  if (out.rank != out_rank) return T4A_ERR_SHAPE_MISMATCH;
  for (int ax = 0; ax < out_rank; ++ax)
    if (out.extents[ax] != derived[ax]) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_destination(out));
  T4A_TRY(check_span(operand, operand_len, dtype_size(dtype)));
  T4A_TRY(check_span(indices, indices_len, index_size(index_dtype)));
  T4A_TRY(check_span(out, out_len, dtype_size(dtype)));
  return T4A_OK;
}

// plan_scatter_add validation (src/lib.rs:2970-3029).
int validate_scatter(int dtype, int index_dtype, const t4a_cuda_layout& out, long long out_len,
                     const t4a_cuda_layout& indices, long long indices_len, const t4a_cuda_layout& updates,
                     long long updates_len, const t4a_cuda_scatter_plan& g) {
  using namespace plan;
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64 && dtype != T4A_CUDA_C32 && dtype != T4A_CUDA_C64)
    return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_index_dtype(index_dtype));
  T4A_TRY(require_compact(indices));
  T4A_TRY(check_counts(g.window_rank, g.window_rank, g.scatter_map_len));
  T4A_TRY(require_unique_axes(g.scatter_dims, g.scatter_map_len, out.rank));
  T4A_TRY(require_unique_axes(g.window_dims, g.window_rank, out.rank));
  T4A_TRY(require_unique_axes(g.update_window_dims, g.window_rank, updates.rank));
  long long vsize = 0;
  T4A_TRY(index_vector_size(indices, g.index_vector_dim, &vsize));
  if (vsize != g.scatter_map_len) return T4A_ERR_INDEX_VECTOR_MISMATCH;
  long long from_updates[T4A_CUDA_MAX_RANK], from_indices[T4A_CUDA_MAX_RANK];
  int nu = 0;
  for (int ax = 0; ax < updates.rank; ++ax) {
    bool window = false;
    for (int q = 0; q < g.window_rank; ++q)
      if (g.update_window_dims[q] == ax) window = true;
    if (!window) from_updates[nu++] = updates.extents[ax];
  }
  const int ni = index_batch_extents(indices, g.index_vector_dim, from_indices);
  if (nu != ni) return T4A_ERR_SHAPE_MISMATCH;
  for (int i = 0; i < nu; ++i)
    if (from_updates[i] != from_indices[i]) return T4A_ERR_SHAPE_MISMATCH;
  long long count = 0;
  T4A_TRY(element_count(updates, &count));
  T4A_TRY(require_destination(out));
  T4A_TRY(check_span(out, out_len, dtype_size(dtype)));
  T4A_TRY(check_span(indices, indices_len, index_size(index_dtype)));
  T4A_TRY(check_span(updates, updates_len, dtype_size(dtype)));
  return T4A_OK;
}

t4a_launch gather_geometry(const WindowPlan& p) {
  using namespace plan;
  const long long units = p.batch.len * p.wrest.len;
  if (units <= 0 || p.run <= 0) return empty_launch();
  const long long nvec = p.run;  // vector count at the narrowest width bounds the piece count
  const Pieces pc = make_pieces(nvec, kGatherPieceVecs);
  const unsigned long long batches = ceil_div(static_cast<unsigned long long>(units * pc.count), 32);
  unsigned long long grid = ceil_div(batches, kGatherThreads / 32);
  if (grid > kResidentBlocks * 4) grid = kResidentBlocks * 4;  // warps are grid-stride
  return make_launch(grid, kGatherThreads, 1, 0, kGatherVariant);
}

t4a_launch scatter_geometry(const WindowPlan& p) {
  using namespace plan;
  const long long units = p.batch.len * p.wrest.len;
  if (units <= 0 || p.run <= 0 || !scatter_windows_fit(p)) return empty_launch();
  const ScatterShape sh = scatter_shape(p.run);  // the narrowest vectors bound the piece count
  const unsigned long long chunks = ceil_div(static_cast<unsigned long long>(units * sh.piece.count), kScatterChunk);
  unsigned long long grid = chunks;
  if (grid > 148 * kScatterBlocksPerSm) grid = 148 * kScatterBlocksPerSm;  // blocks are grid-stride over chunks
  return make_launch(grid, kScatterThreads, 1, 0, kScatterVariant);
}

template <typename I>
int launch_gather_typed(const WindowPlan& p, dim3 grid, cudaStream_t s, void* out, const void* operand,
                        const void* indices) {
  const long long units = p.batch.len * p.wrest.len;
  const int v = window_vec_bytes(p, reinterpret_cast<unsigned long long>(out),
                                 reinterpret_cast<unsigned long long>(operand));
  const long long nvec = p.run * p.esize / v;
  const Pieces pc = make_pieces(nvec, kGatherPieceVecs);
  const int ls = lane_shift_of(pc.vecs);
  const dim3 block(kGatherThreads);
  switch (v) {
    case 16: k_gather<I, 16><<<grid, block, 0, s>>>(p, out, operand, indices, units, nvec, pc, ls); break;
    case 8: k_gather<I, 8><<<grid, block, 0, s>>>(p, out, operand, indices, units, nvec, pc, ls); break;
    case 4: k_gather<I, 4><<<grid, block, 0, s>>>(p, out, operand, indices, units, nvec, pc, ls); break;
    case 2: k_gather<I, 2><<<grid, block, 0, s>>>(p, out, operand, indices, units, nvec, pc, ls); break;
    default: k_gather<I, 1><<<grid, block, 0, s>>>(p, out, operand, indices, units, nvec, pc, ls); break;
  }
  return runtime::check_launch();
}

// Raises a kernel's dynamic shared memory limit once on each device.
template <typename K>
int allow_dynamic_smem(K kernel, unsigned bytes, std::atomic<unsigned long long>& raised) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return runtime::check_launch();
  const unsigned long long bit = 1ull << (dev & 63);
  if ((raised.load(std::memory_order_relaxed) & bit) == 0) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return runtime::check_launch();
    raised.fetch_or(bit);
  }
  return T4A_OK;
}

template <typename F, typename I, int V>
void launch_scatter_width(const WindowPlan& p, dim3 grid, cudaStream_t s, void* out, const void* indices,
                          const void* updates, long long units, long long nvec, void* workspace) {
  if (workspace == nullptr) {
    k_scatter<F, I, V><<<grid, dim3(kScatterThreads), 0, s>>>(p, out, indices, updates, units, nvec);
    return;
  }
  const ScatterShape sh = scatter_shape(nvec);
  const long long total = units * sh.piece.count;
  // Workspace: the status word (16 bytes), then the grouped list.
  int* status = static_cast<int*>(workspace);
  auto* list = reinterpret_cast<GroupedPiece*>(static_cast<unsigned char*>(workspace) + kScatterStatusBytes);
  unsigned long long gg = plan::ceil_div(static_cast<unsigned long long>(total), kGroupChunk);
  if (gg > 148ull * 8) gg = 148ull * 8;
  if (gg == 0) gg = 1;
  k_scatter_group<I, V><<<dim3(static_cast<unsigned>(gg)), dim3(kGroupThreads), 0, s>>>(p, indices, units, nvec,
                                                                                        list, status);
  const dim3 fgrid(148 * kFoldBlocksPerSm);
  if constexpr (V == 16) {
    const unsigned smem = (kFoldThreads / 32) * bulk_stage_bytes_per_warp();
    static std::atomic<unsigned long long> raised{0};
    if (allow_dynamic_smem(k_scatter_fold_bulk<F>, smem, raised) != T4A_OK) return;
    k_scatter_fold_bulk<F><<<fgrid, dim3(kFoldThreads), smem, s>>>(list, total, nvec, out, updates, status);
  } else {
    const unsigned smem = (kFoldThreads / 32) * fold_stage_bytes_per_warp(V);
    static std::atomic<unsigned long long> raised{0};
    if (allow_dynamic_smem(k_scatter_fold<F, V>, smem, raised) != T4A_OK) return;
    k_scatter_fold<F, V><<<fgrid, dim3(kFoldThreads), smem, s>>>(list, total, nvec, out, updates);
  }
}

// The range-filtered two-kernel scatter (workspace: the status word and the list
// counter in its first 16 bytes, then the list).
template <typename F, typename I, int V>
int launch_scatter_range_width(const WindowPlan& p, cudaStream_t s, void* out, const void* indices,
                               const void* updates, long long units, long long nvec, void* workspace,
                               const OwnedPart& own) {
  const ScatterShape sh = scatter_shape(nvec);
  const long long total = units * sh.piece.count;
  int* status = static_cast<int*>(workspace);
  auto* count = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(workspace) + 8);
  auto* list = reinterpret_cast<GroupedPiece*>(static_cast<unsigned char*>(workspace) + kScatterStatusBytes);
  if (cudaMemsetAsync(count, 0, sizeof(*count), s) != cudaSuccess) return runtime::check_launch();
  unsigned long long gg = plan::ceil_div(static_cast<unsigned long long>(total), kGroupChunk);
  if (gg > 148ull * 8) gg = 148ull * 8;
  if (gg == 0) gg = 1;
  k_scatter_group_range<I, V><<<dim3(static_cast<unsigned>(gg)), dim3(kGroupThreads), 0, s>>>(
      p, indices, units, nvec, list, status, own, count);
  const dim3 fgrid(148 * kFoldBlocksPerSm);
  if constexpr (V == 16) {
    const unsigned smem = (kFoldThreads / 32) * bulk_stage_bytes_per_warp();
    static std::atomic<unsigned long long> raised{0};
    T4A_TRY(allow_dynamic_smem(k_scatter_fold_bulk_counted<F>, smem, raised));
    k_scatter_fold_bulk_counted<F><<<fgrid, dim3(kFoldThreads), smem, s>>>(list, count, nvec, out, updates, status);
  } else {
    const unsigned smem = (kFoldThreads / 32) * fold_stage_bytes_per_warp(V);
    static std::atomic<unsigned long long> raised{0};
    T4A_TRY(allow_dynamic_smem(k_scatter_fold_counted<F, V>, smem, raised));
    k_scatter_fold_counted<F, V><<<fgrid, dim3(kFoldThreads), smem, s>>>(list, count, nvec, out, updates);
  }
  return runtime::check_launch();
}

template <typename F, typename I>
int launch_scatter_range_typed(const WindowPlan& p, cudaStream_t s, void* out, const void* indices,
                               const void* updates, void* workspace, const OwnedPart& own) {
  const long long units = p.batch.len * p.wrest.len;
  // Vector width from the alignment of the part's base and of its offsets (its start
  // byte, or its block size) and of the updates.
  const unsigned long long part = static_cast<unsigned long long>(own.block == 0 ? own.lo : own.block);
  const int v = window_vec_bytes(p, reinterpret_cast<unsigned long long>(out) | part,
                                 reinterpret_cast<unsigned long long>(updates));
  const long long nvec = p.run * p.esize / v;
  if (v >= 16) return launch_scatter_range_width<F, I, 16>(p, s, out, indices, updates, units, nvec, workspace, own);
  if (v == 8) return launch_scatter_range_width<F, I, 8>(p, s, out, indices, updates, units, nvec, workspace, own);
  if constexpr (sizeof(F) == 4)
    return launch_scatter_range_width<F, I, 4>(p, s, out, indices, updates, units, nvec, workspace, own);
  return T4A_ERR_UNSUPPORTED_DTYPE;
}

template <typename F, typename I>
int launch_scatter_typed(const WindowPlan& p, dim3 grid, cudaStream_t s, void* out, const void* indices,
                         const void* updates, void* workspace) {
  const long long units = p.batch.len * p.wrest.len;
  const int v = window_vec_bytes(p, reinterpret_cast<unsigned long long>(out),
                                 reinterpret_cast<unsigned long long>(updates));
  const long long nvec = p.run * p.esize / v;
  if (v >= 16) {
    launch_scatter_width<F, I, 16>(p, grid, s, out, indices, updates, units, nvec, workspace);
  } else if (v == 8) {
    launch_scatter_width<F, I, 8>(p, grid, s, out, indices, updates, units, nvec, workspace);
  } else if constexpr (sizeof(F) == 4) {
    launch_scatter_width<F, I, 4>(p, grid, s, out, indices, updates, units, nvec, workspace);
  }
  return runtime::check_launch();
}

template <typename F>
int launch_scatter_index(int index_dtype, const WindowPlan& p, dim3 grid, cudaStream_t s, void* out,
                         const void* indices, const void* updates, void* workspace) {
  switch (index_dtype) {
    case T4A_CUDA_F32: return launch_scatter_typed<F, float>(p, grid, s, out, indices, updates, workspace);
    case T4A_CUDA_F64: return launch_scatter_typed<F, double>(p, grid, s, out, indices, updates, workspace);
    case T4A_CUDA_I32: return launch_scatter_typed<F, int>(p, grid, s, out, indices, updates, workspace);
    case T4A_CUDA_I64: return launch_scatter_typed<F, long long>(p, grid, s, out, indices, updates, workspace);
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
}

}  // namespace
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;

extern "C" {

int t4a_plan_gather(int dtype, int index_dtype, const t4a_cuda_layout* out, long long out_len,
                    const t4a_cuda_layout* operand, long long operand_len, const t4a_cuda_layout* indices,
                    long long indices_len, const t4a_cuda_gather_plan* plan, t4a_launch* launch,
                    long long* output_len) {
  if (plan == nullptr || launch == nullptr || output_len == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(out));
  T4A_TRY(check_layout(operand));
  T4A_TRY(check_layout(indices));
  T4A_TRY(validate_gather(dtype, index_dtype, *out, out_len, *operand, operand_len, *indices, indices_len, *plan));
  long long count = 0;
  T4A_TRY(element_count(*out, &count));
  *output_len = count;
  *launch = gather_geometry(make_gather_plan(*out, *operand, *indices, *plan, dtype_size(dtype)));
  return T4A_OK;
}

int t4a_plan_scatter_add(int dtype, int index_dtype, const t4a_cuda_layout* out, long long out_len,
                         const t4a_cuda_layout* indices, long long indices_len, const t4a_cuda_layout* updates,
                         long long updates_len, const t4a_cuda_scatter_plan* plan, t4a_launch* launch) {
  if (plan == nullptr || launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(out));
  T4A_TRY(check_layout(indices));
  T4A_TRY(check_layout(updates));
  T4A_TRY(
      validate_scatter(dtype, index_dtype, *out, out_len, *indices, indices_len, *updates, updates_len, *plan));
  long long count = 0;
  T4A_TRY(element_count(*out, &count));
  if (count == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  *launch = scatter_geometry(make_scatter_plan(*out, *indices, *updates, *plan, dtype_size(dtype)));
  return T4A_OK;
}

int t4a_launch_gather(const t4a_launch* launch, void* stream, void* out, const void* operand, const void* indices,
                      int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                      const t4a_cuda_layout* operand_layout, const t4a_cuda_layout* indices_layout,
                      const t4a_cuda_gather_plan* plan, long long output_len) {
  if (launch == nullptr || out_layout == nullptr || operand_layout == nullptr || indices_layout == nullptr ||
      plan == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  if (launch->grid[0] == 0 || output_len <= 0) return T4A_OK;
  const int es = dtype_size(dtype);
  if (es == 0) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (!gather_maps_ok(*out_layout, *operand_layout, *indices_layout, *plan)) return T4A_ERR_INVALID_AXIS;
  const WindowPlan p = make_gather_plan(*out_layout, *operand_layout, *indices_layout, *plan, es);
  if (p.run <= 0 || p.batch.len * p.wrest.len <= 0) return T4A_OK;
  const dim3 grid(launch->grid[0]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (index_dtype) {
    case T4A_CUDA_F32: return launch_gather_typed<float>(p, grid, s, out, operand, indices);
    case T4A_CUDA_F64: return launch_gather_typed<double>(p, grid, s, out, operand, indices);
    case T4A_CUDA_I32: return launch_gather_typed<int>(p, grid, s, out, operand, indices);
    case T4A_CUDA_I64: return launch_gather_typed<long long>(p, grid, s, out, operand, indices);
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
}

}  // extern "C"

namespace {

// Launch of a planned scatter; the two-kernel path when `workspace` is given.
int scatter_launch(const t4a_launch* launch, void* stream, void* out, const void* indices, const void* updates,
                   int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                   const t4a_cuda_layout* indices_layout, const t4a_cuda_layout* updates_layout,
                   const t4a_cuda_scatter_plan* plan, long long update_len, void* workspace) {
  if (launch == nullptr || out_layout == nullptr || indices_layout == nullptr || updates_layout == nullptr ||
      plan == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  if (launch->grid[0] == 0 || update_len <= 0) return T4A_OK;
  const int es = dtype_size(dtype);
  if (!scatter_maps_ok(*out_layout, *indices_layout, *updates_layout, *plan)) return T4A_ERR_INVALID_AXIS;
  const WindowPlan p = make_scatter_plan(*out_layout, *indices_layout, *updates_layout, *plan, es);
  if (p.run <= 0 || p.batch.len * p.wrest.len <= 0 || !scatter_windows_fit(p)) return T4A_OK;
  const dim3 grid(launch->grid[0]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case T4A_CUDA_F32:
    case T4A_CUDA_C32: return launch_scatter_index<float>(index_dtype, p, grid, s, out, indices, updates, workspace);
    case T4A_CUDA_F64:
    case T4A_CUDA_C64:
      return launch_scatter_index<double>(index_dtype, p, grid, s, out, indices, updates, workspace);
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
}

// Grouped-list entries the two-kernel path needs: one per piece, counted at the
// narrowest vectors the dtype allows (the most pieces).
int scatter_list_bytes(int dtype, const t4a_cuda_layout& out, const t4a_cuda_layout& indices,
                       const t4a_cuda_layout& updates, const t4a_cuda_scatter_plan& plan, size_t* bytes) {
  const int es = plan::dtype_size(dtype);
  if (es == 0) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (!scatter_maps_ok(out, indices, updates, plan)) return T4A_ERR_INVALID_AXIS;
  const WindowPlan p = make_scatter_plan(out, indices, updates, plan, es);
  const long long units = p.batch.len * p.wrest.len;
  if (p.run <= 0 || units <= 0) {
    *bytes = kScatterStatusBytes;
    return T4A_OK;
  }
  const ScatterShape sh = scatter_shape(p.run);  // vectors are at least one element wide
  long long n = 0;
  if (__builtin_mul_overflow(units, sh.piece.count, &n)) return T4A_ERR_OVERFLOW;
  *bytes = kScatterStatusBytes + static_cast<size_t>(n) * sizeof(GroupedPiece);
  return T4A_OK;
}

}  // namespace

extern "C" {

int t4a_launch_scatter_add(const t4a_launch* launch, void* stream, void* out, const void* indices,
                           const void* updates, int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                           const t4a_cuda_layout* indices_layout, const t4a_cuda_layout* updates_layout,
                           const t4a_cuda_scatter_plan* plan, long long update_len) {
  return scatter_launch(launch, stream, out, indices, updates, dtype, index_dtype, out_layout, indices_layout,
                        updates_layout, plan, update_len, nullptr);
}

int t4a_scatter_add_workspace_bytes(int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                                    const t4a_cuda_layout* indices_layout, const t4a_cuda_layout* updates_layout,
                                    const t4a_cuda_scatter_plan* plan, size_t* bytes) {
  if (out_layout == nullptr || indices_layout == nullptr || updates_layout == nullptr || plan == nullptr ||
      bytes == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(require_index_dtype(index_dtype));
  T4A_TRY(check_layout(out_layout));
  T4A_TRY(check_layout(indices_layout));
  T4A_TRY(check_layout(updates_layout));
  return scatter_list_bytes(dtype, *out_layout, *indices_layout, *updates_layout, *plan, bytes);
}

int t4a_gather(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
               long long out_len, const void* operand, const t4a_cuda_layout* operand_layout, long long operand_len,
               const void* indices, const t4a_cuda_layout* indices_layout, long long indices_len,
               const t4a_cuda_gather_plan* plan) {
  t4a_launch l;
  long long output_len = 0;
  T4A_TRY(t4a_plan_gather(dtype, index_dtype, out_layout, out_len, operand_layout, operand_len, indices_layout,
                          indices_len, plan, &l, &output_len));
  return t4a_launch_gather(&l, stream, out, operand, indices, dtype, index_dtype, out_layout, operand_layout,
                           indices_layout, plan, output_len);
}

int t4a_scatter_add(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                    long long out_len, const void* indices, const t4a_cuda_layout* indices_layout,
                    long long indices_len, const void* updates, const t4a_cuda_layout* updates_layout,
                    long long updates_len, const t4a_cuda_scatter_plan* plan, void* workspace,
                    size_t workspace_bytes) {
  t4a_launch l;
  T4A_TRY(t4a_plan_scatter_add(dtype, index_dtype, out_layout, out_len, indices_layout, indices_len, updates_layout,
                               updates_len, plan, &l));
  long long update_count = 0;
  T4A_TRY(element_count(*updates_layout, &update_count));
  if (workspace != nullptr) {
    size_t need = 0;
    T4A_TRY(scatter_list_bytes(dtype, *out_layout, *indices_layout, *updates_layout, *plan, &need));
    if (workspace_bytes < need) return T4A_ERR_WORKSPACE;
  }
  return scatter_launch(&l, stream, out, indices, updates, dtype, index_dtype, out_layout, indices_layout,
                        updates_layout, plan, update_count, workspace);
}

}  // extern "C"

namespace {

// The owned-part scatter behind t4a_scatter_add_range and t4a_scatter_add_cyclic: `part`
// in elements of the whole destination (block == 0: [lo, hi); else block-cyclic).
int scatter_owned(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                  long long out_len, OwnedPart part, const void* indices, const t4a_cuda_layout* indices_layout,
                  long long indices_len, const void* updates, const t4a_cuda_layout* updates_layout,
                  long long updates_len, const t4a_cuda_scatter_plan* plan, void* workspace, size_t workspace_bytes) {
  t4a_launch l;
  T4A_TRY(t4a_plan_scatter_add(dtype, index_dtype, out_layout, out_len, indices_layout, indices_len, updates_layout,
                               updates_len, plan, &l));
  if (workspace == nullptr) return T4A_ERR_WORKSPACE;
  size_t need = 0;
  T4A_TRY(scatter_list_bytes(dtype, *out_layout, *indices_layout, *updates_layout, *plan, &need));
  if (workspace_bytes < need || workspace_bytes < kScatterStatusBytes) return T4A_ERR_WORKSPACE;
  // The whole destination must be compact (element e at offset e), so that a part is a
  // set of contiguous spans.
  long long count = 0;
  T4A_TRY(element_count(*out_layout, &count));
  long long expect = 1;
  for (int d = 0; d < out_layout->rank; ++d) {
    if (out_layout->extents[d] != 1 && out_layout->strides[d] != expect) return T4A_ERR_INVALID_STRIDE;
    expect *= out_layout->extents[d];
  }
  if (out_layout->offset != 0) return T4A_ERR_INVALID_STRIDE;
  if (part.block == 0) {
    if (part.lo < 0 || part.hi < part.lo || part.hi > count) return T4A_ERR_SHAPE_MISMATCH;
  } else if (part.block < 0 || part.owners < 1 || part.owner < 0 || part.owner >= part.owners) {
    return T4A_ERR_SHAPE_MISMATCH;
  }
  const int es = dtype_size(dtype);
  if (reinterpret_cast<unsigned long long>(workspace) % 16 != 0) return T4A_ERR_INVALID_STRIDE;
  if (out == nullptr || indices == nullptr || updates == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (reinterpret_cast<unsigned long long>(out) % es != 0) return T4A_ERR_INVALID_STRIDE;
  if (l.grid[0] == 0 || (part.block == 0 && part.lo == part.hi)) return T4A_OK;
  if (!scatter_maps_ok(*out_layout, *indices_layout, *updates_layout, *plan)) return T4A_ERR_INVALID_AXIS;
  const WindowPlan p = make_scatter_plan(*out_layout, *indices_layout, *updates_layout, *plan, es);
  if (p.run <= 0 || p.batch.len * p.wrest.len <= 0 || !scatter_windows_fit(p)) return T4A_OK;
  // Every contiguous run of an update window must lie inside one held span: the run
  // covers whole leading destination axes (so runs start at multiples of it), and the
  // span ends (or the block size) are multiples of it.
  long long lead = 1;
  int d = 0;
  while (d < out_layout->rank && lead < p.run) lead *= out_layout->extents[d++];
  if (lead != p.run) return T4A_ERR_SHAPE_MISMATCH;
  if (part.block == 0 ? (part.lo % p.run != 0 || part.hi % p.run != 0) : part.block % p.run != 0)
    return T4A_ERR_SHAPE_MISMATCH;
  OwnedPart own = part;  // in bytes
  own.lo *= es;
  own.hi *= es;
  own.block *= es;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define T4A_OWNED_INDEX(F)                                                                                     \
  switch (index_dtype) {                                                                                       \
    case T4A_CUDA_F32: return launch_scatter_range_typed<F, float>(p, s, out, indices, updates, workspace, own); \
    case T4A_CUDA_F64: return launch_scatter_range_typed<F, double>(p, s, out, indices, updates, workspace, own); \
    case T4A_CUDA_I32: return launch_scatter_range_typed<F, int>(p, s, out, indices, updates, workspace, own);   \
    case T4A_CUDA_I64:                                                                                         \
      return launch_scatter_range_typed<F, long long>(p, s, out, indices, updates, workspace, own);            \
    default: return T4A_ERR_UNSUPPORTED_DTYPE;                                                                 \
  }
  switch (dtype) {
    case T4A_CUDA_F32:
    case T4A_CUDA_C32: T4A_OWNED_INDEX(float)
    case T4A_CUDA_F64:
    case T4A_CUDA_C64: T4A_OWNED_INDEX(double)
    default: return T4A_ERR_UNSUPPORTED_DTYPE;
  }
#undef T4A_OWNED_INDEX
}

}  // namespace

extern "C" {

int t4a_scatter_add_range(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                          long long out_len, long long range_begin, long long range_end, const void* indices,
                          const t4a_cuda_layout* indices_layout, long long indices_len, const void* updates,
                          const t4a_cuda_layout* updates_layout, long long updates_len,
                          const t4a_cuda_scatter_plan* plan, void* workspace, size_t workspace_bytes) {
  return scatter_owned(stream, dtype, index_dtype, out, out_layout, out_len, OwnedPart{range_begin, range_end, 0, 1, 0},
                       indices, indices_layout, indices_len, updates, updates_layout, updates_len, plan, workspace,
                       workspace_bytes);
}

int t4a_scatter_add_cyclic(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                           long long out_len, long long block, long long owners, long long owner, const void* indices,
                           const t4a_cuda_layout* indices_layout, long long indices_len, const void* updates,
                           const t4a_cuda_layout* updates_layout, long long updates_len,
                           const t4a_cuda_scatter_plan* plan, void* workspace, size_t workspace_bytes) {
  if (block <= 0) return T4A_ERR_SHAPE_MISMATCH;
  return scatter_owned(stream, dtype, index_dtype, out, out_layout, out_len, OwnedPart{0, 0, block, owners, owner},
                       indices, indices_layout, indices_len, updates, updates_layout, updates_len, plan, workspace,
                       workspace_bytes);
}

}  // extern "C"

// ---- general-rank twins (`_any`) ------------------------------------------------
// The same bodies as the exported t4a_cuda_gather_any / t4a_cuda_scatter_add_any
// (gather_scatter_any.cuh).  The maps live in device memory, so the host checks what it
// can without reading them; each block checks the maps before it walks.
#include "gather_scatter_any.cuh"

namespace t4a {
namespace {

__global__ void __launch_bounds__(256) k_gather_any(void* out, const void* operand, const void* indices, int dtype,
                                                    int index_dtype, t4a_cuda_layout_any ol, t4a_cuda_layout_any al,
                                                    t4a_cuda_layout_any il, t4a_cuda_gather_plan_any g,
                                                    long long len) {
  any::gather_entry(out, operand, indices, dtype, index_dtype, ol, al, il, g, len);
}

__global__ void __launch_bounds__(256) k_scatter_add_any(void* out, const void* indices, const void* updates,
                                                         int dtype, int index_dtype, t4a_cuda_layout_any ol,
                                                         t4a_cuda_layout_any il, t4a_cuda_layout_any ul,
                                                         t4a_cuda_scatter_plan_any g, long long len) {
  any::scatter_entry(out, indices, updates, dtype, index_dtype, ol, il, ul, g, len);
}

int check_layout_any_gs(const t4a_cuda_layout_any& l) {
  if (l.rank < 0 || l.reserved != 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (l.rank > 0 && (l.extents == nullptr || l.strides == nullptr)) return T4A_ERR_NULL_ARGUMENT;
  return T4A_OK;
}

// The maps' counts against the layouts' ranks, and the index tensor's rank.
int check_maps_any(int plan_rank_a, int layout_rank_a, int plan_rank_b, int layout_rank_b, int window_rank,
                   int map_len, int reserved, int index_vector_dim, int walked_rank, int index_rank,
                   const void* const* arrays, const bool* needed, int n_arrays) {
  if (reserved != 0 || window_rank < 0 || map_len < 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (plan_rank_a != layout_rank_a || plan_rank_b != layout_rank_b) return T4A_ERR_RANK_LENGTH;
  if (window_rank > layout_rank_a || window_rank > layout_rank_b) return T4A_ERR_RANK_OUT_OF_RANGE;
  for (int i = 0; i < n_arrays; ++i)
    if (needed[i] && arrays[i] == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (index_vector_dim < 0 || index_vector_dim > index_rank) return T4A_ERR_INVALID_AXIS;
  if (walked_rank - window_rank + (index_vector_dim < index_rank ? 1 : 0) != index_rank)
    return T4A_ERR_INDEX_VECTOR_MISMATCH;
  return T4A_OK;
}

dim3 dim_of(const unsigned* v) { return dim3(v[0], v[1] ? v[1] : 1, v[2] ? v[2] : 1); }

}  // namespace
}  // namespace t4a

extern "C" {

int t4a_gather_scatter_any_geometry(long long elements, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (elements < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (elements == 0) {
    *launch = plan::empty_launch();
    return T4A_OK;
  }
  const unsigned long long grid = plan::ceil_div(static_cast<unsigned long long>(elements), 256);
  const unsigned long long cap = 148ull * 64;
  *launch = plan::make_launch(grid < cap ? grid : cap, 256, 1, 0, 0);
  return T4A_OK;
}

int t4a_launch_gather_any(const t4a_launch* launch, void* stream, void* out, const void* operand,
                          const void* indices, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
                          t4a_cuda_layout_any operand_layout, t4a_cuda_layout_any indices_layout,
                          t4a_cuda_gather_plan_any plan, long long output_len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (output_len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (dtype_size(dtype) == 0) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_index_dtype(index_dtype));
  T4A_TRY(check_layout_any_gs(out_layout));
  T4A_TRY(check_layout_any_gs(operand_layout));
  T4A_TRY(check_layout_any_gs(indices_layout));
  const void* arrays[] = {plan.window_dims, plan.offset_dims, plan.start_index_map, plan.slice_sizes};
  const bool needed[] = {plan.window_rank > 0, plan.window_rank > 0, plan.start_map_len > 0, plan.start_map_len > 0};
  T4A_TRY(check_maps_any(plan.operand_rank, operand_layout.rank, plan.out_rank, out_layout.rank, plan.window_rank,
                         plan.start_map_len, plan.reserved, plan.index_vector_dim, out_layout.rank,
                         indices_layout.rank, arrays, needed, 4));
  if (output_len == 0 || launch->grid[0] == 0 || launch->block[0] == 0) return T4A_OK;
  if (out == nullptr || operand == nullptr || (plan.start_map_len > 0 && indices == nullptr))
    return T4A_ERR_NULL_ARGUMENT;
  k_gather_any<<<dim_of(launch->grid), dim_of(launch->block), 0, static_cast<cudaStream_t>(stream)>>>(
      out, operand, indices, dtype, index_dtype, out_layout, operand_layout, indices_layout, plan, output_len);
  return runtime::check_launch();
}

int t4a_launch_scatter_add_any(const t4a_launch* launch, void* stream, void* out, const void* indices,
                               const void* updates, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
                               t4a_cuda_layout_any indices_layout, t4a_cuda_layout_any updates_layout,
                               t4a_cuda_scatter_plan_any plan, long long update_len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (update_len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64 && dtype != T4A_CUDA_C32 && dtype != T4A_CUDA_C64)
    return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_index_dtype(index_dtype));
  T4A_TRY(check_layout_any_gs(out_layout));
  T4A_TRY(check_layout_any_gs(indices_layout));
  T4A_TRY(check_layout_any_gs(updates_layout));
  const void* arrays[] = {plan.window_dims, plan.update_window_dims, plan.scatter_dims};
  const bool needed[] = {plan.window_rank > 0, plan.window_rank > 0, plan.scatter_map_len > 0};
  T4A_TRY(check_maps_any(plan.operand_rank, out_layout.rank, plan.updates_rank, updates_layout.rank,
                         plan.window_rank, plan.scatter_map_len, plan.reserved, plan.index_vector_dim,
                         updates_layout.rank, indices_layout.rank, arrays, needed, 3));
  if (update_len == 0 || launch->grid[0] == 0 || launch->block[0] == 0) return T4A_OK;
  if (out == nullptr || updates == nullptr || (plan.scatter_map_len > 0 && indices == nullptr))
    return T4A_ERR_NULL_ARGUMENT;
  k_scatter_add_any<<<dim_of(launch->grid), dim_of(launch->block), 0, static_cast<cudaStream_t>(stream)>>>(
      out, indices, updates, dtype, index_dtype, out_layout, indices_layout, updates_layout, plan, update_len);
  return runtime::check_launch();
}

}  // extern "C"
