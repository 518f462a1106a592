// Per-path reduction kernels and the host launchers of the reduction entries.
//
// The exported symbols (reduce_abi.cu) choose their path at run time, so one register
// allocation serves every path.  The launchers here launch one kernel per path
// instead (t4a_launch.variant, chosen by the planner), each compiled for its own
// register budget.  All of them fold with the same device bodies (reduce_core.cuh),
// so both routes produce the same bits.
#include <cuda_runtime.h>

#include <atomic>

#include "plan_common.h"
#include "reduce_core.cuh"
#include "runtime.h"

namespace t4a {
namespace {

// A split reduction's combine pass is launched with programmatic stream serialization
// after its partials pass (t4a_reduce): it may launch as the partials pass's blocks
// exit, and this wait holds it until that pass has finished and its partials are
// visible.  In every other launch the wait returns at once.
__device__ __forceinline__ void dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename Op, typename T>
__global__ void __launch_bounds__(256) k_strided(T* dst, const T* in, t4a_cuda_layout dst_l,
                                                 t4a_cuda_layout in_l, int axis, long long splits,
                                                 long long chunk, bool partials) {
  dependency_wait();
  constexpr int V = VecOf<T>::kLanes;
  strided_tiles<Op, T, V, 4>(in, dst, in_l, dst_l, strided_ctx(in_l, axis, splits, chunk, V, partials), Op());
}

// The staged strided pass: warp units, 8 plane lanes per thread, a 2-stage cp.async
// ring per thread, two blocks per SM.
constexpr int kStagedLanes = 8;
constexpr int kStagedDepth = 3;
constexpr int kStagedBlocksPerSm = 2;
constexpr unsigned kStagedSmem = kStagedDepth * kStagedLanes * kTileThreads * 16;

template <typename Op, typename T>
__global__ void __launch_bounds__(256, kStagedBlocksPerSm) k_strided_staged(T* dst, const T* in, t4a_cuda_layout dst_l,
                                                                           t4a_cuda_layout in_l, int axis,
                                                                           long long splits, long long chunk,
                                                                           bool partials) {
  dependency_wait();
  constexpr int V = VecOf<T>::kLanes;
  if constexpr (V * sizeof(T) == 16) {
    strided_warp_staged<Op, T, V, kStagedLanes, kStagedDepth>(
        in, dst, in_l, dst_l, strided_ctx(in_l, axis, splits, chunk, V, partials), Op());
  }
}

// Resident blocks asked of the per-cube kernel: 16-byte elements (C64) load a whole
// lane walk of 8 elements at once, so more resident warps keep more bytes in flight.
template <typename T>
struct CubesMinBlocks {
  static constexpr int value = sizeof(T) >= 16 ? 3 : 1;
};

template <typename Op, typename T>
__global__ void __launch_bounds__(256, CubesMinBlocks<T>::value) k_cubes(T* dst, const T* in, t4a_cuda_layout dst_l,
                                                                        t4a_cuda_layout in_l,
                                               int axis, long long outputs, long long splits, long long chunk,
                                               bool partials) {
  dependency_wait();
  plane_cubes<Op, T>(in, dst, in_l, dst_l, axis, outputs, splits, chunk, blockDim.x, partials, partials, Op());
}

template <typename Op, typename T>
__global__ void __launch_bounds__(256) k_unit_rows(T* out, const T* in, t4a_cuda_layout out_l, t4a_cuda_layout in_l,
                                                   long long outputs, int rows) {
  dependency_wait();
  unit_rows<Op, T>(in, out, out_l, in_l, outputs, rows, Op());
}

constexpr int kWarpRowsLen = 32;
constexpr int kWarpRowsThreads = 256;

template <typename Op, typename T>
__global__ void __launch_bounds__(kWarpRowsThreads) k_warp_rows(T* out, const T* in, t4a_cuda_layout out_l,
                                                                t4a_cuda_layout in_l, long long outputs,
                                                                bool dst_linear) {
  dependency_wait();
  extern __shared__ __align__(16) unsigned char warp_slices[];
  if constexpr ((kWarpRowsLen * sizeof(T)) % 128 == 0) {
    unit_warp_rows<Op, T, kWarpRowsLen>(in, out, out_l, in_l, outputs, dst_linear,
                                        warp_slices + (threadIdx.x >> 5) * kWarpRowsLen * sizeof(T) * 32, Op());
  }
}

template <typename Op, typename T>
__global__ void __launch_bounds__(256) k_unit(T* out, const T* in, t4a_cuda_layout out_l, t4a_cuda_layout in_l,
                                              int axis, long long outputs) {
  dependency_wait();
  unit_generic<Op, T>(in, out, out_l, in_l, axis, outputs, Op());
}

template <typename Op, typename T>
__global__ void __launch_bounds__(512) k_wide(T* out, const T* in, t4a_cuda_layout out_l, t4a_cuda_layout in_l,
                                              int axis, long long outputs) {
  dependency_wait();
  wide_plane<Op, T>(in, out, out_l, in_l, axis, outputs, Op());
}

// This launcher's own path ids (the planner never returns them).
constexpr int kPathWarpRows = 64;
constexpr int kPathStridedStaged = 65;

// Output o at dst.offset + o: the destination's strides are compact in axis order.
bool dst_linear(const t4a_cuda_layout& l) {
  long long expect = 1;
  for (int d = 0; d < l.rank; ++d) {
    if (l.extents[d] != 1 && l.strides[d] != expect) return false;
    expect *= l.extents[d];
  }
  return true;
}

// General-rank twins: the same bodies as the exported `_any` symbols.
template <typename Op, typename T>
__global__ void __launch_bounds__(512) k_reduce_any(T* out, const T* in, int strategy, t4a_cuda_layout_any out_l,
                                                    t4a_cuda_layout_any in_l, int axis, long long outputs) {
  reduce_any_body<Op, T>(out, in, strategy, out_l, in_l, axis, outputs, Op());
}
template <typename Op, typename T>
__global__ void __launch_bounds__(256) k_partials_any(T* partials, const T* in, t4a_cuda_layout_any part_l,
                                                      t4a_cuda_layout_any in_l, int axis, long long outputs,
                                                      long long splits, long long chunk) {
  partials_any_body<Op, T>(partials, in, part_l, in_l, axis, outputs, splits, chunk, Op());
}

// Host checks of a general-rank layout that need no device access.
int check_any(const t4a_cuda_layout_any& l) {
  if (l.rank < 0 || l.reserved != 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (l.rank > 0 && (l.extents == nullptr || l.strides == nullptr)) return T4A_ERR_NULL_ARGUMENT;
  return T4A_OK;
}

struct PassArgs {
  void* dst;
  const void* in;
  t4a_cuda_layout dst_l;
  t4a_cuda_layout in_l;
  int axis;
  long long outputs;
  long long splits;
  long long chunk;
  bool partials;
  bool chained = false;  // launched as the link after the partials pass (see dependency_wait)
};

// Launches a pass kernel, as a chained link when `chained`.
template <typename... KArgs, typename... Args>
void go(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned smem, cudaStream_t s, bool chained, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = chained ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);  // an error is left for check_launch
}

template <typename Op, typename T>
void launch_path(int path, dim3 grid, dim3 block, unsigned smem, cudaStream_t stream, const PassArgs& a) {
  T* dst = static_cast<T*>(a.dst);
  const T* in = static_cast<const T*>(a.in);
  switch (path) {
    case kPathStrided:
      go(k_strided<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.axis, a.splits, a.chunk,
         a.partials);
      break;
    case kPathUnitRows: {
      const int rows = unit_rows_per_tile(a.in_l, a.axis, sizeof(T));
      go(k_unit_rows<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.outputs, rows);
      break;
    }
    case kPathStridedStaged: {
      auto kernel = k_strided_staged<Op, T>;
      static std::atomic<unsigned long long> raised{0};
      int dev = 0;
      if (cudaGetDevice(&dev) == cudaSuccess) {
        const unsigned long long bit = 1ull << (dev & 63);
        if ((raised.load(std::memory_order_relaxed) & bit) == 0 &&
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess)
          raised.fetch_or(bit);
      }
      go(kernel, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.axis, a.splits, a.chunk, a.partials);
      break;
    }
    case kPathWarpRows:
      go(k_warp_rows<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.outputs,
         dst_linear(a.dst_l));
      break;
    case kPathUnit:
      go(k_unit<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.axis, a.outputs);
      break;
    case kPathWide:
      go(k_wide<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.axis, a.outputs);
      break;
    default:
      go(k_cubes<Op, T>, grid, block, smem, stream, a.chained, dst, in, a.dst_l, a.in_l, a.axis, a.outputs, a.splits,
         a.chunk, a.partials);
      break;
  }
}

// The rows path for rows of exactly kWarpRowsLen elements of 4 or 8 bytes on a
// 16-byte-aligned base runs the warp-private kernel, with its own geometry (a
// grid-stride walk over groups of 32 outputs).
void prefer_warp_rows(int dtype, const void* in, int* path, dim3* grid, dim3* block, unsigned* smem,
                      const PassArgs& a) {
  if (*path != kPathUnitRows || a.axis != 0 || a.in_l.extents[0] != kWarpRowsLen) return;
  const int esize = plan::dtype_size(dtype);
  if (esize != 4 && esize != 8) return;
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64 && dtype != T4A_CUDA_I32 && dtype != T4A_CUDA_I64) return;
  if (((reinterpret_cast<unsigned long long>(in) + a.in_l.offset * esize) & 15ull) != 0) return;
  const unsigned long long groups = (static_cast<unsigned long long>(a.outputs) + 31) / 32;
  // 8 warps of 4 KiB slices (4-byte elements) or 4 warps of 8 KiB slices: 32 KiB.
  const unsigned warps_per_block = esize == 4 ? kWarpRowsThreads / 32 : kWarpRowsThreads / 64;
  unsigned long long blocks = (groups + warps_per_block - 1) / warps_per_block;
  const unsigned long long cap = 148ull * 16;
  if (blocks > cap) blocks = cap;
  *path = kPathWarpRows;
  *grid = dim3(static_cast<unsigned>(blocks), 1, 1);
  *block = dim3(warps_per_block * 32, 1, 1);
  *smem = warps_per_block * 32 * kWarpRowsLen * esize;
}

// A strided pass over 16-byte vectors with at least kStagedMinTiles tiles per resident
// block runs the staged kernel as a grid-stride walk, each warp walking many units, so
// that its copy ring runs ahead across unit boundaries; smaller passes keep one tile per
// block.  The staged kernel needs every plane lane to own a row: chunks of at least 32
// rows.  The grid is 7/8 of kStagedBlocksPerSm blocks per SM: on config 3's 2.1 GB
// passes 256-264 blocks ran 1.2-2.9 % faster than 296 (fewer copies queued at the
// memory controllers, the same bytes), and config 1's 134 MB pass ran the same down to
// 256 blocks.
constexpr unsigned kStagedMinTiles = 1;
void prefer_strided_staged(int dtype, int* path, dim3* grid, unsigned* smem, const PassArgs& a) {
  if (*path != kPathStrided || strided_vec_lanes(dtype) == 1) return;
  const long long shortest = a.splits > 1 ? a.chunk : a.in_l.extents[a.axis];
  if (shortest < 32) return;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned cap = static_cast<unsigned>(sms * kStagedBlocksPerSm * 7 / 8);
  if (grid->x < kStagedMinTiles * cap) return;
  *path = kPathStridedStaged;
  grid->x = cap;
  *smem = kStagedSmem;
}

// The per-cube walk is grid-stride: a grid of many short-lived blocks (one cube per
// plane) runs as eight resident blocks per SM that each take cubes in turn.
void cap_cube_grid(int path, dim3* grid) {
  if (path != kPathCubes) return;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned cap = static_cast<unsigned>(sms * 8);
  if (grid->x > cap) grid->x = cap;
}

// A 16-byte-vector path needs a 16-byte-aligned base; otherwise the same pass runs on
// the per-cube path, whose geometry is recomputed here.
bool fix_alignment(int dtype, const void* in, int* path, dim3* grid, dim3* block, unsigned* smem,
                   const PassArgs& a) {
  if (*path != kPathStrided || strided_vec_lanes(dtype) == 1) return true;
  const int esize = plan::dtype_size(dtype);
  if (((reinterpret_cast<unsigned long long>(in) + a.in_l.offset * esize) & 15ull) == 0 &&
      (reinterpret_cast<unsigned long long>(in) & 15ull) == 0)
    return true;
  const unsigned w = 32;
  *path = kPathCubes;
  *block = dim3(w, kTileThreads / w, 1);
  *smem = 0;
  const unsigned long long grid_x = plan::ceil_div(static_cast<unsigned long long>(a.outputs) * a.splits, kTileThreads / w);
  if (grid_x > plan::kMaxGridX) return false;
  *grid = dim3(static_cast<unsigned>(grid_x), 1, 1);
  return true;
}

int run_pass(const t4a_launch* launch, void* stream, int dtype, int op, PassArgs a) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch->grid[0] == 0 || launch->grid[1] == 0 || launch->grid[2] == 0) return T4A_OK;
  int path = launch->variant;
  dim3 grid(launch->grid[0], launch->grid[1], launch->grid[2]);
  dim3 block(launch->block[0], launch->block[1], launch->block[2]);
  unsigned smem = launch->shared_bytes;
  if (!fix_alignment(dtype, a.in, &path, &grid, &block, &smem, a)) return T4A_ERR_LAUNCH_LIMIT;
  prefer_warp_rows(dtype, a.in, &path, &grid, &block, &smem, a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {
    // Not reached by the planner's geometry (at most 32 KiB); kept explicit.
    return T4A_ERR_LAUNCH_LIMIT;
  }
  prefer_strided_staged(dtype, &path, &grid, &smem, a);
  cap_cube_grid(path, &grid);
#define T4A_CALL(OP, T) launch_path<OP, T>(path, grid, block, smem, s, a)
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
  return runtime::check_launch();
}

}  // namespace
}  // namespace t4a

using namespace t4a;

extern "C" {

int t4a_launch_reduce(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype, int op,
                      int strategy, t4a_cuda_layout out_layout, t4a_cuda_layout in_layout, int axis,
                      long long output_len) {
  (void)strategy;  // carried by the launch's path
  PassArgs a{out, in, out_layout, in_layout, axis, output_len, 1, in_layout.extents[axis], false};
  return run_pass(launch, stream, dtype, op, a);
}

int t4a_launch_reduce_partials(const t4a_launch* launch, void* stream, void* partials, const void* in,
                               int dtype, int op, t4a_cuda_layout partials_layout, t4a_cuda_layout in_layout,
                               int axis, long long output_len, long long splits, long long chunk_len) {
  PassArgs a{partials, in, partials_layout, in_layout, axis, output_len, splits, chunk_len, true};
  return run_pass(launch, stream, dtype, op, a);
}

int t4a_reduce_any_geometry(int strategy, unsigned w, long long output_len, long long splits, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (output_len < 0 || splits < 1) return T4A_ERR_NEGATIVE_COUNT;
  if (strategy != T4A_CUDA_REDUCE_UNIT && strategy != T4A_CUDA_REDUCE_PLANE) return T4A_ERR_UNSUPPORTED_OP;
  const bool narrow = w == 8 || w == 16 || w == 32;
  const bool wide = w == 64 || w == 128 || w == 256 || w == 512;
  if (!narrow && !(wide && strategy == T4A_CUDA_REDUCE_PLANE && splits == 1)) return T4A_ERR_INVALID_PLANE_WIDTH;
  const unsigned long long cubes = static_cast<unsigned long long>(output_len) * static_cast<unsigned long long>(splits);
  if (cubes == 0) {
    *launch = plan::empty_launch();
    return T4A_OK;
  }
  const unsigned long long cap = 148ull * 64;
  unsigned long long grid;
  if (strategy == T4A_CUDA_REDUCE_UNIT) {
    grid = plan::ceil_div(cubes, kTileThreads);
    *launch = plan::make_launch(grid < cap ? grid : cap, kTileThreads, 1, 0, 0);
  } else if (wide) {
    *launch = plan::make_launch(cubes < cap ? cubes : cap, w, 1, 0, 0);
  } else {
    grid = plan::ceil_div(cubes, kTileThreads / w);
    *launch = plan::make_launch(grid < cap ? grid : cap, w, kTileThreads / w, 0, 0);
  }
  return T4A_OK;
}

int t4a_launch_reduce_any(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype, int op,
                          int strategy, t4a_cuda_layout_any out_layout, t4a_cuda_layout_any in_layout, int axis,
                          long long output_len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_any(out_layout));
  T4A_TRY(check_any(in_layout));
  if (axis < 0 || axis >= in_layout.rank || out_layout.rank != in_layout.rank) return T4A_ERR_INVALID_AXIS;
  if (launch->grid[0] == 0 || launch->grid[1] == 0 || launch->grid[2] == 0 || output_len <= 0) return T4A_OK;
  if (out == nullptr || in == nullptr) return T4A_ERR_NULL_ARGUMENT;
  const dim3 grid(launch->grid[0], launch->grid[1], launch->grid[2]);
  const dim3 block(launch->block[0], launch->block[1], launch->block[2]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define T4A_CALL(OP, T)                                                                                   \
  k_reduce_any<OP, T><<<grid, block, 0, s>>>(static_cast<T*>(out), static_cast<const T*>(in), strategy, \
                                             out_layout, in_layout, axis, output_len)
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
  return runtime::check_launch();
}

int t4a_launch_reduce_partials_any(const t4a_launch* launch, void* stream, void* partials, const void* in,
                                   int dtype, int op, t4a_cuda_layout_any partials_layout,
                                   t4a_cuda_layout_any in_layout, int axis, long long output_len, long long splits,
                                   long long chunk_len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_any(partials_layout));
  T4A_TRY(check_any(in_layout));
  if (axis < 0 || axis >= in_layout.rank || partials_layout.rank != in_layout.rank) return T4A_ERR_INVALID_AXIS;
  if (splits < 1 || chunk_len < 1) return T4A_ERR_INVALID_SPLIT;
  if (launch->grid[0] == 0 || launch->grid[1] == 0 || launch->grid[2] == 0 || output_len <= 0) return T4A_OK;
  if (partials == nullptr || in == nullptr) return T4A_ERR_NULL_ARGUMENT;
  const dim3 grid(launch->grid[0], launch->grid[1], launch->grid[2]);
  const dim3 block(launch->block[0], launch->block[1], launch->block[2]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define T4A_CALL(OP, T)                                                                                          \
  k_partials_any<OP, T><<<grid, block, 0, s>>>(static_cast<T*>(partials), static_cast<const T*>(in),          \
                                               partials_layout, in_layout, axis, output_len, splits, chunk_len)
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
  return runtime::check_launch();
}

int t4a_reduce_workspace_bytes(int dtype, int op, const t4a_cuda_layout* out, long long out_len,
                               const t4a_cuda_layout* in, long long in_len, unsigned axis, unsigned w,
                               size_t* bytes) {
  if (bytes == nullptr) return T4A_ERR_NULL_ARGUMENT;
  t4a_reduction_plan plan;
  T4A_TRY(t4a_plan_reduction(dtype, op, out, out_len, in, in_len, axis, w, &plan));
  *bytes = 0;
  if (!plan.is_split) return T4A_OK;
  t4a_cuda_layout partials;
  T4A_TRY(t4a_reduction_partials_layout(in, axis, plan.split.splits, &partials));
  long long count;
  T4A_TRY(plan::element_count(partials, &count));
  *bytes = static_cast<size_t>(count) * plan::dtype_size(dtype);
  return T4A_OK;
}

int t4a_reduce(void* stream, int dtype, int op, void* out, const t4a_cuda_layout* out_layout, long long out_len,
               const void* in, const t4a_cuda_layout* in_layout, long long in_len, unsigned axis, unsigned w,
               void* workspace, size_t workspace_bytes) {
  if (out == nullptr || in == nullptr) return T4A_ERR_NULL_ARGUMENT;
  t4a_reduction_plan plan;
  T4A_TRY(t4a_plan_reduction(dtype, op, out_layout, out_len, in_layout, in_len, axis, w, &plan));
  long long outputs;
  T4A_TRY(plan::element_count(*out_layout, &outputs));
  if (!plan.is_split) {
    return t4a_launch_reduce(&plan.launch, stream, out, in, dtype, op, plan.strategy, *out_layout, *in_layout,
                             static_cast<int>(axis), outputs);
  }
  t4a_cuda_layout partials;
  T4A_TRY(t4a_reduction_partials_layout(in_layout, axis, plan.split.splits, &partials));
  long long count;
  T4A_TRY(plan::element_count(partials, &count));
  const size_t need = static_cast<size_t>(count) * plan::dtype_size(dtype);
  if (workspace == nullptr || workspace_bytes < need) return T4A_ERR_WORKSPACE;
  T4A_TRY(t4a_launch_reduce_partials(&plan.pass1, stream, workspace, in, dtype, op, partials, *in_layout,
                                     static_cast<int>(axis), outputs, plan.split.splits, plan.split.chunk_len));
  PassArgs a{out, workspace, *out_layout, partials, static_cast<int>(axis), outputs, 1, partials.extents[axis], false,
             true};
  return run_pass(&plan.pass2, stream, dtype, plan.combine_op, a);
}

}  // extern "C"
