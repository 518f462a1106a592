// Exported gather / scatter symbols of the kernel ABI, for callers that load the
// module and launch by name (reference signatures cuda/src/gather_scatter.cu:454-458,
// :486-492).  Each block builds the window plan once into shared memory, then runs
// the warp paths of gather_scatter_core.cuh.  Any geometry is correct: a block that
// is not whole warps takes the element-per-thread walk.
#include "gather_scatter_core.cuh"

namespace t4a {
namespace {

__device__ __forceinline__ int gs_esize(int dtype) {
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

__device__ __forceinline__ bool whole_warps() {
  return blockDim.y == 1 && blockDim.z == 1 && (blockDim.x & 31) == 0;
}

template <typename I>
__device__ __forceinline__ void gather_dispatch(const WindowPlan& p, void* out, const void* operand,
                                                const void* indices, long long units, GatherSlot* slots) {
  auto* o = static_cast<unsigned char*>(out);
  const auto* a = static_cast<const unsigned char*>(operand);
  const I* idx = static_cast<const I*>(indices);
  if (!whole_warps()) {
    gather_elements<I>(p, o, a, idx, units);
    return;
  }
  const int v = window_vec_bytes(p, reinterpret_cast<unsigned long long>(out),
                                 reinterpret_cast<unsigned long long>(operand));
  const long long nvec = p.run * p.esize / v;
  const Pieces pc = make_pieces(nvec, kGatherPieceVecs);
  const int ls = lane_shift_of(pc.vecs);
  switch (v) {
    case 16: gather_units<I, 16>(p, o, a, idx, units, nvec, pc, ls, slots); break;
    case 8: gather_units<I, 8>(p, o, a, idx, units, nvec, pc, ls, slots); break;
    case 4: gather_units<I, 4>(p, o, a, idx, units, nvec, pc, ls, slots); break;
    case 2: gather_units<I, 2>(p, o, a, idx, units, nvec, pc, ls, slots); break;
    default: gather_units<I, 1>(p, o, a, idx, units, nvec, pc, ls, slots); break;
  }
}

template <typename F, typename I>
__device__ __forceinline__ void scatter_dispatch(const WindowPlan& p, void* out, const void* indices,
                                                 const void* updates, long long units, ScatterSmem& sm,
                                                 long long max_dst_bytes) {
  auto* o = static_cast<unsigned char*>(out);
  const auto* u = static_cast<const unsigned char*>(updates);
  const I* idx = static_cast<const I*>(indices);
  const int v = window_vec_bytes(p, reinterpret_cast<unsigned long long>(out),
                                 reinterpret_cast<unsigned long long>(updates));
  // The grouped path packs destination offsets / v beside the position bits.
  if (!whole_warps() || max_dst_bytes / v >= kScatterMaxVecOffset) {
    scatter_elements<F, I>(p, o, u, idx, units);
    return;
  }
  const long long nvec = p.run * p.esize / v;
  if (v >= 16) {
    scatter_units<F, I, 16>(p, o, u, idx, units, nvec, sm);
  } else if (v == 8) {
    scatter_units<F, I, 8>(p, o, u, idx, units, nvec, sm);
  } else if constexpr (sizeof(F) == 4) {
    scatter_units<F, I, 4>(p, o, u, idx, units, nvec, sm);
  }
}

}  // namespace
}  // namespace t4a

using namespace t4a;

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_gather(
    void* out, const void* operand, const void* indices, int dtype, int index_dtype, t4a_cuda_layout out_layout,
    t4a_cuda_layout operand_layout, t4a_cuda_layout indices_layout, t4a_cuda_gather_plan plan, long long output_len) {
  __shared__ WindowPlan sp;
  __shared__ GatherSlot slots[256];  // 32 per warp of the (at most 256-thread) block
  const int es = gs_esize(dtype);
  if (es == 0 || output_len <= 0 || !gather_maps_ok(out_layout, operand_layout, indices_layout, plan)) return;
  if (flat_tid() == 0) sp = make_gather_plan(out_layout, operand_layout, indices_layout, plan, es);
  __syncthreads();
  if (sp.run <= 0) return;
  const long long units = sp.batch.len * sp.wrest.len;
  switch (index_dtype) {
    case T4A_CUDA_F32: gather_dispatch<float>(sp, out, operand, indices, units, slots); break;
    case T4A_CUDA_F64: gather_dispatch<double>(sp, out, operand, indices, units, slots); break;
    case T4A_CUDA_I32: gather_dispatch<int>(sp, out, operand, indices, units, slots); break;
    case T4A_CUDA_I64: gather_dispatch<long long>(sp, out, operand, indices, units, slots); break;
    default: break;
  }
}

extern "C" __global__ void __launch_bounds__(512) t4a_cuda_scatter_add(
    void* out, const void* indices, const void* updates, int dtype, int index_dtype, t4a_cuda_layout out_layout,
    t4a_cuda_layout indices_layout, t4a_cuda_layout updates_layout, t4a_cuda_scatter_plan plan,
    long long update_len) {
  __shared__ WindowPlan sp;
  __shared__ ScatterSmem sm;
  int es = 0;
  switch (dtype) {
    case T4A_CUDA_F32: es = 4; break;
    case T4A_CUDA_F64: es = 8; break;
    case T4A_CUDA_C32: es = 8; break;
    case T4A_CUDA_C64: es = 16; break;
    default: return;
  }
  if (update_len <= 0 || !scatter_maps_ok(out_layout, indices_layout, updates_layout, plan)) return;
  if (flat_tid() == 0) sp = make_scatter_plan(out_layout, indices_layout, updates_layout, plan, es);
  __syncthreads();
  if (sp.run <= 0 || !scatter_windows_fit(sp)) return;
  const long long units = sp.batch.len * sp.wrest.len;
  const long long max_dst = (layout_max_offset(out_layout) + 1) * es;
  const bool dbl = dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_C64;  // component type
  switch (index_dtype) {
    case T4A_CUDA_F32:
      if (dbl) scatter_dispatch<double, float>(sp, out, indices, updates, units, sm, max_dst);
      else scatter_dispatch<float, float>(sp, out, indices, updates, units, sm, max_dst);
      break;
    case T4A_CUDA_F64:
      if (dbl) scatter_dispatch<double, double>(sp, out, indices, updates, units, sm, max_dst);
      else scatter_dispatch<float, double>(sp, out, indices, updates, units, sm, max_dst);
      break;
    case T4A_CUDA_I32:
      if (dbl) scatter_dispatch<double, int>(sp, out, indices, updates, units, sm, max_dst);
      else scatter_dispatch<float, int>(sp, out, indices, updates, units, sm, max_dst);
      break;
    case T4A_CUDA_I64:
      if (dbl) scatter_dispatch<double, long long>(sp, out, indices, updates, units, sm, max_dst);
      else scatter_dispatch<float, long long>(sp, out, indices, updates, units, sm, max_dst);
      break;
    default: break;
  }
}

// ---- general-rank twins (`_any`, reference cuda/src/gather_scatter.cu:587, :619) ----
// Element-wise walks over layouts and maps in device memory (gather_scatter_any.cuh).
#include "gather_scatter_any.cuh"

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_gather_any(
    void* out, const void* operand, const void* indices, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
    t4a_cuda_layout_any operand_layout, t4a_cuda_layout_any indices_layout, t4a_cuda_gather_plan_any plan,
    long long output_len) {
  t4a::any::gather_entry(out, operand, indices, dtype, index_dtype, out_layout, operand_layout, indices_layout, plan,
                         output_len);
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_scatter_add_any(
    void* out, const void* indices, const void* updates, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
    t4a_cuda_layout_any indices_layout, t4a_cuda_layout_any updates_layout, t4a_cuda_scatter_plan_any plan,
    long long update_len) {
  t4a::any::scatter_entry(out, indices, updates, dtype, index_dtype, out_layout, indices_layout, updates_layout, plan,
                          update_len);
}
