// Device bodies of the single-axis reductions (sm_100a), shared by the exported ABI
// symbols (reduce_abi.cu) and the per-path kernels the host launchers use
// (reduce_fast.cu).
//
// Both entries keep the reference ABI's symbols, signatures and numerical topology
// (reference cuda/src/reduce.cu:765-852; topology: docs/abi/c-kernel-abi.md
// "Revision 3: reductions", revisions 12-14):
//   * pass 1 folds cube (output o, split s) = chunk [s*chunk, end) of the axis with W
//     lanes: the revision-13 group walk on a contiguous chunk of a regroupable op over
//     4/8-byte reals and integers, the serial lane-strided walk otherwise, then the
//     ascending xor tree;
//   * `t4a_cuda_reduce` folds a whole axis: serially per output (UNIT) or with a
//     blockDim.x-lane plane (PLANE; lanes walk serially, then the balanced tree).
// What differs from the reference is only which thread computes what, so every result
// is bit-identical to the reference topology:
//   * a strided reduce axis with a unit-stride run of outputs is walked by tiles of
//     contiguous outputs (16-byte loads across outputs, W lanes spread over threads),
//     and the lane tree finishes in registers and shared memory;
//   * a short contiguous axis under UNIT is staged through shared memory so that the
//     global loads are coalesced 16-byte vectors and each thread folds one output;
//   * everything else uses one W-lane plane per cube, like the reference.
// The plane width W is blockDim.x (<= 32; 32 for a wider pass-1 block, the reference's
// rule), so a launch with the reference's own geometry computes the same values.
// All loops are grid-stride, so any grid is correct.
#pragma once

#include "common.cuh"
#include "reduce_paths.h"

namespace t4a {
namespace {

__device__ __forceinline__ unsigned dynamic_smem_bytes() {
  unsigned r;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

extern __shared__ __align__(16) unsigned char t4a_dyn_smem[];

// ---------------------------------------------------------------------------
// Lane walks (one lane of one W-lane plane).
// ---------------------------------------------------------------------------

// Serial walk: lane t seeds from start + t and folds start + t + k*W in order.  The
// loads of a batch are issued before any is folded; the fold order is unchanged.
template <typename Op, typename T>
__device__ __forceinline__ T serial_walk(const T* in, long long base, long long stride,
                                         long long start, long long end, int W, int lane, Op op) {
  // Loads per batch: 64 bytes' worth (at least 4), and 8 for 16-byte elements, whose
  // lane walks over a 256-element chunk are then a single batch.
  constexpr int B = sizeof(T) >= 16 ? 8 : ((64 / static_cast<int>(sizeof(T))) < 4 ? 4 : 64 / static_cast<int>(sizeof(T)));
  long long i = start + lane;
  if (end > 0x7fffffffffffffffLL - static_cast<long long>(B) * W) {
    T acc = op.seed(in[base + i * stride]);
    for (i += W; i < end; i += W) acc = op.fold(acc, in[base + i * stride]);
    return acc;
  }
  T buf[B];
#pragma unroll
  for (int b = 0; b < B; ++b)
    if (b == 0 || i + b * W < end) buf[b] = in[base + (i + b * W) * stride];
  T acc = op.seed(buf[0]);
#pragma unroll
  for (int b = 1; b < B; ++b)
    if (i + b * W < end) acc = op.fold(acc, buf[b]);
  for (i += static_cast<long long>(B) * W; i < end; i += static_cast<long long>(B) * W) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (i + b * W < end) buf[b] = in[base + (i + b * W) * stride];
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (i + b * W < end) acc = op.fold(acc, buf[b]);
  }
  return acc;
}

// Value of one V-element group: the pairwise tree of its seeded elements.
template <typename Op, typename T, int V>
__device__ __forceinline__ T group_value(const Vec<T, V>& x, Op op) {
  if constexpr (V == 4) {
    return op.combine(op.combine(op.seed(x.v[0]), op.seed(x.v[1])),
                      op.combine(op.seed(x.v[2]), op.seed(x.v[3])));
  } else {
    return op.combine(op.seed(x.v[0]), op.seed(x.v[1]));
  }
}

// The revision-13 group walk over a contiguous chunk of `len` elements: lane t takes
// groups t, t+W, ... in batches of four (first group seeds, next three join one at a
// time; each later whole batch joins as (g0.g1).(g2.g3); the remainder joins one at a
// time), then folds tail element groups*V + t.  `Aligned` only selects 16-byte loads.
template <typename Op, typename T, bool Aligned>
__device__ __noinline__ T group_walk(const T* chunk, long long len, int W, int lane, Op op) {
  constexpr int V = VecOf<T>::kLanes;
  using G = Vec<T, V>;
  auto load = [&](long long g) -> G {
    if constexpr (Aligned) {
      return reinterpret_cast<const G*>(chunk)[g];
    } else {
      G x;
#pragma unroll
      for (int c = 0; c < V; ++c) x.v[c] = chunk[g * V + c];
      return x;
    }
  };
  const long long groups = len / V;
  const long long w = W;
  G batch[4];
#pragma unroll
  for (int b = 0; b < 4; ++b)
    if (b == 0 || lane + b * w < groups) batch[b] = load(lane + b * w);
  T acc = group_value<Op, T, V>(batch[0], op);
#pragma unroll
  for (int b = 1; b < 4; ++b)
    if (lane + b * w < groups) acc = op.combine(acc, group_value<Op, T, V>(batch[b], op));
  long long index = lane + 4 * w;
  for (; index + 3 * w < groups; index += 4 * w) {
#pragma unroll
    for (int b = 0; b < 4; ++b) batch[b] = load(index + b * w);
    const T low = op.combine(group_value<Op, T, V>(batch[0], op), group_value<Op, T, V>(batch[1], op));
    const T high = op.combine(group_value<Op, T, V>(batch[2], op), group_value<Op, T, V>(batch[3], op));
    acc = op.combine(acc, op.combine(low, high));
  }
#pragma unroll
  for (int b = 0; b < 3; ++b)
    if (index + b * w < groups) batch[b] = load(index + b * w);
#pragma unroll
  for (int b = 0; b < 3; ++b)
    if (index + b * w < groups) acc = op.combine(acc, group_value<Op, T, V>(batch[b], op));
  const long long tail = groups * V;
  if (lane < len - tail) acc = op.fold(acc, chunk[tail + lane]);
  return acc;
}

template <typename Op, typename T>
__device__ __forceinline__ constexpr bool group_walk_enabled() {
  return Op::kRegroup && (sizeof(T) == 4 || sizeof(T) == 8) && VecOf<T>::kLanes >= 2;
}

// Fold of one cube's chunk by one lane: group walk or serial walk (reference rule).
template <typename Op, typename T>
__device__ __forceinline__ T cube_lane(const T* in, long long base, long long stride, long long start,
                                       long long end, int W, int lane, bool allow_groups, Op op) {
  if constexpr (group_walk_enabled<Op, T>()) {
    constexpr int V = VecOf<T>::kLanes;
    if (allow_groups && stride == 1 && (end - start) / V >= W) {
      const T* chunk = in + base + start;
      if ((reinterpret_cast<unsigned long long>(chunk) & 15ull) == 0)
        return group_walk<Op, T, true>(chunk, end - start, W, lane, op);
      return group_walk<Op, T, false>(chunk, end - start, W, lane, op);
    }
  }
  return serial_walk<Op, T>(in, base, stride, start, end, W, lane, op);
}

// ---------------------------------------------------------------------------
// Output addressing.
// ---------------------------------------------------------------------------

// Input base and destination offset of output `o` (flat over the output extents,
// whose reduce axis has extent one).
__device__ __forceinline__ void output_offsets(long long o, const t4a_cuda_layout& dst,
                                               const t4a_cuda_layout& in, long long* in_base,
                                               long long* dst_offset) {
  long long rest = o, base = in.offset, off = dst.offset;
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d < dst.rank) {
      const long long e = dst.extents[d];
      const long long c = rest % e;
      rest /= e;
      base += c * in.strides[d];
      off += c * dst.strides[d];
    }
  }
  *in_base = base;
  *dst_offset = off;
}

// Same for a partials destination, whose `axis` extent is the split count: the output
// index runs over the other axes only.
__device__ __forceinline__ void partial_offsets(long long o, const t4a_cuda_layout& dst,
                                                const t4a_cuda_layout& in, int axis,
                                                long long* in_base, long long* dst_offset) {
  long long rest = o, base = in.offset, off = dst.offset;
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d < dst.rank && d != axis) {
      const long long e = dst.extents[d];
      const long long c = rest % e;
      rest /= e;
      base += c * in.strides[d];
      off += c * dst.strides[d];
    }
  }
  *in_base = base;
  *dst_offset = off;
}

// Output decoders shared by the plane, wide and unit walks: (output, split) -> input
// base and destination offset, for the by-value layouts (rank <= 8) and for the
// general-rank `_any` layouts, whose arrays live in device memory (reference
// reduce.cu:641-656, :726-745: the same walk over the operand's runtime rank).
struct FastDecode {
  const t4a_cuda_layout* dst;
  const t4a_cuda_layout* in;
  int axis;
  bool partials;
  __device__ __forceinline__ void operator()(long long o, long long s, long long* base, long long* off) const {
    if (partials) {
      partial_offsets(o, *dst, *in, axis, base, off);
      *off += s * dst->strides[axis];
    } else {
      output_offsets(o, *dst, *in, base, off);
    }
  }
};

struct AnyDecode {
  const t4a_cuda_layout_any* dst;
  const t4a_cuda_layout_any* in;
  int axis;
  bool partials;
  __device__ __forceinline__ void operator()(long long o, long long s, long long* in_base,
                                             long long* dst_offset) const {
    long long rest = o, base = in->offset, off = dst->offset;
    for (int d = 0; d < dst->rank; ++d) {
      if (partials && d == axis) {
        off += s * dst->strides[d];
        continue;
      }
      const long long e = dst->extents[d];
      const long long c = rest % e;
      rest /= e;
      base += c * in->strides[d];
      off += c * dst->strides[d];
    }
    *in_base = base;
    *dst_offset = off;
  }
};

// ---------------------------------------------------------------------------
// Strided axis: one tile = 32 vector slots (V contiguous outputs each, slots run over
// the unit-stride output run, then the outer outputs) x all W = 8*LPT lanes x one
// split.  Thread (tx, ty) walks lanes ty*LPT .. ty*LPT+LPT-1 of slot tx serially (the
// reference's serial lane walk, rows start + lane + k*W), folds its lanes with the
// balanced tree, and the 8 lane groups meet in shared memory, lower lanes on the left.
// ---------------------------------------------------------------------------
struct StridedCtx {
  long long len;        // axis length
  long long astride;    // axis stride
  long long splits;     // 1 for a direct plane
  long long chunk;
  long long vectors;    // vectors per inner run
  long long slots;      // vectors * outer outputs
  int inner_r;          // axes [0, inner_r) form the unit-stride run
  int axis;
  bool partials;        // destination is a partials layout
};

__device__ __forceinline__ StridedCtx strided_ctx(const t4a_cuda_layout& in_l, int axis, long long splits,
                                                  long long chunk, int V, bool partials) {
  const InnerRun run = inner_run(in_l, axis);
  StridedCtx c;
  c.len = in_l.extents[axis];
  c.astride = in_l.strides[axis];
  c.splits = splits;
  c.chunk = chunk;
  c.vectors = run.ext / V;
  c.slots = c.vectors * outer_count(in_l, axis, run.r);
  c.inner_r = run.r;
  c.axis = axis;
  c.partials = partials;
  return c;
}

template <typename Op, typename T, int V, int LPT>
__device__ __forceinline__ void strided_tiles(const T* __restrict__ in, T* __restrict__ dst,
                                              const t4a_cuda_layout& in_l, const t4a_cuda_layout& dst_l,
                                              const StridedCtx& c, Op op) {
  constexpr int W = LPT * kLaneGroups;
  constexpr int MB = LPT >= 8 ? 1 : 8 / LPT;  // rows per lane per load batch
  T* red = reinterpret_cast<T*>(t4a_dyn_smem);
  const int tid = flat_tid();
  const int tx = tid % kSlotsPerTile;
  const int ty = tid / kSlotsPerTile;
  const long long slot_tiles = (c.slots + kSlotsPerTile - 1) / kSlotsPerTile;
  const long long tiles = slot_tiles * c.splits;
  const long long lane0 = static_cast<long long>(ty) * LPT;

  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const long long s = tile / slot_tiles;
    const long long slot = (tile % slot_tiles) * kSlotsPerTile + tx;
    const bool valid = slot < c.slots;
    const long long q = valid ? slot / c.vectors : 0;
    const long long vi = valid ? slot % c.vectors : 0;
    long long in_q = in_l.offset, dst_q = dst_l.offset;
    {
      long long rest = q;
#pragma unroll
      for (int d = 0; d < kMaxRank; ++d) {
        if (d < in_l.rank && d >= c.inner_r && d != c.axis) {
          const long long e = in_l.extents[d];
          const long long k = rest % e;
          rest /= e;
          in_q += k * in_l.strides[d];
          dst_q += k * dst_l.strides[d];
        }
      }
    }
    const T* base = in + in_q + vi * V;
    const long long start = s * c.chunk;
    const long long end = s + 1 == c.splits ? c.len : start + c.chunk;

    Vec<T, V> acc[LPT];
    Vec<T, V> buf[MB][LPT];
    for (long long m = 0;; m += MB) {
      const long long row_m = start + lane0 + m * W;
      if (row_m >= end) break;
#pragma unroll
      for (int mb = 0; mb < MB; ++mb)
#pragma unroll
        for (int l = 0; l < LPT; ++l) {
          const long long row = row_m + l + static_cast<long long>(mb) * W;
          if (valid && row < end) buf[mb][l] = load_vec<T, V>(base + row * c.astride);
        }
#pragma unroll
      for (int mb = 0; mb < MB; ++mb)
#pragma unroll
        for (int l = 0; l < LPT; ++l) {
          const long long row = row_m + l + static_cast<long long>(mb) * W;
          if (row < end) {
#pragma unroll
            for (int v = 0; v < V; ++v)
              acc[l].v[v] = (m + mb == 0) ? op.seed(buf[mb][l].v[v]) : op.fold(acc[l].v[v], buf[mb][l].v[v]);
          }
        }
    }
#pragma unroll
    for (int w = 1; w < LPT; w *= 2)
#pragma unroll
      for (int l = 0; l + w < LPT; l += 2 * w)
#pragma unroll
        for (int v = 0; v < V; ++v) acc[l].v[v] = op.combine(acc[l].v[v], acc[l + w].v[v]);
    Vec<T, V> mine = acc[0];
#pragma unroll
    for (int w = 1; w < kLaneGroups; w *= 2) {
      if (ty % (2 * w) == w) {
#pragma unroll
        for (int v = 0; v < V; ++v) red[(ty * kSlotsPerTile + tx) * V + v] = mine.v[v];
      }
      __syncthreads();
      if (ty % (2 * w) == 0) {
#pragma unroll
        for (int v = 0; v < V; ++v) mine.v[v] = op.combine(mine.v[v], red[((ty + w) * kSlotsPerTile + tx) * V + v]);
      }
      __syncthreads();
    }
    if (ty == 0 && valid) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        long long rest = vi * V + v, off = dst_q;
#pragma unroll
        for (int d = 0; d < kMaxRank; ++d) {
          if (d < c.inner_r) {
            const long long e = in_l.extents[d];
            off += (rest % e) * dst_l.strides[d];
            rest /= e;
          }
        }
        if (c.partials) off += s * dst_l.strides[c.axis];
        dst[off] = mine.v[v];
      }
    }
  }
}

// One (slot, split) unit of the staged strided pass: rows [start, end) of the chunk,
// the slot's input and destination bases, and its stage count.
struct StridedTile {
  long long start, end, s, vi, in_q, dst_q;
  int nk;       // stages of W rows
  bool valid;   // the slot exists
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}

// Staged variant of strided_tiles for 16-byte vectors (V > 1): the same lanes, folds
// and tree, with every warp working on its own units so that no block barrier is needed.  A unit is kWarpSlots
// consecutive vector slots of one split; lane = ty * kWarpSlots + tx holds slot tx and
// the plane lanes [ty * LPT, ty * LPT + LPT) (LPT * 32 / kWarpSlots == 32 plane lanes).
// Each thread copies its LPT rows of a stage with 16-byte cp.async into its own slice
// of a D-stage ring and folds them once its own copies have landed; a producer cursor
// runs D stages ahead across the warp's units.  The plane tree pairs lanes at distances
// 1, 2, 4 inside the thread, then 8 and 16 across threads by shuffles, each pair
// combined as (lower, higher), the order of strided_tiles' tree.  Every lane must own
// at least one row (chunk >= 32): the host takes this path only then.
// Shared memory: D * LPT * blockDim * 16 bytes.
constexpr int kWarpSlots = 8;

template <typename Op, typename T, int V, int LPT, int D>
__device__ __forceinline__ void strided_warp_staged(const T* __restrict__ in, T* __restrict__ dst,
                                                    const t4a_cuda_layout& in_l, const t4a_cuda_layout& dst_l,
                                                    const StridedCtx& c, Op op) {
  static_assert(V * sizeof(T) == 16, "16-byte vectors");
  static_assert(LPT * (32 / kWarpSlots) == 32, "LPT lanes per thread cover the 32-lane plane");
  constexpr int W = 32;
  const int nthreads = block_threads();
  Vec<T, V>* ring = reinterpret_cast<Vec<T, V>*>(t4a_dyn_smem);  // [D][LPT][nthreads]
  const int tid = flat_tid();
  const int lane = tid & 31;
  const int tx = lane % kWarpSlots;
  const int ty = lane / kWarpSlots;
  const long long gw = static_cast<long long>(blockIdx.x) * (nthreads >> 5) + (tid >> 5);
  const long long nw = static_cast<long long>(gridDim.x) * (nthreads >> 5);
  const long long slot_units = (c.slots + kWarpSlots - 1) / kWarpSlots;
  const long long units = slot_units * c.splits;
  const long long lane0 = static_cast<long long>(ty) * LPT;

  auto unit_of = [&](long long u) {
    StridedTile t;
    t.s = u / slot_units;
    const long long slot = (u % slot_units) * kWarpSlots + tx;
    t.valid = slot < c.slots;
    const long long q = t.valid ? slot / c.vectors : 0;
    t.vi = t.valid ? slot % c.vectors : 0;
    t.in_q = in_l.offset;
    t.dst_q = dst_l.offset;
    long long rest = q;
#pragma unroll
    for (int d = 0; d < kMaxRank; ++d) {
      if (d < in_l.rank && d >= c.inner_r && d != c.axis) {
        const long long e = in_l.extents[d];
        const long long k = rest % e;
        rest /= e;
        t.in_q += k * in_l.strides[d];
        t.dst_q += k * dst_l.strides[d];
      }
    }
    t.start = t.s * c.chunk;
    t.end = t.s + 1 == c.splits ? c.len : t.start + c.chunk;
    t.nk = static_cast<int>((t.end - t.start + W - 1) / W);
    return t;
  };

  long long p_unit = gw;
  int p_k = 0;
  StridedTile pt{};
  if (p_unit < units) pt = unit_of(p_unit);
  int p_slot = 0;
  auto issue = [&]() {
    if (p_unit < units) {
      const T* base = in + pt.in_q + pt.vi * V;
#pragma unroll
      for (int l = 0; l < LPT; ++l) {
        const long long row = pt.start + static_cast<long long>(p_k) * W + lane0 + l;
        if (pt.valid && row < pt.end) cp_async16(&ring[(p_slot * LPT + l) * nthreads + tid], base + row * c.astride);
      }
      if (++p_k == pt.nk) {
        p_k = 0;
        p_unit += nw;
        if (p_unit < units) pt = unit_of(p_unit);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    p_slot = p_slot + 1 == D ? 0 : p_slot + 1;
  };
#pragma unroll
  for (int i = 0; i < D; ++i) issue();

  int c_slot = 0;
  for (long long u = gw; u < units; u += nw) {
    const StridedTile t = unit_of(u);
    Vec<T, V> acc[LPT];
    // The first stage seeds every accumulator: a tile holds at least 32 rows (the
    // planner's condition for this pass), so each plane lane owns row lane0 + l.
    // Peeling it keeps the seed-or-fold select out of the per-element loop.
    asm volatile("cp.async.wait_group %0;" ::"n"(D - 1) : "memory");
#pragma unroll
    for (int l = 0; l < LPT; ++l) {
      const Vec<T, V> x = ring[(c_slot * LPT + l) * nthreads + tid];
#pragma unroll
      for (int v = 0; v < V; ++v) acc[l].v[v] = op.seed(x.v[v]);
    }
    c_slot = c_slot + 1 == D ? 0 : c_slot + 1;
    issue();
    for (int k = 1; k < t.nk; ++k) {
      asm volatile("cp.async.wait_group %0;" ::"n"(D - 1) : "memory");
      const long long row0 = t.start + static_cast<long long>(k) * W + lane0;
      if (row0 + LPT <= t.end) {
#pragma unroll
        for (int l = 0; l < LPT; ++l) {
          const Vec<T, V> x = ring[(c_slot * LPT + l) * nthreads + tid];
#pragma unroll
          for (int v = 0; v < V; ++v) acc[l].v[v] = op.fold(acc[l].v[v], x.v[v]);
        }
      } else {
#pragma unroll
        for (int l = 0; l < LPT; ++l) {
          if (row0 + l < t.end) {
            const Vec<T, V> x = ring[(c_slot * LPT + l) * nthreads + tid];
#pragma unroll
            for (int v = 0; v < V; ++v) acc[l].v[v] = op.fold(acc[l].v[v], x.v[v]);
          }
        }
      }
      c_slot = c_slot + 1 == D ? 0 : c_slot + 1;
      issue();  // into the slot just folded
    }
#pragma unroll
    for (int w = 1; w < LPT; w *= 2)
#pragma unroll
      for (int l = 0; l + w < LPT; l += 2 * w)
#pragma unroll
        for (int v = 0; v < V; ++v) acc[l].v[v] = op.combine(acc[l].v[v], acc[l + w].v[v]);
    Vec<T, V> mine = acc[0];
#pragma unroll
    for (int w = 1; w < 32 / kWarpSlots; w *= 2) {
      const bool upper = (ty & w) != 0;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const T other = shfl_xor<T>(mine.v[v], w * kWarpSlots, 0xffffffffu);
        if (!upper) mine.v[v] = op.combine(mine.v[v], other);
      }
    }
    if (ty == 0 && t.valid) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        long long rest = t.vi * V + v, off = t.dst_q;
#pragma unroll
        for (int d = 0; d < kMaxRank; ++d) {
          if (d < c.inner_r) {
            const long long e = in_l.extents[d];
            off += (rest % e) * dst_l.strides[d];
            rest /= e;
          }
        }
        if (c.partials) off += t.s * dst_l.strides[c.axis];
        dst[off] = mine.v[v];
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------------------
// One W-lane plane per cube (contiguous axis, and the general fallback).  Planes of
// one block are consecutive cubes; every lane of a warp reaches the shuffles.
// ---------------------------------------------------------------------------
template <typename Op, typename T, typename Dec>
__device__ __forceinline__ void plane_cubes_walk(const T* in, T* dst, const Dec& decode, long long astride,
                                                 long long len, long long outputs, long long splits, long long chunk,
                                                 int W, bool allow_groups, Op op) {
  const int tid = flat_tid();
  const int planes = block_threads() / W;
  const int plane = tid / W;
  const int lane = tid % W;
  const long long cubes = outputs * splits;
  for (long long first = static_cast<long long>(blockIdx.x) * planes; first < cubes;
       first += static_cast<long long>(gridDim.x) * planes) {
    const long long cube = first + plane;
    const bool valid = plane < planes && cube < cubes;
    T acc{};
    long long dst_off = 0;
    if (valid) {
      const long long o = cube / splits;
      const long long s = cube % splits;
      long long base;
      decode(o, s, &base, &dst_off);
      const long long start = s * chunk;
      const long long end = s + 1 == splits ? len : start + chunk;
      acc = cube_lane<Op, T>(in, base, astride, start, end, W, lane, allow_groups, op);
    }
    acc = lane_tree(acc, W, op);
    if (valid && lane == 0) dst[dst_off] = acc;
  }
}

template <typename Op, typename T>
__device__ __forceinline__ void plane_cubes(const T* in, T* dst, const t4a_cuda_layout& in_l,
                                            const t4a_cuda_layout& dst_l, int axis, long long outputs,
                                            long long splits, long long chunk, int W, bool partials,
                                            bool allow_groups, Op op) {
  const FastDecode decode{&dst_l, &in_l, axis, partials};
  plane_cubes_walk<Op, T>(in, dst, decode, in_l.strides[axis], in_l.extents[axis], outputs, splits, chunk, W,
                          allow_groups, op);
}

// ---------------------------------------------------------------------------
// UNIT: one serial fold per output.
// ---------------------------------------------------------------------------

// Short contiguous axis over a compact input: tiles of `rows` outputs (rows*len
// contiguous elements) are loaded with 16-byte vectors into shared memory with an odd
// row pitch, then thread r folds row r in order.
template <typename Op, typename T>
__device__ __forceinline__ void unit_rows(const T* in, T* out, const t4a_cuda_layout& out_l,
                                          const t4a_cuda_layout& in_l, long long outputs, int rows,
                                          Op op) {
  T* tile = reinterpret_cast<T*>(t4a_dyn_smem);
  const int len = static_cast<int>(in_l.extents[0]);
  const int pitch = len | 1;
  const int tid = flat_tid();
  const int threads = block_threads();
  constexpr int V = VecOf<T>::kLanes;
  const T* src = in + in_l.offset;
  const bool vec = V > 1 && (reinterpret_cast<unsigned long long>(src) & 15ull) == 0 &&
                   (static_cast<long long>(rows) * len) % V == 0;
  for (long long o0 = static_cast<long long>(blockIdx.x) * rows; o0 < outputs;
       o0 += static_cast<long long>(gridDim.x) * rows) {
    const int n_rows = static_cast<int>(outputs - o0 < rows ? outputs - o0 : rows);
    const int n_el = n_rows * len;
    const T* seg = src + o0 * len;
    int e0 = 0;
    if constexpr (V > 1) {
      if (vec) {
        const int n_vec = n_el / V;
        for (int i = tid; i < n_vec; i += threads) {
          const Vec<T, V> x = reinterpret_cast<const Vec<T, V>*>(seg)[i];
#pragma unroll
          for (int k = 0; k < V; ++k) {
            const int e = i * V + k;
            tile[(e / len) * pitch + e % len] = x.v[k];
          }
        }
        e0 = n_vec * V;
      }
    }
    for (int e = e0 + tid; e < n_el; e += threads) tile[(e / len) * pitch + e % len] = seg[e];
    __syncthreads();
    for (int r = tid; r < n_rows; r += threads) {
      const T* row = tile + r * pitch;
      T acc = op.seed(row[0]);
      for (int k = 1; k < len; ++k) acc = op.fold(acc, row[k]);
      long long base, off;
      output_offsets(o0 + r, out_l, in_l, &base, &off);
      out[off] = acc;
    }
    __syncthreads();
  }
}

// Warp-private variant of the rows path for rows of exactly L elements (L * sizeof(T) a
// multiple of 128 bytes): each warp stages the 32 rows of its outputs (a contiguous
// 32 L-element block) with coalesced 16-byte loads into its own shared slice, chunk c
// of row r at slot c ^ (r mod C) (C chunks per row, so both the staging stores and
// each lane's reads of its own row fill whole wavefronts), then lane r folds row r
// serially: the same fold as unit_rows, with no block barrier and no index division.
// `dst_linear`: output o lives at dst.offset + o.
template <typename Op, typename T, int L>
__device__ __forceinline__ void unit_warp_rows(const T* in, T* out, const t4a_cuda_layout& out_l,
                                               const t4a_cuda_layout& in_l, long long outputs, bool dst_linear,
                                               unsigned char* slice, Op op) {
  constexpr int kRowBytes = L * static_cast<int>(sizeof(T));
  constexpr int C = kRowBytes / 16;     // 16-byte chunks per row
  constexpr int E = 16 / sizeof(T);     // elements per chunk
  static_assert(kRowBytes % 128 == 0, "rows of whole 128-byte lines");
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const T* src = in + in_l.offset;
  const long long groups = (outputs + 31) / 32;
  for (long long g = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
       g += warps) {
    const long long o0 = g * 32;
    const int n = outputs - o0 < 32 ? static_cast<int>(outputs - o0) : 32;
    const uint4* gsrc = reinterpret_cast<const uint4*>(src + o0 * L);
    uint4 v[C];
#pragma unroll
    for (int k = 0; k < C; ++k) {
      const int q = lane + 32 * k;
      if (q < n * C) v[k] = gsrc[q];
    }
    __syncwarp();  // the previous group's reads of the slice are done
#pragma unroll
    for (int k = 0; k < C; ++k) {
      const int q = lane + 32 * k;
      const int r = q / C, c = q % C;
      if (q < n * C) *reinterpret_cast<uint4*>(slice + r * kRowBytes + ((c ^ (r % C)) << 4)) = v[k];
    }
    __syncwarp();
    if (lane < n) {
      const unsigned char* row = slice + lane * kRowBytes;
      T acc;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + ((c ^ (lane % C)) << 4));
        const T* x = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int j = 0; j < E; ++j) acc = (c == 0 && j == 0) ? op.seed(x[0]) : op.fold(acc, x[j]);
      }
      long long off;
      if (dst_linear) {
        off = out_l.offset + o0 + lane;
      } else {
        long long base;
        output_offsets(o0 + lane, out_l, in_l, &base, &off);
      }
      out[off] = acc;
    }
  }
}

template <typename Op, typename T, typename Dec>
__device__ __forceinline__ void unit_walk(const T* in, T* out, const Dec& decode, long long len, long long stride,
                                          long long outputs, Op op) {
  const long long threads = static_cast<long long>(gridDim.x) * block_threads();
  for (long long o = static_cast<long long>(blockIdx.x) * block_threads() + flat_tid(); o < outputs;
       o += threads) {
    long long base, off;
    decode(o, 0, &base, &off);
    T buf[8];
    T acc = op.seed(in[base]);
    long long i = 1;
    for (; i + 8 <= len; i += 8) {
#pragma unroll
      for (int b = 0; b < 8; ++b) buf[b] = in[base + (i + b) * stride];
#pragma unroll
      for (int b = 0; b < 8; ++b) acc = op.fold(acc, buf[b]);
    }
    for (; i < len; ++i) acc = op.fold(acc, in[base + i * stride]);
    out[off] = acc;
  }
}

template <typename Op, typename T>
__device__ __forceinline__ void unit_generic(const T* in, T* out, const t4a_cuda_layout& out_l,
                                             const t4a_cuda_layout& in_l, int axis, long long outputs,
                                             Op op) {
  const FastDecode decode{&out_l, &in_l, axis, false};
  unit_walk<Op, T>(in, out, decode, in_l.extents[axis], in_l.strides[axis], outputs, op);
}

// PLANE wider than a warp (the combine pass over many partials): one block per output;
// blockDim.x lanes walk serially, warp trees meet in shared memory, so the result is
// the balanced tree over all lanes.  Per-warp results: at most 16 warps of 16 bytes.
__shared__ __align__(16) unsigned char t4a_warp_results[16 * 16];

template <typename Op, typename T, typename Dec>
__device__ __forceinline__ void wide_walk(const T* in, T* out, const Dec& decode, long long len, long long stride,
                                          long long outputs, Op op) {
  T* warp_results = reinterpret_cast<T*>(t4a_warp_results);
  const int W = blockDim.x;
  const int lane = threadIdx.x;
  const int warps = W / kWarp;
  for (long long o = blockIdx.x; o < outputs; o += gridDim.x) {
    long long base, off;
    decode(o, 0, &base, &off);
    T acc = serial_walk<Op, T>(in, base, stride, 0, len, W, lane, op);
    acc = lane_tree(acc, kWarp, op);
    if ((lane & 31) == 0) warp_results[lane >> 5] = acc;
    __syncthreads();
    if (lane < kWarp) {
      T v = lane < warps ? warp_results[lane] : acc;
      v = lane_tree(v, warps, op);
      if (lane == 0) out[off] = v;
    }
    __syncthreads();
  }
}

template <typename Op, typename T>
__device__ __forceinline__ void wide_plane(const T* in, T* out, const t4a_cuda_layout& out_l,
                                           const t4a_cuda_layout& in_l, int axis, long long outputs,
                                           Op op) {
  const FastDecode decode{&out_l, &in_l, axis, false};
  wide_walk<Op, T>(in, out, decode, in_l.extents[axis], in_l.strides[axis], outputs, op);
}

// ---------------------------------------------------------------------------
// Runtime path selection for the exported ABI symbols (uniform per launch).
// ---------------------------------------------------------------------------
template <typename Op, typename T>
__device__ __forceinline__ bool strided_fits_launch(const T* in, const t4a_cuda_layout& in_l, int axis, int W) {
  constexpr int V = VecOf<T>::kLanes;
  if (block_threads() != kTileThreads || dynamic_smem_bytes() < static_cast<unsigned>(kStridedSmem)) return false;
  if (!strided_path_applies(in_l, axis, W, V)) return false;
  return V == 1 || (reinterpret_cast<unsigned long long>(in) & 15ull) == 0;
}

template <typename Op, typename T>
__device__ __forceinline__ void reduce_abi_body(void* out_p, const void* in_p, int strategy,
                                                const t4a_cuda_layout& out_l, const t4a_cuda_layout& in_l,
                                                int axis, long long outputs, Op op) {
  const T* in = static_cast<const T*>(in_p);
  T* out = static_cast<T*>(out_p);
  if (strategy == T4A_CUDA_REDUCE_UNIT) {
    const int rows = unit_rows_per_tile(in_l, axis, sizeof(T));
    if (rows > 0 && dynamic_smem_bytes() >= static_cast<unsigned>(unit_rows_smem(in_l, rows, sizeof(T)))) {
      unit_rows<Op, T>(in, out, out_l, in_l, outputs, rows, op);
    } else {
      unit_generic<Op, T>(in, out, out_l, in_l, axis, outputs, op);
    }
    return;
  }
  const int W = blockDim.x;
  if (W > kWarp) {
    wide_plane<Op, T>(in, out, out_l, in_l, axis, outputs, op);
    return;
  }
  const long long len = in_l.extents[axis];
  if (strided_fits_launch<Op, T>(in, in_l, axis, W)) {
    constexpr int V = VecOf<T>::kLanes;
    strided_tiles<Op, T, V, 4>(in, out, in_l, out_l, strided_ctx(in_l, axis, 1, len, V, false), op);
    return;
  }
  plane_cubes<Op, T>(in, out, in_l, out_l, axis, outputs, 1, len, W, false, false, op);
}

template <typename Op, typename T>
__device__ __forceinline__ void partials_abi_body(void* partials_p, const void* in_p,
                                                  const t4a_cuda_layout& part_l, const t4a_cuda_layout& in_l,
                                                  int axis, long long outputs, long long splits,
                                                  long long chunk, Op op) {
  const T* in = static_cast<const T*>(in_p);
  T* partials = static_cast<T*>(partials_p);
  const int W = blockDim.x <= 32 ? static_cast<int>(blockDim.x) : kWarp;
  if (strided_fits_launch<Op, T>(in, in_l, axis, W)) {
    constexpr int V = VecOf<T>::kLanes;
    strided_tiles<Op, T, V, 4>(in, partials, in_l, part_l, strided_ctx(in_l, axis, splits, chunk, V, true), op);
    return;
  }
  plane_cubes<Op, T>(in, partials, in_l, part_l, axis, outputs, splits, chunk, W, true, true, op);
}

// General-rank entries (reference reduce.cu:854-940): the same walks and trees as the
// by-value entries (unit fold, W-lane planes, wider planes, split partials), with the
// outputs decoded over the layouts' runtime rank.  Any launch geometry is correct: a
// block of W = blockDim.x lanes (at most a warp: blockDim.y planes of W lanes; wider:
// one output per block) walks outputs grid-stride.
template <typename Op, typename T>
__device__ __forceinline__ void reduce_any_body(void* out_p, const void* in_p, int strategy,
                                                const t4a_cuda_layout_any& out_l, const t4a_cuda_layout_any& in_l,
                                                int axis, long long outputs, Op op) {
  if (axis < 0 || axis >= in_l.rank || outputs <= 0) return;
  const T* in = static_cast<const T*>(in_p);
  T* out = static_cast<T*>(out_p);
  const AnyDecode decode{&out_l, &in_l, axis, false};
  const long long len = in_l.extents[axis];
  const long long stride = in_l.strides[axis];
  if (strategy == T4A_CUDA_REDUCE_UNIT) {
    unit_walk<Op, T>(in, out, decode, len, stride, outputs, op);
    return;
  }
  const int W = blockDim.x;
  if (W > kWarp) {
    wide_walk<Op, T>(in, out, decode, len, stride, outputs, op);
    return;
  }
  plane_cubes_walk<Op, T>(in, out, decode, stride, len, outputs, 1, len, W, false, op);
}

template <typename Op, typename T>
__device__ __forceinline__ void partials_any_body(void* partials_p, const void* in_p,
                                                  const t4a_cuda_layout_any& part_l,
                                                  const t4a_cuda_layout_any& in_l, int axis, long long outputs,
                                                  long long splits, long long chunk, Op op) {
  if (axis < 0 || axis >= in_l.rank || outputs <= 0 || splits <= 0) return;
  const int W = blockDim.x <= 32 ? static_cast<int>(blockDim.x) : kWarp;
  const AnyDecode decode{&part_l, &in_l, axis, true};
  plane_cubes_walk<Op, T>(static_cast<const T*>(in_p), static_cast<T*>(partials_p), decode, in_l.strides[axis],
                          in_l.extents[axis], outputs, splits, chunk, W, true, op);
}

}  // namespace
}  // namespace t4a

// Dispatch over the reference's (op, dtype) matrix: SUM/PROD F32 F64 I32 I64 C32 C64,
// SUM_SQUARES F32 F64, MAX/MIN F32 F64 I32 I64.  Unknown tags do no work.
#define T4A_REDUCE_SWITCH(OPTAG, DTYPE, CALL)                     \
  switch (OPTAG) {                                                \
    case T4A_CUDA_REDUCE_SUM:                                     \
      switch (DTYPE) {                                            \
        case T4A_CUDA_F32: CALL(t4a::OpSum, float); break;        \
        case T4A_CUDA_F64: CALL(t4a::OpSum, double); break;       \
        case T4A_CUDA_I32: CALL(t4a::OpSum, int); break;          \
        case T4A_CUDA_I64: CALL(t4a::OpSum, long long); break;    \
        case T4A_CUDA_C32: CALL(t4a::OpSum, t4a::c32); break;     \
        case T4A_CUDA_C64: CALL(t4a::OpSum, t4a::c64); break;     \
        default: break;                                           \
      }                                                           \
      break;                                                      \
    case T4A_CUDA_REDUCE_PROD:                                    \
      switch (DTYPE) {                                            \
        case T4A_CUDA_F32: CALL(t4a::OpProd, float); break;       \
        case T4A_CUDA_F64: CALL(t4a::OpProd, double); break;      \
        case T4A_CUDA_I32: CALL(t4a::OpProd, int); break;         \
        case T4A_CUDA_I64: CALL(t4a::OpProd, long long); break;   \
        case T4A_CUDA_C32: CALL(t4a::OpProd, t4a::c32); break;    \
        case T4A_CUDA_C64: CALL(t4a::OpProd, t4a::c64); break;    \
        default: break;                                           \
      }                                                           \
      break;                                                      \
    case T4A_CUDA_REDUCE_SUM_SQUARES:                             \
      switch (DTYPE) {                                            \
        case T4A_CUDA_F32: CALL(t4a::OpSumSq, float); break;      \
        case T4A_CUDA_F64: CALL(t4a::OpSumSq, double); break;     \
        default: break;                                           \
      }                                                           \
      break;                                                      \
    case T4A_CUDA_REDUCE_MAX:                                     \
      switch (DTYPE) {                                            \
        case T4A_CUDA_F32: CALL(t4a::OpMax, float); break;        \
        case T4A_CUDA_F64: CALL(t4a::OpMax, double); break;       \
        case T4A_CUDA_I32: CALL(t4a::OpMax, int); break;          \
        case T4A_CUDA_I64: CALL(t4a::OpMax, long long); break;    \
        default: break;                                           \
      }                                                           \
      break;                                                      \
    case T4A_CUDA_REDUCE_MIN:                                     \
      switch (DTYPE) {                                            \
        case T4A_CUDA_F32: CALL(t4a::OpMin, float); break;        \
        case T4A_CUDA_F64: CALL(t4a::OpMin, double); break;       \
        case T4A_CUDA_I32: CALL(t4a::OpMin, int); break;          \
        case T4A_CUDA_I64: CALL(t4a::OpMin, long long); break;    \
        default: break;                                           \
      }                                                           \
      break;                                                      \
    default:                                                      \
      break;                                                      \
  }
