// Device bodies of the strided movement entries (sm_100a), shared by the exported
// ABI symbols (movement_abi.cu) and the host launchers (movement_fast.cu).
//
// Movement is a bit copy, so the bodies are templated on the element size only.
// Every path is a grid-stride loop over its work units.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "movement_plan.h"

namespace t4a {
namespace {

template <int kBytes>
struct Elem;
template <>
struct Elem<1> {
  using T = unsigned char;
};
template <>
struct Elem<4> {
  using T = unsigned int;
};
template <>
struct Elem<8> {
  using T = unsigned long long;
};
struct alignas(8) Bytes16 {
  unsigned long long lo, hi;
};
template <>
struct Elem<16> {
  using T = Bytes16;
};

extern __shared__ __align__(16) unsigned char t4a_move_smem[];

// One 16-byte vector of `V` elements (V * sizeof(E) == 16), or a single element.
template <typename E, int V>
__device__ __forceinline__ void copy_vec(E* dst, const E* src) {
  if constexpr (V > 1) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  } else {
    *dst = *src;
  }
}

// ---------------------------------------------------------------------------
// Rows: the shared run is contiguous on both sides.  A work unit is R rows x one
// segment of up to `seg` elements of the run; row offsets are decoded once per
// unit into shared memory, then the block copies V-element vectors.
// ---------------------------------------------------------------------------
template <typename E, int V>
__device__ __forceinline__ void perm_rows(const PermPlan& p, E* __restrict__ dst, const E* __restrict__ src) {
  long long* row_src = reinterpret_cast<long long*>(t4a_move_smem);
  const long long run = p.run.len;
  const long long seg = run < kPermRowsBytes / p.esize ? run : kPermRowsBytes / p.esize;
  const int rows_per_unit = static_cast<int>(kPermRowsBytes / p.esize / seg);  // >= 1
  long long* row_dst = row_src + rows_per_unit;
  const long long segs = (run + seg - 1) / seg;
  const long long row_units = (p.rest.len + rows_per_unit - 1) / rows_per_unit;
  const long long units = row_units * segs;
  const int tid = flat_tid();
  const int threads = block_threads();
  for (long long u = blockIdx.x; u < units; u += gridDim.x) {
    const long long g = u % segs;
    const long long r0 = (u / segs) * rows_per_unit;
    const int nrows = static_cast<int>(p.rest.len - r0 < rows_per_unit ? p.rest.len - r0 : rows_per_unit);
    for (int r = tid; r < nrows; r += threads) {
      long long so, dof;
      group_offsets(p.rest, r0 + r, &so, &dof);
      row_src[r] = p.src_offset + so;
      row_dst[r] = p.dst_offset + dof;
    }
    __syncthreads();
    const long long c0 = g * seg;
    const long long clen = run - c0 < seg ? run - c0 : seg;
    const long long vecs_per_row = clen / V;
    const long long total = vecs_per_row * nrows;
    for (long long i = tid; i < total; i += threads) {
      const int r = static_cast<int>(i / vecs_per_row);
      const long long c = c0 + (i - r * vecs_per_row) * V;
      copy_vec<E, V>(dst + row_dst[r] + c, src + row_src[r] + c);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Tiles: EDGE positions of the D run (contiguous in the destination) x EDGE
// positions of the S run (contiguous in the source) per batch index.  Loads run
// along S with VS-element vectors into a padded shared tile; stores run along D
// with VD-element vectors.
// ---------------------------------------------------------------------------
template <typename E, int VS, int VD, int EDGE>
__device__ __forceinline__ void perm_tiles(const PermPlan& p, E* __restrict__ dst, const E* __restrict__ src) {
  constexpr int PITCH = EDGE + 1;
  E* tile = reinterpret_cast<E*>(t4a_move_smem);
  long long* off_d = reinterpret_cast<long long*>(t4a_move_smem + ((EDGE * PITCH * sizeof(E) + 15) & ~15));
  long long* off_s = off_d + EDGE;
  const long long dlen = p.run.len, slen = p.srun.len;
  const long long nt_d = (dlen + EDGE - 1) / EDGE, nt_s = (slen + EDGE - 1) / EDGE;
  const long long tiles = p.rest.len * nt_d * nt_s;
  const int tid = flat_tid();
  const int threads = block_threads();
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const long long ts = t % nt_s;
    const long long td = (t / nt_s) % nt_d;
    const long long bi = t / (nt_s * nt_d);
    const long long d0 = td * EDGE, s0 = ts * EDGE;
    long long src_b, dst_b;
    group_offsets(p.rest, bi, &src_b, &dst_b);
    src_b += p.src_offset;
    dst_b += p.dst_offset;
    // Source offset of each D position and destination offset of each S position.
    for (int i = tid; i < 2 * EDGE; i += threads) {
      long long so, dof;
      if (i < EDGE) {
        if (d0 + i < dlen) {
          group_offsets(p.run, d0 + i, &so, &dof);
          off_d[i] = src_b + so;
        }
      } else if (s0 + (i - EDGE) < slen) {
        group_offsets(p.srun, s0 + (i - EDGE), &so, &dof);
        off_s[i - EDGE] = dst_b + dof;
      }
    }
    __syncthreads();
    const int drows = static_cast<int>(dlen - d0 < EDGE ? dlen - d0 : EDGE);
    const int scols = static_cast<int>(slen - s0 < EDGE ? slen - s0 : EDGE);
    // Loads: row d of the tile is contiguous in the source.
    {
      constexpr int per_row = EDGE / VS;
      for (int i = tid; i < EDGE * per_row; i += threads) {
        const int d = i / per_row;
        const int sv = (i % per_row) * VS;
        if (d < drows && sv < scols) {
          const E* from = src + off_d[d] + s0 + sv;
          if constexpr (VS > 1) {
            const uint4 x = *reinterpret_cast<const uint4*>(from);
            const E* xe = reinterpret_cast<const E*>(&x);
#pragma unroll
            for (int c = 0; c < VS; ++c) tile[d * PITCH + sv + c] = xe[c];
          } else {
            tile[d * PITCH + sv] = *from;
          }
        }
      }
    }
    __syncthreads();
    // Stores: column s of the tile is contiguous in the destination.
    {
      constexpr int per_col = EDGE / VD;
      for (int i = tid; i < EDGE * per_col; i += threads) {
        const int s = i / per_col;
        const int dv = (i % per_col) * VD;
        if (s < scols && dv < drows) {
          E* to = dst + off_s[s] + d0 + dv;
          if constexpr (VD > 1) {
            uint4 x;
            E* xe = reinterpret_cast<E*>(&x);
#pragma unroll
            for (int c = 0; c < VD; ++c) xe[c] = tile[(dv + c) * PITCH + s];
            *reinterpret_cast<uint4*>(to) = x;
          } else {
            *to = tile[dv * PITCH + s];
          }
        }
      }
    }
    __syncthreads();
  }
}

// One element per thread.  The three groups partition the axes, so decoding a flat
// index over (run, srun, rest) visits every element once, whatever the plan's kind.
template <typename E>
__device__ __forceinline__ void perm_generic(const PermPlan& p, E* dst, const E* src) {
  const long long stride = static_cast<long long>(gridDim.x) * block_threads();
  for (long long f = static_cast<long long>(blockIdx.x) * block_threads() + flat_tid(); f < p.len; f += stride) {
    long long s1, d1, s2, d2, s3, d3;
    const long long a = f % p.run.len;
    const long long q = f / p.run.len;
    group_offsets(p.run, a, &s1, &d1);
    group_offsets(p.srun, q % p.srun.len, &s2, &d2);
    group_offsets(p.rest, q / p.srun.len, &s3, &d3);
    dst[p.dst_offset + d1 + d2 + d3] = src[p.src_offset + s1 + s2 + s3];
  }
}

// Shared memory a plan's path needs (bytes).
T4A_HD int perm_smem_bytes(const PermPlan& p) {
  if (p.kind == kPermRows) {
    const long long seg = p.run.len < kPermRowsBytes / p.esize ? p.run.len : kPermRowsBytes / p.esize;
    const long long rows = kPermRowsBytes / p.esize / seg;
    return static_cast<int>(2 * rows * 8);
  }
  if (p.kind == kPermTiles) {
    const int edge = perm_tile_edge(p.esize);
    return ((edge * (edge + 1) * p.esize + 15) & ~15) + 2 * edge * 8;
  }
  return 0;
}

__device__ __forceinline__ unsigned move_dynamic_smem() {
  unsigned r;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

// Run a plan with the widest vectors the pointers allow; `smem_ok` says whether the
// launch has the shared memory the tiled paths need.
template <int B>
__device__ __forceinline__ void perm_run(const PermPlan& p, void* dst_p, const void* src_p, bool smem_ok) {
  using E = typename Elem<B>::T;
  E* dst = static_cast<E*>(dst_p);
  const E* src = static_cast<const E*>(src_p);
  constexpr int VV = B >= 16 ? 1 : 16 / B;
  const bool src_al = (reinterpret_cast<unsigned long long>(src) & 15ull) == 0;
  const bool dst_al = (reinterpret_cast<unsigned long long>(dst) & 15ull) == 0;
  if (p.kind == kPermRows && smem_ok) {
    const bool vec = VV > 1 && src_al && dst_al && perm_vec(p, 0) == VV && perm_vec(p, 1) == VV;
    if constexpr (VV > 1) {
      if (vec) {
        perm_rows<E, VV>(p, dst, src);
        return;
      }
    }
    perm_rows<E, 1>(p, dst, src);
    return;
  }
  if (p.kind == kPermTiles && smem_ok) {
    constexpr int EDGE = B >= 16 ? 32 : 64;
    const bool vs = VV > 1 && src_al && perm_vec(p, 0) == VV;
    const bool vd = VV > 1 && dst_al && perm_vec(p, 1) == VV;
    if constexpr (VV > 1) {
      if (vs && vd) return perm_tiles<E, VV, VV, EDGE>(p, dst, src);
      if (vs) return perm_tiles<E, VV, 1, EDGE>(p, dst, src);
      if (vd) return perm_tiles<E, 1, VV, EDGE>(p, dst, src);
    }
    perm_tiles<E, 1, 1, EDGE>(p, dst, src);
    return;
  }
  if (p.kind != kPermEmpty) perm_generic<E>(p, dst, src);
}

}  // namespace
}  // namespace t4a
