// Device bodies of the strided movement entries (sm_100a), shared by the exported
// ABI symbols (movement_abi.cu) and the host launchers (movement_fast.cu).
//
// Movement is a bit copy, so the bodies are templated on the element size only.
// Every path is a grid-stride loop over its work units.
#pragma once

#include <cstdint>
#include <type_traits>

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

// complex64 elements are only 4-byte aligned in the ABI: an 8-byte element walk whose
// bases are off 8 bytes moves each element as two 4-byte words.
struct alignas(4) Words8 {
  unsigned lo, hi;
};
__host__ __device__ __forceinline__ bool off8(const void* a, const void* b) {
  return ((reinterpret_cast<unsigned long long>(a) | reinterpret_cast<unsigned long long>(b)) & 7ull) != 0;
}

// out[view(f)] = 0 for f < len; the view is the identity when `l` is null.
template <typename E>
__device__ __forceinline__ void zero_walk(void* out, const t4a_cuda_layout* l, long long len) {
  E* o = static_cast<E*>(out);
  E z;
  memset(&z, 0, sizeof(E));
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long f = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; f < len; f += stride)
    o[l == nullptr ? f : decode_offset(f, *l, l->strides, l->offset)] = z;
}

template <int B>
__device__ __forceinline__ void zero_fill(void* out, const t4a_cuda_layout* l, long long len) {
  if constexpr (B == 8) {
    if (off8(out, out)) {
      zero_walk<Words8>(out, l, len);
      return;
    }
  }
  zero_walk<typename Elem<B>::T>(out, l, len);
}

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

// Offsets of flat index f of a group, in 32-bit arithmetic when the group's length
// fits (the common case: one 64-bit division costs several 32-bit ones).
T4A_HD void group_offsets_fast(const PermGroup& g, long long f, long long* so, long long* dof) {
  if (g.len <= 0x7fffffffLL) {
    unsigned x = static_cast<unsigned>(f);
    long long s = 0, d = 0;
    for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) {
      if (i < g.n) {
        const unsigned e = static_cast<unsigned>(g.ext[i]);
        const unsigned c = x % e;
        x /= e;
        s += static_cast<long long>(c) * g.ss[i];
        d += static_cast<long long>(c) * g.ds[i];
      }
    }
    *so = s;
    *dof = d;
    return;
  }
  group_offsets(g, f, so, dof);
}

// Per-warp work units: no block-wide barrier anywhere in the movement paths, so a
// warp's memory latency is hidden by the other warps of the SM, not by waiting for
// its block.
constexpr int kWarpUnitBytes = 4096;

// Warp-tile shape per element size: TD D positions x TS S positions = 4 KiB, rows of
// 16-byte chunks (CE elements per chunk).
template <int B>
struct WarpTile {
  static constexpr int CE = B >= 16 ? 1 : 16 / B;
  static constexpr int TS = B == 1 ? 64 : (B >= 16 ? 16 : 32);
  static constexpr int TD = kWarpUnitBytes / B / TS;
};

// Lanes 0, 1, 2 decode one group each; every lane gets the three results.
__device__ __forceinline__ void warp_decode3(const PermGroup& g0, long long f0, const PermGroup& g1, long long f1,
                                             const PermGroup& g2, long long f2, int lane, long long* s0,
                                             long long* d0, long long* s1, long long* d1, long long* s2,
                                             long long* d2) {
  long long so = 0, dof = 0;
  if (lane == 0) group_offsets_fast(g0, f0, &so, &dof);
  if (lane == 1) group_offsets_fast(g1, f1, &so, &dof);
  if (lane == 2) group_offsets_fast(g2, f2, &so, &dof);
  *s0 = __shfl_sync(0xffffffffu, so, 0);
  *d0 = __shfl_sync(0xffffffffu, dof, 0);
  *s1 = __shfl_sync(0xffffffffu, so, 1);
  *d1 = __shfl_sync(0xffffffffu, dof, 1);
  *s2 = __shfl_sync(0xffffffffu, so, 2);
  *d2 = __shfl_sync(0xffffffffu, dof, 2);
}

// ---------------------------------------------------------------------------
// Rows: the shared run is contiguous on both sides.  A warp unit is R rows x one
// segment of the run (about 4 KiB); each lane loads its vectors of the unit into
// registers, then stores them.  Row offsets are one decode plus an affine step when
// the rest axes allow it, else decoded per row by the lanes (R <= 32).
// ---------------------------------------------------------------------------
template <typename E, int V, bool A16, bool AFF>
__device__ __forceinline__ void perm_rows(const PermPlan& p, E* __restrict__ dst, const E* __restrict__ src) {
  using Chunk = typename std::conditional<V * sizeof(E) == 16 && A16, uint4, E>::type;
  constexpr int kCB = static_cast<int>(sizeof(Chunk));
  constexpr int kPerLane = kWarpUnitBytes / kCB / kWarp;  // chunks per lane per unit
  constexpr int kBatch = kPerLane < 8 ? kPerLane : 8;     // loads in flight per lane
  const PermRowsShape shape = perm_rows_shape(p, V);
  const int R = shape.rows;
  const int lv = shape.lv;
  const AffineSpan as = affine_span(p.rest, 0, R);
  const AffineSpan ad = affine_span(p.rest, 1, R);
  const long long run = p.run.len;
  const long long segs = (run + shape.seg - 1) / shape.seg;
  const long long units = ((p.rest.len + R - 1) / R) * segs;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (block_threads() / kWarp);
  const long long first = static_cast<long long>(blockIdx.x) * (block_threads() / kWarp) + flat_tid() / kWarp;
  for (long long u = first; u < units; u += warps) {
    const long long g = u % segs;
    const long long r0 = (u / segs) * R;
    const int nrows = static_cast<int>(p.rest.len - r0 < R ? p.rest.len - r0 : R);
    long long src_base, dst_base;
    {
      long long so = 0, dof = 0;
      if (AFF ? lane == 0 : lane < nrows) group_offsets_fast(p.rest, r0 + (AFF ? 0 : lane), &so, &dof);
      if (AFF) {
        so = __shfl_sync(0xffffffffu, so, 0);
        dof = __shfl_sync(0xffffffffu, dof, 0);
      }
      src_base = p.src_offset + so;  // AFF: the unit's base; else: this lane's row
      dst_base = p.dst_offset + dof;
    }
    const long long c0 = g * shape.seg;
    const int cchunks = static_cast<int>((run - c0 < shape.seg ? run - c0 : shape.seg) / V);
    const int total = nrows << lv;
    for (int base = 0; base < total; base += kWarp * kBatch) {
      Chunk buf[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int v = base + lane + k * kWarp;
        const int r = v >> lv, c = v & ((1 << lv) - 1);
        const long long row = AFF ? src_base + r * as.s0 : __shfl_sync(0xffffffffu, src_base, r & 31);
        if (v < total && c < cchunks)
          buf[k] = *reinterpret_cast<const Chunk*>(src + row + c0 + static_cast<long long>(c) * V);
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int v = base + lane + k * kWarp;
        const int r = v >> lv, c = v & ((1 << lv) - 1);
        const long long row = AFF ? dst_base + r * ad.s0 : __shfl_sync(0xffffffffu, dst_base, r & 31);
        if (v < total && c < cchunks) *reinterpret_cast<Chunk*>(dst + row + c0 + static_cast<long long>(c) * V) = buf[k];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tiles: a warp tile is TD positions of the D run (contiguous in the destination)
// x TS positions of the S run (contiguous in the source) of one batch index, in the
// warp's own 4 KiB of shared memory.  Loads are cp.async copies of 16-byte chunks
// (or elements) of source rows; chunk c of tile row d sits at chunk c ^ ((d / CE) %
// chunks-per-row), so the store phase's column reads hit distinct banks.  Stores
// assemble CE consecutive D positions of one S position into a 16-byte vector.
// Offsets: source (d, s) = A + run_src(d) + s, destination (d, s) = B + srun_dst(s) + d,
// with run_src / srun_dst affine within a tile when the runs' leading axes allow,
// else decoded per position by the lanes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async(void* smem, const void* gmem, int bytes) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  if (bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
  } else if (bytes == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
  }
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

template <typename E, bool VS, bool VD, bool AFF>
__device__ __forceinline__ void perm_tiles(const PermPlan& p, E* __restrict__ dst, const E* __restrict__ src) {
  constexpr int B = static_cast<int>(sizeof(E));
  using Shape = WarpTile<B>;
  constexpr int CE = Shape::CE, TS = Shape::TS, TD = Shape::TD;
  constexpr int CL = TS / CE;                    // chunks per tile row
  constexpr int GS = VS ? CE : 1;                // elements per load
  constexpr int GD = VD ? CE : 1;                // elements per store
  constexpr int NLOAD = TD * (TS / GS) / kWarp;  // loads per lane
  constexpr int NSTORE = TS * (TD / GD) / kWarp; // stores per lane
  constexpr int LOADB = GS * B;
  const int lane = threadIdx.x & 31;
  const int warp_in_block = flat_tid() / kWarp;
  E* tile = reinterpret_cast<E*>(t4a_move_smem + warp_in_block * kWarpUnitBytes);
  const long long dlen = p.run.len, slen = p.srun.len;
  const long long nt_d = (dlen + TD - 1) / TD, nt_s = (slen + TS - 1) / TS;
  const long long total = p.rest.len * nt_d * nt_s;
  const AffineSpan ad = affine_span(p.run, 0, TD);
  const AffineSpan as = affine_span(p.srun, 1, TS);
  constexpr bool affine = AFF;
  auto at = [](int d, int s) -> int { return d * TS + ((((s / CE) ^ ((d / CE) % CL))) * CE) + (s % CE); };
  const long long warps = static_cast<long long>(gridDim.x) * (block_threads() / kWarp);
  for (long long t = static_cast<long long>(blockIdx.x) * (block_threads() / kWarp) + warp_in_block; t < total;
       t += warps) {
    const long long ts = t % nt_s, td = (t / nt_s) % nt_d, bi = t / (nt_s * nt_d);
    long long rest_s, rest_d, run_s, run_d, srun_s, srun_d;
    warp_decode3(p.rest, bi, p.run, td * TD, p.srun, ts * TS, lane, &rest_s, &rest_d, &run_s, &run_d, &srun_s,
                 &srun_d);
    const int drows = static_cast<int>(dlen - td * TD < TD ? dlen - td * TD : TD);
    const int scols = static_cast<int>(slen - ts * TS < TS ? slen - ts * TS : TS);
    // Per-position tables (lane i holds positions i and i + 32) when not affine.
    long long tab_d[TD > 32 ? 2 : 1], tab_s[TS > 32 ? 2 : 1];
    if constexpr (!affine) {
#pragma unroll
      for (int h = 0; h < (TD > 32 ? 2 : 1); ++h) {
        const int i = lane + 32 * h;
        long long so = 0, dof = 0;
        if (i < drows) group_offsets_fast(p.run, td * TD + i, &so, &dof);
        tab_d[h] = so - run_s;
      }
#pragma unroll
      for (int h = 0; h < (TS > 32 ? 2 : 1); ++h) {
        const int i = lane + 32 * h;
        long long so = 0, dof = 0;
        if (i < scols) group_offsets_fast(p.srun, ts * TS + i, &so, &dof);
        tab_s[h] = dof - srun_d;
      }
    }
    const long long a = p.src_offset + rest_s + run_s + ts * TS;
    const long long b = p.dst_offset + rest_d + srun_d + td * TD;
    __syncwarp();  // the previous tile's reads of this slice are done
#pragma unroll 8
    for (int k = 0; k < NLOAD; ++k) {
      const int i = lane + k * kWarp;
      const int d = i / (TS / GS);
      const int sv = (i % (TS / GS)) * GS;
      long long row = 0;
      if constexpr (affine) {
        row = affine_at(ad, d);
      } else {
        const long long v0 = __shfl_sync(0xffffffffu, tab_d[0], d & 31);
        row = v0;
        if constexpr (TD > 32) {
          const long long v1 = __shfl_sync(0xffffffffu, tab_d[TD > 32 ? 1 : 0], d & 31);
          row = d >= 32 ? v1 : v0;
        }
      }
      if (d < drows && sv < scols) {
        const E* from = src + a + row + sv;
        if constexpr (LOADB >= 4) {
          if constexpr (B == 16 && !VS) {
            cp_async(tile + at(d, sv), from, 8);
            cp_async(reinterpret_cast<char*>(tile + at(d, sv)) + 8, reinterpret_cast<const char*>(from) + 8, 8);
          } else {
            cp_async(tile + at(d, sv), from, LOADB);
          }
        } else {
          tile[at(d, sv)] = *from;  // narrower than cp.async's 4-byte minimum
        }
      }
    }
    cp_async_wait_all();
    __syncwarp();
    if constexpr (VS && VD && CE > 1 && CE <= 4) {
      // CE x CE register blocks: CE 16-byte shared loads (rows d..d+CE-1 of one chunk)
      // become CE 16-byte destination vectors (columns s..s+CE-1 of rows d..d+CE-1).
      constexpr int BD = TD / CE, BS = TS / CE;  // blocks along D and S
      constexpr int PER_LANE = BD * BS / kWarp;
      static_assert(BD <= kWarp && kWarp % BD == 0, "block rows per warp");
#pragma unroll
      for (int k = 0; k < PER_LANE; ++k) {
        const int bd = lane % BD;
        const int bs = lane / BD + k * (kWarp / BD);
        const int d0 = bd * CE, s0 = bs * CE;
        if (d0 < drows && s0 < scols) {
          E blk[CE][CE];
#pragma unroll
          for (int r = 0; r < CE; ++r) {
            const uint4 x = *reinterpret_cast<const uint4*>(tile + at(d0 + r, s0));
            const E* xe = reinterpret_cast<const E*>(&x);
#pragma unroll
            for (int c = 0; c < CE; ++c) blk[r][c] = xe[c];
          }
#pragma unroll
          for (int c = 0; c < CE; ++c) {
            long long col;
            if constexpr (affine) {
              col = affine_at(as, s0 + c);
            } else {
              const long long v0 = __shfl_sync(0xffffffffu, tab_s[0], (s0 + c) & 31);
              col = v0;
              if constexpr (TS > 32) {
                const long long v1 = __shfl_sync(0xffffffffu, tab_s[TS > 32 ? 1 : 0], (s0 + c) & 31);
                col = s0 + c >= 32 ? v1 : v0;
              }
            }
            uint4 y;
            E* ye = reinterpret_cast<E*>(&y);
#pragma unroll
            for (int r = 0; r < CE; ++r) ye[r] = blk[r][c];
            *reinterpret_cast<uint4*>(dst + b + col + d0) = y;
          }
        } else {
          // Keep the shuffles of the table path convergent.
          if constexpr (!affine) {
#pragma unroll
            for (int c = 0; c < CE; ++c) {
              __shfl_sync(0xffffffffu, tab_s[0], (s0 + c) & 31);
              if constexpr (TS > 32) __shfl_sync(0xffffffffu, tab_s[TS > 32 ? 1 : 0], (s0 + c) & 31);
            }
          }
        }
      }
      continue;
    }
#pragma unroll 8
    for (int k = 0; k < NSTORE; ++k) {
      const int i = lane + k * kWarp;
      const int sp = i / (TD / GD);
      const int dv = (i % (TD / GD)) * GD;
      long long col = 0;
      if constexpr (affine) {
        col = affine_at(as, sp);
      } else {
        const long long v0 = __shfl_sync(0xffffffffu, tab_s[0], sp & 31);
        col = v0;
        if constexpr (TS > 32) {
          const long long v1 = __shfl_sync(0xffffffffu, tab_s[TS > 32 ? 1 : 0], sp & 31);
          col = sp >= 32 ? v1 : v0;
        }
      }
      if (sp < scols && dv < drows) {
        E* to = dst + b + col + dv;
        if constexpr (GD > 1) {
          uint4 x;
          E* xe = reinterpret_cast<E*>(&x);
#pragma unroll
          for (int c = 0; c < GD; ++c) xe[c] = tile[at(dv + c, sp)];
          *reinterpret_cast<uint4*>(to) = x;
        } else if constexpr (B == 16 && VD) {
          *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(tile + at(dv, sp));
        } else {
          *to = tile[at(dv, sp)];
        }
      }
    }
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

// Shared memory a plan's path needs for a block of `threads` threads (bytes).
T4A_HD int perm_smem_bytes(const PermPlan& p, int threads = kPermThreads) {
  return p.kind == kPermTiles ? (threads / 32) * kWarpUnitBytes : 0;
}

__device__ __forceinline__ unsigned move_dynamic_smem() {
  unsigned r;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

// Run a plan with the widest vectors the pointers allow; `smem_ok` says whether the
// launch has the shared memory the tiled paths need.
// Whether the offsets inside one work unit are affine (rows: over R rows; tiles:
// over a warp tile's D and S positions).
T4A_HD bool perm_affine(const PermPlan& p, int rows_vec) {
  if (p.kind == kPermRows) {
    const int r = perm_rows_shape(p, rows_vec).rows;
    return affine_span(p.rest, 0, r).ok && affine_span(p.rest, 1, r).ok;
  }
  if (p.kind == kPermTiles) {
    return affine_span(p.run, 0, warp_tile_d(p.esize)).ok && affine_span(p.srun, 1, warp_tile_s(p.esize)).ok;
  }
  return false;
}

template <typename E, bool VS, bool VD>
__device__ __forceinline__ void perm_tiles_any(const PermPlan& p, E* dst, const E* src, bool aff) {
  if (aff) {
    perm_tiles<E, VS, VD, true>(p, dst, src);
  } else {
    perm_tiles<E, VS, VD, false>(p, dst, src);
  }
}

template <typename E, int V, bool A16>
__device__ __forceinline__ void perm_rows_any(const PermPlan& p, E* dst, const E* src, bool aff) {
  if (aff) {
    perm_rows<E, V, A16, true>(p, dst, src);
  } else {
    perm_rows<E, V, A16, false>(p, dst, src);
  }
}

template <int B>
__device__ __forceinline__ void perm_run(const PermPlan& p, void* dst_p, const void* src_p, bool smem_ok) {
  if constexpr (B == 8) {
    if (off8(dst_p, src_p)) {
      if (p.kind != kPermEmpty) perm_generic<Words8>(p, static_cast<Words8*>(dst_p), static_cast<const Words8*>(src_p));
      return;
    }
  }
  using E = typename Elem<B>::T;
  E* dst = static_cast<E*>(dst_p);
  const E* src = static_cast<const E*>(src_p);
  constexpr int VV = B >= 16 ? 1 : 16 / B;
  const bool src_al = (reinterpret_cast<unsigned long long>(src) & 15ull) == 0;
  const bool dst_al = (reinterpret_cast<unsigned long long>(dst) & 15ull) == 0;
  const bool warps_ok = block_threads() % kWarp == 0;
  const bool rows_vec = VV > 1 && src_al && dst_al && perm_vec(p, 0) == VV && perm_vec(p, 1) == VV;
  const bool aff = perm_affine(p, rows_vec ? VV : 1);
  if (p.kind == kPermRows && warps_ok) {
    if constexpr (VV > 1) {
      if (rows_vec) {
        perm_rows_any<E, VV, true>(p, dst, src, aff);
        return;
      }
    }
    if (B == 16 && src_al && dst_al) {
      perm_rows_any<E, 1, true>(p, dst, src, aff);
    } else {
      perm_rows_any<E, 1, false>(p, dst, src, aff);
    }
    return;
  }
  if (p.kind == kPermTiles && smem_ok && warps_ok) {
    const bool vs = src_al && (VV == 1 || perm_vec(p, 0) == VV);
    const bool vd = dst_al && (VV == 1 || perm_vec(p, 1) == VV);
    if (vs && vd) return perm_tiles_any<E, true, true>(p, dst, src, aff);
    if (vs) return perm_tiles_any<E, true, false>(p, dst, src, aff);
    if (vd) return perm_tiles_any<E, false, true>(p, dst, src, aff);
    perm_tiles_any<E, false, false>(p, dst, src, aff);
    return;
  }
  if (p.kind != kPermEmpty) perm_generic<E>(p, dst, src);
}

}  // namespace
}  // namespace t4a
