// Permutation plan of the strided movement entries, shared by the host planner and
// the kernels.
//
// Every movement entry copies the logical elements of one index space:
// dst[dst_offset + sum c_k * ds_k] = src[src_offset + sum c_k * ss_k] for all
// coordinates c of the common extents.  The plan coalesces that space and classifies
// it:
//   * kPermRows: a run of axes is contiguous in both source and destination (same
//     fastest axis); the space is rows of that run, copied with vectors;
//   * kPermTiles: the fastest destination axis differs from the fastest source axis;
//     the space is (D run: dst-contiguous axes) x (S run: src-contiguous axes) x
//     batch axes, moved through shared-memory tiles so that both the loads and the
//     stores are contiguous;
//   * kPermGeneric: anything else, one element per thread.
#pragma once

#include "../../include/t4a_b200/abi.h"

#if defined(__CUDACC__)
#define T4A_HD __host__ __device__ __forceinline__
#else
#define T4A_HD inline
#endif

namespace t4a {

enum PermKind { kPermEmpty = 0, kPermRows = 1, kPermTiles = 2, kPermGeneric = 3 };

struct PermGroup {
  int n;                        // axes in the group
  long long ext[T4A_CUDA_MAX_RANK];
  long long ss[T4A_CUDA_MAX_RANK];   // source strides
  long long ds[T4A_CUDA_MAX_RANK];   // destination strides
  long long len;                // product of the extents
};

struct PermPlan {
  int kind;
  int esize;
  long long src_offset;
  long long dst_offset;
  long long len;                // logical elements
  PermGroup run;                // kPermRows: the shared run; kPermTiles: the D run
  PermGroup srun;               // kPermTiles: the S run
  PermGroup rest;               // rows (kPermRows) / batch axes (kPermTiles) / all axes (generic)
};

T4A_HD void group_clear(PermGroup& g) {
  g.n = 0;
  g.len = 1;
  for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) g.ext[i] = g.ss[i] = g.ds[i] = 0;
}

T4A_HD void group_push(PermGroup& g, long long e, long long s, long long d) {
  g.ext[g.n] = e;
  g.ss[g.n] = s;
  g.ds[g.n] = d;
  ++g.n;
  g.len *= e;
}

// Offsets of flat index `f` of a group (axis 0 fastest) in source and destination.
T4A_HD void group_offsets(const PermGroup& g, long long f, long long* so, long long* dof) {
  long long s = 0, d = 0;
  for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) {
    if (i < g.n) {
      const long long c = f % g.ext[i];
      f /= g.ext[i];
      s += c * g.ss[i];
      d += c * g.ds[i];
    }
  }
  *so = s;
  *dof = d;
}

// Build the plan of a copy over `rank` axes with extents `ext`, source strides `ss`
// and destination strides `ds`.
T4A_HD PermPlan make_perm_plan(int rank, const long long* ext_in, const long long* ss_in,
                               const long long* ds_in, long long src_offset, long long dst_offset,
                               int esize) {
  PermPlan p;
  p.esize = esize;
  p.src_offset = src_offset;
  p.dst_offset = dst_offset;
  group_clear(p.run);
  group_clear(p.srun);
  group_clear(p.rest);
  // 1. Drop extent-1 axes and merge neighbours that are contiguous on both sides.
  long long e[T4A_CUDA_MAX_RANK], s[T4A_CUDA_MAX_RANK], d[T4A_CUDA_MAX_RANK];
  int n = 0;
  long long len = 1;
  for (int i = 0; i < rank && i < T4A_CUDA_MAX_RANK; ++i) {
    len *= ext_in[i];
    if (ext_in[i] == 1) continue;
    if (n > 0 && ss_in[i] == s[n - 1] * e[n - 1] && ds_in[i] == d[n - 1] * e[n - 1]) {
      e[n - 1] *= ext_in[i];
      continue;
    }
    e[n] = ext_in[i];
    s[n] = ss_in[i];
    d[n] = ds_in[i];
    ++n;
  }
  p.len = len;
  if (len == 0) {
    p.kind = kPermEmpty;
    return p;
  }
  // 2. The source-contiguous chain (S) and the destination-contiguous chain (D).
  //    When the fastest axes differ, the two runs of a tile must stay disjoint.
  bool in_d[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
  bool in_s[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
  int dchain[T4A_CUDA_MAX_RANK], schain[T4A_CUDA_MAX_RANK];
  int nd = 0, ns = 0;
  long long want = 1;
  for (bool grew = true; grew && ns < n;) {
    grew = false;
    for (int i = 0; i < n; ++i) {
      if (!in_s[i] && s[i] == want) {
        in_s[i] = true;
        schain[ns++] = i;
        want *= e[i];
        grew = true;
        break;
      }
    }
  }
  // The shortest prefix of the S chain that fills a tile edge is reserved for the S
  // run; the D chain stops at any reserved axis.
  const long long edge = esize >= 16 ? 32 : 64;
  bool reserved[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
  {
    long long filled = 1;
    for (int k = 0; k < ns && filled < edge; ++k) {
      reserved[schain[k]] = true;
      filled *= e[schain[k]];
    }
  }
  want = 1;
  for (bool grew = true; grew && nd < n;) {
    grew = false;
    for (int i = 0; i < n; ++i) {
      if (!in_d[i] && d[i] == want) {
        if (nd > 0 && reserved[i]) break;
        in_d[i] = true;
        dchain[nd++] = i;
        want *= e[i];
        grew = true;
        break;
      }
    }
  }
  if (nd > 0 && ns > 0 && dchain[0] == schain[0]) {
    // 3a. Shared run: the common prefix of both chains.
    int k = 0;
    while (k < nd && k < ns && dchain[k] == schain[k]) ++k;
    bool used[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
    for (int i = 0; i < k; ++i) {
      group_push(p.run, e[dchain[i]], s[dchain[i]], d[dchain[i]]);
      used[dchain[i]] = true;
    }
    for (int i = 0; i < n; ++i)
      if (!used[i]) group_push(p.rest, e[i], s[i], d[i]);
    p.kind = kPermRows;
    return p;
  }
  if (nd > 0 && ns > 0) {
    // 3b. Transpose-like: D run, S run (axes of the S chain outside the D chain), batch.
    bool used[T4A_CUDA_MAX_RANK] = {false, false, false, false, false, false, false, false};
    for (int i = 0; i < nd; ++i) {
      group_push(p.run, e[dchain[i]], s[dchain[i]], d[dchain[i]]);
      used[dchain[i]] = true;
    }
    for (int i = 0; i < ns; ++i) {
      if (used[schain[i]]) break;  // the S chain stops where it meets the D run
      group_push(p.srun, e[schain[i]], s[schain[i]], d[schain[i]]);
      used[schain[i]] = true;
    }
    for (int i = 0; i < n; ++i)
      if (!used[i]) group_push(p.rest, e[i], s[i], d[i]);
    p.kind = kPermTiles;
    return p;
  }
  for (int i = 0; i < n; ++i) group_push(p.rest, e[i], s[i], d[i]);
  p.kind = kPermGeneric;
  return p;
}

// Whether every offset a vector of `v` elements starts at is a multiple of `v` on
// the given side (0 = source, 1 = destination), for the groups listed.
T4A_HD bool group_strides_divisible(const PermGroup& g, int side, long long v) {
  for (int i = 0; i < T4A_CUDA_MAX_RANK; ++i) {
    if (i < g.n) {
      const long long st = side == 0 ? g.ss[i] : g.ds[i];
      if (st % v != 0) return false;
    }
  }
  return true;
}

// Vector widths (elements) of the tiles: along the S run for loads and along the D
// run for stores; of the rows: along the shared run.  1 = element accesses.
T4A_HD int perm_vec(const PermPlan& p, int side) {
  const int v = p.esize >= 16 ? 1 : 16 / p.esize;
  if (v == 1) return 1;
  if (p.kind == kPermRows) {
    if (p.run.len % v != 0) return 1;
    if ((side == 0 ? p.src_offset : p.dst_offset) % v != 0) return 1;
    if (!group_strides_divisible(p.rest, side, v)) return 1;
    return v;
  }
  if (p.kind == kPermTiles) {
    // Loads run along the S run (side 0), stores along the D run (side 1).
    const PermGroup& along = side == 0 ? p.srun : p.run;
    if (along.len % v != 0) return 1;
    if ((side == 0 ? p.src_offset : p.dst_offset) % v != 0) return 1;
    if (!group_strides_divisible(side == 0 ? p.run : p.srun, side, v)) return 1;
    if (!group_strides_divisible(p.rest, side, v)) return 1;
    return v;
  }
  return 1;
}

// Warp-tile shape of kPermTiles (4 KiB per warp): S positions per tile and D positions
// per tile for an element size.
T4A_HD int warp_tile_s(int esize) { return esize == 1 ? 64 : (esize >= 16 ? 16 : 32); }
T4A_HD int warp_tile_d(int esize) { return 4096 / esize / warp_tile_s(esize); }

constexpr int kPermThreads = 256;
constexpr int kPermRowsBytes = 4096;   // bytes per (warp) work unit of the rows path
constexpr int kPermRowsMax = 32;       // rows per unit: one per lane

struct PermRowsShape {
  long long seg;  // run elements per unit: chunks * V, chunks a power of two
  int lv;         // log2 of the chunks per unit row
  int rows;       // rows per unit, a power of two
};

// Unit shape of the rows path for chunks of `v` elements (v divides the run when v > 1):
// a power-of-two number of chunks per row segment and of rows, about 4 KiB in all.
T4A_HD PermRowsShape perm_rows_shape(const PermPlan& p, int v) {
  PermRowsShape s;
  const long long run_chunks = p.run.len / v;
  long long cap = kPermRowsBytes / (v * p.esize);  // chunks per unit
  if (cap < 1) cap = 1;
  const long long want = run_chunks < cap ? run_chunks : cap;
  int lv = 0;
  while ((2LL << lv) <= want) ++lv;
  s.lv = lv;
  s.seg = (1LL << lv) * v;
  long long rows = cap >> lv;
  if (rows > kPermRowsMax) rows = kPermRowsMax;
  int r = 1;
  while (2 * r <= rows) r *= 2;
  s.rows = r;
  return s;
}

// Vector width (elements) of the rows path for 16-byte-aligned pointers.
T4A_HD int perm_rows_vec(const PermPlan& p);

// Offsets of T consecutive flat indices f0 + i (f0 a multiple of T) of a group on one
// side are linear, i * s0, when axis 0 alone holds the span (e0 a multiple of T) or
// the group is empty.  `ok` is false otherwise (decode every index).
struct AffineSpan {
  bool ok;
  long long s0;
};

T4A_HD AffineSpan affine_span(const PermGroup& g, int side, long long t) {
  AffineSpan a;
  a.ok = g.n == 0 || g.ext[0] % t == 0;
  a.s0 = g.n == 0 ? 0 : (side == 0 ? g.ss[0] : g.ds[0]);
  return a;
}

T4A_HD long long affine_at(const AffineSpan& a, int i) { return i * a.s0; }

}  // namespace t4a

namespace t4a {
T4A_HD int perm_rows_vec(const PermPlan& p) {
  const int v = p.esize >= 16 ? 1 : 16 / p.esize;
  return (v > 1 && perm_vec(p, 0) == v && perm_vec(p, 1) == v) ? v : 1;
}
}  // namespace t4a
