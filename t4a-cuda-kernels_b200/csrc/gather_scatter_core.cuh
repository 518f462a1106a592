// Gather and additive scatter bodies for sm_100a, shared by the per-path kernels
// (gather_scatter_fast.cu) and the exported ABI symbols (gather_scatter_abi.cu).
//
// The work is a list of units: one unit is one contiguous run of a window (the
// gathered row, or one update row), optionally cut into pieces of at most
// kPieceVecs vectors so that long runs spread over many warps.
//
// Gather: each warp takes 32 units, every lane decodes one unit (index read, starts
// clamped) into shared memory, then the warp copies the 32 runs with V-byte vectors,
// kGatherDepth loads in flight per lane before their stores.
//
// Scatter: update rows are grouped by destination inside chunks (a counting sort
// through a shared-memory hash table), and each group is summed in registers and
// added to memory with one vector of `red.global.add` per lane; details at the
// scatter section below.
#pragma once

#include "common.cuh"
#include "gather_scatter_plan.h"

namespace t4a {

constexpr int kGatherThreads = 256;
constexpr int kGatherDepth = 8;
constexpr int kScatterThreads = 512;

// ---- raw vectors of V bytes ---------------------------------------------------
template <int V> struct Raw;
template <> struct Raw<16> { using T = uint4; };
template <> struct Raw<8> { using T = uint2; };
template <> struct Raw<4> { using T = unsigned; };
template <> struct Raw<2> { using T = unsigned short; };
template <> struct Raw<1> { using T = unsigned char; };

// Read-only load through the non-coherent path (table rows may be re-read from L2).
template <int V>
__device__ __forceinline__ typename Raw<V>::T ld_ro(const unsigned char* p) {
  typename Raw<V>::T r;
  if constexpr (V == 16) {
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  } else if constexpr (V == 8) {
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  } else if constexpr (V == 4) {
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  } else if constexpr (V == 2) {
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  } else {
    unsigned short t;
    asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(t) : "l"(p));
    r = static_cast<unsigned char>(t);
  }
  return r;
}

// Streaming load (read once, evict first).
template <int V>
__device__ __forceinline__ typename Raw<V>::T ld_stream(const unsigned char* p) {
  typename Raw<V>::T r;
  if constexpr (V == 16) {
    asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  } else if constexpr (V == 8) {
    asm volatile("ld.global.cs.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  } else {
    static_assert(V == 4, "scatter vectors are 4, 8 or 16 bytes");
    asm volatile("ld.global.cs.u32 %0, [%1];" : "=r"(r) : "l"(p));
  }
  return r;
}

// Streaming store (written once).
template <int V>
__device__ __forceinline__ void st_stream(unsigned char* p, typename Raw<V>::T v) {
  if constexpr (V == 16) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  } else if constexpr (V == 8) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
  } else if constexpr (V == 4) {
    asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  } else if constexpr (V == 2) {
    asm volatile("st.global.cs.u16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
  } else {
    const unsigned short t = v;
    asm volatile("st.global.cs.u8 [%0], %1;" ::"l"(p), "h"(t) : "memory");
  }
}

// ---- unit decoding ------------------------------------------------------------
// Mixed-radix decode of `f` over a group; the last axis needs no division.
__device__ __forceinline__ void group_offsets(const IdxGroup& g, long long f, long long* sa, long long* sb) {
  long long a = 0, b = 0;
#pragma unroll
  for (int i = 0; i < kMaxRank; ++i) {
    if (i < g.n) {
      long long c = f;
      if (i + 1 < g.n) {
        c = f % g.ext[i];
        f /= g.ext[i];
      }
      a += c * g.a[i];
      b += c * g.b[i];
    }
  }
  *sa = a;
  *sb = b;
}

// Element offsets of the run of unit `u`: side A (with the clamped starts) and side B.
template <typename I>
__device__ __forceinline__ void unit_offsets(const WindowPlan& p, const I* idx, long long u, long long* oa,
                                             long long* ob) {
  long long bu = u, wu = 0;
  if (p.wrest.n > 0) {
    wu = u % p.wrest.len;
    bu = u / p.wrest.len;
  }
  long long ia = 0, ib = 0, wa = 0, wb = 0;
  group_offsets(p.batch, bu, &ia, &ib);
  if (p.wrest.n > 0) group_offsets(p.wrest, wu, &wa, &wb);
  long long a = p.a_offset + wa;
  const long long ibase = p.idx_offset + ia;
#pragma unroll
  for (int c = 0; c < kMaxRank; ++c) {
    if (c < p.ncomp) {
      const I start = idx[ibase + static_cast<long long>(c) * p.comp_stride];
      a += clamp_start<I>(start, p.comp_dim[c], p.comp_window[c]) * p.comp_stride_a[c];
    }
  }
  *oa = a;
  *ob = p.b_offset + ib + wb;
}

// Pieces of a run of `nvec` vectors: count and vectors per piece.
struct Pieces {
  long long count;
  long long vecs;  // vectors per piece (the last piece may be shorter)
};

__host__ __device__ __forceinline__ Pieces make_pieces(long long nvec, long long max_vecs) {
  Pieces r;
  r.vecs = nvec < max_vecs ? nvec : max_vecs;
  r.count = r.vecs > 0 ? (nvec + r.vecs - 1) / r.vecs : 0;
  return r;
}

__host__ __device__ __forceinline__ int lane_shift_of(long long vecs) {
  int s = 0;
  while (s < 5 && (1ll << s) < vecs) ++s;
  return s;
}

constexpr long long kGatherPieceVecs = 256;

// ---- gather -------------------------------------------------------------------
struct GatherSlot {
  long long src;  // operand byte offset of the piece, -1 when the unit is past the end
  long long dst;  // output byte offset
};

// Copies `units` run pieces.  `slots` holds 32 entries per warp of the block; the
// block is whole warps.  `piece` = run cut for this launch, `lshift` = log2 lanes per
// unit (lanes per unit = min(32, next pow2 of piece.vecs)).
template <typename I, int V>
__device__ __forceinline__ void gather_units(const WindowPlan& p, unsigned char* __restrict__ out,
                                             const unsigned char* __restrict__ operand, const I* __restrict__ idx,
                                             long long units, long long nvec, Pieces piece, int lshift,
                                             GatherSlot* slots) {
  using R = typename Raw<V>::T;
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const long long gw = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + wib;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int L = 1 << lshift;
  const int gshift = 5 - lshift;  // log2 groups per warp
  const int g = lane >> lshift;
  const int lig = lane & (L - 1);
  const int J = static_cast<int>((piece.vecs + L - 1) >> lshift);  // vector steps per unit and lane
  const int T = L * J;                                              // slots per lane and batch
  const long long total = units * piece.count;
  GatherSlot* my = slots + wib * 32;
  for (long long b = gw; b * 32 < total; b += nw) {
    const long long w = b * 32 + lane;
    GatherSlot s{-1, 0};
    if (w < total) {
      long long u = w, pc = 0;
      if (piece.count > 1) {
        u = w / piece.count;
        pc = w - u * piece.count;
      }
      long long oa, ob;
      unit_offsets<I>(p, idx, u, &oa, &ob);
      const long long shift = pc * piece.vecs * V;
      s.src = oa * p.esize + shift;
      s.dst = ob * p.esize + shift;
    }
    __syncwarp();
    my[lane] = s;
    __syncwarp();
    int k = 0, j = 0;
    for (int t0 = 0; t0 < T; t0 += kGatherDepth) {
      R buf[kGatherDepth];
      long long dst[kGatherDepth];
#pragma unroll
      for (int d = 0; d < kGatherDepth; ++d) {
        dst[d] = -1;
        if (t0 + d < T) {
          const int uu = g + (k << gshift);
          const GatherSlot o = my[uu];
          const long long v = lig + (static_cast<long long>(j) << lshift);
          if (o.src >= 0) {
            // Vectors of this piece: the full piece, or what is left of the run.
            const long long pc = piece.count > 1 ? (b * 32 + uu) % piece.count : 0;
            const long long left = nvec - pc * piece.vecs;
            const long long len = left < piece.vecs ? left : piece.vecs;
            if (v < len) {
              buf[d] = ld_ro<V>(operand + o.src + v * V);
              dst[d] = o.dst + v * V;
            }
          }
        }
        if (++j == J) {
          j = 0;
          ++k;
        }
      }
#pragma unroll
      for (int d = 0; d < kGatherDepth; ++d)
        if (dst[d] >= 0) st_stream<V>(out + dst[d], buf[d]);
    }
  }
}

// One element per thread over the units' runs (any geometry).
template <typename I>
__device__ __forceinline__ void gather_elements(const WindowPlan& p, unsigned char* out, const unsigned char* operand,
                                                const I* idx, long long units) {
  const long long total = units * p.run;
  const long long stride = static_cast<long long>(gridDim.x) * block_threads();
  for (long long f = static_cast<long long>(blockIdx.x) * block_threads() + flat_tid(); f < total; f += stride) {
    const long long u = f / p.run;
    const long long e = f - u * p.run;
    long long oa, ob;
    unit_offsets<I>(p, idx, u, &oa, &ob);
    const unsigned char* s = operand + (oa + e) * p.esize;
    unsigned char* d = out + (ob + e) * p.esize;
    for (int c = 0; c < p.esize; ++c) d[c] = s[c];
  }
}

// ---- scatter ------------------------------------------------------------------
// Work unit: a piece = up to 32 * kScatterVecs vectors of one update run.  Pieces are
// grouped by destination inside chunks (a hash table in shared memory counts each
// destination's pieces, a block scan turns the counts into group offsets: a counting
// sort), then folded by sub-warps of L lanes (kScatterVecs vectors a lane):
// consecutive pieces with one destination are summed in registers and reach memory
// as one vector of `red.global.add` per lane.  Under Zipf indices a hot destination
// therefore costs one atomic row per chunk instead of one per update.  Results equal
// the reference's up to the order of floating additions, which the reference leaves
// to its atomics as well.
//
// Two ways to run it:
//  * two kernels (library launcher with a workspace): k_scatter_group writes each
//    chunk's grouped (destination, source) list to the workspace; k_scatter_fold then
//    streams the list with no block barrier, each lane keeping kFoldSlots pieces in
//    flight through a cp.async ring in shared memory;
//  * one kernel (the exported ABI symbol, or no workspace): each block groups a chunk
//    in shared memory and folds it from there.
constexpr int kScatterVecs = 4;  // vectors per lane and piece
constexpr unsigned long long kEmptySlot = ~0ull;
// Keys pack (destination / V) << 1 | short-piece flag.
constexpr long long kScatterMaxVecOffset = 1ll << 62;

// Reductions without a return value; V-byte vectors of F components.
template <typename F, int V>
__device__ __forceinline__ void red_add(unsigned char* p, const F (&x)[V / sizeof(F)]) {
  if constexpr (sizeof(F) == 4) {
    if constexpr (V == 16) {
      asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3])
                   : "memory");
    } else if constexpr (V == 8) {
      asm volatile("red.global.add.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(x[0]), "f"(x[1]) : "memory");
    } else {
      asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(x[0]) : "memory");
    }
  } else {
#pragma unroll
    for (int i = 0; i < static_cast<int>(V / sizeof(F)); ++i)
      asm volatile("red.global.add.f64 [%0], %1;" ::"l"(p + 8 * i), "d"(x[i]) : "memory");
  }
}

template <typename F, int V>
__device__ __forceinline__ void raw_to_f(typename Raw<V>::T r, F (&x)[V / sizeof(F)]) {
  static_assert(sizeof(r) == sizeof(x), "vector size");
  memcpy(&x, &r, sizeof(x));
}

// Geometry of a launch's pieces and sub-warps.
struct ScatterShape {
  Pieces piece;    // pieces of at most 32 * kScatterVecs vectors
  long long last;  // vectors of a unit's last piece
  int lshift;      // log2 lanes per piece
};

__host__ __device__ __forceinline__ ScatterShape scatter_shape(long long nvec) {
  ScatterShape r;
  r.piece = make_pieces(nvec, 32ll * kScatterVecs);
  r.last = r.piece.count > 0 ? nvec - (r.piece.count - 1) * r.piece.vecs : 0;
  const long long per_lane = (r.piece.vecs + kScatterVecs - 1) / kScatterVecs;
  r.lshift = lane_shift_of(per_lane);
  return r;
}

// Destination and updates byte offsets of piece w; the destination carries the
// short-piece flag in bit 0 (destinations are multiples of V >= 4).
template <typename I, int V>
__device__ __forceinline__ void piece_offsets(const WindowPlan& p, const I* __restrict__ idx, long long w,
                                              const ScatterShape& sh, long long* dflag, long long* s) {
  long long u = w, pc = 0;
  if (sh.piece.count > 1) {
    u = w / sh.piece.count;
    pc = w - u * sh.piece.count;
  }
  long long oa, ob;
  unit_offsets<I>(p, idx, u, &oa, &ob);
  const long long shift = pc * sh.piece.vecs * V;
  const bool short_piece = pc == sh.piece.count - 1 && sh.last != sh.piece.vecs;
  *dflag = (oa * p.esize + shift) | static_cast<long long>(short_piece);
  *s = ob * p.esize + shift;
}

__device__ __forceinline__ unsigned long long key_of(long long dflag, int vbytes) {
  return (static_cast<unsigned long long>((dflag & ~1ll) / vbytes) << 1) | static_cast<unsigned long long>(dflag & 1);
}

__device__ __forceinline__ long long dflag_of(unsigned long long key, int vbytes) {
  return static_cast<long long>(key >> 1) * vbytes | static_cast<long long>(key & 1);
}

// Hash table of a chunk of C pieces: 3C/2 slots, so a free or matching slot exists.
template <int C>
struct GroupTable {
  static constexpr int H = C + C / 2;
  unsigned long long key[H];
  unsigned count[H];  // pieces per slot, then the exclusive group offsets
  unsigned warp_total[32];
};

template <int C>
__device__ __forceinline__ void clear_table(GroupTable<C>& t, int tid, int nthreads) {
  for (int q = tid; q < GroupTable<C>::H; q += nthreads) {
    t.key[q] = kEmptySlot;
    t.count[q] = 0;
  }
}

// Slot of a key, inserting it.  At most C keys live in 3C/2 slots, so a free or
// matching slot exists and the probe ends within H steps.
template <int C>
__device__ __forceinline__ unsigned find_slot(GroupTable<C>& t, unsigned long long key) {
  constexpr unsigned H = GroupTable<C>::H;
  unsigned h = __umulhi(static_cast<unsigned>((key * 0x9E3779B97F4A7C15ull) >> 32), H);
  for (unsigned probe = 0; probe < H; ++probe) {
    const unsigned long long prev = atomicCAS(&t.key[h], kEmptySlot, key);
    if (prev == kEmptySlot || prev == key) break;
    h = h + 1 == H ? 0 : h + 1;
  }
  return h;
}

// Warp-aggregated insert, called by all 32 lanes (`key` == kEmptySlot: no piece):
// lanes holding the same key elect one leader that inserts it and reserves their
// ranks with one atomic, so a hot destination costs one shared atomic per warp.
template <int C>
__device__ __forceinline__ unsigned insert_key(GroupTable<C>& t, unsigned long long key, unsigned* rank) {
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(peers) - 1;
  unsigned slot = 0, base = 0;
  if (lane == leader && key != kEmptySlot) {
    slot = find_slot(t, key);
    base = atomicAdd(&t.count[slot], static_cast<unsigned>(__popc(peers)));
  }
  slot = __shfl_sync(0xffffffffu, slot, leader);
  base = __shfl_sync(0xffffffffu, base, leader);
  *rank = base + static_cast<unsigned>(__popc(peers & ((1u << lane) - 1u)));
  return slot;
}

// Exclusive block scan of t.count in place (block of whole warps; barriers inside).
template <int C>
__device__ __forceinline__ void scan_counts(GroupTable<C>& t, int tid, int nthreads) {
  constexpr int n = GroupTable<C>::H;
  const int per = (n + nthreads - 1) / nthreads;
  const int lo = tid * per;
  unsigned local = 0;
  for (int q = 0; q < per; ++q)
    if (lo + q < n) local += t.count[lo + q];
  const int lane = tid & 31, warp = tid >> 5;
  unsigned incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) t.warp_total[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = nthreads >> 5;
    const unsigned v = lane < nw ? t.warp_total[lane] : 0;
    unsigned vi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, vi, o);
      if (lane >= o) vi += y;
    }
    if (lane < nw) t.warp_total[lane] = vi - v;
  }
  __syncthreads();
  unsigned run = t.warp_total[warp] + incl - local;
  for (int q = 0; q < per; ++q) {
    if (lo + q < n) {
      const unsigned c = t.count[lo + q];
      t.count[lo + q] = run;
      run += c;
    }
  }
  __syncthreads();
}

// One sub-warp's running sum over consecutive grouped pieces with one destination.
// The sum starts at -0.0, the exact identity of IEEE addition (x + -0.0 == x for
// every x, signed zeros included), so every piece is simply added.
template <typename F, int V>
struct Fold {
  static constexpr int VE = V / sizeof(F);
  using R = typename Raw<V>::T;
  F acc[kScatterVecs][VE];
  long long dflag = -1;

  __device__ __forceinline__ void flush(unsigned char* out, int lig, int L, const ScatterShape& sh) {
    if (dflag < 0) return;
    const int len = static_cast<int>((dflag & 1) ? sh.last : sh.piece.vecs);
    unsigned char* base = out + (dflag & ~1ll);
#pragma unroll
    for (int j = 0; j < kScatterVecs; ++j) {
      const int v = lig + L * j;
      if (v < len) red_add<F, V>(base + static_cast<long long>(v) * V, acc[j]);
    }
  }

  // Adds one piece (its lane's vectors in x); a new destination first flushes.
  __device__ __forceinline__ void take(unsigned char* out, int lig, int L, const ScatterShape& sh, long long edflag,
                                       const R (&x)[kScatterVecs]) {
    if (edflag != dflag) {
      flush(out, lig, L, sh);
      dflag = edflag;
#pragma unroll
      for (int j = 0; j < kScatterVecs; ++j)
#pragma unroll
        for (int q = 0; q < VE; ++q) acc[j][q] = F(-0.0);
    }
    const int len = static_cast<int>((edflag & 1) ? sh.last : sh.piece.vecs);
#pragma unroll
    for (int j = 0; j < kScatterVecs; ++j) {
      if (lig + L * j < len) {
        F y[VE];
        raw_to_f<F, V>(x[j], y);
#pragma unroll
        for (int q = 0; q < VE; ++q) acc[j][q] += y[q];
      }
    }
  }
};

// ---- one-kernel path ----------------------------------------------------------
constexpr int kScatterChunk = 1024;  // pieces grouped per block and step

struct ScatterSmem {
  GroupTable<kScatterChunk> t;
  long long src[kScatterChunk];          // updates byte offset, by position in the chunk
  unsigned short slot[kScatterChunk];    // hash slot, by position
  unsigned short rank[kScatterChunk];    // rank within the slot's pieces, by position
  unsigned short order[kScatterChunk];   // positions in group order
};

// Groups the chunk of pieces [c0, c0 + n) into sm.order (barriers included).
template <typename I, int V>
__device__ __forceinline__ void group_chunk(const WindowPlan& p, const I* __restrict__ idx, long long c0, int n,
                                            const ScatterShape& sh, ScatterSmem& sm, int tid, int nthreads) {
  clear_table(sm.t, tid, nthreads);
  __syncthreads();
  // Every lane of a warp takes the same number of turns (insert_key is warp-wide).
  for (int i0 = tid - (tid & 31); i0 < kScatterChunk; i0 += nthreads) {
    const int i = i0 + (tid & 31);
    long long dflag = 0, s = 0;
    unsigned long long key = kEmptySlot;
    if (i < n) {
      piece_offsets<I, V>(p, idx, c0 + i, sh, &dflag, &s);
      key = key_of(dflag, V);
    }
    unsigned rank;
    const unsigned slot = insert_key(sm.t, key, &rank);
    if (i < n) {
      sm.slot[i] = static_cast<unsigned short>(slot);
      sm.rank[i] = static_cast<unsigned short>(rank);
      sm.src[i] = s;
    }
  }
  __syncthreads();
  scan_counts(sm.t, tid, nthreads);
  for (int i = tid; i < n; i += nthreads) sm.order[sm.t.count[sm.slot[i]] + sm.rank[i]] = static_cast<unsigned short>(i);
  __syncthreads();
}

// Folds the grouped chunk, warp w taking [beg, end), sub-warps consecutive pieces.
template <typename F, int V>
__device__ __forceinline__ void fold_chunk(const ScatterSmem& sm, unsigned char* __restrict__ out,
                                           const unsigned char* __restrict__ upd, const ScatterShape& sh, int beg,
                                           int end, int lane) {
  using R = typename Raw<V>::T;
  const int L = 1 << sh.lshift;
  const int E = 32 >> sh.lshift;
  const int sub = lane >> sh.lshift;
  const int lig = lane & (L - 1);
  Fold<F, V> f;
  for (int e0 = beg; e0 < end; e0 += E) {
    const int e = e0 + sub;
    if (e < end) {
      const int i = sm.order[e];
      const long long dflag = dflag_of(sm.t.key[sm.slot[i]], V);
      const long long src = sm.src[i];
      const int len = static_cast<int>((dflag & 1) ? sh.last : sh.piece.vecs);
      R x[kScatterVecs];
#pragma unroll
      for (int j = 0; j < kScatterVecs; ++j) {
        const int v = lig + L * j;
        if (v < len) x[j] = ld_stream<V>(upd + src + static_cast<long long>(v) * V);
      }
      f.take(out, lig, L, sh, dflag, x);
    }
  }
  f.flush(out, lig, L, sh);
}

// One-kernel scatter of `units` update runs of `nvec` V-byte vectors (block of whole warps).
template <typename F, typename I, int V>
__device__ __forceinline__ void scatter_units(const WindowPlan& p, unsigned char* __restrict__ out,
                                              const unsigned char* __restrict__ upd, const I* __restrict__ idx,
                                              long long units, long long nvec, ScatterSmem& sm) {
  const ScatterShape sh = scatter_shape(nvec);
  const long long total = units * sh.piece.count;
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = nthreads >> 5;
  for (long long c0 = static_cast<long long>(blockIdx.x) * kScatterChunk; c0 < total;
       c0 += static_cast<long long>(gridDim.x) * kScatterChunk) {
    const int n = total - c0 < kScatterChunk ? static_cast<int>(total - c0) : kScatterChunk;
    group_chunk<I, V>(p, idx, c0, n, sh, sm, tid, nthreads);
    const int per_warp = (n + nwarps - 1) / nwarps;
    const int beg = warp * per_warp < n ? warp * per_warp : n;
    const int end = beg + per_warp < n ? beg + per_warp : n;
    fold_chunk<F, V>(sm, out, upd, sh, beg, end, lane);
    __syncthreads();
  }
}

// ---- two-kernel path ---------------------------------------------------------
// A grouped piece in the workspace list.
struct alignas(16) GroupedPiece {
  long long dflag;  // destination byte offset | short-piece flag
  long long src;    // updates byte offset
};

constexpr int kGroupChunk = 2048;  // pieces grouped per block and step of pass 1
constexpr int kGroupThreads = 512;
constexpr int kGroupPer = kGroupChunk / kGroupThreads;

// Pass 1: the grouped list of every chunk, in chunk order (one entry per piece).
// Each thread keeps its kGroupPer pieces in registers and writes them straight to
// their grouped positions.  Block of kGroupThreads.
//
// The part of a destination one caller holds, in bytes of the whole destination:
// block == 0: the span [lo, hi), held from its first byte;
// block > 0:  the blocks b (bytes [b block, (b + 1) block)) with b % owners == owner,
//             held back to back in block order (block-cyclic ownership).
struct OwnedPart {
  long long lo, hi;
  long long block, owners, owner;
};

// Offset within the held part of destination byte `at`, or -1 when another part holds it.
__host__ __device__ __forceinline__ long long owned_offset(const OwnedPart& o, long long at) {
  if (o.block == 0) return at >= o.lo && at < o.hi ? at - o.lo : -1;
  const long long b = at / o.block;
  if (b % o.owners != o.owner) return -1;
  return (b / o.owners) * o.block + (at - b * o.block);
}

// kRange: only pieces whose destination bytes lie in the part `own` holds are listed,
// with the offset taken within that part; each chunk reserves its slice of the list
// with one atomic on *reserve (so the list holds the kept pieces only, chunk by chunk, in
// the order the chunks reserved), and *reserve ends as the list's length.
template <typename I, int V, bool kRange = false>
__device__ __forceinline__ void scatter_group_pass(const WindowPlan& p, const I* __restrict__ idx, long long units,
                                                   long long nvec, GroupedPiece* __restrict__ list,
                                                   GroupTable<kGroupChunk>& t, OwnedPart own = OwnedPart{},
                                                   unsigned long long* reserve = nullptr) {
  __shared__ unsigned kept;
  __shared__ unsigned long long base;
  const ScatterShape sh = scatter_shape(nvec);
  const long long total = units * sh.piece.count;
  const int tid = threadIdx.x;
  for (long long c0 = static_cast<long long>(blockIdx.x) * kGroupChunk; c0 < total;
       c0 += static_cast<long long>(gridDim.x) * kGroupChunk) {
    const int n = total - c0 < kGroupChunk ? static_cast<int>(total - c0) : kGroupChunk;
    clear_table(t, tid, kGroupThreads);
    if (kRange && tid == 0) kept = 0;
    __syncthreads();
    long long dflag[kGroupPer], src[kGroupPer];
    unsigned long long key[kGroupPer];
    unsigned slot[kGroupPer], rank[kGroupPer];
    // Phases across the thread's pieces, so their index loads and shared atomics
    // overlap instead of forming one dependent chain per piece.
#pragma unroll
    for (int q = 0; q < kGroupPer; ++q) {
      const int i = tid + q * kGroupThreads;
      dflag[q] = -1;
      src[q] = 0;
      if (i < n) piece_offsets<I, V>(p, idx, c0 + i, sh, &dflag[q], &src[q]);
      if (kRange && dflag[q] >= 0) {
        const long long local = owned_offset(own, dflag[q] & ~1ll);
        dflag[q] = local >= 0 ? local | (dflag[q] & 1) : -1;
      }
      key[q] = dflag[q] >= 0 ? key_of(dflag[q], V) : kEmptySlot;
      slot[q] = __umulhi(static_cast<unsigned>((key[q] * 0x9E3779B97F4A7C15ull) >> 32), GroupTable<kGroupChunk>::H);
    }
    unsigned long long prev[kGroupPer];
#pragma unroll
    for (int q = 0; q < kGroupPer; ++q)
      prev[q] = key[q] != kEmptySlot ? atomicCAS(&t.key[slot[q]], kEmptySlot, key[q]) : kEmptySlot;
#pragma unroll
    for (int q = 0; q < kGroupPer; ++q)
      if (prev[q] != kEmptySlot && prev[q] != key[q]) slot[q] = find_slot(t, key[q]);  // occupied by another key
    unsigned mine = 0;
#pragma unroll
    for (int q = 0; q < kGroupPer; ++q)
      if (key[q] != kEmptySlot) {
        rank[q] = atomicAdd(&t.count[slot[q]], 1u);
        ++mine;
      }
    if (kRange && mine) atomicAdd(&kept, mine);
    __syncthreads();
    scan_counts(t, tid, kGroupThreads);
    if (kRange) {
      if (tid == 0) base = kept ? atomicAdd(reserve, static_cast<unsigned long long>(kept)) : 0;
      __syncthreads();
    }
    const long long first = kRange ? static_cast<long long>(base) : c0;
#pragma unroll
    for (int q = 0; q < kGroupPer; ++q) {
      if (dflag[q] >= 0) {
        GroupedPiece g;
        g.dflag = dflag[q];
        g.src = src[q];
        list[first + t.count[slot[q]] + rank[q]] = g;
      }
    }
    __syncthreads();
  }
}

constexpr int kFoldSlots = 4;  // steps in flight per lane in the streaming fold

__host__ __device__ __forceinline__ int fold_stage_bytes_per_warp(int vbytes) {
  return kFoldSlots * kScatterVecs * 32 * vbytes;
}

template <int V>
__device__ __forceinline__ void cp_async_v(void* smem, const void* gmem) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  if constexpr (V == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(gmem) : "memory");
  } else if constexpr (V == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(a), "l"(gmem) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(a), "l"(gmem) : "memory");
  }
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The list pieces of one warp, read 32 at a time (one per lane, the next batch
// prefetched) and handed to the sub-warps by shuffles.  `at` must be called with
// non-decreasing batches, advancing at most one batch a call, by the whole warp.
struct ListCursor {
  const GroupedPiece* list;
  long long beg, end;
  long long batch;
  longlong2 cur, next;

  __device__ __forceinline__ longlong2 load(long long b, int lane) const {
    const long long q = beg + (b << 5) + lane;
    if (q < end) return __ldg(reinterpret_cast<const longlong2*>(list) + q);
    return make_longlong2(-1, 0);
  }

  __device__ __forceinline__ void start(int lane) {
    batch = 0;
    cur = load(0, lane);
    next = load(1, lane);
  }

  __device__ __forceinline__ void at(long long e, int lane, long long* dflag, long long* src) {
    if ((e >> 5) != batch) {
      ++batch;
      cur = next;
      next = load(batch + 1, lane);
    }
    const int from = static_cast<int>(e & 31);
    *dflag = __shfl_sync(0xffffffffu, cur.x, from);
    *src = __shfl_sync(0xffffffffu, cur.y, from);
  }
};

// Pass 2: fold the grouped list.  Warp w of the grid takes a contiguous range of the
// list; step t hands piece t*E + sub of the range to sub-warp sub.  Each lane keeps
// kFoldSlots steps of its own vectors in flight (cp.async into its ring slots; it
// reads back only what it copied, so no warp barrier is needed).  The loop is
// unrolled by kFoldSlots so the ring slot and the remembered destinations are static.
template <typename F, int V>
__device__ __forceinline__ void scatter_fold_pass(const GroupedPiece* __restrict__ list, long long total,
                                                  long long nvec, unsigned char* __restrict__ out,
                                                  const unsigned char* __restrict__ upd, unsigned char* stage) {
  using R = typename Raw<V>::T;
  constexpr int S = kFoldSlots;
  const ScatterShape sh = scatter_shape(nvec);
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long per = (total + nw - 1) / nw;
  const long long beg = w * per < total ? w * per : total;
  const long long end = beg + per < total ? beg + per : total;
  const int L = 1 << sh.lshift;
  const int E = 32 >> sh.lshift;
  const int sub = lane >> sh.lshift;
  const int lig = lane & (L - 1);
  const long long steps = (end - beg + E - 1) / E;
  unsigned char* ring = stage + (threadIdx.x >> 5) * fold_stage_bytes_per_warp(V);
  ListCursor cur{list, beg, end, 0, {}, {}};
  cur.start(lane);
  long long pend[S];  // destination | flag of the step in each slot (-1: none)
  auto issue = [&](long long t, int slot) {
    long long dflag = -1, src = 0;
    if (t < steps) {
      cur.at(t * E + sub, lane, &dflag, &src);
      if (dflag >= 0) {
        const int len = static_cast<int>((dflag & 1) ? sh.last : sh.piece.vecs);
#pragma unroll
        for (int j = 0; j < kScatterVecs; ++j) {
          const int v = lig + L * j;
          if (v < len)
            cp_async_v<V>(ring + ((slot * kScatterVecs + j) * 32 + lane) * V, upd + src + static_cast<long long>(v) * V);
        }
      }
    }
    cp_async_commit();
    return dflag;
  };
  Fold<F, V> f;
#pragma unroll
  for (int k = 0; k < S - 1; ++k) pend[k] = issue(k, k);
  for (long long t0 = 0; t0 < steps; t0 += S) {
#pragma unroll
    for (int k = 0; k < S; ++k) {
      pend[(k + S - 1) % S] = issue(t0 + k + S - 1, (k + S - 1) % S);
      cp_async_wait<S - 1>();
      const long long dflag = pend[k];
      if (dflag >= 0) {
        const int len = static_cast<int>((dflag & 1) ? sh.last : sh.piece.vecs);
        R x[kScatterVecs];
#pragma unroll
        for (int j = 0; j < kScatterVecs; ++j)
          if (lig + L * j < len) x[j] = *reinterpret_cast<const R*>(ring + ((k * kScatterVecs + j) * 32 + lane) * V);
        f.take(out, lig, L, sh, dflag, x);
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  f.flush(out, lig, L, sh);
}

// ---- TMA fold (16-byte vectors) ------------------------------------------------
// The streaming fold for rows whose pieces are whole 16-byte vectors: lane 0 moves
// every piece with one bulk copy (cp.async.bulk, completion on a per-slot mbarrier)
// into a ring in shared memory, and adds every group to memory with one bulk
// reduction (cp.reduce.async.bulk .add) from there: a group of one piece goes back
// out untouched, a longer group is summed by the warp into its last piece's slot
// first.  Per piece the warp executes a few dozen instructions, whatever its size.
constexpr int kBulkRingBytes = 8192;  // per warp
constexpr int kBulkMaxSlots = 16;
// try_wait rounds of a staged-data wait before it gives up (a build may lower it: the
// tests build the library once with 0, so that every such wait runs out at once).
#ifndef T4A_STAGE_WAIT_LIMIT
#define T4A_STAGE_WAIT_LIMIT (1u << 20)
#endif
constexpr unsigned kBulkWaitLimit = T4A_STAGE_WAIT_LIMIT;
// Rounds of the drain of loads still in flight when a warp stops: never lowered.
constexpr unsigned kBulkDrainLimit = 1u << 22;

__host__ __device__ __forceinline__ int bulk_stage_bytes_per_warp() { return kBulkRingBytes + kBulkMaxSlots * 8; }

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

// Bounded wait for phase `parity` of an mbarrier; false when the limit ran out.  Each
// try may suspend the thread for up to kBulkSuspendNs while the phase is pending,
// so a waiting warp does not spin on the issue slots.
constexpr unsigned kBulkSuspendNs = 2000;
__device__ __forceinline__ bool bar_wait(unsigned bar, unsigned parity, unsigned limit = kBulkWaitLimit) {
  for (unsigned it = 0; it < limit; ++it) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "n"(kBulkSuspendNs)
        : "memory");
    if (ok) return true;
  }
  return false;
}

template <typename F>
__device__ __forceinline__ void bulk_reduce(unsigned char* gdst, unsigned ssrc, unsigned bytes) {
  if constexpr (sizeof(F) == 8) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f64 [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc),
                 "r"(bytes)
                 : "memory");
  } else {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc),
                 "r"(bytes)
                 : "memory");
  }
}

// Consume-side view of the list: the piece at e and the destination of e + 1.
__device__ __forceinline__ long long next_dflag(const ListCursor& c, long long e, long long n) {
  if (e + 1 >= n) return -1;
  const int q = static_cast<int>((e + 1) & 31);
  const long long from_cur = __shfl_sync(0xffffffffu, c.cur.x, q);
  const long long from_next = __shfl_sync(0xffffffffu, c.next.x, 0);
  return q == 0 ? from_next : from_cur;
}

// `status` receives 1 when a wait ran out (the warp then stops).
template <typename F>
__device__ __forceinline__ void scatter_fold_bulk(const GroupedPiece* __restrict__ list, long long total,
                                                  long long nvec, unsigned char* __restrict__ out,
                                                  const unsigned char* __restrict__ upd, unsigned char* stage,
                                                  int* status) {
  constexpr int V = 16;
  constexpr int VE = V / sizeof(F);
  const ScatterShape sh = scatter_shape(nvec);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp;
  const long long per = (total + nw - 1) / nw;
  const long long beg = w * per < total ? w * per : total;
  const long long end = beg + per < total ? beg + per : total;
  const long long n = end - beg;
  const int full_bytes = static_cast<int>(sh.piece.vecs) * V;
  int slots = kBulkRingBytes / full_bytes;
  if (slots > kBulkMaxSlots) slots = kBulkMaxSlots;
  unsigned char* ring = stage + warp * bulk_stage_bytes_per_warp();
  const unsigned bars = smem_addr(ring + kBulkRingBytes);
  if (lane == 0) {
    for (int q = 0; q < slots; ++q) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bars + 8 * q) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  ListCursor ic{list, beg, end, 0, {}, {}};
  ListCursor fc{list, beg, end, 0, {}, {}};
  ic.start(lane);
  fc.start(lane);
  const int ahead = slots - 2;  // loads in flight; two slots drain their reductions
  unsigned pending = 0;          // bit q: a load into slot q is in flight
  // Lane 0 loads piece k into slot `slot`; reuse waits for the slot's previous
  // reduction to finish reading (one bulk group is committed per consumed piece).
  auto issue = [&](long long k, int slot) {
    long long dflag, src;
    ic.at(k, lane, &dflag, &src);
    if (lane == 0) {
      const unsigned bytes = static_cast<unsigned>(((dflag & 1) ? sh.last : sh.piece.vecs) * V);
      if (k >= slots) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bars + 8 * slot), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       smem_addr(ring + slot * full_bytes)),
                   "l"(upd + src), "r"(bytes), "r"(bars + 8 * slot)
                   : "memory");
    }
    pending |= 1u << slot;
  };
  int islot = 0;
  for (long long k = 0; k < ahead && k < n; ++k) {
    issue(k, islot);
    islot = islot + 1 == slots ? 0 : islot + 1;
  }
  unsigned phases = 0;  // bit q: parity to wait for on slot q
  long long prev = -1;
  F acc[kScatterVecs][VE];
  bool failed = false;
  int slot = 0;
  for (long long k = 0; k < n; ++k) {
    if (k + ahead < n) {
      issue(k + ahead, islot);
      islot = islot + 1 == slots ? 0 : islot + 1;
    }
    // The warp stops together if any lane's wait ran out.
    if (__any_sync(0xffffffffu, !bar_wait(bars + 8 * slot, (phases >> slot) & 1u))) {
      failed = true;
      break;
    }
    phases ^= 1u << slot;
    pending &= ~(1u << slot);
    long long dflag, src;
    fc.at(k, lane, &dflag, &src);
    const long long nd = next_dflag(fc, k, n);
    const bool first = dflag != prev;
    const bool last = dflag != nd;
    prev = dflag;
    const int len = static_cast<int>((dflag & 1) ? sh.last : sh.piece.vecs);
    unsigned char* sp = ring + slot * full_bytes;
    if (!(first && last)) {
#pragma unroll
      for (int j = 0; j < kScatterVecs; ++j) {
        const int v = lane + 32 * j;
        if (v < len) {
          F y[VE];
          raw_to_f<F, V>(*reinterpret_cast<const uint4*>(sp + v * V), y);
#pragma unroll
          for (int q = 0; q < VE; ++q) acc[j][q] = first ? y[q] : acc[j][q] + y[q];
        }
      }
      if (last) {
#pragma unroll
        for (int j = 0; j < kScatterVecs; ++j) {
          const int v = lane + 32 * j;
          if (v < len) memcpy(sp + v * V, &acc[j][0], V);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
    }
    __syncwarp();
    if (lane == 0) {
      if (last) bulk_reduce<F>(out + (dflag & ~1ll), smem_addr(sp), static_cast<unsigned>(len * V));
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    slot = slot + 1 == slots ? 0 : slot + 1;
  }
  if (failed) {
    if (lane == 0) atomicExch(status, 1);
    // Drain the loads still in flight (each wait bounded) before the ring goes away.
    for (int q = 0; q < slots; ++q)
      if ((pending >> q) & 1u) bar_wait(bars + 8 * q, (phases >> q) & 1u, kBulkDrainLimit);
  }
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  __syncwarp();
}

// One element per thread (any geometry): atomics per component, as the reference.
template <typename F, typename I>
__device__ __forceinline__ void scatter_elements(const WindowPlan& p, unsigned char* out, const unsigned char* upd,
                                                 const I* idx, long long units) {
  const long long total = units * p.run;
  const int comps = p.esize / static_cast<int>(sizeof(F));
  const long long stride = static_cast<long long>(gridDim.x) * block_threads();
  for (long long f = static_cast<long long>(blockIdx.x) * block_threads() + flat_tid(); f < total; f += stride) {
    const long long u = f / p.run;
    const long long e = f - u * p.run;
    long long oa, ob;
    unit_offsets<I>(p, idx, u, &oa, &ob);
    F* d = reinterpret_cast<F*>(out + (oa + e) * p.esize);
    const F* s = reinterpret_cast<const F*>(upd + (ob + e) * p.esize);
    for (int c = 0; c < comps; ++c) atomicAdd(d + c, s[c]);
  }
}

}  // namespace t4a
