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
// Scatter: each block takes a chunk of kScatterChunk units, sorts it by destination
// (bitonic, in shared memory), and each warp folds its share of the sorted chunk in
// registers: consecutive units with the same destination are summed in update order
// and reach memory as one vector of `red.global.add` per distinct destination.
// Collisions on hot destinations (Zipf indices) therefore cost one atomic row per
// chunk instead of one per update.  Results equal the reference's up to the order of
// floating additions, which the reference leaves to its atomics as well.
#pragma once

#include "common.cuh"
#include "gather_scatter_plan.h"

namespace t4a {

constexpr int kGatherThreads = 256;
constexpr int kGatherDepth = 8;
constexpr int kScatterThreads = 512;
constexpr int kScatterChunk = 2048;
constexpr long long kScatterSentinel = 0x7fffffffffffffffll;

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
struct ScatterSmem {
  long long dst[kScatterChunk];  // destination byte offset of the piece (sort key)
  long long src[kScatterChunk];  // updates byte offset of the piece (second key)
  int piece[kScatterChunk];      // piece of the run
};

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

// Block-wide ascending sort of the chunk by (dst, src): bitonic network, every stage
// ends with a block barrier.  `n` is a power of two.
__device__ __forceinline__ void sort_chunk(ScatterSmem& sm, int n, int tid, int nthreads) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < (n >> 1); i += nthreads) {
        const int lo = ((i & ~(j - 1)) << 1) | (i & (j - 1));
        const int hi = lo + j;
        const bool up = (lo & k) == 0;
        const long long dl = sm.dst[lo], dh = sm.dst[hi];
        const long long sl = sm.src[lo], sh = sm.src[hi];
        const bool greater = dl > dh || (dl == dh && sl > sh);
        if (greater == up) {
          sm.dst[lo] = dh;
          sm.dst[hi] = dl;
          sm.src[lo] = sh;
          sm.src[hi] = sl;
          const int pl = sm.piece[lo];
          sm.piece[lo] = sm.piece[hi];
          sm.piece[hi] = pl;
        }
      }
      __syncthreads();
    }
  }
}

// Scatters `units` update runs of `nvec` V-byte vectors into `out`.  The block is
// whole warps; JB = vectors per lane per piece (pieces are 32 * JB vectors).
template <typename F, typename I, int V, int JB>
__device__ __forceinline__ void scatter_units(const WindowPlan& p, unsigned char* __restrict__ out,
                                              const unsigned char* __restrict__ upd, const I* __restrict__ idx,
                                              long long units, long long nvec, ScatterSmem& sm) {
  using R = typename Raw<V>::T;
  constexpr int VE = V / sizeof(F);
  constexpr int D = JB >= 4 ? 2 : 4;  // pieces in flight per warp
  const Pieces piece = make_pieces(nvec, 32ll * JB);
  const long long total = units * piece.count;
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31;
  const int nwarps = nthreads >> 5;
  const int per_warp = (kScatterChunk + nwarps - 1) / nwarps;
  const int beg = (tid >> 5) * per_warp;
  const int end = beg + per_warp < kScatterChunk ? beg + per_warp : kScatterChunk;
  for (long long c0 = static_cast<long long>(blockIdx.x) * kScatterChunk; c0 < total;
       c0 += static_cast<long long>(gridDim.x) * kScatterChunk) {
    for (int i = tid; i < kScatterChunk; i += nthreads) {
      const long long w = c0 + i;
      long long d = kScatterSentinel, s = 0, pc = 0;
      if (w < total) {
        long long u = w;
        if (piece.count > 1) {
          u = w / piece.count;
          pc = w - u * piece.count;
        }
        long long oa, ob;
        unit_offsets<I>(p, idx, u, &oa, &ob);
        d = oa * p.esize + pc * piece.vecs * V;
        s = ob * p.esize + pc * piece.vecs * V;
      }
      sm.dst[i] = d;
      sm.src[i] = s;
      sm.piece[i] = static_cast<int>(pc);
    }
    __syncthreads();
    sort_chunk(sm, kScatterChunk, tid, nthreads);

    F acc[JB][VE];
    long long cur_d = -1, cur_p = -1, cur_len = 0;
    for (int e0 = beg; e0 < end; e0 += D) {
      R x[D][JB];
      long long ed[D], ep[D], elen[D];
#pragma unroll
      for (int dd = 0; dd < D; ++dd) {
        const int e = e0 + dd;
        ed[dd] = kScatterSentinel;
        if (e < end) ed[dd] = sm.dst[e];
        if (ed[dd] != kScatterSentinel) {
          const long long s = sm.src[e];
          ep[dd] = sm.piece[e];
          const long long left = nvec - ep[dd] * piece.vecs;
          elen[dd] = left < piece.vecs ? left : piece.vecs;
#pragma unroll
          for (int j = 0; j < JB; ++j) {
            const long long v = lane + 32 * j;
            if (v < elen[dd]) x[dd][j] = ld_stream<V>(upd + s + v * V);
          }
        }
      }
#pragma unroll
      for (int dd = 0; dd < D; ++dd) {
        if (ed[dd] == kScatterSentinel) continue;
        const bool same = ed[dd] == cur_d && ep[dd] == cur_p;
        if (!same && cur_d >= 0) {
#pragma unroll
          for (int j = 0; j < JB; ++j) {
            const long long v = lane + 32 * j;
            if (v < cur_len) red_add<F, V>(out + cur_d + v * V, acc[j]);
          }
        }
#pragma unroll
        for (int j = 0; j < JB; ++j) {
          const long long v = lane + 32 * j;
          if (v < elen[dd]) {
            F y[VE];
            raw_to_f<F, V>(x[dd][j], y);
#pragma unroll
            for (int q = 0; q < VE; ++q) acc[j][q] = same ? acc[j][q] + y[q] : y[q];
          }
        }
        cur_d = ed[dd];
        cur_p = ep[dd];
        cur_len = elen[dd];
      }
    }
    if (cur_d >= 0) {
#pragma unroll
      for (int j = 0; j < JB; ++j) {
        const long long v = lane + 32 * j;
        if (v < cur_len) red_add<F, V>(out + cur_d + v * V, acc[j]);
      }
    }
    __syncthreads();
  }
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
