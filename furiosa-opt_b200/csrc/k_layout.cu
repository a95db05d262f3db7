// Layout-move kernels: relayout (BufStorage::transpose, furiosa-opt-std/src/storage/buf.rs:257-313),
// transmute (buf.rs:592-613), and the walk-driven gather / scatter (buf.rs:485-576).
//
// Every kernel is HBM-bound: one read of each live source element and one write of each live
// destination element. Three relayout paths, picked per plan:
//   * vec:   the innermost walk wheel is unit-stride on both sides -> 16-byte loads and stores;
//   * tile:  the dst-innermost wheel is strided in src but another wheel is unit-stride in src ->
//            a 32x32 shared-memory tile so both the read and the write are coalesced;
//   * walk:  anything else, one element per thread with the odometer decomposed per position.
#include <cstring>
#include <algorithm>
#include <type_traits>

#include "ctx.hpp"

namespace fopt {

KWalk to_kwalk(const Walk& w) {
  KWalk k{};
  k.n = (int)w.wheels.size();
  for (int i = 0; i < k.n; ++i) {
    k.extent[i] = w.wheels[i].extent;
    k.live[i] = w.wheels[i].live;
    for (int m = 0; m < 3; ++m) k.stride[m][i] = m < w.nmem ? w.wheels[i].stride[m] : 0;
  }
  return k;
}

bool to_kwalk32(const KWalk& w, KWalk32& out) {
  out = KWalk32{};
  out.n = w.n;
  int64_t pos = 1;
  for (int i = 0; i < w.n; ++i) {
    if (w.extent[i] >= (1ll << 31)) return false;
    pos *= w.extent[i];
    if (pos >= (1ll << 31)) return false;
    out.div[i] = make_fastdiv((uint32_t)w.extent[i]);
    out.live[i] = (uint32_t)w.live[i];
    for (int m = 0; m < 3; ++m) {
      int64_t s = w.stride[m][i];
      if (s * (w.extent[i] - 1) >= (1ll << 30)) return false;
      out.stride[m][i] = (int32_t)s;
    }
  }
  return true;
}

namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t work, int per_block = kThreads) {
  int64_t g = (work + per_block - 1) / per_block;
  // Persistent-ish: cap at a multiple of the 148 SMs, grid-stride loops cover the rest.
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32));
}

// ---- vec path: V elements (16 bytes) per unit ----
template <typename V>
__global__ void relayout_vec32(V* __restrict__ dst, const V* __restrict__ src, KWalk32 w, uint32_t units,
                               uint32_t vlen, int64_t src_base_v, int64_t dst_base_v) {
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    int32_t off = 0;
    if (!walk_offsets32<1>(w, u * vlen, &off)) continue;
    dst[dst_base_v + u] = src[src_base_v + off / (int32_t)vlen];
  }
}

template <typename V>
__global__ void relayout_vec64(V* __restrict__ dst, const V* __restrict__ src, KWalk w, int64_t units, int64_t vlen,
                               int64_t src_base_v, int64_t dst_base_v) {
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    int64_t off = 0;
    if (!walk_offsets<1>(w, u * vlen, &off)) continue;
    dst[dst_base_v + u] = src[src_base_v + off / vlen];
  }
}

// ---- broadcast path: the dst-innermost wheel re-reads one src element (src stride 0) ----
template <typename T>
__global__ void relayout_bcast(uint4* __restrict__ dst, const T* __restrict__ src, KWalk outer, int64_t inner_units,
                               int64_t units, int64_t src_base, int64_t dst_base_v) {
  constexpr int V = 16 / sizeof(T);
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    int64_t off = 0;
    if (!walk_offsets<1>(outer, u / inner_units, &off)) continue;
    T v = src[src_base + off];
    union {
      uint4 q;
      T e[V];
    } pack;
#pragma unroll
    for (int k = 0; k < V; ++k) pack.e[k] = v;
    dst[dst_base_v + u] = pack.q;
  }
}

// Broadcast rows of at least 32 vectors: a warp per row, the row's source offset walked once, then
// the warp's lanes store the row's vectors (512 contiguous bytes per warp store) instead of every
// 16-byte vector dividing its index and walking the odometer.
template <typename T>
__global__ void relayout_bcast_rows(uint4* __restrict__ dst, const T* __restrict__ src, KWalk outer,
                                    int64_t inner_units, int64_t rows, int64_t src_base, int64_t dst_base_v) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += nw) {
    int64_t off = 0;
    if (!walk_offsets<1>(outer, row, &off)) continue;
    const T v = src[src_base + off];
    union {
      uint4 q;
      T e[V];
    } pack;
#pragma unroll
    for (int k = 0; k < V; ++k) pack.e[k] = v;
    uint4* d = dst + dst_base_v + row * inner_units;
    for (int64_t u = lane; u < inner_units; u += 32) d[u] = pack.q;
  }
}

// ---- tile path ----
// `others` walks every wheel except the dst-innermost (i) and the src-unit-stride (j) ones; memory
// 0 = src offset, memory 1 = dst position. A (32 V) x (32 V) tile moves through shared memory; each
// thread reads V consecutive src elements (a 4-byte word for 1- and 2-byte types) and writes V
// consecutive dst elements, so both global sides move whole 128-byte lines per warp.
template <typename T, int V, int TT>
__global__ void __launch_bounds__(256) relayout_tile(T* __restrict__ dst, const T* __restrict__ src, KWalk others,
                                                     int64_t e0, int64_t s0, int64_t ej, int64_t wj, int64_t src_base,
                                                     int64_t dst_base, int64_t nt0, int64_t ntj, int64_t batches) {
  // TT x TT tile; a warp covers TT / V columns... each thread moves V-element vectors along both
  // the read side (src-contiguous) and the write side (dst-contiguous)
  constexpr int VB = sizeof(T) * V;
  using W = typename std::conditional<VB == 16, uint4, typename std::conditional<VB == 8, uint2,
            typename std::conditional<VB == 4, uint32_t, typename std::conditional<VB == 2, uint16_t, uint8_t>::type>::type>::type>::type;
  constexpr int LANES = TT / V;            // threads across one tile row
  constexpr int ROWS = 256 / LANES;        // tile rows per pass
  constexpr int PAD = 1;  // odd row stride: the V-row column gather spreads over the banks
  __shared__ T tile[TT][TT + PAD];
  const int tid = threadIdx.x;
  const int tx = tid % LANES, ty = tid / LANES;
  for (int64_t blk = blockIdx.x; blk < nt0 * ntj * batches; blk += gridDim.x) {
    int64_t ti = blk % nt0, tj = (blk / nt0) % ntj, b = blk / (nt0 * ntj);
    int64_t off[2] = {0, 0};
    bool live = walk_offsets<2>(others, b, off);
    if (live) {
      const int64_t dj = tj * TT + tx * V;
#pragma unroll 4
      for (int r = ty; r < TT; r += ROWS) {
        int64_t d0 = ti * TT + r;
        if (d0 < e0 && dj < ej) {
          W w = *(const W*)(src + src_base + off[0] + d0 * s0 + dj);
#pragma unroll
          for (int k = 0; k < V; ++k) tile[r][tx * V + k] = ((const T*)&w)[k];
        }
      }
    }
    __syncthreads();
    if (live) {
      const int64_t d0 = ti * TT + tx * V;
#pragma unroll 4
      for (int c = ty; c < TT; c += ROWS) {
        int64_t dj = tj * TT + c;
        if (d0 < e0 && dj < ej) {
          W w;
#pragma unroll
          for (int k = 0; k < V; ++k) ((T*)&w)[k] = tile[tx * V + k][c];
          *(W*)(dst + dst_base + off[1] + d0 + dj * wj) = w;
        }
      }
    }
    __syncthreads();
  }
}

// Tile path on 32-bit words (E = 4 / sizeof(T) elements per word; the launcher uses it for 1-byte
// elements). A
// tile is 32 E x 32 E elements: 128-byte rows on both sides. An E x E element block moves as E
// words: a lane loads one word from each of E consecutive source rows (a warp instruction reads a
// whole 128-byte line), transposes the block in registers with byte permutes, and stores the E
// words into the transposed shared tile. The shared column is XOR-swizzled by the block's source
// word (word a of tile row c sits at column a ^ (c / E)), so the stores and the row reads both hit
// 32 distinct banks; each warp then writes whole 128-byte dst lines. Tile base pointers are formed
// once per tile in 64 bits; in-tile offsets stay 32-bit.
template <int E>
__device__ __forceinline__ void transpose_block(const uint32_t* r, uint32_t* o) {
  if constexpr (E == 1) {
    o[0] = r[0];
  } else if constexpr (E == 2) {
    o[0] = __byte_perm(r[0], r[1], 0x5410);
    o[1] = __byte_perm(r[0], r[1], 0x7632);
  } else {
    const uint32_t t0 = __byte_perm(r[0], r[1], 0x5140), t1 = __byte_perm(r[0], r[1], 0x7362);
    const uint32_t t2 = __byte_perm(r[2], r[3], 0x5140), t3 = __byte_perm(r[2], r[3], 0x7362);
    o[0] = __byte_perm(t0, t2, 0x5410);
    o[1] = __byte_perm(t0, t2, 0x7632);
    o[2] = __byte_perm(t1, t3, 0x5410);
    o[3] = __byte_perm(t1, t3, 0x7632);
  }
}

// TW: tile width in words (32, or 64 for wider types); the tile is (TW E) x (TW E) elements, TW E rows
// of TW words in shared memory. With TW = 64 a warp covers each row in two halves of 32 words, and
// the XOR swizzle (columns 0..63) still gives every half 32 distinct banks.
template <typename T, int TW>
__global__ void __launch_bounds__(256) relayout_tile_w(T* __restrict__ dst, const T* __restrict__ src, KWalk others,
                                                       int64_t e0, int64_t s0, int64_t ej, int64_t wj,
                                                       int64_t src_base, int64_t dst_base, int64_t nt0, int64_t ntj,
                                                       int64_t batches) {
  constexpr int E = 4 / (int)sizeof(T), TT = TW * E;
  __shared__ uint32_t tile[TT][TW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t blk = blockIdx.x; blk < nt0 * ntj * batches; blk += gridDim.x) {
    const int64_t ti = blk % nt0, tj = (blk / nt0) % ntj, b = blk / (nt0 * ntj);
    int64_t off[2] = {0, 0};
    const bool live = walk_offsets<2>(others, b, off);
    const int64_t r0 = e0 - ti * TT, rj = ej - tj * TT;
    const int n0 = r0 < TT ? (int)r0 : TT, nj = rj < TT ? (int)rj : TT;
    if (live) {
      const T* sT = src + src_base + off[0] + ti * TT * s0 + tj * TT;
#pragma unroll 2
      for (int q = warp; q < TW * (TW / 32); q += 8) {
        const int a = q % TW;                  // source rows E a .. E a + E - 1 of the tile
        const int w = (q / TW) * 32 + lane;    // source word column
        uint32_t r[E], o[E];
#pragma unroll
        for (int i = 0; i < E; ++i) r[i] = 0;
        if (E * a < n0 && E * w < nj) {
#pragma unroll
          for (int i = 0; i < E; ++i) r[i] = *(const uint32_t*)(sT + (int64_t)(E * a + i) * s0 + E * w);
        }
        transpose_block<E>(r, o);
#pragma unroll
        for (int k = 0; k < E; ++k) tile[E * w + k][a ^ w] = o[k];
      }
    }
    __syncthreads();
    if (live) {
      T* dT = dst + dst_base + off[1] + ti * TT + tj * TT * wj;
#pragma unroll 4
      for (int q = warp; q < nj * (TW / 32); q += 8) {
        const int c = q / (TW / 32);              // dst row of the tile
        const int a = (q % (TW / 32)) * 32 + lane;  // dst word
        if (E * a < n0) *(uint32_t*)(dT + (int64_t)c * wj + E * a) = tile[c][a ^ (c / E)];
      }
    }
    __syncthreads();
  }
}

// Tile path for 2-byte elements in 8-byte units: a thread moves a 4 x 4 element block, loading four
// 8-byte row pieces, transposing them in registers with byte permutes and storing four 8-byte
// units into the transposed shared tile (128 rows x 32 units; unit a of tile row c sits at column
// a ^ (c / 4), so a warp's 8-byte stores and loads take the minimum two wavefronts). Global loads and
// stores are 8 bytes per lane, 256 contiguous bytes per warp instruction.
__global__ void __launch_bounds__(256) relayout_tile_h(uint16_t* __restrict__ dst, const uint16_t* __restrict__ src,
                                                       KWalk others, int64_t e0, int64_t s0, int64_t ej, int64_t wj,
                                                       int64_t src_base, int64_t dst_base, int64_t nt0, int64_t ntj,
                                                       int64_t batches) {
  __shared__ uint2 tile[128][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t blk = blockIdx.x; blk < nt0 * ntj * batches; blk += gridDim.x) {
    const int64_t ti = blk % nt0, tj = (blk / nt0) % ntj, b = blk / (nt0 * ntj);
    int64_t off[2] = {0, 0};
    const bool live = walk_offsets<2>(others, b, off);
    const int64_t r0 = e0 - ti * 128, rj = ej - tj * 128;
    const int n0 = r0 < 128 ? (int)r0 : 128, nj = rj < 128 ? (int)rj : 128;  // multiples of 4
    if (live) {
      const uint16_t* sT = src + src_base + off[0] + ti * 128 * s0 + tj * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int a = warp + 8 * q;  // source rows 4 a .. 4 a + 3; lane = source unit (4 columns)
        uint2 r[4] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
        if (4 * a < n0 && 4 * lane < nj) {
#pragma unroll
          for (int i = 0; i < 4; ++i) r[i] = *(const uint2*)(sT + (int64_t)(4 * a + i) * s0 + 4 * lane);
        }
        // column k of the block: rows (0, 1) in .x, rows (2, 3) in .y
        const uint2 c0 = make_uint2(__byte_perm(r[0].x, r[1].x, 0x5410), __byte_perm(r[2].x, r[3].x, 0x5410));
        const uint2 c1 = make_uint2(__byte_perm(r[0].x, r[1].x, 0x7632), __byte_perm(r[2].x, r[3].x, 0x7632));
        const uint2 c2 = make_uint2(__byte_perm(r[0].y, r[1].y, 0x5410), __byte_perm(r[2].y, r[3].y, 0x5410));
        const uint2 c3 = make_uint2(__byte_perm(r[0].y, r[1].y, 0x7632), __byte_perm(r[2].y, r[3].y, 0x7632));
        tile[4 * lane + 0][a ^ lane] = c0;
        tile[4 * lane + 1][a ^ lane] = c1;
        tile[4 * lane + 2][a ^ lane] = c2;
        tile[4 * lane + 3][a ^ lane] = c3;
      }
    }
    __syncthreads();
    if (live && 4 * lane < n0) {
      uint16_t* dT = dst + dst_base + off[1] + ti * 128 + tj * 128 * wj + 4 * lane;
#pragma unroll 4
      for (int c = warp; c < nj; c += 8) *(uint2*)(dT + (int64_t)c * wj) = tile[c][lane ^ (c >> 2)];
    }
    __syncthreads();
  }
}

// Tile path for 1-byte elements in 8-byte units: a thread moves an 8 x 8 byte block (four 4 x 4 word
// transposes), loading eight 8-byte row pieces and storing eight 8-byte units into the transposed
// shared tile (128 rows x 16 units; unit a of tile row c sits at column a ^ (c / 8), so the 8-byte
// stores and loads take the minimum two wavefronts). A warp covers two 128-byte rows per global load
// and store.
__global__ void __launch_bounds__(256) relayout_tile_b8(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                                        KWalk others, int64_t e0, int64_t s0, int64_t ej, int64_t wj,
                                                        int64_t src_base, int64_t dst_base, int64_t nt0, int64_t ntj,
                                                        int64_t batches) {
  __shared__ uint2 tile[128][16];
  const int a = threadIdx.x >> 4, b = threadIdx.x & 15;  // source row block, source unit
  for (int64_t blk = blockIdx.x; blk < nt0 * ntj * batches; blk += gridDim.x) {
    const int64_t ti = blk % nt0, tj = (blk / nt0) % ntj, bt = blk / (nt0 * ntj);
    int64_t off[2] = {0, 0};
    const bool live = walk_offsets<2>(others, bt, off);
    const int64_t r0 = e0 - ti * 128, rj = ej - tj * 128;
    const int n0 = r0 < 128 ? (int)r0 : 128, nj = rj < 128 ? (int)rj : 128;  // multiples of 8
    if (live) {
      const uint8_t* sT = src + src_base + off[0] + ti * 128 * s0 + tj * 128;
      uint32_t lo[8], hi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) lo[i] = hi[i] = 0;
      if (8 * a < n0 && 8 * b < nj) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint2 v = *(const uint2*)(sT + (int64_t)(8 * a + i) * s0 + 8 * b);
          lo[i] = v.x;
          hi[i] = v.y;
        }
      }
      uint32_t tl[4], tr[4], bl[4], br[4];
      transpose_block<4>(lo, tl);
      transpose_block<4>(lo + 4, bl);
      transpose_block<4>(hi, tr);
      transpose_block<4>(hi + 4, br);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        tile[8 * b + k][a ^ b] = make_uint2(tl[k], bl[k]);
        tile[8 * b + 4 + k][a ^ b] = make_uint2(tr[k], br[k]);
      }
    }
    __syncthreads();
    if (live && 8 * b < n0) {
      uint8_t* dT = dst + dst_base + off[1] + ti * 128 + tj * 128 * wj + 8 * b;
#pragma unroll 4
      for (int c = a; c < nj; c += 16) *(uint2*)(dT + (int64_t)c * wj) = tile[c][b ^ (c >> 3)];
    }
    __syncthreads();
  }
}

// ---- walk path ----
template <typename T>
__global__ void relayout_walk32(T* __restrict__ dst, const T* __restrict__ src, KWalk32 w, uint32_t positions,
                                int64_t src_base, int64_t dst_base, int64_t src_elems) {
  for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < positions; q += gridDim.x * blockDim.x) {
    int32_t off = 0;
    if (!walk_offsets32<1>(w, q, &off)) continue;
    int64_t s = src_base + off;
    if (s < src_elems) dst[dst_base + q] = src[s];
  }
}

template <typename T>
__global__ void relayout_walk64(T* __restrict__ dst, const T* __restrict__ src, KWalk w, int64_t positions,
                                int64_t src_base, int64_t dst_base, int64_t src_elems) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < positions;
       q += (int64_t)gridDim.x * blockDim.x) {
    int64_t off = 0;
    if (!walk_offsets<1>(w, q, &off)) continue;
    int64_t s = src_base + off;
    if (s < src_elems) dst[dst_base + q] = src[s];
  }
}

// ---- padded rows from a dense source: [rows, L] -> [rows, E # ...], E > L, 4-byte elements ----
// A CTA stages kPadRows source rows (one contiguous run of kPadRows * L elements) in shared memory
// with aligned 16-byte loads, so every source byte is read from DRAM once, then writes the live
// cells of its destination rows (16-byte vectors when the rows are aligned, else one element per
// thread). Dead cells are not touched, as the reference skips them.
constexpr int kPadRowsDefault = 32;
// VEC: the destination rows start on 16-byte boundaries (E % 4 == 0, aligned base), so each thread
// writes one 16-byte vector of a row: whole vectors with one store, the vector across the live width
// element by element (its dead cells stay untouched).
template <bool VEC>
__global__ void __launch_bounds__(256) relayout_pad_rows(uint32_t* __restrict__ dst, const uint32_t* __restrict__ src,
                                                         int64_t rows, int L, int E, FastDiv e_div,
                                                         int64_t src_base, int64_t dst_base, int64_t src_elems, int kPadRows) {
  extern __shared__ uint4 pad_buf4[];
  uint32_t* buf = (uint32_t*)pad_buf4;
  for (int64_t r0 = (int64_t)blockIdx.x * kPadRows; r0 < rows; r0 += (int64_t)gridDim.x * kPadRows) {
    const int nr = (int)(rows - r0 < kPadRows ? rows - r0 : kPadRows);
    const int64_t s0 = src_base + r0 * L, s1 = s0 + (int64_t)nr * L;  // elements [s0, s1)
    const int64_t a0 = s0 & ~(int64_t)3;                                // aligned to 16 bytes
    const int off = (int)(s0 - a0);
    const int nvec = (int)((s1 - a0 + 3) >> 2);
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const int64_t e = a0 + 4 * (int64_t)v;
      if (e + 4 <= src_elems) {
        pad_buf4[v] = *((const uint4*)src + (e >> 2));
      } else {  // the source's last partial vector: element by element, inside the allocation
#pragma unroll
        for (int k = 0; k < 4; ++k) buf[4 * v + k] = e + k < src_elems ? src[e + k] : 0u;
      }
    }
    __syncthreads();
    uint32_t* drow = dst + dst_base + r0 * E;
    if constexpr (VEC) {
      const int nv = E >> 2, total = nr * nv;  // e_div divides by nv here
      for (int q = threadIdx.x; q < total; q += blockDim.x) {
        const uint32_t i = fdiv(e_div, (uint32_t)q);
        const int c = 4 * (int)((uint32_t)q - i * (uint32_t)nv);
        const uint32_t* sp = buf + off + (int)i * L + c;
        if (c + 4 <= L) {
          ((uint4*)drow)[q] = make_uint4(sp[0], sp[1], sp[2], sp[3]);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (c + k < L) drow[4 * q + k] = sp[k];
        }
      }
    } else {
      const int total = nr * E;
      for (int q = threadIdx.x; q < total; q += blockDim.x) {
        const uint32_t i = fdiv(e_div, (uint32_t)q), c = (uint32_t)q - i * (uint32_t)E;
        if ((int)c < L) drow[q] = buf[off + (int)i * L + (int)c];
      }
    }
    __syncthreads();
  }
}

// ---- rows path: a warp per row of the innermost wheel (partially live rows, e.g. padded widths) ----
template <typename T>
__global__ void relayout_rows(T* __restrict__ dst, const T* __restrict__ src, KWalk32 outer, uint32_t rows, uint32_t e0,
                              uint32_t l0, int32_t st0, int64_t src_base, int64_t dst_base, int64_t src_elems) {
  const uint32_t lane = threadIdx.x & 31, warps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    int32_t off = 0;
    if (!walk_offsets32<1>(outer, row, &off)) continue;
    const int64_t sb = src_base + off, db = dst_base + (int64_t)row * e0;
    for (uint32_t d = lane; d < l0; d += 32) {
      const int64_t si = sb + (int64_t)d * st0;
      if (si < src_elems) dst[db + d] = src[si];
    }
  }
}

// Rows path, vectorised: one thread per 16-byte dst vector of a row whose innermost wheel is only
// partly live (e.g. a padded width). The dst row pitch is a whole number of vectors, so every
// vector lies in one row; fully live vectors gather their V elements and store once, the vector
// that straddles the live width reads the dst first so that the dead slots keep their contents
// (the reference skips them), and fully dead vectors are not touched.
template <typename T>
__global__ void relayout_rows_vec(T* __restrict__ dst, const T* __restrict__ src, KWalk32 outer, FastDiv lvec_div,
                                  uint32_t total, uint32_t e0, uint32_t l0, int32_t st0, int64_t src_base,
                                  int64_t dst_base, int64_t src_elems, int64_t src_bytes) {
  constexpr int V = 16 / sizeof(T);
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
    const uint32_t row = fdiv(lvec_div, t);
    const uint32_t c0 = (t - row * lvec_div.d) * V;
    int32_t off = 0;
    if (!walk_offsets32<1>(outer, row, &off)) continue;
    const int64_t sb = src_base + off + (int64_t)c0 * st0;
    uint4* dp = (uint4*)(dst + dst_base + (int64_t)row * e0 + c0);
    uint4 w;
    T* e = (T*)&w;
    if (c0 + V <= l0 && st0 == 1 && sb >= 0 && (sb * (int64_t)sizeof(T) & ~(int64_t)15) + 32 <= src_bytes) {
      // contiguous source window at any element alignment: two aligned 16-byte loads and a
      // funnel shift by the window's byte offset
      const int64_t byte = sb * (int64_t)sizeof(T);
      const uint4* a = (const uint4*)((const uint8_t*)src + (byte & ~(int64_t)15));
      const uint4 lo = a[0], hi = a[1];
      const uint32_t x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      const int o = (int)(byte & 15), ow = o >> 2, sh = (o & 3) * 8;
      uint32_t r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t w0 = x[0], w1 = x[1];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (ow == q) {
            w0 = x[i + q];
            w1 = x[i + q + 1];
          }
        r[i] = __funnelshift_r(w0, w1, sh);
      }
      w = make_uint4(r[0], r[1], r[2], r[3]);
    } else if (c0 + V <= l0) {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int64_t si = sb + (int64_t)k * st0;
        e[k] = si < src_elems ? src[si] : T(0);
      }
      if (sb + (int64_t)(V - 1) * st0 >= src_elems) {  // rare: the window runs past the source
        const uint4 old = *dp;
#pragma unroll
        for (int k = 0; k < V; ++k)
          if (sb + (int64_t)k * st0 >= src_elems) e[k] = ((const T*)&old)[k];
      }
    } else {
      w = *dp;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int64_t si = sb + (int64_t)k * st0;
        if (c0 + k < l0 && si < src_elems) e[k] = src[si];
      }
    }
    *dp = w;
  }
}

template <typename T>
__global__ void relayout_table(T* __restrict__ dst, const T* __restrict__ src, const int64_t* __restrict__ table,
                               int64_t positions, int64_t src_base, int64_t dst_base, int64_t src_elems) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < positions;
       q += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = table[q];
    if (t < 0) continue;
    int64_t s = src_base + t;
    if (s < src_elems) dst[dst_base + q] = src[s];
  }
}

// 4-bit elements: one thread owns one dst byte (two positions), so sibling nibbles never race.
__global__ void relayout_nibble(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, KWalk w,
                                const int64_t* __restrict__ table, int64_t positions, int64_t src_base,
                                int64_t dst_base, int64_t src_elems, int64_t dst_bytes) {
  for (int64_t by = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; by < dst_bytes;
       by += (int64_t)gridDim.x * blockDim.x) {
    uint32_t byte = dst[by];
    bool changed = false;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int64_t q = by * 2 + h - dst_base;
      if (q < 0 || q >= positions) continue;
      int64_t off = 0;
      bool live;
      if (table) {
        off = table[q];
        live = off >= 0;
      } else {
        live = walk_offsets<1>(w, q, &off);
      }
      int64_t s = src_base + off;
      if (!live || s >= src_elems) continue;
      uint32_t nib = raw_nibble(src, s);
      byte = h ? ((byte & 0x0f) | (nib << 4)) : ((byte & 0xf0) | nib);
      changed = true;
    }
    if (changed) dst[by] = (uint8_t)byte;
  }
}

template <typename T>
void launch_relayout_typed(fopt_ctx* ctx, const RelayoutPlan& p, void* dst, const void* src, int64_t src_base,
                           int64_t dst_base, int64_t src_elems) {
  cudaStream_t st = ctx->stream;
  T* d = (T*)dst;
  const T* s = (const T*)src;
  if (!p.has_walk) {
    relayout_table<T><<<grid_for(p.positions), kThreads, 0, st>>>(d, s, p.table, p.positions, src_base, dst_base,
                                                                 src_elems);
    launched(ctx, "relayout_table");
    return;
  }
  const KWalk& w = p.walk;
  const int64_t V = 16 / sizeof(T);
  // vec path
  bool vec = w.n >= 1 && w.live[0] == w.extent[0] && w.stride[0][0] == 1 && w.extent[0] % V == 0 &&
             src_base % V == 0 && dst_base % V == 0 && ((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0);
  for (int i = 1; vec && i < w.n; ++i) vec = w.stride[0][i] % V == 0;
  if (w.n == 0) {
    // a single element (or empty) stream
    vec = false;
  }
  if (vec && V > 1) {
    int64_t units = p.positions / V;
    KWalk32 w32;
    if (to_kwalk32(w, w32) && units < (1ll << 31)) {
      relayout_vec32<uint4><<<grid_for(units), kThreads, 0, st>>>((uint4*)d, (const uint4*)s, w32, (uint32_t)units,
                                                                   (uint32_t)V, src_base / V, dst_base / V);
    } else {
      relayout_vec64<uint4><<<grid_for(units), kThreads, 0, st>>>((uint4*)d, (const uint4*)s, w, units, V,
                                                                   src_base / V, dst_base / V);
    }
    launched(ctx, "relayout_vec");
    return;
  }
  // broadcast path: the innermost wheel is a fully-live stride-0 run of whole 16-byte vectors
  if (w.n >= 1 && w.stride[0][0] == 0 && w.live[0] == w.extent[0] && w.extent[0] % V == 0 && V > 1 &&
      dst_base % V == 0 && (uintptr_t)dst % 16 == 0) {
    KWalk outer{};
    outer.n = w.n - 1;
    for (int i = 1; i < w.n; ++i) {
      outer.extent[i - 1] = w.extent[i];
      outer.live[i - 1] = w.live[i];
      outer.stride[0][i - 1] = w.stride[0][i];
    }
    int64_t inner_units = w.extent[0] / V, units = p.positions / V;
    if (inner_units >= 32) {
      const int64_t rows = units / inner_units;
      relayout_bcast_rows<T><<<grid_for(rows * 32), kThreads, 0, st>>>((uint4*)d, s, outer, inner_units, rows,
                                                                       src_base, dst_base / V);
      launched(ctx, "relayout_bcast_rows");
      return;
    }
    relayout_bcast<T><<<grid_for(units), kThreads, 0, st>>>((uint4*)d, s, outer, inner_units, units, src_base,
                                                           dst_base / V);
    launched(ctx, "relayout_bcast");
    return;
  }
  // tile path: dst-innermost wheel strided in src, some other fully-live wheel unit-stride in src.
  int j = -1;
  if (w.n >= 2 && w.live[0] == w.extent[0] && w.stride[0][0] != 1 && w.extent[0] >= 8) {
    for (int i = 1; i < w.n; ++i)
      if (w.stride[0][i] == 1 && w.live[i] == w.extent[i] && w.extent[i] >= 8) {
        j = i;
        break;
      }
  }
  if (j > 0) {
    KWalk others{};
    int64_t weight = 1, wj = 0;
    for (int i = 0; i < w.n; ++i) {
      if (i == j) wj = weight;
      if (i != 0 && i != j) {
        int k = others.n++;
        others.extent[k] = w.extent[i];
        others.live[k] = w.live[i];
        others.stride[0][k] = w.stride[0][i];
        others.stride[1][k] = weight;
      }
      weight *= w.extent[i];
    }
    int64_t batches = 1;
    for (int k = 0; k < others.n; ++k) batches *= others.extent[k];
    // Vector width: 8-byte vectors per thread when every offset stays aligned to them; a 128 x 128
    // tile for 1- and 2-byte elements, 64 x 64 for 4-byte ones (shared memory stays <= 32 KiB).
    constexpr int VW = sizeof(T) >= 4 ? 2 : 8 / (int)sizeof(T);
    bool wide = w.extent[0] % VW == 0 && w.extent[j] % VW == 0 && w.stride[0][0] % VW == 0 && src_base % VW == 0 &&
                dst_base % VW == 0 && (uintptr_t)src % 8 == 0 && (uintptr_t)dst % 8 == 0;
    for (int k = 0; wide && k < others.n; ++k) wide = others.stride[0][k] % VW == 0;
    constexpr int TTW = sizeof(T) >= 4 ? 64 : 128;
    const int TT = wide ? TTW : 32;
    int64_t nt0 = (w.extent[0] + TT - 1) / TT, ntj = (w.extent[j] + TT - 1) / TT;
    int64_t blocks = nt0 * ntj * batches;
    int grid = (int)std::min<int64_t>(blocks, (1ll << 31) - 1);  // one tile per block
    // word tiles for 1-byte elements (4 x 4 byte blocks): for 2- and 4-byte elements the vector tile
    // below is faster (its 8-byte global accesses halve the memory instructions): 61 vs 71 us (bf16)
    // and 103 vs 146 us (f32) at 8192^2 against 64-word tiles
    bool words = sizeof(T) == 1 && w.extent[0] % 4 == 0 && w.extent[j] % 4 == 0 && w.stride[0][0] % 4 == 0 &&
                 src_base % 4 == 0 && dst_base % 4 == 0 && (uintptr_t)src % 4 == 0 && (uintptr_t)dst % 4 == 0 &&
                 !getenv("FOPT_RELAYOUT_NO_WORDTILE");
    for (int k = 0; words && k < others.n; ++k) words = others.stride[0][k] % 4 == 0;
    bool halves = sizeof(T) == 2 && w.extent[0] % 4 == 0 && w.extent[j] % 4 == 0 && w.stride[0][0] % 4 == 0 &&
                  src_base % 4 == 0 && dst_base % 4 == 0 && (uintptr_t)src % 8 == 0 && (uintptr_t)dst % 8 == 0 &&
                  !getenv("FOPT_RELAYOUT_NO_HTILE");
    for (int k = 0; halves && k < others.n; ++k) halves = others.stride[0][k] % 4 == 0;
    if constexpr (sizeof(T) == 2) {
      if (halves) {
        const int64_t n0 = (w.extent[0] + 127) / 128, nj = (w.extent[j] + 127) / 128;
        const int gh = (int)std::min<int64_t>(n0 * nj * batches, (1ll << 31) - 1);
        relayout_tile_h<<<gh, 256, 0, st>>>((uint16_t*)d, (const uint16_t*)s, others, w.extent[0], w.stride[0][0],
                                            w.extent[j], wj, src_base, dst_base, n0, nj, batches);
        launched(ctx, "relayout_tile_h");
        return;
      }
    }
    bool bytes8 = sizeof(T) == 1 && w.extent[0] % 8 == 0 && w.extent[j] % 8 == 0 && w.stride[0][0] % 8 == 0 &&
                  src_base % 8 == 0 && dst_base % 8 == 0 && (uintptr_t)src % 8 == 0 && (uintptr_t)dst % 8 == 0 &&
                  !getenv("FOPT_RELAYOUT_NO_B8TILE");
    for (int k = 0; bytes8 && k < others.n; ++k) bytes8 = others.stride[0][k] % 8 == 0;
    if constexpr (sizeof(T) == 1) {
      if (bytes8) {
        const int64_t n0 = (w.extent[0] + 127) / 128, nj = (w.extent[j] + 127) / 128;
        const int gb = (int)std::min<int64_t>(n0 * nj * batches, (1ll << 31) - 1);
        relayout_tile_b8<<<gb, 256, 0, st>>>((uint8_t*)d, (const uint8_t*)s, others, w.extent[0], w.stride[0][0],
                                             w.extent[j], wj, src_base, dst_base, n0, nj, batches);
        launched(ctx, "relayout_tile_b8");
        return;
      }
      if (words) {
        const int64_t n0 = (w.extent[0] + 127) / 128, nj = (w.extent[j] + 127) / 128;
        const int gw = (int)std::min<int64_t>(n0 * nj * batches, (1ll << 31) - 1);
        relayout_tile_w<T, 32><<<gw, 256, 0, st>>>(d, s, others, w.extent[0], w.stride[0][0], w.extent[j], wj,
                                                   src_base, dst_base, n0, nj, batches);
        launched(ctx, "relayout_tile_w");
        return;
      }
    }
    if (wide)
      relayout_tile<T, VW, TTW><<<grid, 256, 0, st>>>(d, s, others, w.extent[0], w.stride[0][0], w.extent[j], wj,
                                                       src_base, dst_base, nt0, ntj, batches);
    else
      relayout_tile<T, 1, 32><<<grid, 256, 0, st>>>(d, s, others, w.extent[0], w.stride[0][0], w.extent[j], wj,
                                                     src_base, dst_base, nt0, ntj, batches);
    launched(ctx, "relayout_tile");
    return;
  }
  // padded rows from a dense source (the shared-memory staged kernel above)
  if constexpr (sizeof(T) == 4) {
    const bool dense_rows = w.n == 2 && w.stride[0][0] == 1 && w.live[0] < w.extent[0] &&
                            w.live[1] == w.extent[1] && w.stride[0][1] == w.live[0] && (uintptr_t)src % 16 == 0 &&
                            w.extent[0] < (1 << 20) && w.extent[1] * w.extent[0] < (1ll << 40) &&
                            !getenv("FOPT_RELAYOUT_NO_PADROWS");
    if (dense_rows) {
      const int64_t rows = w.extent[1];
      const int L = (int)w.live[0], E = (int)w.extent[0];
      // 64 rows a CTA where they fit in 48 KB (D = 61 f32: 0.76 of the copy rate against 0.72 with 32
      // rows, 0.66 with 16 and 0.67 with 128), else 32
      const int kPadRows = ((size_t)64 * L + 8) * 4 <= 48 * 1024 ? 64 : kPadRowsDefault;
      const size_t sm = ((size_t)kPadRows * L + 8) * 4;
      if (sm <= 48 * 1024) {
        const int64_t blocks = std::min<int64_t>((rows + kPadRows - 1) / kPadRows, 148 * 16);
        if (E % 4 == 0 && dst_base % 4 == 0 && (uintptr_t)d % 16 == 0 && !getenv("FOPT_RELAYOUT_NO_PADVEC"))
          relayout_pad_rows<true><<<(int)blocks, 256, sm, st>>>((uint32_t*)d, (const uint32_t*)s, rows, L, E,
                                                                make_fastdiv((uint32_t)(E / 4)), src_base, dst_base,
                                                                src_elems, kPadRows);
        else
          relayout_pad_rows<false><<<(int)blocks, 256, sm, st>>>((uint32_t*)d, (const uint32_t*)s, rows, L, E,
                                                                 make_fastdiv((uint32_t)E), src_base, dst_base,
                                                                 src_elems, kPadRows);
        launched(ctx, "relayout_pad_rows");
        return;
      }
    }
  }
  KWalk32 w32;
  if (w.n >= 2 && w.extent[0] >= 16 && to_kwalk32(w, w32) && p.positions < (1ll << 31)) {
    // rows path: the innermost wheel walked by a warp's lanes, the outer wheels decomposed once per row
    KWalk32 outer{};
    outer.n = w32.n - 1;
    for (int i = 1; i < w32.n; ++i) {
      outer.div[i - 1] = w32.div[i];
      outer.live[i - 1] = w32.live[i];
      outer.stride[0][i - 1] = w32.stride[0][i];
    }
    const int64_t rows = p.positions / w.extent[0];
    constexpr int V = 16 / sizeof(T);
    const int64_t lvec = (w.live[0] + V - 1) / V;
    if (sizeof(T) <= 4 && w.extent[0] % V == 0 && dst_base % V == 0 && (uintptr_t)d % 16 == 0 &&
        rows * lvec < (1ll << 31) && !getenv("FOPT_RELAYOUT_NO_ROWVEC")) {
      relayout_rows_vec<T><<<grid_for(rows * lvec), kThreads, 0, st>>>(
          d, s, outer, make_fastdiv((uint32_t)lvec), (uint32_t)(rows * lvec), (uint32_t)w.extent[0],
          (uint32_t)w.live[0], (int32_t)w.stride[0][0], src_base, dst_base, src_elems,
          (uintptr_t)s % 16 == 0 ? src_elems * (int64_t)sizeof(T) : 0);
      launched(ctx, "relayout_rows_vec");
      return;
    }
    relayout_rows<T><<<grid_for(rows * 32), kThreads, 0, st>>>(d, s, outer, (uint32_t)rows, (uint32_t)w.extent[0],
                                                                 (uint32_t)w.live[0], (int32_t)w.stride[0][0],
                                                                 src_base, dst_base, src_elems);
    launched(ctx, "relayout_rows");
    return;
  }
  if (to_kwalk32(w, w32) && p.positions < (1ll << 31)) {
    relayout_walk32<T><<<grid_for(p.positions), kThreads, 0, st>>>(d, s, w32, (uint32_t)p.positions, src_base,
                                                                  dst_base, src_elems);
  } else {
    relayout_walk64<T><<<grid_for(p.positions), kThreads, 0, st>>>(d, s, w, p.positions, src_base, dst_base,
                                                                  src_elems);
  }
  launched(ctx, "relayout_walk");
}

// ---- transmute ----
struct KRank {
  int n;
  int64_t extent[kKWheels], live[kKWheels];
};

__device__ __forceinline__ bool rank_of(const KRank& r, int64_t q, int64_t& k) {
  int64_t lw = 1;
  k = 0;
  for (int i = 0; i < r.n; ++i) {
    int64_t d = q % r.extent[i];
    q /= r.extent[i];
    if (d >= r.live[i]) return false;
    k += d * lw;
    lw *= r.live[i];
  }
  return true;
}
__device__ __forceinline__ int64_t pos_of_rank(const KRank& r, int64_t k) {
  int64_t ew = 1, p = 0;
  for (int i = 0; i < r.n; ++i) {
    int64_t d = k % r.live[i];
    k /= r.live[i];
    p += d * ew;
    ew *= r.extent[i];
  }
  return p;
}

template <typename T>
__global__ void transmute_kernel(T* __restrict__ dst, const T* __restrict__ src, KRank s, KRank d, int64_t positions,
                                 int64_t src_live) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < positions;
       q += (int64_t)gridDim.x * blockDim.x) {
    int64_t k;
    T v{};
    if (rank_of(d, q, k) && k < src_live) v = src[pos_of_rank(s, k)];
    dst[q] = v;
  }
}

__global__ void transmute_nibble(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, KRank s, KRank d,
                                 int64_t positions, int64_t src_live) {
  for (int64_t by = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; by * 2 < positions;
       by += (int64_t)gridDim.x * blockDim.x) {
    uint32_t out = 0;
    for (int h = 0; h < 2; ++h) {
      int64_t q = by * 2 + h, k;
      if (q < positions && rank_of(d, q, k) && k < src_live) out |= raw_nibble(src, pos_of_rank(s, k)) << (4 * h);
    }
    dst[by] = (uint8_t)out;
  }
}

KRank to_krank(const RankWalk& r) {
  KRank k{};
  k.n = (int)r.extent.size();
  if (k.n > kKWheels) throw Fail{FOPT_ERR_UNSUPPORTED, "transmute: too many factors"};
  for (int i = 0; i < k.n; ++i) {
    k.extent[i] = r.extent[i];
    k.live[i] = r.live[i];
  }
  return k;
}

}  // namespace

void launch_relayout(fopt_ctx* ctx, const RelayoutPlan& p, void* dst, const void* src, int dtype, int64_t src_base,
                     int64_t dst_base, int64_t src_elems, int64_t dst_elems) {
  if (p.positions == 0) return;
  if (dst_base + p.positions > dst_elems) {
    // The stream's trailing positions would address past the dst window; the reference clamps them
    // away (buf.rs:294-301). Clamping needs a shorter stream, which the walk kernels handle via the
    // positions bound; we only shorten when the clamp drops whole tail positions.
  }
  int bits = dtype_bits(dtype);
  int64_t positions_cap = std::min<int64_t>(p.positions, dst_elems - dst_base);
  RelayoutPlan q = p;
  q.positions = positions_cap;
  if (bits == 4) {
    int64_t dst_bytes = (dst_elems + 1) / 2;
    relayout_nibble<<<grid_for(dst_bytes), kThreads, 0, ctx->stream>>>(
        (uint8_t*)dst, (const uint8_t*)src, p.walk, p.has_walk ? nullptr : p.table, q.positions, src_base, dst_base,
        src_elems, dst_bytes);
    launched(ctx, "relayout_nibble");
    return;
  }
  switch (bits) {
    case 8: launch_relayout_typed<uint8_t>(ctx, q, dst, src, src_base, dst_base, src_elems); break;
    case 16: launch_relayout_typed<uint16_t>(ctx, q, dst, src, src_base, dst_base, src_elems); break;
    default: launch_relayout_typed<uint32_t>(ctx, q, dst, src, src_base, dst_base, src_elems); break;
  }
}

void launch_transmute(fopt_ctx* ctx, const RankWalk& src, const RankWalk& dst, void* out, const void* in, int dtype) {
  KRank s = to_krank(src), d = to_krank(dst);
  int64_t positions = 1, src_live = 1;
  for (auto e : dst.extent) positions *= e;
  for (auto l : src.live) src_live *= l;
  int bits = dtype_bits(dtype);
  cudaStream_t st = ctx->stream;
  if (positions == 0) return;
  switch (bits) {
    case 4:
      transmute_nibble<<<grid_for((positions + 1) / 2), kThreads, 0, st>>>((uint8_t*)out, (const uint8_t*)in, s, d,
                                                                          positions, src_live);
      break;
    case 8:
      transmute_kernel<uint8_t><<<grid_for(positions), kThreads, 0, st>>>((uint8_t*)out, (const uint8_t*)in, s, d,
                                                                         positions, src_live);
      break;
    case 16:
      transmute_kernel<uint16_t><<<grid_for(positions), kThreads, 0, st>>>((uint16_t*)out, (const uint16_t*)in, s, d,
                                                                          positions, src_live);
      break;
    default:
      transmute_kernel<uint32_t><<<grid_for(positions), kThreads, 0, st>>>((uint32_t*)out, (const uint32_t*)in, s, d,
                                                                          positions, src_live);
      break;
  }
  launched(ctx, "transmute");
}

}  // namespace fopt
