// Streaming kernels of the adapter phase on sm_100a: persistent CTAs, one producer warp
// that moves each tile of TV vectors into a shared-memory ring (1-D bulk copies with
// mbarrier transaction counts for contiguous tiles, 16-byte cp.async chunks tracked on the
// same mbarrier for strided or padded rows), and consumer warps that run the math on the
// staged tile while the next tiles are in flight.
//
//   k_draw_zca     Zc_A draws of every module, materialised in torch's launch layout
//   k_sperturb     z = eps * (Zc_A Q^T | Zc_B V^T), pos/neg, Kalman partial sums
//   k_sgram        fp64 Gram of the momentum (plain, or after the Kalman update, which it
//                  also writes back to mu/var)
//   k_sapply       param -= eta * X with X = mu Pm (Newton-Schulz apply)
//   k_sqr_apply    V = W R^-1 in fp64 (power-iteration CholeskyQR) and [V_hi | V_lo]^T
//
// Tiles: a segment (MatD::segv vectors of one matrix) is cut into tiles of TV vectors; CTA
// b takes segments b, b + grid, ... . Perturb / apply / QR apply hand consecutive tiles to
// four consumer teams of two warps (a 4 x 8 register block per thread covers a whole tile
// per team); the Gram uses all eight consumer warps on one tile. Every wait is bounded
// (mbar_wait), and a consumer verdict is agreed with bar.red before any barrier that
// depends on it, so a timeout ends the kernel instead of hanging it.
#pragma once

#include <type_traits>

#include "dsmz_kernels.cuh"
#include "dsmz_ptx.cuh"

namespace dsmz {
namespace sk {

constexpr int kCW = 8;                   // consumer warps
constexpr int kCT = 32 * kCW;            // consumer threads
constexpr int kST = kCT + 32;            // + producer warp 0
// Team kernels and the QR apply: two producer warps (0 and 1) take alternate tiles. A TMA
// issue costs a producer a few hundred cycles while the consumers keep the memory
// instruction queue busy, and a tile needs up to five of them.
constexpr int kProd = 2;
constexpr int kSTP = kCT + 32 * kProd;
constexpr int kTeams = 4;                // perturb / apply / QR apply
// Tile i goes to team i % kTeams and ring stage i % S. With S a multiple of kTeams each
// stage only ever holds one team's tiles, so the phase a team waits on directly follows the
// phase it consumed itself there (a stage two phases behind would alias on the phase
// parity). The team kernels' layouts round S down to a multiple of kTeams.
constexpr int kTT = kCT / kTeams;        // threads per team (two warps)
// QR apply: four groups of four consumer warps take tiles i % kQrGroups (four consumer
// warps per scheduler, to hide the fp64 MMA and shared-memory latencies of its short tiles).
constexpr int kQrGroups = 4;
constexpr int kQrGroupWarps = 4;
constexpr int kQrCT = 32 * kQrGroups * kQrGroupWarps;   // consumer threads
constexpr int kQrThreads = kQrCT + 32 * kProd;
constexpr int kBarAll = 1;               // named barrier: all consumer threads (one role)
// Role-split fp64 Gram: producer warp, prep warps, MMA warps.
constexpr int kPrepWarps = 6, kMmaWarps = 8;
constexpr int kSTG = 32 * (1 + kPrepWarps + kMmaWarps);
constexpr int kBarTeam0 = 2;             // named barriers 2..5: one per team

// Vectors per tile: ~2048 elements, a multiple of 8 (16-byte bf16 rows of side-B tiles).
__host__ __device__ inline int stream_tv(int r) {
  int tv = (2048 / (r < 1 ? 1 : r)) & ~7;
  return tv < 8 ? 8 : (tv > 512 ? 512 : tv);
}
__host__ __device__ inline int al16(int b) { return (b + 15) & ~15; }
__host__ __device__ inline int al128(int b) { return (b + 127) & ~127; }
__host__ __device__ inline int al1024(int b) { return (b + 1023) & ~1023; }

// Swizzled row image: rows of a tile (TV vectors, each of w fp32 components) stored as
// ceil(w / 32) boxes of TV rows x 128 bytes with the 128-byte swizzle of a 2-D TMA copy
// (16-byte chunk c of row v at chunk c ^ (v % 8)). A box is 1024-byte aligned (TV % 8 == 0).
// Four consecutive components of a row are one aligned 16-byte chunk, and eight rows read
// at the same column fall into eight different chunks.
__host__ __device__ inline int swz_boxes(int w) { return (w + 31) / 32; }
__host__ __device__ inline int swz_bytes(int w, int TV) { return swz_boxes(w) * TV * 128; }
__host__ __device__ inline int swz_off(int v, int a, int TV) {
  return (a >> 5) * TV * 128 + v * 128 + ((((a >> 2) & 7) ^ (v & 7)) << 4) + (a & 3) * 4;
}

// One input array of a tile. Side 0: vector v is the row at v*ld (components k*cs);
// side 1: vector v is the column at v*cs (components k*ld). In shared memory, side 0
// keeps vector v at dst + v*pitch and side 1 component row k at dst + k*pitch.
struct Src {
  const char* base;
  int64_t ld, cs;
  int32_t es, side, r, swz;   // swz: the stage holds the swizzled row image (side-0 fp32 rows)
  const CUtensorMap* map;     // side 1: tile-box tensor map (one TMA copy); swz: 32-column
                              // swizzled boxes (one TMA copy per box)
};

// Array `which` (0 param, 1 mu, 2 var, 3 z) of matrix M, with its tensor map when M has them.
__device__ __forceinline__ Src make_src(const void* base, const MatD& M, int es, const Tables& tb, int which) {
  Src a;
  a.base = reinterpret_cast<const char*>(base);
  a.ld = M.ld; a.cs = M.cs; a.es = es; a.side = M.side; a.r = static_cast<int>(M.r); a.swz = 0;
  a.map = (M.side == 1 && M.tmap >= 0 && tb.smaps != nullptr) ? tb.smaps + M.tmap + which : nullptr;
  return a;
}

// How one array of a tile reaches shared memory: one bulk copy when the tile image is a
// contiguous run of global memory (side-0 rows of exactly r elements, unpadded); 16-byte
// cp.async chunks spread over the producer lanes when every row is 16-byte aligned (strided
// or padded rows: many short rows would starve the bulk engine); element copies otherwise.
enum { kCopyBulk = 0, kCopy16 = 1, kCopyPlain = 2, kCopyTensor = 3, kCopySwzTma = 4, kCopySwzPlain = 5 };

__device__ __forceinline__ int copy_mode(const Src& a, int64_t s0, int nv, int pitch, const void* dst) {
  // swizzled row image: a TMA copy per 32-column box (zero fill past the rows and columns),
  // or element copies into the same image
  if (a.swz) return (a.map != nullptr && (reinterpret_cast<uintptr_t>(dst) & 1023) == 0) ? kCopySwzTma : kCopySwzPlain;
  // side 1 with a tensor map: one 2-D TMA box (TV x r, dense rows of TV, zero fill past
  // the matrix end); x = s0 is a multiple of the tile width (16-byte aligned)
  if (a.map != nullptr && ((reinterpret_cast<uintptr_t>(dst) & 127) == 0)) return kCopyTensor;
  if (a.cs != 1 || (reinterpret_cast<uintptr_t>(a.base) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15) ||
      (pitch & 15))
    return kCopyPlain;
  const int64_t ldb = a.ld * a.es;
  if (a.side == 0) {
    const int rowb = a.r * a.es;
    if (rowb & 15) return kCopyPlain;
    if (a.ld == a.r && pitch == rowb) return kCopyBulk;
    return (ldb & 15) ? kCopyPlain : kCopy16;
  }
  if ((ldb & 15) || ((s0 * a.es) & 15) || ((static_cast<int64_t>(nv) * a.es) & 15)) return kCopyPlain;
  return kCopy16;
}

// 16-byte chunks of the tile's rows, lane-parallel: side 0 has nv rows of r*es bytes,
// side 1 has r rows of nv*es bytes. When the chunks per row divide 32, each lane keeps one
// chunk column and walks the rows by pointer increments (no per-chunk division).
__device__ __forceinline__ void copy16_issue(const Src& a, int64_t s0, int nv, char* dst, int pitch, int lane) {
  const int nrow = (a.side == 0) ? nv : a.r;
  const int cpr = ((a.side == 0) ? a.r : nv) * a.es / 16;      // chunks per row
  const int64_t srow = a.ld * a.es;                              // bytes between source rows
  const char* src0 = (a.side == 0) ? a.base + s0 * srow : a.base + s0 * a.es;
  if (cpr <= 32 && (32 % cpr) == 0) {
    const int rstep = 32 / cpr;
    int row = lane / cpr;
    const int c = lane - row * cpr;
    const char* sp = src0 + row * srow + c * 16;
    char* dp = dst + row * pitch + c * 16;
    const int64_t sstep = rstep * srow;
    const int dstep = rstep * pitch;
    for (; row < nrow; row += rstep, sp += sstep, dp += dstep) cp16(dp, sp);
    return;
  }
  const int n = nrow * cpr;
  for (int e = lane; e < n; e += 32) {
    const int row = e / cpr, c = e - row * cpr;
    cp16(dst + row * pitch + c * 16, src0 + row * srow + c * 16);
  }
}

// Element-by-element copy for layouts neither engine can take (strides, odd sizes).
__device__ __forceinline__ void plain_copy(const Src& a, int64_t s0, int nv, char* dst, int pitch, int lane) {
  const int n = nv * a.r;
  for (int e = lane; e < n; e += 32) {
    int v, k;
    if (a.side == 0) { v = e / a.r; k = e - v * a.r; } else { k = e / nv; v = e - k * nv; }
    const int64_t off = (a.side == 0) ? ((s0 + v) * a.ld + k * a.cs) : (k * a.ld + (s0 + v) * a.cs);
    char* d = dst + (a.side == 0 ? v * pitch + k * a.es : k * pitch + v * a.es);
    if (a.es == 4) *reinterpret_cast<uint32_t*>(d) = *reinterpret_cast<const uint32_t*>(a.base + off * 4);
    else *reinterpret_cast<uint16_t*>(d) = *reinterpret_cast<const uint16_t*>(a.base + off * 2);
  }
}

// Element copies of side-0 fp32 rows into the swizzled row image (pitch = bytes per box,
// TV x 128): every column of the boxes is written, zeros past the row width r.
__device__ __forceinline__ void swz_plain_copy(const Src& a, int64_t s0, int nv, char* dst, int pitch, int lane) {
  const int TV = pitch / 128;
  const int w = 32 * swz_boxes(a.r);
  const int n = nv * w;
  for (int e = lane; e < n; e += 32) {
    const int v = e / w, k = e - v * w;
    const float x = (k < a.r) ? *reinterpret_cast<const float*>(a.base + ((s0 + v) * a.ld + k * a.cs) * 4) : 0.f;
    *reinterpret_cast<float*>(dst + swz_off(v, k, TV)) = x;
  }
}

// Fills one stage with up to NA arrays (null base: absent). The stage's `full` barrier
// expects 33 arrivals: lane 0's expect_tx (bulk bytes, after the element copies) and one
// cp.async-tracking arrival per lane. Called by all 32 producer lanes.
constexpr int kFullArrivals = 33;
template <int NA>
__device__ __forceinline__ void produce(const Src (&a)[NA], const int (&off)[NA], const int (&pitch)[NA],
                                        int64_t s0, int nv, char* stage, uint64_t* full, int lane, bool acquire) {
  int mode[NA];
  uint32_t tx = 0;
#pragma unroll
  for (int i = 0; i < NA; ++i) {
    mode[i] = -1;
    if (a[i].base == nullptr) continue;
    mode[i] = copy_mode(a[i], s0, nv, pitch[i], stage + off[i]);
    if (mode[i] == kCopyBulk) tx += static_cast<uint32_t>(nv) * a[i].r * a[i].es;
    else if (mode[i] == kCopyTensor) tx += static_cast<uint32_t>(pitch[i]) * a[i].r;   // the whole box
    else if (mode[i] == kCopySwzTma) tx += static_cast<uint32_t>(pitch[i]) * swz_boxes(a[i].r);   // whole boxes
    else if (mode[i] == kCopyPlain) plain_copy(a[i], s0, nv, stage + off[i], pitch[i], lane);
    else if (mode[i] == kCopySwzPlain) swz_plain_copy(a[i], s0, nv, stage + off[i], pitch[i], lane);
  }
  __syncwarp();
  if (lane == 0) mbar_expect_tx(full, tx);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NA; ++i) {
    if (mode[i] == kCopyBulk) {
      if (lane == 0)
        bulk_g2s(stage + off[i], a[i].base + s0 * a[i].ld * a[i].es, static_cast<uint32_t>(nv) * a[i].r * a[i].es,
                 full);
    } else if (mode[i] == kCopy16) {
      copy16_issue(a[i], s0, nv, stage + off[i], pitch[i], lane);
    } else if (mode[i] == kCopyTensor) {
      if (lane == 0) {
        if (acquire) tmap_acquire(a[i].map);       // once per matrix (maps are fixed per launch)
        tma_load_2d(stage + off[i], a[i].map, static_cast<int>(s0), 0, full);
      }
    } else if (mode[i] == kCopySwzTma) {
      if (lane == 0) {
        if (acquire) tmap_acquire(a[i].map);
        for (int b = 0; b < swz_boxes(a[i].r); ++b)
          tma_load_2d(stage + off[i] + b * pitch[i], a[i].map, 32 * b, static_cast<int>(s0), full);
      }
    }
  }
  cp16_arrive(full);
}

// Stage pitch of an unpadded tile image: side 0 rows of r elements, side 1 rows of TV.
__device__ __forceinline__ int side_pitch(int side, int r, int TV, int es) { return (side == 0 ? r : TV) * es; }

// Every consumer thread of a group of n threads passes `ok`; all get the AND.
__device__ __forceinline__ bool agree(int bar_id, int n, bool ok) {
  uint32_t all;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(all)
      : "r"(static_cast<uint32_t>(ok)), "r"(bar_id), "r"(n)
      : "memory");
  return all != 0;
}

// The CTA's tile sequence: chunk blockIdx.x of the global tile space, tiles
// [c*T/G, (c+1)*T/G) (T tiles, G CTAs), walked in matrix order. A segment is the run of
// the chunk's tiles inside one matrix (global index MatD::seg0 + c - MatD::chunk0).
struct TileIt {
  const MatD* mats; int nmats, TV;
  int t, t1;            // current global tile, end of the chunk
  int mi, seg;
  int64_t s0, nvec;     // first vector of the tile, vectors of the matrix
  bool fresh;           // the tile is the first of its segment
  __device__ void init(const MatD* m, int n, int tv) {
    mats = m; nmats = n; TV = tv;
    const int64_t T = static_cast<int64_t>(m[n - 1].tile0) + m[n - 1].ntile;
    const int64_t G = gridDim.x, c = blockIdx.x;
    t = static_cast<int>((c * T) / G);
    t1 = static_cast<int>(((c + 1) * T) / G);
  }
  __device__ void load() {
    const MatD& M = mats[mi];
    nvec = M.nvec;
    seg = M.seg0 + static_cast<int>(blockIdx.x) - M.chunk0;
  }
  __device__ bool start_seg() {
    if (t >= t1) return false;
    mi = find_owner(mats, nmats, t, [](const MatD& m) { return m.tile0; });
    load();
    s0 = static_cast<int64_t>(t - mats[mi].tile0) * TV;
    fresh = true;
    return true;
  }
  __device__ int nv() const { return static_cast<int>(min(static_cast<int64_t>(TV), nvec - s0)); }
  // advance; returns 1 on a new tile of the same segment, 2 on a new segment, 0 at the end
  __device__ int next() {
    if (++t >= t1) return 0;
    s0 += TV;
    fresh = s0 >= nvec;
    if (!fresh) return 1;
    ++mi;
    s0 = 0;
    load();
    return 2;
  }
};

// (d0, d1) += (a, a) * (b0, b1) as one packed fp32x2 FMA: each component rounds exactly as
// fmaf, and one instruction issues both, which leaves the row products' issue slots to
// their shared-memory operand loads.
__device__ __forceinline__ void fma2_bcast(float& d0, float& d1, float a, float b0, float b1) {
  asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %2};\n mov.b64 rb, {%3, %4};\n mov.b64 rc, {%0, %1};\n"
      " fma.rn.f32x2 rc, ra, rb, rc;\n mov.b64 {%0, %1}, rc;\n}"
      : "+f"(d0), "+f"(d1)
      : "f"(a), "f"(b0), "f"(b1));
}

// out(v, c) = sum_a X(v, a) P[a*pld + c] with X(v, a) = X[v*vs + a*as] (as = 1 when AS1).
// A thread block owns vectors {vb + i*Q} (Q = ceil(nv/4)) and columns {4cb..4cb+3,
// pld/2 + 4cb..+3}: the four vectors a warp reads per step are consecutive rows (distinct
// banks when vs = 4 mod 32, or vs = 1) and its eight column blocks one contiguous 128-byte
// run of a P row. pld % 8 == 0, P padded with zero columns to pld; rows up to 4Q - 1
// must be readable.
template <bool AS1, typename Sink>
__device__ __forceinline__ void mm_rows(const float* __restrict__ X, int vs, int as, const float* __restrict__ P,
                                        int pld, int nv, int K, int nc, int t, int nt, Sink sink) {
  const int cbs = pld >> 3, half = pld >> 1;
  const int Q = (nv + 3) >> 2;
  const int ast = AS1 ? 1 : as;
  for (int blk = t; blk < Q * cbs; blk += nt) {
    const int vb = blk / cbs, cb = blk - vb * cbs;
    const int c0 = cb * 4;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    const float* x0 = X + vb * vs;
    const float* x1 = x0 + Q * vs;
    const float* x2 = x1 + Q * vs;
    const float* x3 = x2 + Q * vs;
    const float* pr = P + c0;
#pragma unroll 4
    for (int a = 0; a < K; ++a) {
      const float4 p0 = *reinterpret_cast<const float4*>(pr);
      const float4 p1 = *reinterpret_cast<const float4*>(pr + half);
      pr += pld;
      const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      const float xv[4] = {x0[a * ast], x1[a * ast], x2[a * ast], x3[a * ast]};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; j += 2) fma2_bcast(acc[i][j], acc[i][j + 1], xv[i], pv[j], pv[j + 1]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = vb + i * Q;
      if (v >= nv) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = (j < 4) ? c0 + j : half + c0 + j - 4;
        if (c < nc) sink(v, c, acc[i][j]);
      }
    }
  }
}

// mm_rows with X the swizzled row image of the tile (boxes of TV rows, swz_off): a thread
// block's four vectors read four consecutive components as one 16-byte chunk each (eight
// distinct chunks for the rows a warp touches: no bank conflicts). K4 = K rounded up to 4;
// the image's columns K .. K4-1 are zero and P has K4 rows (zero past K).
template <typename Sink>
__device__ __forceinline__ void mm_rows_sw(const unsigned char* __restrict__ X, int TV, const float* __restrict__ P,
                                           int pld, int nv, int K4, int nc, int t, int nt, Sink sink) {
  const int cbs = pld >> 3, half = pld >> 1;
  const int Q = (nv + 3) >> 2;
  const int boxb = TV * 128;
  for (int blk = t; blk < Q * cbs; blk += nt) {
    const int vb = blk / cbs, cb = blk - vb * cbs;
    const int c0 = cb * 4;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    const unsigned char* xr[4];
    int sw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = vb + i * Q;
      xr[i] = X + v * 128;
      sw[i] = v & 7;
    }
    const float* pr = P + c0;
    for (int a4 = 0; a4 < K4; a4 += 4) {
      const int boff = (a4 >> 5) * boxb, ch = (a4 >> 2) & 7;
      float4 x4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x4[i] = *reinterpret_cast<const float4*>(xr[i] + boff + ((ch ^ sw[i]) << 4));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 p0 = *reinterpret_cast<const float4*>(pr);
        const float4 p1 = *reinterpret_cast<const float4*>(pr + half);
        pr += pld;
        const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = u == 0 ? x4[i].x : u == 1 ? x4[i].y : u == 2 ? x4[i].z : x4[i].w;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 8; j += 2) fma2_bcast(acc[i][j], acc[i][j + 1], xv[i], pv[j], pv[j + 1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = vb + i * Q;
      if (v >= nv) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = (j < 4) ? c0 + j : half + c0 + j - 4;
        if (c < nc) sink(v, c, acc[i][j]);
      }
    }
  }
}

// fp64 variant: P is r x pld doubles; columns {2cb, 2cb+1} + g*pld/4 for g < 4 (each
// thread's double2 loads of a warp cover contiguous 256-byte runs). pld % 8 == 0.
template <typename Sink>
__device__ __forceinline__ void mm_rows_f64(const float* __restrict__ X, int vs, const double* __restrict__ P,
                                            int pld, int nv, int K, int nc, int t, int nt, Sink sink) {
  const int cbs = pld >> 3, quarter = pld >> 2;
  const int Q = (nv + 3) >> 2;
  for (int blk = t; blk < Q * cbs; blk += nt) {
    const int vb = blk / cbs, cb = blk - vb * cbs;
    const int c0 = cb * 2;
    double acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
    const float* x0 = X + vb * vs;
    const float* x1 = x0 + Q * vs;
    const float* x2 = x1 + Q * vs;
    const float* x3 = x2 + Q * vs;
    const double* pr = P + c0;
#pragma unroll 2
    for (int a = 0; a < K; ++a) {
      double pv[8];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const double2 tt = *reinterpret_cast<const double2*>(pr + g * quarter);
        pv[2 * g] = tt.x;
        pv[2 * g + 1] = tt.y;
      }
      pr += pld;
      const double xv[4] = {static_cast<double>(x0[a]), static_cast<double>(x1[a]), static_cast<double>(x2[a]),
                            static_cast<double>(x3[a])};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fma(xv[i], pv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = vb + i * Q;
      if (v >= nv) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = (j >> 1) * quarter + c0 + (j & 1);
        if (c < nc) sink(v, c, acc[i][j]);
      }
    }
  }
}

// Elements e = e0, e0 + step, ... of an nv x r tile in global memory order, as (vector v,
// component k), advanced without division. Side 0 walks each vector's components, side 1
// each component row along the vectors.
template <int SIDE>
struct Walk {
  int v, k, dv, dk, lim;
  __device__ __forceinline__ Walk(int e0, int step, int r, int nv) {
    if (SIDE == 0) { v = e0 / r; k = e0 - v * r; dv = step / r; dk = step - dv * r; lim = r; }
    else { k = e0 / nv; v = e0 - k * nv; dk = step / nv; dv = step - dk * nv; lim = nv; }
  }
  __device__ __forceinline__ void next() {
    if (SIDE == 0) { k += dk; v += dv; if (k >= lim) { k -= lim; ++v; } }
    else { v += dv; k += dk; if (v >= lim) { v -= lim; ++k; } }
  }
  // element offset from the tile's first element in global memory (32-bit) and in the
  // unpadded shared-memory image
  __device__ __forceinline__ int goff(int ld, int cs) const { return SIDE == 0 ? v * ld + k * cs : k * ld + v * cs; }
  __device__ __forceinline__ int soff(int r, int TV) const { return SIDE == 0 ? v * r + k : k * TV + v; }
};

template <int FES>
__device__ __forceinline__ void st_fac(void* p, int i, float x) {
  if (FES == 2) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}
// Stores four consecutive copy-dtype elements (8 bytes of bf16 or 16 of fp32, aligned).
template <int FES>
__device__ __forceinline__ void st_fac4(void* p, int i, float4 x) {
  if (FES == 2) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y), b = __floats2bfloat162_rn(x.z, x.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = u;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = x;
  }
}
__device__ __forceinline__ bool aligned_to(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) & static_cast<uintptr_t>(bytes - 1)) == 0;
}
// Steps of four consecutive elements of a tile along its contiguous direction (component
// k on side 0, vector v on side 1): (v, k) of the step's first element.
template <int SIDE>
struct Walk4 {
  Walk<SIDE> w;
  __device__ __forceinline__ Walk4(int e0, int step, int r, int nv)
      : w(e0, step, SIDE == 0 ? r / 4 : r, SIDE == 0 ? nv : nv / 4) {}
  __device__ __forceinline__ int v() const { return SIDE == 0 ? w.v : 4 * w.v; }
  __device__ __forceinline__ int k() const { return SIDE == 0 ? 4 * w.k : w.k; }
  __device__ __forceinline__ void next() { w.next(); }
};
// Element pointer of the tile's first element (vector s0, component 0).
template <typename T>
__device__ __forceinline__ T* tile_ptr(T* base, const MatD& M, int64_t s0, int es) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(const_cast<typename std::remove_const<T>::type*>(base)) +
                              s0 * (M.side == 0 ? M.ld : M.cs) * es);
}

// =====================================================================================
// Layouts (host and device): stage ring and fixed buffers, byte offsets from a 128-byte
// aligned base. Every plan has one rank r (modules) or R (bases).
// =====================================================================================
struct Layout {
  int TV, S;             // vectors per tile, ring stages
  int stage_bytes;
  int off[4], pitch[4];  // per array in a stage
  int fixed0;            // first byte after the ring
  int o_c, o_z, o_x, o_red, o_tab, o_bar;
  int total;             // dynamic shared memory bytes (+128 alignment slack)
  int r, pld, zp, rp, xp, nsb, ng;
};

// Perturb: p, mu, var (fp32, unpadded) and the K operand rows (Zc_A rows of width RCA, or
// basis rows of width RC) as a swizzled row image (pitch[3]: bytes per box); the
// coefficient matrix with KW rounded up to 4 rows (zero rows past KW).
__host__ __device__ inline Layout perturb_layout(int r, int R, int RC, int RCA, int budget, int TV) {
  Layout L{};
  L.r = r;
  L.TV = TV;
  const int KW = RC > RCA ? RC : RCA;
  const int K4 = (KW + 3) & ~3;
  int o = 0;
  L.off[0] = o; L.pitch[0] = r * 4;                                   o += al128(TV * r * 4);
  L.off[1] = o; L.pitch[1] = r * 4;                                   o += al128(TV * r * 4);
  L.off[2] = o; L.pitch[2] = r * 4;                                   o += al128(TV * r * 4);
  o = al1024(o);
  L.off[3] = o; L.pitch[3] = TV * 128;                                o += swz_bytes(KW, TV);
  L.stage_bytes = al1024(o);
  L.pld = pad8(R);
  L.zp = r + 1;
  const int fixed = al128(K4 * L.pld * 4) + kTeams * al128(TV * L.zp * 4) + al128(2 * kCW * 8 * 2) + 2048;
  int S = (budget - fixed) / L.stage_bytes;
  S = S > 8 ? 8 : S / kTeams * kTeams;
  L.S = S;
  L.fixed0 = S * L.stage_bytes;
  L.o_c = L.fixed0;
  L.o_z = L.o_c + al128(K4 * L.pld * 4);
  L.o_red = L.o_z + kTeams * al128(TV * L.zp * 4);
  L.o_bar = L.o_red + al128(2 * kCW * 8 * 2);
  L.total = L.o_bar + 2 * 8 * S + 1024 + 128;
  return L;
}

// Apply: p (fp32, unpadded) and mu (side 0: swizzled row image, pitch[1] bytes per box;
// side 1: dense rows of TV); the r x r apply matrix with r rounded up to 4 rows (zero rows
// past r).
__host__ __device__ inline Layout apply_layout(int r, int budget, int TV) {
  Layout L{};
  L.r = r;
  L.TV = TV;
  const int r4 = (r + 3) & ~3;
  const int mub = swz_bytes(r, TV) > TV * r * 4 ? swz_bytes(r, TV) : TV * r * 4;
  int o = 0;
  L.off[0] = o; L.pitch[0] = r * 4;                                     o += al128(TV * r * 4);
  o = al1024(o);
  L.off[1] = o; L.pitch[1] = TV * 128;                                  o += mub;
  L.stage_bytes = al1024(o);
  L.pld = pad8(r);
  L.zp = r + 1;
  const int fixed = al128(r4 * L.pld * 4) + kTeams * al128(TV * L.zp * 4) + 2048;
  int S = (budget - fixed) / L.stage_bytes;
  S = S > 8 ? 8 : S / kTeams * kTeams;
  L.S = S;
  L.fixed0 = S * L.stage_bytes;
  L.o_c = L.fixed0;
  L.o_z = L.o_c + al128(r4 * L.pld * 4);
  L.o_bar = L.o_z + kTeams * al128(TV * L.zp * 4);
  L.total = L.o_bar + 2 * 8 * S + 1024 + 128;
  return L;
}

// QR apply: W rows as a swizzled row image per stage (a multiple of kQrGroups stages, at most 8);
// fp64 R^{-1} zero-padded to rp x pld (rp = R rounded up to 8, pld = rp + 4: each half-warp's
// B fragment on distinct banks); two fp32 result tiles (TV x zp, zp = rp + 1) per group.
__host__ __device__ inline Layout qr_layout(int R, int budget, int TV) {
  Layout L{};
  L.r = R;
  L.TV = TV;
  const int rp = pad8(R);
  L.off[0] = 0; L.pitch[0] = TV * 128;
  L.stage_bytes = swz_bytes(R, TV);
  L.rp = rp;
  L.pld = rp + 4;
  L.zp = rp + 1;
  const int osz = al128(TV * L.zp * 4);
  const int fixed = al128(rp * L.pld * 8) + 2 * kQrGroups * osz + 2048;
  int S = (budget - fixed) / L.stage_bytes;
  S = S > 8 ? 8 : S - S % kQrGroups;               // each stage serves one consumer group
  L.S = S;
  L.fixed0 = S * L.stage_bytes;
  L.o_c = L.fixed0;
  L.o_z = L.o_c + al128(rp * L.pld * 8);
  L.o_bar = L.o_z + 2 * kQrGroups * osz;
  L.total = L.o_bar + 2 * 8 * S + 1024 + 128;
  return L;
}

__host__ __device__ inline Layout gram_layout(int r, int kalman, int budget, int TV) {
  Layout L{};
  L.r = r;
  L.TV = TV;
  int o = 0;
  L.off[0] = o; L.pitch[0] = r * 4; o += al128(TV * r * 4);
  L.off[1] = o; L.pitch[1] = kalman ? r * 4 : 0; o += al128(kalman ? TV * r * 4 : 0);
  L.off[2] = o; L.pitch[2] = kalman ? r * 4 : 0; o += al128(kalman ? TV * r * 4 : 0);
  L.stage_bytes = o;
  L.rp = pad8(r);
  L.xp = L.rp + 8;                 // side 0 rows of the fp64 tile
  L.zp = TV + 4;                   // side 1 rows
  const int xa = TV * L.xp, xb = L.rp * L.zp;
  const int xbytes = al128((xa > xb ? xa : xb) * 8);   // one buffer; two are kept
  const int fixed = 2 * xbytes + 1024 + 1024;
  int S = (budget - fixed) / L.stage_bytes;
  S = S > 8 ? 8 : S;
  L.S = S;
  L.fixed0 = S * L.stage_bytes;
  L.o_x = L.fixed0;
  L.o_red = L.o_x + 2 * xbytes;    // block table (<= 136 ints)
  L.o_bar = L.o_red + 1024;
  L.total = L.o_bar + 2 * 8 * S + 4 * 8 + 1024 + 128;
  return L;
}

__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

// Producer loop shared by every streaming kernel: NP producer warps (warps 0 .. NP-1) walk
// the CTA's tiles; warp p fills the tiles i with i % NP == p (every stage then has one
// producer: S is a multiple of NP). Waits for the stage to be free, then
// `fill(it, stage, full, lane, fresh)` issues the copies; fresh: the first tile of a
// matrix this warp fills (copy sources are rebuilt, tensor maps acquired).
template <int NP, typename Fill>
__device__ __forceinline__ void producer_loop(TileIt it, const Layout& L, unsigned char* smem, uint64_t* full,
                                              uint64_t* empty, int* err, Fill fill) {
  const int lane = threadIdx.x & 31, pw = static_cast<int>(threadIdx.x >> 5);
  int i = 0;
  int cur = -1;
  if (it.start_seg()) {
    while (true) {
      if (i % NP == pw) {
        const int s = i % L.S;
        if (i >= L.S) {
          const bool w = mbar_wait(empty + s, (static_cast<uint32_t>(i / L.S) & 1u) ^ 1u, err);
          if (!__all_sync(0xffffffffu, w)) break;
        }
        const bool fresh = it.mi != cur;
        cur = it.mi;
        fill(it, smem + s * L.stage_bytes, full + s, lane, fresh);
      }
      ++i;
      if (it.next() == 0) break;
    }
  }
  // the copies already issued land before the CTA can exit, whatever the consumers did
  if (lane == 0)
    for (int j = (i > L.S ? i - L.S : 0); j < i; ++j)
      if (j % NP == pw) mbar_drain(full + (j % L.S), static_cast<uint32_t>(j / L.S) & 1u);
}

__device__ __forceinline__ void init_bars(uint64_t* full, uint64_t* empty, int S, int empty_count) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(full + s, kFullArrivals); mbar_init(empty + s, empty_count); }
    mbar_init_fence();
  }
  __syncthreads();
}

// =====================================================================================
// Zc_A draws (controller.py:187-188) of every module, in torch's own launch layout: one
// thread per torch thread idx, curand_init(seed, idx, offset) and one curand_normal4 per
// grid-stride round, component c of round j -> element idx + threads*(4j + c). A draw no
// larger than its thread count only ever uses component 0 of round 0 (curand_normal,
// which returns the same first value of the Box-Muller pair).
// =====================================================================================
__global__ void __launch_bounds__(256) k_draw_zca(Tables tb, uint64_t seed, uint64_t base_off) {
  // grid-stride over the torch launch's blocks (256 of its threads each); the module index
  // only moves forward, so one search per CTA
  int mi = -1;
  for (int vb = static_cast<int>(blockIdx.x); vb < tb.ndblk; vb += static_cast<int>(gridDim.x)) {
    if (mi < 0) mi = find_owner(tb.mods, tb.nmods, vb, [](const ModD& d) { return d.dblk0; });
    while (mi + 1 < tb.nmods && tb.mods[mi + 1].dblk0 <= vb) ++mi;
    const ModD& D = tb.mods[mi];
    const int64_t idx = static_cast<int64_t>(vb - D.dblk0) * 256 + threadIdx.x;
    const int64_t thr = D.thrA;
    const int64_t n = D.d_out * D.rca;
    if (idx >= thr || idx >= n) continue;
    float* out = reinterpret_cast<float*>(tb.ws) + D.zca_off;
    curandStatePhilox4_32_10_t st;
    curand_init(seed, static_cast<unsigned long long>(idx), base_off + D.offA, &st);
    if (n <= thr) {
      out[idx] = curand_normal(&st);
      continue;
    }
    for (int64_t base = idx; base < n; base += 4 * thr) {
      const float4 g = curand_normal4(&st);
      out[base] = g.x;
      if (base + thr < n) out[base + thr] = g.y;
      if (base + 2 * thr < n) out[base + 2 * thr] = g.z;
      if (base + 3 * thr < n) out[base + 3 * thr] = g.w;
    }
  }
}

// =====================================================================================
// Consumer-side failure protocol of the team kernels: a team whose bounded wait failed is
// "dead" (agreed within the team); it stops waiting and processing but keeps walking the
// tile sequence, so every CTA-wide barrier (segment ends, matrix switches) is still met.
// A failed wait sets the error word, which makes every later wait of the CTA fail fast.
// =====================================================================================

// =====================================================================================
// Perturbation (controller.py:178-193, 241-248, 262-270; ds_mezo/kernels.py:290-368,
// 399-412). Side A: z[i,:] = eps * Zc_A[i,:] Q^T; side B: z[:,j] = eps * Zc_B V[j,:]^T.
// z, pos = copy(p + z), neg = copy(p - z) (p the fp32 master, the sum rounded to the copy
// dtype of FES bytes per element, as the reference's fp32 pos/neg are cast at export), and
// the per-segment Kalman partials (sum z * beta*mu, sum z*z * (beta^2 var + q)).
// =====================================================================================
template <int FES>
__global__ void __launch_bounds__(kSTP, 1) k_sperturb(Tables tb, Layout L, uint64_t seed, uint64_t base_off, float eps,
                                                     KalmanIn kin, GatherPeers gp, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + L.S;
  init_bars(full, empty, L.S, 2);
  TileIt it;
  it.init(tb.mats, tb.nmats, L.TV);
  const int warp = threadIdx.x >> 5;
  (void)seed; (void)base_off;

  if (warp < kProd) {
    Src a[4];                                   // the segment's copy sources, built at its first tile
    int pitch[4];
    producer_loop<kProd>(it, L, smem, full, empty, err, [&](const TileIt& t, unsigned char* stage, uint64_t* fb, int lane, bool fresh) {
      if (fresh) {
      const MatD& M = t.mats[t.mi];
      const ModD& D = tb.mods[M.owner];
      const int r = static_cast<int>(M.r);
      a[0] = make_src(M.param, M, 4, tb, 0);
      a[1] = make_src(M.mu, M, 4, tb, 1);
      a[2] = make_src(M.var, M, 4, tb, 2);
      // K operand: rows s0.. of Zc_A (d_out x RCA) or of the basis (d_in x RC)
      Src k{};
      k.es = 4; k.side = 0; k.cs = 1; k.swz = 1;
      k.map = (M.kmap >= 0 && tb.smaps != nullptr) ? tb.smaps + M.kmap : nullptr;
      if (M.side == 0) {
        k.base = reinterpret_cast<const char*>(reinterpret_cast<const float*>(tb.ws) + D.zca_off);
        k.ld = D.rca; k.r = D.rca;
      } else {
        const BasisD& Bd = tb.bases[D.basis];
        k.base = reinterpret_cast<const char*>(Bd.Vin);
        k.ld = Bd.v_s0; k.cs = Bd.v_s1; k.r = D.rc;
      }
      a[3] = k;
      pitch[0] = pitch[1] = pitch[2] = side_pitch(M.side, r, L.TV, 4);
      pitch[3] = L.pitch[3];
      }
      const int off[4] = {L.off[0], L.off[1], L.off[2], L.off[3]};
      produce<4>(a, off, pitch, t.s0, t.nv(), reinterpret_cast<char*>(stage), fb, lane, fresh);
    });
    return;
  }

  const int ct = threadIdx.x - 32 * kProd;
  const int team = ct / kTT, tt = ct - team * kTT;
  float* Cs = reinterpret_cast<float*>(smem + L.o_c);
  float* zs = reinterpret_cast<float*>(smem + L.o_z + team * al128(L.TV * L.zp * 4));
  double* red = reinterpret_cast<double*>(smem + L.o_red);
  float s_zmu = 0.f, s_zzv = 0.f;
  int i = 0;
  bool dead = false;
  bool more = it.start_seg();
  while (more) {
    // segment start: the module side's coefficient matrix, shared by the four teams
    const MatD M = it.mats[it.mi];
    const ModD D = tb.mods[M.owner];
    const int r = static_cast<int>(M.r);
    const int KW = (M.side == 0) ? D.rca : D.rc;
    const float* coef = reinterpret_cast<const float*>(tb.ws) + D.coef_off;
    named_sync(kBarAll, kCT);                         // every team is done with the previous segment
    const int K4 = (KW + 3) & ~3;                     // rows past KW are zero
    if (M.side == 0) {
      const float* Qm = coef + static_cast<int64_t>(D.r) * D.rc;   // R x RCA
      for (int e = ct; e < K4 * L.pld; e += kCT) {
        const int k = e / L.pld, c = e - k * L.pld;
        Cs[e] = (k < KW && c < D.r) ? Qm[c * D.rca + k] : 0.f;
      }
    } else {
      for (int e = ct; e < K4 * L.pld; e += kCT) {
        const int k = e / L.pld, c = e - k * L.pld;
        Cs[e] = (k < KW && c < D.r) ? coef[c * D.rc + k] : 0.f;
      }
    }
    named_sync(kBarAll, kCT);
    int adv, seg_done;
    do {
      const int nv = it.nv();
      if ((i % kTeams) == team && !dead) {
        const int s = i % L.S;
        const bool w = mbar_wait(full + s, static_cast<uint32_t>(i / L.S) & 1u, err);
        dead = !agree(kBarTeam0 + team, kTT, w);
        if (!dead) {
          const unsigned char* stage = smem + s * L.stage_bytes;
          mm_rows_sw(stage + L.off[3], L.TV, Cs, L.pld, nv, K4, r, tt, kTT,
                     [&](int v, int c, float x) { zs[v * L.zp + c] = x * eps; });
          named_sync(kBarTeam0 + team, kTT);
          const int n = nv * r;
          const int ld = static_cast<int>(M.ld), cs = static_cast<int>(M.cs);
          // this launch's direction: its z and +/- copies sit a fixed stride past direction 0's
          float* zt = tile_ptr(M.z + static_cast<int64_t>(tb.dir) * tb.dstride_z, M, it.s0, 4);
          const int64_t fo = static_cast<int64_t>(tb.dir) * tb.dstride_f * FES;
          void* post = tile_ptr(reinterpret_cast<char*>(M.pos) + fo, M, it.s0, FES);
          void* negt = tile_ptr(reinterpret_cast<char*>(M.neg) + fo, M, it.s0, FES);
          const float* ps = reinterpret_cast<const float*>(stage + L.off[0]);
          const float* ms = reinterpret_cast<const float*>(stage + L.off[1]);
          const float* vsg = reinterpret_cast<const float*>(stage + L.off[2]);
          // four elements per step along the contiguous direction when rows and pointers
          // allow vector accesses; element by element otherwise
          const bool vec = cs == 1 && (ld & 3) == 0 && ((M.side == 0 ? r : nv) & 3) == 0 && aligned_to(zt, 16) &&
                           aligned_to(post, 4 * FES) && aligned_to(negt, 4 * FES);
          auto body4 = [&](auto side_tag) {
            constexpr int SIDE = decltype(side_tag)::value;
            Walk4<SIDE> w(tt, kTT, r, nv);
            const int n4 = n / 4;
            for (int e = tt; e < n4; e += kTT, w.next()) {
              const int v = w.v(), k = w.k();
              float z[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) z[q] = SIDE == 0 ? zs[v * L.zp + k + q] : zs[(v + q) * L.zp + k];
              const int g = SIDE == 0 ? v * ld + k : k * ld + v;
              *reinterpret_cast<float4*>(zt + g) = make_float4(z[0], z[1], z[2], z[3]);
              {
                const int so = SIDE == 0 ? v * r + k : k * L.TV + v;
                const float4 p4 = *reinterpret_cast<const float4*>(ps + so);
                const float4 m4 = *reinterpret_cast<const float4*>(ms + so);
                const float4 w4 = *reinterpret_cast<const float4*>(vsg + so);
                const float4 pv = make_float4(__fadd_rn(p4.x, z[0]), __fadd_rn(p4.y, z[1]), __fadd_rn(p4.z, z[2]),
                                              __fadd_rn(p4.w, z[3]));
                const float4 nv4 = make_float4(__fsub_rn(p4.x, z[0]), __fsub_rn(p4.y, z[1]), __fsub_rn(p4.z, z[2]),
                                               __fsub_rn(p4.w, z[3]));
                st_fac4<FES>(post, g, pv);
                st_fac4<FES>(negt, g, nv4);
#pragma unroll
                for (int pp = 0; pp < kMaxPeers; ++pp) {   // the peers' copies of the +/- buffers
                  if (pp >= gp.n) break;
                  st_fac4<FES>(reinterpret_cast<char*>(post) + gp.dpos[pp], g, pv);
                  st_fac4<FES>(reinterpret_cast<char*>(negt) + gp.dneg[pp], g, nv4);
                }
                const float mv[4] = {m4.x, m4.y, m4.z, m4.w}, wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float mu1 = __fmul_rn(mv[q], kin.beta);
                  const float var1 = __fadd_rn(__fmul_rn(wv[q], kin.beta2), kin.q);
                  s_zmu = fmaf(z[q], mu1, s_zmu);
                  s_zzv = fmaf(__fmul_rn(z[q], z[q]), var1, s_zzv);
                }
              }
            }
          };
          auto body = [&](auto side_tag) {
            constexpr int SIDE = decltype(side_tag)::value;
            Walk<SIDE> w(tt, kTT, r, nv);
            for (int e = tt; e < n; e += kTT, w.next()) {
              const float z = zs[w.v * L.zp + w.k];
              const int g = w.goff(ld, cs);
              zt[g] = z;
              {
                const int so = w.soff(r, L.TV);
                const float p0 = ps[so];
                const float m0 = ms[so];
                const float w0 = vsg[so];
                st_fac<FES>(post, g, __fadd_rn(p0, z));
                st_fac<FES>(negt, g, __fsub_rn(p0, z));
#pragma unroll
                for (int pp = 0; pp < kMaxPeers; ++pp) {
                  if (pp >= gp.n) break;
                  st_fac<FES>(reinterpret_cast<char*>(post) + gp.dpos[pp], g, __fadd_rn(p0, z));
                  st_fac<FES>(reinterpret_cast<char*>(negt) + gp.dneg[pp], g, __fsub_rn(p0, z));
                }
                const float mu1 = __fmul_rn(m0, kin.beta);
                const float var1 = __fadd_rn(__fmul_rn(w0, kin.beta2), kin.q);
                s_zmu = fmaf(z, mu1, s_zmu);
                s_zzv = fmaf(__fmul_rn(z, z), var1, s_zzv);
              }
            }
          };
          if (vec) {
            if (M.side == 0) body4(std::integral_constant<int, 0>{});
            else body4(std::integral_constant<int, 1>{});
          } else {
            if (M.side == 0) body(std::integral_constant<int, 0>{});
            else body(std::integral_constant<int, 1>{});
          }
          __syncwarp();
          if ((tt & 31) == 0) mbar_arrive(empty + s);
          named_sync(kBarTeam0 + team, kTT);          // zs is rewritten by the team's next tile
        }
      }
      ++i;
      seg_done = it.seg;
      adv = it.next();
    } while (adv == 1);
    {
      // segment end: Kalman partials of the segment (fixed reduction order)
      double a = s_zmu, b = s_zzv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
      }
      if ((ct & 31) == 0) { red[2 * (ct >> 5)] = a; red[2 * (ct >> 5) + 1] = b; }
      named_sync(kBarAll, kCT);
      if (ct == 0) {
        double sa = 0.0, sb = 0.0;
        for (int w = 0; w < kCW; ++w) { sa += red[2 * w]; sb += red[2 * w + 1]; }
        double* out = reinterpret_cast<double*>(tb.ws) + tb.seg_kal_off + 2 * static_cast<int64_t>(seg_done);
        out[0] = sa;
        out[1] = sb;
      }
      s_zmu = 0.f;
      s_zzv = 0.f;
    }
    more = (adv == 2);
  }
  if (gp.n > 0) __threadfence_system();   // the peer stores precede this rank's next collective
}

// =====================================================================================
// Newton-Schulz apply (ds_mezo/kernels.py:84-92 rewritten in Gram space):
// param -= eta * X on the fp32 master, X[v,:] = x_v^T Pm with x_v the (already
// Kalman-updated) momentum; optional shadow = copy(param) in the copy dtype of FES bytes per
// element (what the rollout loads), optional scratch = X.
// =====================================================================================
template <int FES>
__global__ void __launch_bounds__(kSTP, 1) k_sapply(Tables tb, const MatD* __restrict__ mats, int nmats, int nsegs,
                                                   Layout L, float eta, GatherPeers gp, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + L.S;
  init_bars(full, empty, L.S, 2);
  TileIt it;
  it.init(mats, nmats, L.TV);
  const int warp = threadIdx.x >> 5;

  if (warp < kProd) {
    Src a[2];                                   // the segment's copy sources, built at its first tile
    int pitch[2];
    producer_loop<kProd>(it, L, smem, full, empty, err, [&](const TileIt& t, unsigned char* stage, uint64_t* fb, int lane, bool fresh) {
      if (fresh) {
        const MatD& M = t.mats[t.mi];
        a[0] = make_src(M.param, M, 4, tb, 0);
        a[1] = make_src(M.mu, M, 4, tb, 1);
        if (M.side == 0) {                      // mu rows as the swizzled row image
          a[1].swz = 1;
          a[1].map = (M.rmap >= 0 && tb.smaps != nullptr) ? tb.smaps + M.rmap : nullptr;
        }
        pitch[0] = side_pitch(M.side, static_cast<int>(M.r), L.TV, 4);
        pitch[1] = M.side == 0 ? L.pitch[1] : L.TV * 4;
      }
      const int off[2] = {L.off[0], L.off[1]};
      produce<2>(a, off, pitch, t.s0, t.nv(), reinterpret_cast<char*>(stage), fb, lane, fresh);
    });
    return;
  }

  const int ct = threadIdx.x - 32 * kProd;
  const int team = ct / kTT, tt = ct - team * kTT;
  float* Ps = reinterpret_cast<float*>(smem + L.o_c);
  float* os = reinterpret_cast<float*>(smem + L.o_z + team * al128(L.TV * L.zp * 4));
  int i = 0;
  bool dead = false;
  bool more = it.start_seg();
  int cur = -1;
  while (more) {
    const MatD M = it.mats[it.mi];
    const int r = static_cast<int>(M.r);
    if (it.mi != cur) {
      named_sync(kBarAll, kCT);
      const float* Pm = reinterpret_cast<const float*>(tb.ws) + M.p_off;
      for (int e = ct; e < ((r + 3) & ~3) * L.pld; e += kCT) {   // rows past r are zero
        const int a = e / L.pld, c = e - a * L.pld;
        Ps[e] = (a < r && c < r) ? Pm[a * r + c] : 0.f;
      }
      named_sync(kBarAll, kCT);
      cur = it.mi;
    }
    const int as = L.TV;                        // side 1: mu dense along the tile
    int adv;
    do {
      const int nv = it.nv();
      if ((i % kTeams) == team && !dead) {
        const int s = i % L.S;
        const bool w = mbar_wait(full + s, static_cast<uint32_t>(i / L.S) & 1u, err);
        dead = !agree(kBarTeam0 + team, kTT, w);
        if (!dead) {
          const unsigned char* stage = smem + s * L.stage_bytes;
          if (M.side == 0) {
            mm_rows_sw(stage + L.off[1], L.TV, Ps, L.pld, nv, (r + 3) & ~3, r, tt, kTT,
                       [&](int v, int c, float x) { os[v * L.zp + c] = x; });
          } else {
            const float* Xs = reinterpret_cast<const float*>(stage + L.off[1]);
            mm_rows<false>(Xs, 1, as, Ps, L.pld, nv, r, r, tt, kTT, [&](int v, int c, float x) { os[v * L.zp + c] = x; });
          }
          named_sync(kBarTeam0 + team, kTT);
          const int n = nv * r;
          const int ld = static_cast<int>(M.ld), cs = static_cast<int>(M.cs);
          float* pt = tile_ptr(reinterpret_cast<float*>(M.param), M, it.s0, 4);
          void* sht = M.shadow ? tile_ptr(reinterpret_cast<char*>(M.shadow), M, it.s0, FES) : nullptr;
          float* sct = M.scratch ? tile_ptr(M.scratch, M, it.s0, 4) : nullptr;
          const float* ps = reinterpret_cast<const float*>(stage + L.off[0]);
          const bool vec = cs == 1 && (ld & 3) == 0 && ((M.side == 0 ? r : nv) & 3) == 0 && aligned_to(pt, 16) &&
                           aligned_to(sht, 4 * FES) && aligned_to(sct, 16);
          auto body4 = [&](auto side_tag) {             // four elements per step
            constexpr int SIDE = decltype(side_tag)::value;
            Walk4<SIDE> w(tt, kTT, r, nv);
            const int n4 = n / 4;
            for (int e = tt; e < n4; e += kTT, w.next()) {
              const int v = w.v(), k = w.k();
              float X[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) X[q] = SIDE == 0 ? os[v * L.zp + k + q] : os[(v + q) * L.zp + k];
              const float4 p4 = *reinterpret_cast<const float4*>(ps + (SIDE == 0 ? v * r + k : k * L.TV + v));
              const int g = SIDE == 0 ? v * ld + k : k * ld + v;
              const float4 np = make_float4(__fsub_rn(p4.x, __fmul_rn(eta, X[0])), __fsub_rn(p4.y, __fmul_rn(eta, X[1])),
                                            __fsub_rn(p4.z, __fmul_rn(eta, X[2])), __fsub_rn(p4.w, __fmul_rn(eta, X[3])));
              *reinterpret_cast<float4*>(pt + g) = np;
              if (sht) {
                st_fac4<FES>(sht, g, np);
#pragma unroll
                for (int pp = 0; pp < kMaxPeers; ++pp) {   // the peers' copies of the shadow (dpos)
                  if (pp >= gp.n) break;
                  st_fac4<FES>(reinterpret_cast<char*>(sht) + gp.dpos[pp], g, np);
                }
              }
              if (sct) *reinterpret_cast<float4*>(sct + g) = make_float4(X[0], X[1], X[2], X[3]);
            }
          };
          auto body = [&](auto side_tag) {
            constexpr int SIDE = decltype(side_tag)::value;
            Walk<SIDE> w(tt, kTT, r, nv);
            for (int e = tt; e < n; e += kTT, w.next()) {
              const float X = os[w.v * L.zp + w.k];
              const float p0 = ps[w.soff(r, L.TV)];
              const int g = w.goff(ld, cs);
              const float np = __fsub_rn(p0, __fmul_rn(eta, X));
              pt[g] = np;
              if (sht) {
                st_fac<FES>(sht, g, np);
#pragma unroll
                for (int pp = 0; pp < kMaxPeers; ++pp) {
                  if (pp >= gp.n) break;
                  st_fac<FES>(reinterpret_cast<char*>(sht) + gp.dpos[pp], g, np);
                }
              }
              if (sct) sct[g] = X;
            }
          };
          if (vec) {
            if (M.side == 0) body4(std::integral_constant<int, 0>{});
            else body4(std::integral_constant<int, 1>{});
          } else {
            if (M.side == 0) body(std::integral_constant<int, 0>{});
            else body(std::integral_constant<int, 1>{});
          }
          __syncwarp();
          if ((tt & 31) == 0) mbar_arrive(empty + s);
          named_sync(kBarTeam0 + team, kTT);
        }
      }
      ++i;
      adv = it.next();
    } while (adv == 1);
    more = (adv == 2);
  }
  if (gp.n > 0) __threadfence_system();   // the peer stores precede this rank's next collective
}

// =====================================================================================
// CholeskyQR apply of the power iteration: V = W R^{-1} in fp64 (R^{-1}, upper
// triangular, exported by k_chol after the fp64 workspace's first r*r doubles), V rows out
// and, when the next product runs on the tensor cores, [V_hi | V_lo]^T (bf16, 2R x D).
// Four groups of four warps take tiles i % 4 straight from the ring (a multiple of four
// stages, so each stage has one consumer group). In a group each warp owns MV row
// blocks x MC column blocks of 8 x 8 and forms them with the fp64 MMA: A fragments are
// fp32 W read from the stage and widened in registers, B fragments R^{-1} in fp64. Column
// blocks are dealt snake-wise (ascending per warp), so the k-extent of block column cb
// (k < 8cb + 8, R^{-1} being upper triangular) shrinks the active set one block at a time
// and every warp has the same number of MMAs. V rows are stored from the accumulators;
// the bf16 pair goes through an fp32 tile per group (two, alternating), eight vectors per
// thread and 16-byte stores. Waits are bounded; a group agrees on each tile's verdict.
// =====================================================================================

// Warp shape of the QR apply for tiles of TV vectors and width R: the first of
// (MV, MC) = (2,4), (4,2), (1,8), (8,1) whose warp grid fits a group; -1 if none.
__host__ __device__ inline int qr_variant(int TV, int R) {
  const int nvb = (TV + 7) / 8, ncb = (R + 7) / 8;
  const int mv[4] = {2, 4, 1, 8}, mc[4] = {4, 2, 8, 1};
  for (int v = 0; v < 4; ++v)
    if (((nvb + mv[v] - 1) / mv[v]) * ((ncb + mc[v] - 1) / mc[v]) <= kQrGroupWarps) return v;
  return -1;
}

// [hi | lo] bf16 rows of eight fp32 values x[0..7] (hi = bf16(x), lo = bf16(x - hi)).
__device__ __forceinline__ void bf16_pair8(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(x[2 * q], x[2 * q + 1]);
    const float2 hf = __bfloat1622float2(hh);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(x[2 * q] - hf.x, x[2 * q + 1] - hf.y);
    h[q] = *reinterpret_cast<const uint32_t*>(&hh);
    l[q] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int MV, int MC>
__global__ void __launch_bounds__(kQrThreads, 1) k_sqr_apply(Tables tb, const MatD* __restrict__ mats, int nmats,
                                                      int nsegs, Layout L, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + L.S;
  double* Ps = reinterpret_cast<double*>(smem + L.o_c);        // rp x pld fp64 R^{-1}
  const int osz = (L.o_bar - L.o_z) / (8 * kQrGroups);           // floats per fp32 tile (two per group)
  if (threadIdx.x == 0) {
    for (int i = 0; i < L.S; ++i) { mbar_init(full + i, kFullArrivals); mbar_init(empty + i, kQrGroupWarps); }
    mbar_init_fence();
  }
  __syncthreads();
  TileIt it;
  it.init(mats, nmats, L.TV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp < kProd) {
    Src a[1];                                       // the segment's copy source, built at its first tile
    producer_loop<kProd>(it, L, smem, full, empty, err, [&](const TileIt& t, unsigned char* stage, uint64_t* fb, int ln, bool fresh) {
      if (fresh) {
        const MatD& M = t.mats[t.mi];
        a[0] = make_src(M.mu, M, 4, tb, 1);
        a[0].swz = 1;                               // W rows as the swizzled row image
        a[0].map = (M.rmap >= 0 && tb.smaps != nullptr) ? tb.smaps + M.rmap : nullptr;
      }
      const int off[1] = {0};
      const int pitch[1] = {L.pitch[0]};
      produce<1>(a, off, pitch, t.s0, t.nv(), reinterpret_cast<char*>(stage), fb, ln, fresh);
    });
    return;
  }

  const int mw = warp - kProd;
  const int grp = mw / kQrGroupWarps, gw = mw - grp * kQrGroupWarps;
  const int ct = threadIdx.x - 32 * kProd, gt = ct - grp * 32 * kQrGroupWarps;
  const int g = lane >> 2, kq = lane & 3;
  const int boxb = L.TV * 128;
  const int WV = ((L.TV + 7) / 8 + MV - 1) / MV;
  const int wv = gw % WV, wc = gw / WV;
  int i = 0, jt = 0;
  bool dead = false;
  int cur = -1;
  if (!it.start_seg()) return;
  int adv;
  do {
    const MatD& M = it.mats[it.mi];
    const int r = static_cast<int>(M.r), nv = it.nv();
    if (it.mi != cur) {                            // R^{-1} of this basis (both groups)
      named_sync(kBarAll, kQrCT);
      const double* Rd = reinterpret_cast<const double*>(tb.ws) + M.dw_off + static_cast<int64_t>(r) * r;
      for (int e = ct; e < L.rp * L.pld; e += kQrCT) {
        const int a2 = e / L.pld, c = e - a2 * L.pld;
        Ps[e] = (a2 < r && c < r) ? Rd[a2 * r + c] : 0.0;
      }
      named_sync(kBarAll, kQrCT);
      cur = it.mi;
    }
    if ((i % kQrGroups) == grp) {
      const int s = i % L.S;
      const bool w = dead ? false : mbar_wait(full + s, static_cast<uint32_t>(i / L.S) & 1u, err);
      dead = !agree(kBarTeam0 + grp, 32 * kQrGroupWarps, w);
      if (!dead) {
        const unsigned char* Ws = smem + s * L.stage_bytes;   // swizzled row image of W
        const int nvb = (nv + 7) >> 3, ncb = (r + 7) >> 3;
        const int WC = (ncb + MC - 1) / MC;
        int rv[MV], cc[MC], kb[MC];
        bool rok[MV], cok[MC];
#pragma unroll
        for (int j = 0; j < MV; ++j) { rv[j] = wv + WV * j; rok[j] = wc < WC && rv[j] < nvb; }
#pragma unroll
        for (int j = 0; j < MC; ++j) {              // ascending; k-extent 8cc + 8 (0 if none)
          cc[j] = (j >> 1) * 2 * WC + ((j & 1) ? 2 * WC - 1 - wc : wc);
          cok[j] = wc < WC && cc[j] < ncb;
          kb[j] = cok[j] ? 8 * cc[j] + 8 : (j > 0 ? kb[j - 1] : 0);
          if (!cok[j]) cc[j] = 0;
        }
        double acc[MV][MC][2];
#pragma unroll
        for (int jv = 0; jv < MV; ++jv)
#pragma unroll
          for (int jc = 0; jc < MC; ++jc) { acc[jv][jc][0] = 0.0; acc[jv][jc][1] = 0.0; }
        // A fragment (row 8 rv + g, column k0 + kq): row start + chunk ((k0 / 4) % 8) ^ g
        // (the row's swizzle is g) of box k0 / 32
        const unsigned char* xa[MV];
        const double* pb[MC];
#pragma unroll
        for (int jv = 0; jv < MV; ++jv) xa[jv] = Ws + (8 * (rok[jv] ? rv[jv] : 0) + g) * 128 + kq * 4;
#pragma unroll
        for (int jc = 0; jc < MC; ++jc) pb[jc] = Ps + kq * L.pld + 8 * cc[jc] + g;
        const int pstep = 4 * L.pld;
        int k0 = 0;
#pragma unroll
        for (int j0 = 0; j0 < MC; ++j0) {           // blocks j0 .. MC-1 active for k < kb[j0]
          for (; k0 < kb[j0]; k0 += 4) {
            double av[MV];
            const int xo = (k0 >> 5) * boxb + ((((k0 >> 2) & 7) ^ g) << 4);
#pragma unroll
            for (int jv = 0; jv < MV; ++jv) av[jv] = static_cast<double>(*reinterpret_cast<const float*>(xa[jv] + xo));
            const int po = (k0 >> 2) * pstep;
#pragma unroll
            for (int jc = j0; jc < MC; ++jc) {
              const double bv = pb[jc][po];
#pragma unroll
              for (int jv = 0; jv < MV; ++jv)
                if (rok[jv] && cok[jc]) dmma8x8x4(acc[jv][jc][0], acc[jv][jc][1], av[jv], bv);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);      // W tile consumed
        float* V = reinterpret_cast<float*>(M.param);
        const int64_t ldV = M.ld;
        __nv_bfloat16* const v2t = M.v2t;
        const int64_t ldv2 = M.ldv2;
        const bool vec2 = (ldV % 2) == 0 && (reinterpret_cast<uintptr_t>(V) % 8) == 0;
        float* os = reinterpret_cast<float*>(smem + L.o_z) + (2 * grp + (jt & 1)) * osz;
#pragma unroll
        for (int jv = 0; jv < MV; ++jv) {
#pragma unroll
          for (int jc = 0; jc < MC; ++jc) {
            if (!rok[jv] || !cok[jc]) continue;
            const int v = 8 * rv[jv] + g, c = 8 * cc[jc] + 2 * kq;
            const float x0 = static_cast<float>(acc[jv][jc][0]), x1 = static_cast<float>(acc[jv][jc][1]);
            if (v < nv) {                           // V rows, from the accumulators
              float* row = V + static_cast<int64_t>(it.s0 + v) * ldV;
              if (vec2 && c + 1 < r) {
                *reinterpret_cast<float2*>(row + c) = make_float2(x0, x1);
              } else {
                if (c < r) row[c] = x0;
                if (c + 1 < r) row[c + 1] = x1;
              }
            }
            if (v2t) { os[v * L.zp + c] = x0; os[v * L.zp + c + 1] = x1; }
          }
        }
        if (v2t) {                                  // [V_hi | V_lo]^T, coalesced along d
          named_sync(kBarTeam0 + grp, 32 * kQrGroupWarps);
          const int nu = r * (nv >> 3);             // eight vectors per unit
          for (int u = gt; u < nu; u += 32 * kQrGroupWarps) {
            const int c = u % r, v0 = (u / r) * 8;
            float x[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) x[q] = os[(v0 + q) * L.zp + c];
            uint4 hi, lo;
            bf16_pair8(x, hi, lo);
            *reinterpret_cast<uint4*>(v2t + static_cast<int64_t>(c) * ldv2 + it.s0 + v0) = hi;
            *reinterpret_cast<uint4*>(v2t + static_cast<int64_t>(r + c) * ldv2 + it.s0 + v0) = lo;
          }
          for (int e = (nv & ~7) * r + gt; e < nv * r; e += 32 * kQrGroupWarps) {   // ragged tail
            const int v = e / r, c = e - v * r;
            const float x = os[v * L.zp + c];
            const __nv_bfloat16 h = __float2bfloat16_rn(x);
            v2t[static_cast<int64_t>(c) * ldv2 + it.s0 + v] = h;
            v2t[static_cast<int64_t>(r + c) * ldv2 + it.s0 + v] = __float2bfloat16_rn(x - __bfloat162float(h));
          }
        }
        // the group's next tile writes the other fp32 tile; the barrier there orders the
        // reads above before this tile is written again
      }
      ++jt;
    }
    ++i;
    adv = it.next();
  } while (adv != 0);
}

// =====================================================================================
// Gram partials per segment: G_seg = sum_v x_v x_v^T in fp64 (products of fp32 values are
// exact in fp64). SRC 0: x = mu. SRC 1: x = mu2 of the Kalman update (controller.py:
// 267-268, 283-285), and mu2 / var2 are written back to mu / var.
// Warp roles after the producer: four prep warps turn each staged tile into an fp64 tile
// (Kalman update and write-back on the way) in one of two buffers; four MMA warps
// accumulate the upper-triangle 8 x 8 blocks of G from the other buffer with the fp64
// MMA (m8n8k4), each block owned by one warp for the whole segment (fragments in
// registers) and written out, mirrored, at the segment end. Prep and MMA warps hand the
// buffers over through mbarriers only (bounded waits), so a failed wait cannot leave one
// role blocked at a barrier the other never reaches.
// Tile image: side 0 X[v][c] with pitch rp + 8 doubles, side 1 X[c][v] with pitch TV + 4
// (either way a fragment load of a warp touches 256 bytes in two wavefronts).
// =====================================================================================
// MAXB: upper 8 x 8 blocks per MMA warp (5 up to r = 64, 17 up to r = 128)
__host__ __device__ inline int gram_maxb(int r) {
  const int nb = (r + 7) / 8;
  return (nb * (nb + 1) / 2 + kMmaWarps - 1) / kMmaWarps;
}

template <int SRC, int MAXB>
__global__ void __launch_bounds__(kSTG, 1) k_sgram(Tables tb, const MatD* __restrict__ mats, int nmats, int nsegs,
                                                  Layout L, KalmanIn kin, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + L.S;
  uint64_t* xfull = empty + L.S;                 // [2]: prep -> MMA
  uint64_t* xempty = xfull + 2;                  // [2]: MMA -> prep
  const int rp = L.rp, nb = rp / 8;
  const int nblk = nb * (nb + 1) / 2;
  double* X0 = reinterpret_cast<double*>(smem + L.o_x);
  const int xbuf = (L.o_red - L.o_x) / 16;       // doubles per buffer (two buffers)
  int* btab = reinterpret_cast<int*>(smem + L.o_red);
  // zero both fp64 buffers (padding columns stay zero), block table, barriers
  for (int e = threadIdx.x; e < 2 * xbuf; e += kSTG) X0[e] = 0.0;
  if (threadIdx.x == 0) {
    int q = 0;
    for (int bi = 0; bi < nb; ++bi)
      for (int bj = bi; bj < nb; ++bj) btab[q++] = (bi << 8) | bj;
    for (int i = 0; i < L.S; ++i) { mbar_init(full + i, kFullArrivals); mbar_init(empty + i, kPrepWarps); }
    for (int i = 0; i < 2; ++i) { mbar_init(xfull + i, kPrepWarps); mbar_init(xempty + i, kMmaWarps); }
    mbar_init_fence();
  }
  __syncthreads();
  TileIt it;
  it.init(mats, nmats, L.TV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0) {
    Src a[3];                                       // the segment's copy sources, built at its first tile
    int pitch[3];
    producer_loop<1>(it, L, smem, full, empty, err, [&](const TileIt& t, unsigned char* stage, uint64_t* fb, int ln, bool fresh) {
      if (fresh) {
        const MatD& M = t.mats[t.mi];
        a[0] = make_src(M.mu, M, 4, tb, 1);
        a[1] = make_src(SRC == 1 ? M.var : nullptr, M, 4, tb, 2);
        a[2] = make_src(SRC == 1 ? M.z : nullptr, M, 4, tb, 3);
        pitch[0] = pitch[1] = pitch[2] = side_pitch(M.side, static_cast<int>(M.r), L.TV, 4);
      }
      const int off[3] = {L.off[0], L.off[1], L.off[2]};
      produce<3>(a, off, pitch, t.s0, t.nv(), reinterpret_cast<char*>(stage), fb, ln, fresh);
    });
    return;
  }

  if (warp <= kPrepWarps) {
    // ------------------------------------------------------------ prep warps
    const int pt = threadIdx.x - 32, npt = 32 * kPrepWarps;
    KalScal ks{};
    if (SRC == 1) ks = kal_derive(kin, reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off);
    int i = 0;
    bool dead = false;
    if (!it.start_seg()) return;
    int adv;
    do {
      const MatD& M = it.mats[it.mi];
      const int r = static_cast<int>(M.r), nv = it.nv();
      const int s = i % L.S, b = i & 1;
      if (!dead) {
        bool w = mbar_wait(full + s, static_cast<uint32_t>(i / L.S) & 1u, err);
        if (w && i >= 2) w = mbar_wait(xempty + b, (static_cast<uint32_t>(i >> 1) & 1u) ^ 1u, err);
        dead = !__all_sync(0xffffffffu, w);
      }
      if (!dead) {
        double* X = X0 + b * xbuf;
        const int sv = (M.side == 0) ? L.xp : 1;
        const int sc = (M.side == 0) ? 1 : L.zp;
        const unsigned char* stage = smem + s * L.stage_bytes;
        const float* mus = reinterpret_cast<const float*>(stage + L.off[0]);
        const float* vas = reinterpret_cast<const float*>(stage + L.off[1]);
        const float* zss = reinterpret_cast<const float*>(stage + L.off[2]);
        const int n = nv * r;
        const int ld = static_cast<int>(M.ld), cs = static_cast<int>(M.cs);
        float* mut = tile_ptr(M.mu, M, it.s0, 4);
        float* vat = tile_ptr(M.var, M, it.s0, 4);
        auto body = [&](auto side_tag) {
          constexpr int SIDE = decltype(side_tag)::value;
          constexpr int U = 4;
          Walk<SIDE> wk(pt, npt, r, nv);
          for (int e = pt; e < n; e += U * npt) {
            int vv[U], kk[U], so[U];
            float x[U], va[U], zz[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {                   // every load before any use
              vv[u] = wk.v; kk[u] = wk.k;
              so[u] = wk.soff(r, L.TV);
              wk.next();
              if (e + u * npt < n) {
                x[u] = mus[so[u]];
                if (SRC == 1) { va[u] = vas[so[u]]; zz[u] = zss[so[u]]; }
              }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
              if (e + u * npt >= n) continue;
              float xv = x[u];
              if (SRC == 1) {
                float mu1, var1, mu2, var2;
                kal_predict(xv, va[u], ks, mu1, var1);
                kal_observe(mu1, var1, zz[u], ks, mu2, var2);
                const int g = SIDE == 0 ? vv[u] * ld + kk[u] * cs : kk[u] * ld + vv[u] * cs;
                mut[g] = mu2;
                vat[g] = var2;
                xv = mu2;
              }
              X[vv[u] * sv + kk[u] * sc] = static_cast<double>(xv);
            }
          }
        };
        // four consecutive elements per step along the contiguous direction when rows and
        // pointers allow 16-byte accesses (fp64 tile: two 16-byte stores)
        const bool vec = cs == 1 && (ld & 3) == 0 && ((M.side == 0 ? r : nv) & 3) == 0 &&
                         (SRC == 0 || (aligned_to(mut, 16) && aligned_to(vat, 16)));
        auto body4 = [&](auto side_tag) {
          constexpr int SIDE = decltype(side_tag)::value;
          Walk4<SIDE> wk(pt, npt, r, nv);
          const int n4 = n / 4;
          for (int e = pt; e < n4; e += npt, wk.next()) {
            const int v = wk.v(), k = wk.k();
            const int so = SIDE == 0 ? v * r + k : k * L.TV + v;
            float4 x4 = *reinterpret_cast<const float4*>(mus + so);
            if (SRC == 1) {
              const float4 va4 = *reinterpret_cast<const float4*>(vas + so);
              const float4 zz4 = *reinterpret_cast<const float4*>(zss + so);
              const float xi[4] = {x4.x, x4.y, x4.z, x4.w}, vi[4] = {va4.x, va4.y, va4.z, va4.w};
              const float zi[4] = {zz4.x, zz4.y, zz4.z, zz4.w};
              float mo[4], vo[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float mu1, var1;
                kal_predict(xi[q], vi[q], ks, mu1, var1);
                kal_observe(mu1, var1, zi[q], ks, mo[q], vo[q]);
              }
              const int g = SIDE == 0 ? v * ld + k : k * ld + v;
              *reinterpret_cast<float4*>(mut + g) = make_float4(mo[0], mo[1], mo[2], mo[3]);
              *reinterpret_cast<float4*>(vat + g) = make_float4(vo[0], vo[1], vo[2], vo[3]);
              x4 = make_float4(mo[0], mo[1], mo[2], mo[3]);
            }
            if (SIDE == 0) {
              double2* xd = reinterpret_cast<double2*>(X + v * sv + k);
              xd[0] = make_double2(x4.x, x4.y);
              xd[1] = make_double2(x4.z, x4.w);
            } else {
              double2* xd = reinterpret_cast<double2*>(X + v + k * sc);
              xd[0] = make_double2(x4.x, x4.y);
              xd[1] = make_double2(x4.z, x4.w);
            }
          }
        };
        if (vec) {
          if (M.side == 0) body4(std::integral_constant<int, 0>{});
          else body4(std::integral_constant<int, 1>{});
        } else {
          if (M.side == 0) body(std::integral_constant<int, 0>{});
          else body(std::integral_constant<int, 1>{});
        }
        const int nv4 = (nv + 3) & ~3;                        // zero vectors nv .. nv4-1
        for (int e = pt; e < (nv4 - nv) * r; e += npt) {
          const int v = nv + e / r, c = e - (e / r) * r;
          X[v * sv + c * sc] = 0.0;
        }
        __syncwarp();
        if (lane == 0) { mbar_arrive(empty + s); mbar_arrive(xfull + b); }
      }
      ++i;
      adv = it.next();
    } while (adv != 0);
    return;
  }

  // -------------------------------------------------------------- MMA warps
  const int mw = warp - 1 - kPrepWarps;
  const int fv = lane & 3, fc = lane >> 2;
  const int nmine = (nblk - mw + kMmaWarps - 1) / kMmaWarps;
  double acc[MAXB][2];
#pragma unroll
  for (int q = 0; q < MAXB; ++q) { acc[q][0] = 0.0; acc[q][1] = 0.0; }
  int i = 0;
  bool dead = false;
  if (!it.start_seg()) return;
  int adv;
  do {
    const MatD& M = it.mats[it.mi];
    const int r = static_cast<int>(M.r), nv = it.nv();
    const int b = i & 1;
    if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(xfull + b, static_cast<uint32_t>(i >> 1) & 1u, err));
    if (!dead) {
      const double* X = X0 + b * xbuf;
      const int sv = (M.side == 0) ? L.xp : 1;
      const int sc = (M.side == 0) ? 1 : L.zp;
      int oa[MAXB], ob[MAXB];
#pragma unroll
      for (int q = 0; q < MAXB; ++q) {
        const int t = (q < nmine) ? btab[mw + q * kMmaWarps] : 0;
        oa[q] = 8 * (t >> 8) * sc;
        ob[q] = 8 * (t & 0xff) * sc;
      }
      const int nv4 = (nv + 3) & ~3;
      const double* xr = X + fv * sv + fc * sc;
      for (int v0 = 0; v0 < nv4; v0 += 4, xr += 4 * sv) {
#pragma unroll
        for (int q = 0; q < MAXB; ++q)
          if (q < nmine) dmma8x8x4(acc[q][0], acc[q][1], xr[oa[q]], xr[ob[q]]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(xempty + b);
    }
    ++i;
    const int seg_done = it.seg;
    adv = it.next();
    if (adv != 1) {
      // segment end: this warp's blocks (and their mirror images) of the partial
      if (!dead) {
        double* gout = reinterpret_cast<double*>(tb.ws) + M.gram_off + static_cast<int64_t>(seg_done - M.seg0) * r * r;
#pragma unroll
        for (int q = 0; q < MAXB; ++q) {
          if (q < nmine) {
            const int t = btab[mw + q * kMmaWarps];
            const int bi = t >> 8, bj = t & 0xff;
            const int row = 8 * bi + (lane >> 2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int col = 8 * bj + 2 * (lane & 3) + h;
              if (row < r && col < r) {
                gout[row * r + col] = acc[q][h];
                gout[col * r + row] = acc[q][h];
              }
            }
          }
        }
      }
#pragma unroll
      for (int q = 0; q < MAXB; ++q) { acc[q][0] = 0.0; acc[q][1] = 0.0; }
    }
  } while (adv != 0);
}

// =====================================================================================
// Kalman observation update for K directions (no reference counterpart; the reference
// observes one direction per step): with innov_k = dd_k - y_hat_k and
// inv_k = 1 / (s_k + norm_floor), per element
//   mu1 = mu * beta, var1 = var * beta^2 + q                 (controller.py:267-268)
//   mu2 = mu1 + var1 * sum_k z_k * inv_k * innov_k
//   var2 = var1 * (1 - var1 * sum_k z_k^2 * inv_k)
// i.e. the joint observation of the K directions with the innovation covariance's
// diagonal (its off-diagonal terms are O(1/sqrt(n)) for independent directions). A plain
// coalesced pass over a chunk of tiles per CTA (any grid: no per-segment output); the
// fp64 Gram of mu2 follows (k_sgram<0>).
// =====================================================================================
struct KalmanDirs {
  float beta, beta2, q, floor_;
  int32_t n;
  float dd[DSMZ_MAX_DIRECTIONS];
};

__global__ void __launch_bounds__(256) k_kalman_dirs(Tables tb, KalmanDirs kd, int TV) {
  __shared__ float innov[DSMZ_MAX_DIRECTIONS], invs[DSMZ_MAX_DIRECTIONS];
  const double* sums = reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off;
  if (threadIdx.x < kd.n) {
    const int k = threadIdx.x;
    const float y_hat = static_cast<float>(sums[2 * k]);
    const float S = __fadd_rn(static_cast<float>(sums[2 * k + 1]), kd.floor_);
    invs[k] = __fdiv_rn(1.0f, S);
    innov[k] = __fsub_rn(kd.dd[k], y_hat);
  }
  __syncthreads();
  TileIt it;
  it.init(tb.mats, tb.nmats, TV);
  if (!it.start_seg()) return;
  int adv;
  do {
    const MatD& M = it.mats[it.mi];
    const int r = static_cast<int>(M.r), nv = it.nv();
    const int ld = static_cast<int>(M.ld), cs = static_cast<int>(M.cs);
    float* mut = tile_ptr(M.mu, M, it.s0, 4);
    float* vat = tile_ptr(M.var, M, it.s0, 4);
    const float* zt = tile_ptr(M.z, M, it.s0, 4);
    auto body = [&](auto side_tag) {
      constexpr int SIDE = decltype(side_tag)::value;
      Walk<SIDE> w(threadIdx.x, 256, r, nv);
      for (int e = threadIdx.x; e < nv * r; e += 256, w.next()) {
        const int g = w.goff(ld, cs);
        const float mu1 = __fmul_rn(mut[g], kd.beta);
        const float var1 = __fadd_rn(__fmul_rn(vat[g], kd.beta2), kd.q);
        float am = 0.f, av = 0.f;
        for (int k0 = 0; k0 < kd.n; k0 += 8) {       // eight independent loads in flight
          float z[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            z[u] = (k0 + u < kd.n) ? zt[static_cast<int64_t>(k0 + u) * tb.dstride_z + g] : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (k0 + u >= kd.n) break;
            const float zi = __fmul_rn(z[u], invs[k0 + u]);
            am = __fmaf_rn(zi, innov[k0 + u], am);
            av = __fmaf_rn(zi, z[u], av);
          }
        }
        mut[g] = __fmaf_rn(var1, am, mu1);
        vat[g] = __fmul_rn(var1, __fsub_rn(1.0f, __fmul_rn(var1, av)));
      }
    };
    if (M.side == 0) body(std::integral_constant<int, 0>{});
    else body(std::integral_constant<int, 1>{});
    adv = it.next();
  } while (adv != 0);
}

}  // namespace sk
}  // namespace dsmz
