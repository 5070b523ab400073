// Tensor-core (tcgen05 + TMEM + TMA) kernels for the power-iteration products on sm_100a.
//
// Y = H V and W = H^T Y with bf16 H. Three iterations of the reference power iteration
// are not converged, so an operand rounded to bf16 once shows up in the result (measured
// subspace sine ~1e-2); both products therefore take the fp32 operand as a bf16 hi/lo
// pair, B = [X_hi | X_lo] with N = 2R columns, and add the two halves of the fp32 TMEM
// accumulator in the epilogue (sine ~1e-5 against the exact algorithm).
//
// Both kernels run six warps:
//   warp 0     TMA producer (one lane): A and B tiles into a ring of smem stages
//   warp 1     TMEM owner + MMA issuer (one lane): tcgen05.mma kind::f16, M=128, N=2R
//   warps 2-5  epilogue: tcgen05.ld of the 128 x 2R fp32 accumulator, hi+lo, stores
// Both are persistent (one CTA per SM) over tiles of one or two 128-row halves (w_halves).
// Every mbarrier wait gives up after ~1 s of globaltimer, sets the error word and lets
// the CTA drain and free its TMEM.
#pragma once

#include <cuda.h>

#include "dsmz_internal.cuh"
#include "dsmz_ptx.cuh"

namespace dsmz {
namespace tc {

constexpr int kBM = 128;         // output rows per CTA (MMA M)
constexpr int kBK = 64;          // bf16 elements of K per stage (one 128-byte swizzle row)
constexpr int kThreadsTC = 192;  // 6 warps

// Per-basis operands of the tensor-core power iteration. Tensor maps come first (64-byte
// alignment); they are encoded on the host once the workspace addresses are known.
struct alignas(64) TCBasis {
  CUtensorMap mapHy;      // H (T x D), box {64 cols, 128 rows}: A of Y = H [V_hi|V_lo], K-major
  CUtensorMap mapHw;      // H (T x D), box {64 cols, 64 rows}:  A of W = H^T [Y_hi|Y_lo], MN-major
  CUtensorMap mapV2;      // V2T (2R x D) bf16, box {64, 2R}: B of the Y product, K-major
  CUtensorMap mapY2;      // Y2T (2R x T) bf16, box {64, 2R}: B of the W product, K-major
  __nv_bfloat16* V2T;     // [V_hi | V_lo]^T, row stride ldv2
  __nv_bfloat16* Y2T;     // [Y_hi | Y_lo]^T, row stride ldy2
  float* W;               // D x R fp32
  const float* Vsrc;      // caller's basis, read on the first iteration (strides v_s0, v_s1)
  const float* Vout;      // D x R contiguous basis of later iterations
  int64_t v_s0, v_s1;
  int64_t ldv2, ldy2;
  int64_t T, D;
  int32_t R, pad0;
  int32_t ytile0, nytile, wtile0, nwtile;
  int32_t vt0, nvt;       // blocks of the split kernel
  double* Gp;             // fused W Gram (R <= 64): per W tile, its upper 8 x 8 blocks of
                          // W_tile^T W_tile (block-major, 64 doubles each); NULL: not fused
  int32_t nq, pad1;       // upper blocks per tile
};

// Pitch (doubles) of the fp64 W tile staged by the W kernel's epilogue for the fused Gram:
// R + 4 (R % 16 == 0, so 4 mod 16): each half-warp's fragment (four rows x four columns of
// 8-byte words) falls on distinct banks.
__host__ __device__ inline int w_stage_ld(int R) { return R + 4; }
constexpr int kGramMaxBlocks = 9;   // upper blocks per epilogue warp (R <= 64: 36 / 4)

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}
// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulator, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Instruction descriptor, kind::tf32: tf32 A and B (32-bit operands whose low 13 mantissa
// bits the tensor core does not use), fp32 accumulator, M = 128, N = n, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// x rounded to the nearest tf32 value (low 13 mantissa bits zero); x - tf32_hi(x) is exact.
__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// Shared-memory writes of this thread become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 lanes x 16 consecutive fp32 columns of TMEM -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__host__ __device__ inline int tmem_cols(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

// Upper 8 x 8 blocks of a W tile's Gram W_tile^T W_tile on the fp64 MMA, accumulated over
// rows staged in shared memory as fp64 (pitch tld); epilogue warp q (of four) owns the
// blocks q, q + 4, ..., stored block-major (64 doubles each).
struct TileGram {
  int oa[kGramMaxBlocks], ob[kGramMaxBlocks];
  bool on[kGramMaxBlocks];
  double acc[kGramMaxBlocks][2];
  int q, g, kq;
  __device__ __forceinline__ TileGram(int tld, int R, int nq, int q_, int lane) : q(q_), g(lane >> 2), kq(lane & 3) {
    const int nb = R >> 3;
#pragma unroll
    for (int u = 0; u < kGramMaxBlocks; ++u) {
      int qq = q + 4 * u;
      int bi = 0, bj = 0;
      on[u] = qq < nq;
      if (on[u]) {
        while (qq >= nb - bi) { qq -= nb - bi; ++bi; }
        bj = bi + qq;
      }
      oa[u] = kq * tld + 8 * bi + g;
      ob[u] = kq * tld + 8 * bj + g;
      acc[u][0] = 0.0; acc[u][1] = 0.0;
    }
  }
  // rows [0, nrows) of the staged tile (nrows a multiple of 4)
  __device__ __forceinline__ void rows(const double* wt, int tld, int nrows) {
    for (int k0 = 0; k0 < nrows; k0 += 4) {        // all of a step's loads, then its MMAs
      const double* wr = wt + k0 * tld;
      double ca[kGramMaxBlocks], cb[kGramMaxBlocks];
#pragma unroll
      for (int u = 0; u < kGramMaxBlocks; ++u) { ca[u] = wr[oa[u]]; cb[u] = wr[ob[u]]; }
#pragma unroll
      for (int u = 0; u < kGramMaxBlocks; ++u)
        if (on[u]) dmma8x8x4(acc[u][0], acc[u][1], ca[u], cb[u]);
    }
  }
  __device__ __forceinline__ void store(double* gp) const {
#pragma unroll
    for (int u = 0; u < kGramMaxBlocks; ++u)
      if (on[u]) *reinterpret_cast<double2*>(gp + (q + 4 * u) * 64 + g * 8 + 2 * kq) = make_double2(acc[u][0], acc[u][1]);
  }
};

// Shared-memory bytes of the fp64 staging region of the persistent W kernel's fused Gram
// (R <= 64), beside the stage ring: one epilogue warp's 32 rows at a time.
__host__ __device__ inline int w_stage_bytes(int R) { return R <= 64 ? 32 * w_stage_ld(R) * 8 : 0; }
// 128-row halves per W tile: two for R <= 64 (two accumulators of 2R columns per TMEM
// buffer, 2 x 2 x 128 = 512 columns), one above.
__host__ __device__ inline int w_halves(int R) { return R <= 64 ? 2 : 1; }
// One stage of the W ring: MT x 128 rows of H (two 64 x 64 boxes per half) and the 2R x 64
// Y operand they share.
__host__ __device__ inline int ring_stage_bytes(int R, int MT) { return MT * kBM * kBK * 2 + 2 * R * kBK * 2; }

// Persistent W = H^T [Y_hi | Y_lo] (+ the fused fp64 Gram of each W tile for R <= 64).
// One CTA per SM walks the W tiles of every basis, last basis first: the first tiles then
// read the activations that the Y product read last, while they are still in L2. TMEM holds
// two accumulators, so the epilogue of tile j (W rows stored from the accumulator, the tile
// staged in fp64 and its Gram formed on the fp64 MMA) runs while the MMA warp accumulates
// tile j + 1; the stage ring runs on across tiles. Every basis of a plan has the same R.
// A tile is MT halves of 128 rows: both halves' MMAs read the same Y stage, so the Y
// operand crosses from L2 once per MT x 128 rows of H, and the Gram partial covers them all.
//   warp 0     TMA producer (one lane)
//   warp 1     TMEM owner + MMA issuer (one lane); buffer j & 1 for the CTA's j-th tile
//   warps 2-5  epilogue; each frees its share of the buffer once its tcgen05.ld are done
// Barriers per TMEM buffer: tfull (one commit per tile) and tempty (one arrival per
// epilogue warp). Every wait is bounded; on an error each role stops, waits for its own
// copies or MMAs in flight, and the CTA frees its TMEM.
template <int MT>
__global__ void __launch_bounds__(kThreadsTC, 1) k_pi_w(const TCBasis* __restrict__ bases, int nb, int ntiles,
                                                       int stages, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared pointer
  const int R = bases[0].R;
  const int N = 2 * R;
  const int sbytes = ring_stage_bytes(R, MT);
  const int a_bytes = MT * kBM * kBK * 2;
  double* wt = reinterpret_cast<double*>(smem + stages * sbytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * sbytes + w_stage_bytes(R));
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;     // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int acc_cols = tmem_cols(N);
  const int ncols = 2 * MT * acc_cols;
  const int G = gridDim.x;
  const int nmine = (ntiles - static_cast<int>(blockIdx.x) + G - 1) / G;
  auto item_of = [&](int j) { return ntiles - 1 - (static_cast<int>(blockIdx.x) + j * G); };
  auto basis_of = [&](int item) { return find_owner(bases, nb, item, [](const TCBasis& b) { return b.wtile0; }); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 4); }
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;                        // k-steps issued (position in the ring)
      int cur = -1;
      bool ok = true;
      for (int j = 0; j < nmine && ok; ++j) {
        const int item = item_of(j);
        const int bi = basis_of(item);
        const TCBasis* B = bases + bi;
        if (bi != cur) { tmap_acquire(&B->mapHw); tmap_acquire(&B->mapY2); cur = bi; }
        const int tile = item - B->wtile0;
        const int nk = static_cast<int>((B->T + kBK - 1) / kBK);
        for (int i = 0; i < nk; ++i) {
          const int s = g % stages;
          const uint32_t u = static_cast<uint32_t>(g / stages);
          if (g >= stages && !mbar_wait(empty + s, (u & 1u) ^ 1u, err)) { ok = false; break; }
          unsigned char* As = smem + s * sbytes;
          mbar_expect_tx(full + s, static_cast<uint32_t>(sbytes));
#pragma unroll
          for (int h = 0; h < MT; ++h) {
            const int x = (tile * MT + h) * kBM;
            tma_load_2d(As + h * (kBM * kBK * 2), &B->mapHw, x, i * kBK, full + s);
            tma_load_2d(As + h * (kBM * kBK * 2) + kBM * kBK, &B->mapHw, x + 64, i * kBK, full + s);
          }
          tma_load_2d(As + a_bytes, &B->mapY2, i * kBK, 0, full + s);
          ++g;
        }
      }
      if (!ok) {
        // let the loads already issued land before the CTA can exit
        for (int i = (g > stages ? g - stages : 0); i < g; ++i)
          mbar_drain(full + (i % stages), static_cast<uint32_t>(i / stages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(N, 1, 0);
      int g = 0;
      bool ok = true;
      int last = -1;                    // the CTA's last tile whose accumulator was committed
      for (int j = 0; j < nmine && ok; ++j) {
        const int a = j & 1;
        if (j >= 2 && !mbar_wait(tempty + a, static_cast<uint32_t>((j >> 1) - 1) & 1u, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dacc = tmem + static_cast<uint32_t>(a * MT * acc_cols);
        const TCBasis* B = bases + basis_of(item_of(j));
        const int nk = static_cast<int>((B->T + kBK - 1) / kBK);
        for (int i = 0; i < nk; ++i) {
          const int s = g % stages;
          if (!mbar_wait(full + s, static_cast<uint32_t>(g / stages) & 1u, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * sbytes);
          const uint32_t b0 = a0 + static_cast<uint32_t>(a_bytes);
#pragma unroll
          for (int h = 0; h < MT; ++h)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              // A: MN-major 64 x 8 atoms, two along MN 8 KB apart (half h 16 KB on); B: K-major
              // rows of 128 B, the same for both halves
              mma_bf16(dacc + static_cast<uint32_t>(h * acc_cols), sdesc(a0 + h * 16384 + kk * 2048, 8192, 1024),
                       sdesc(b0 + kk * 32, 16, 1024), idesc, (i > 0 || kk > 0) ? 1u : 0u);
            }
          mma_commit(empty + s);
          ++g;
        }
        mma_commit(tfull + a);          // on an error too: it completes once the issued MMAs have
        last = j;
      }
      if (!ok && last >= 0) mbar_drain(tfull + (last & 1), static_cast<uint32_t>(last >> 1) & 1u);
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int tld = w_stage_ld(R);
    for (int j = 0; j < nmine; ++j) {
      const int a = j & 1;
      const bool mine = mbar_wait(tfull + a, static_cast<uint32_t>(j >> 1) & 1u, err);
      // one verdict for the four epilogue warps, so none waits at a barrier the others skip
      uint32_t all_ok;
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 1, 128, q;\n selp.u32 %0, 1, 0, p;\n}\n"
          : "=r"(all_ok)
          : "r"(static_cast<uint32_t>(mine))
          : "memory");
      if (all_ok == 0) break;
      tc_fence_after();
      const int item = item_of(j);
      const TCBasis* B = bases + basis_of(item);
      const int tile = item - B->wtile0;
      const bool gram = B->Gp != nullptr;
      const uint32_t tbase = tmem + static_cast<uint32_t>(a * MT * acc_cols) + (static_cast<uint32_t>(q * 32) << 16);
      if (!gram) {
#pragma unroll
        for (int h = 0; h < MT; ++h) {
          const uint32_t trow = tbase + static_cast<uint32_t>(h * acc_cols);
          const int64_t d = (static_cast<int64_t>(tile) * MT + h) * kBM + row;
          float* wrow = B->W + d * R;
          for (int c0 = 0; c0 < R; c0 += 16) {
            float hi[16], lo[16];
            tmem_ld16(trow + c0, hi);
            tmem_ld16(trow + R + c0, lo);
#pragma unroll
            for (int c = 0; c < 16; c += 4)
              if (d < B->D)
                *reinterpret_cast<float4*>(wrow + c0 + c) =
                    make_float4(hi[c] + lo[c], hi[c + 1] + lo[c + 1], hi[c + 2] + lo[c + 2], hi[c + 3] + lo[c + 3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + a);    // this warp's lanes of the buffer are read
        continue;
      }
      // R <= 64: half by half, each thread's row stays in registers for the Gram; the buffer
      // is released once the last half is read. The Gram runs over the tile's 32-row
      // quarters in row order, one epilogue warp's rows staged at a time (rows past D are
      // zero: the H box there is zero filled).
      TileGram gr(tld, R, B->nq, q, lane);
#pragma unroll 1
      for (int h = 0; h < MT; ++h) {
        const uint32_t trow = tbase + static_cast<uint32_t>(h * acc_cols);
        const int64_t d = (static_cast<int64_t>(tile) * MT + h) * kBM + row;
        const bool live = d < B->D;
        float* wrow = B->W + d * R;
        float w[64];
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          if (c0 < R) {
            float hi[16], lo[16];
            tmem_ld16(trow + c0, hi);
            tmem_ld16(trow + R + c0, lo);
#pragma unroll
            for (int c = 0; c < 16; ++c) w[c0 + c] = hi[c] + lo[c];
#pragma unroll
            for (int c = 0; c < 16; c += 4)
              if (live) *reinterpret_cast<float4*>(wrow + c0 + c) = make_float4(w[c0 + c], w[c0 + c + 1], w[c0 + c + 2], w[c0 + c + 3]);
          }
        }
        if (h == MT - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty + a);
        }
#pragma unroll 1
        for (int r = 0; r < 4; ++r) {
          if (q == r) {
            double* st = wt + lane * tld;
#pragma unroll
            for (int c = 0; c < 64; c += 2)
              if (c < R) *reinterpret_cast<double2*>(st + c) = make_double2(w[c], w[c + 1]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");   // the quarter is staged
          gr.rows(wt, tld, 32);
          asm volatile("bar.sync 1, 128;" ::: "memory");   // the staging region is free again
        }
      }
      gr.store(B->Gp + static_cast<int64_t>(tile) * B->nq * 64);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// Persistent Y2T = split(H [V_hi | V_lo]) for tiles of MT x 128 tokens: one CTA per SM, two
// TMEM accumulators (the epilogue of tile j overlaps the mainloop of tile j + 1), the ring
// running on across tiles, both halves' MMAs sharing each V stage. Tiles cost ceil(D / 64)
// k-steps, so bases of different widths make them uneven: with `sched` (built on the host,
// longest tiles first, each to the least-loaded CTA) CTA b takes the tiles
// sched[G + 1 + sched[b] .. G + 1 + sched[b + 1]); without it, tiles b, b + G, ...
// Roles, barriers and error handling as in k_pi_w.
template <int MT>
__global__ void __launch_bounds__(kThreadsTC, 1) k_pi_yp(const TCBasis* __restrict__ bases, int nb, int ntiles,
                                                        const int32_t* __restrict__ sched, int stages, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared pointer
  const int R = bases[0].R;
  const int N = 2 * R;
  const int sbytes = ring_stage_bytes(R, MT);
  const int a_bytes = MT * kBM * kBK * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * sbytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;     // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int acc_cols = tmem_cols(N);
  const int ncols = 2 * MT * acc_cols;
  const int G = gridDim.x;
  const int b = static_cast<int>(blockIdx.x);
  const int first = sched ? sched[b] : 0;
  const int nmine = sched ? sched[b + 1] - first : (ntiles - b + G - 1) / G;
  auto item_of = [&](int j) { return sched ? sched[G + 1 + first + j] : b + j * G; };
  auto basis_of = [&](int item) { return find_owner(bases, nb, item, [](const TCBasis& c) { return c.ytile0; }); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 4); }
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      int cur = -1;
      bool ok = true;
      for (int j = 0; j < nmine && ok; ++j) {
        const int item = item_of(j);
        const int bi = basis_of(item);
        const TCBasis* B = bases + bi;
        if (bi != cur) { tmap_acquire(&B->mapHy); tmap_acquire(&B->mapV2); cur = bi; }
        const int tile = item - B->ytile0;
        const int nk = static_cast<int>((B->D + kBK - 1) / kBK);
        for (int i = 0; i < nk; ++i) {
          const int s = g % stages;
          const uint32_t u = static_cast<uint32_t>(g / stages);
          if (g >= stages && !mbar_wait(empty + s, (u & 1u) ^ 1u, err)) { ok = false; break; }
          unsigned char* As = smem + s * sbytes;
          mbar_expect_tx(full + s, static_cast<uint32_t>(sbytes));
#pragma unroll
          for (int h = 0; h < MT; ++h)
            tma_load_2d(As + h * (kBM * kBK * 2), &B->mapHy, i * kBK, (tile * MT + h) * kBM, full + s);
          tma_load_2d(As + a_bytes, &B->mapV2, i * kBK, 0, full + s);
          ++g;
        }
      }
      if (!ok) {
        for (int i = (g > stages ? g - stages : 0); i < g; ++i)
          mbar_drain(full + (i % stages), static_cast<uint32_t>(i / stages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(N, 0, 0);
      int g = 0;
      bool ok = true;
      int last = -1;
      for (int j = 0; j < nmine && ok; ++j) {
        const int a = j & 1;
        if (j >= 2 && !mbar_wait(tempty + a, static_cast<uint32_t>((j >> 1) - 1) & 1u, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dacc = tmem + static_cast<uint32_t>(a * MT * acc_cols);
        const TCBasis* B = bases + basis_of(item_of(j));
        const int nk = static_cast<int>((B->D + kBK - 1) / kBK);
        for (int i = 0; i < nk; ++i) {
          const int s = g % stages;
          if (!mbar_wait(full + s, static_cast<uint32_t>(g / stages) & 1u, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * sbytes);
          const uint32_t b0 = a0 + static_cast<uint32_t>(a_bytes);
#pragma unroll
          for (int h = 0; h < MT; ++h)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)   // A and B: K-major rows of 128 B (half h 16 KB on)
              mma_bf16(dacc + static_cast<uint32_t>(h * acc_cols), sdesc(a0 + h * 16384 + kk * 32, 16, 1024),
                       sdesc(b0 + kk * 32, 16, 1024), idesc, (i > 0 || kk > 0) ? 1u : 0u);
          mma_commit(empty + s);
          ++g;
        }
        mma_commit(tfull + a);
        last = j;
      }
      if (!ok && last >= 0) mbar_drain(tfull + (last & 1), static_cast<uint32_t>(last >> 1) & 1u);
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    for (int j = 0; j < nmine; ++j) {
      const int a = j & 1;
      const bool mine = mbar_wait(tfull + a, static_cast<uint32_t>(j >> 1) & 1u, err);
      uint32_t all_ok;
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 1, 128, q;\n selp.u32 %0, 1, 0, p;\n}\n"
          : "=r"(all_ok)
          : "r"(static_cast<uint32_t>(mine))
          : "memory");
      if (all_ok == 0) break;
      tc_fence_after();
      const int item = item_of(j);
      const TCBasis* B = bases + basis_of(item);
      const int tile = item - B->ytile0;
      const uint32_t tbase = tmem + static_cast<uint32_t>(a * MT * acc_cols) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int h = 0; h < MT; ++h) {
        const int64_t t = (static_cast<int64_t>(tile) * MT + h) * kBM + row;
        for (int c0 = 0; c0 < R; c0 += 16) {
          float hi[16], lo[16];
          tmem_ld16(tbase + static_cast<uint32_t>(h * acc_cols) + c0, hi);
          tmem_ld16(tbase + static_cast<uint32_t>(h * acc_cols) + R + c0, lo);
          if (t < B->T) {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const float y = hi[c] + lo[c];
              const __nv_bfloat16 yh = __float2bfloat16_rn(y);
              const __nv_bfloat16 yl = __float2bfloat16_rn(y - __bfloat162float(yh));
              B->Y2T[static_cast<int64_t>(c0 + c) * B->ldy2 + t] = yh;
              B->Y2T[static_cast<int64_t>(R + c0 + c) * B->ldy2 + t] = yl;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + a);    // this warp's lanes of the buffer are read
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// Sums the fused W Gram's per-tile partials of every basis (fixed order over the tiles)
// into the basis's Gram, the first partial slot of its W table (r x r, mirrored): per
// CTA 256 entries of the block-major partial; gpb CTAs per basis.
__global__ void __launch_bounds__(kThreads) k_gsum(const TCBasis* __restrict__ bases, Tables tb,
                                                   const MatD* __restrict__ wA, int gpb) {
  const int bi = blockIdx.x / gpb, blk = blockIdx.x - bi * gpb;
  const TCBasis* B = bases + bi;
  const int e = blk * kThreads + threadIdx.x;
  if (e >= B->nq * 64) return;
  const int R = B->R, nb = R >> 3;
  int q = e >> 6, rb = 0;
  while (q >= nb - rb) { q -= nb - rb; ++rb; }
  const int row = 8 * rb + ((e & 63) >> 3), col = 8 * (rb + q) + (e & 7);
  if (q == 0 && row > col) return;                    // diagonal block: its upper half suffices
  const double* p = B->Gp + e;
  const int64_t st = static_cast<int64_t>(B->nq) * 64;
  constexpr int kU = 8;                               // independent loads in flight
  double acc[kU];
#pragma unroll
  for (int u = 0; u < kU; ++u) acc[u] = 0.0;
  int t = 0;
  for (; t + kU <= B->nwtile; t += kU) {
#pragma unroll
    for (int u = 0; u < kU; ++u) acc[u] += p[(t + u) * st];
  }
  for (; t < B->nwtile; ++t) acc[0] += p[t * st];
  const double sum = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
  double* G = reinterpret_cast<double*>(tb.ws) + wA[bi].gram_off;
  G[row * R + col] = sum;
  G[col * R + row] = sum;
}

// [V_hi | V_lo]^T (2R x D bf16) from the fp32 basis, grouped over bases: one CTA per tile of
// kSplitD vectors. The tile's rows are read coalesced into shared memory (pitch R + 1), and
// each thread writes eight consecutive vectors of one component as two 16-byte stores.
constexpr int kSplitD = 64;
__global__ void __launch_bounds__(kThreads) k_split_vt(const TCBasis* __restrict__ bases, int nb, int first) {
  __shared__ float tile[kSplitD * (DSMZ_MAX_RANK + 1)];
  const int item = blockIdx.x;
  const int bi = find_owner(bases, nb, item, [](const TCBasis& b) { return b.vt0; });
  const TCBasis* B = bases + bi;
  const int R = B->R, tp = R + 1;
  const int64_t d0 = static_cast<int64_t>(item - B->vt0) * kSplitD;
  const int nd = static_cast<int>(min(static_cast<int64_t>(kSplitD), B->D - d0));
  const int64_t s0 = first ? B->v_s0 : R, s1 = first ? B->v_s1 : 1;
  const float* V = first ? B->Vsrc : B->Vout;
  for (int e = threadIdx.x; e < nd * R; e += kThreads) {
    const int d = e / R, r = e - d * R;
    tile[d * tp + r] = V[(d0 + d) * s0 + r * s1];
  }
  __syncthreads();
  const int nu = R * (nd >> 3);                       // eight vectors per unit
  for (int u = threadIdx.x; u < nu; u += kThreads) {
    const int r = u / (nd >> 3), j = (u - r * (nd >> 3)) * 8;
    uint32_t h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float x0 = tile[(j + 2 * q) * tp + r], x1 = tile[(j + 2 * q + 1) * tp + r];
      const __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
      const float2 hf = __bfloat1622float2(hh);
      const __nv_bfloat162 ll = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
      h[q] = *reinterpret_cast<const uint32_t*>(&hh);
      l[q] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    *reinterpret_cast<uint4*>(B->V2T + static_cast<int64_t>(r) * B->ldv2 + d0 + j) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(B->V2T + static_cast<int64_t>(R + r) * B->ldv2 + d0 + j) = make_uint4(l[0], l[1], l[2], l[3]);
  }
  for (int e = (nd & ~7) + threadIdx.x % 8; e < nd; e += 8) {   // ragged tail (D % 8 != 0)
    for (int r = threadIdx.x / 8; r < R; r += kThreads / 8) {
      const float x = tile[e * tp + r];
      const __nv_bfloat16 hh = __float2bfloat16_rn(x);
      B->V2T[static_cast<int64_t>(r) * B->ldv2 + d0 + e] = hh;
      B->V2T[static_cast<int64_t>(R + r) * B->ldv2 + d0 + e] = __float2bfloat16_rn(x - __bfloat162float(hh));
    }
  }
}

}  // namespace tc
}  // namespace dsmz
