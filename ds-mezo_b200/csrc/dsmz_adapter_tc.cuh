// Perturbation of the adapter phase on the tensor cores (controller.py:178-193, 241-248,
// 262-270; ds_mezo/kernels.py:290-368, 399-412), for r <= 64 and a basis width <= 64.
//
// A tile is 128 vectors of one matrix (rows of a tall A, columns of a wide B). Its z^T /
// eps is a 128 x r product D = X C^T with K = the draw width: X the tile's K rows (Zc_A
// rows, or basis rows), C the module side's coefficient matrix (Q, or Zc_B * sqrt(var_B
// V^2)). Both are fp32; each is split into a tf32 pair (x = hi + lo, hi = tf32(x), lo
// exact) and D = X_hi C_hi^T + X_hi C_lo^T + X_lo C_hi^T on tcgen05 (kind::tf32, fp32
// accumulation in TMEM): the dropped X_lo C_lo^T and lo's own tf32 rounding are below 2^-21
// of each product term. TMEM lane v holds vector v; the group moves z into shared memory in
// the matrix's own element order, then streams the tile's fp32 master, momentum and
// variance from global memory in that order (16-byte units, coalesced) and writes z, pos,
// neg and the Kalman partials.
//
// Warps: 0 TMA producer (one lane); 1 spare; 2-9 two groups of four (one warp per TMEM lane
// quadrant) that take alternate tiles: wait for the tile, split it (hi in the stage, lo in
// the group's buffer), issue its MMAs (one thread), wait for them, release the stage, run
// the epilogue. Every wait is bounded (error word); TMEM is freed at exit after in-flight
// MMAs land.
#pragma once

#include "dsmz_stream.cuh"
#include "dsmz_tc.cuh"

namespace dsmz {
namespace atc {

constexpr int kTile = 128;                 // vectors per tile (MMA M)
constexpr int kGroups = 2;                 // epilogue groups of four warps
constexpr int kThreads = 32 * (2 + 4 * kGroups);
constexpr int kBarGroup0 = 6;              // named barriers 6, 7

struct PLayout {
  int S;                // stages (one TMA'd tile of K rows each)
  int nbk;              // 32-column boxes of the K rows (K <= 64: 1 or 2)
  int npad;             // r rounded up to 16 (MMA N)
  int stage_bytes;      // nbk * 16 KB
  int o_lo, lo_bytes;   // per group: lo half of the tile
  int o_c, c_bytes;     // per group: [C_hi | C_lo] images (npad rows)
  int o_red, o_bar;
  int total;
};

// Stages: as many as fit in `budget` bytes beside the fixed buffers, 2 to 6.
__host__ __device__ inline PLayout perturb_layout(int r, int KW, int budget) {
  PLayout L{};
  L.nbk = (KW + 31) / 32;
  L.npad = (r + 15) & ~15;
  L.stage_bytes = L.nbk * kTile * 128;
  L.lo_bytes = L.stage_bytes > kTile * L.npad * 4 ? L.stage_bytes : kTile * L.npad * 4;   // lo half, then the z tile
  L.c_bytes = 2 * L.nbk * L.npad * 128;
  const int fixed = kGroups * L.lo_bytes + kGroups * ((L.c_bytes + 1023) & ~1023) + 2048;
  L.S = (budget - fixed) / L.stage_bytes;
  L.S = L.S > 6 ? 6 : L.S;
  int o = L.S * L.stage_bytes;
  L.o_lo = o;   o += kGroups * L.lo_bytes;
  L.o_c = o;    o += kGroups * ((L.c_bytes + 1023) & ~1023);
  L.o_red = o;  o += 8 * 2 * 8 * 4 + 128;
  L.o_bar = o;  o += 8 * (2 * L.S + kGroups) + 16;
  L.total = o + 1024;
  return L;
}
// r padded to 16, 32 or 64 (the z tile's 16-byte chunks swizzle within groups of eight)
__host__ __device__ inline bool perturb_ok(int r, int KW) {
  return r >= 1 && r <= 64 && ((r + 15) & ~15) != 48 && KW >= 1 && KW <= 64;
}

using dsmz::GatherPeers;
using dsmz::kMaxPeers;

// the tile's matrix: last m with tt[m] <= t
__device__ __forceinline__ int tile_owner(const int32_t* tt, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tt[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int FES>
__global__ void __launch_bounds__(kThreads, 1) k_perturb_tc(Tables tb, const int32_t* __restrict__ ttab, int ntiles,
                                                            int nsegs, PLayout L, float eps, KalmanIn kin,
                                                            GatherPeers gp, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = sk::aligned_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + L.S;
  uint64_t* mbar = empty + L.S;                         // per group: its MMAs landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + kGroups);
  double* red = reinterpret_cast<double*>(smem + L.o_red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncols = tc::tmem_cols(kGroups * L.npad);
  if (threadIdx.x == 0) {
    for (int s = 0; s < L.S; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 4); }
    for (int g = 0; g < kGroups; ++g) mbar_init(mbar + g, 1);
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(static_cast<uint32_t>(ncols))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // this CTA's tiles: a contiguous range of the global tile list
  const int64_t G = gridDim.x, b = blockIdx.x;
  const int t0 = static_cast<int>((b * ntiles) / G), t1 = static_cast<int>(((b + 1) * ntiles) / G);

  if (warp == 0) {
    if (lane == 0) {
      int cur = -1;
      const CUtensorMap* map = nullptr;
      int64_t nvec = 0;
      int j = 0;
      for (int t = t0; t < t1; ++t, ++j) {
        const int s = j % L.S;
        if (j >= L.S && !mbar_wait(empty + s, (static_cast<uint32_t>(j / L.S) & 1u) ^ 1u, err)) {
          // the consumers stopped: drain what is in flight and leave
          for (int i = (j > L.S ? j - L.S : 0); i < j; ++i)
            mbar_drain(full + (i % L.S), static_cast<uint32_t>(i / L.S) & 1u);
          j = -1;
          break;
        }
        const int mi = tile_owner(ttab, tb.nmats, t);
        if (mi != cur) {
          const MatD& M = tb.mats[mi];
          map = tb.smaps + M.kmap;
          tmap_acquire(map);
          nvec = M.nvec;
          cur = mi;
        }
        (void)nvec;
        const int row0 = (t - ttab[mi]) * kTile;
        unsigned char* st = smem + s * L.stage_bytes;
        mbar_expect_tx(full + s, static_cast<uint32_t>(L.stage_bytes));
        for (int k = 0; k < L.nbk; ++k) tma_load_2d(st + k * kTile * 128, map, 32 * k, row0, full + s);
      }
      if (j > 0)
        for (int i = (j > L.S ? j - L.S : 0); i < j; ++i) mbar_drain(full + (i % L.S), static_cast<uint32_t>(i / L.S) & 1u);
    }
  } else if (warp >= 2) {
    const int gw = warp - 2, grp = gw / 4, gt = gw % 4 * 32 + lane;   // group thread 0..127
    const int q = warp & 3;                                            // TMEM lane quadrant
    const int v = 32 * q + lane;                                       // this thread's vector in the tile
    unsigned char* lo = smem + L.o_lo + grp * L.lo_bytes;
    unsigned char* cimg = smem + L.o_c + grp * ((L.c_bytes + 1023) & ~1023);
    const uint32_t acc = tmem + static_cast<uint32_t>(grp * L.npad);
    const uint32_t idesc = tc::idesc_tf32(L.npad);
    float s_zmu = 0.f, s_zzv = 0.f;
    uint32_t mphase = 0;
    bool dead = false, pending = false;
    int cur = -1;
    int j = 0;
    for (int t = t0; t < t1 && !dead; ++t, ++j) {
      if ((j % kGroups) != grp) continue;
      const int s = j % L.S;
      const bool w = mbar_wait(full + s, static_cast<uint32_t>(j / L.S) & 1u, err);
      dead = !sk::agree(kBarGroup0 + grp, 128, w);
      if (dead) break;
      const int mi = tile_owner(ttab, tb.nmats, t);
      // the matrix's fields in registers (the stores below could alias the tables as far as
      // the compiler can tell, which would reload them every unit)
      const MatD& Mg = tb.mats[mi];
      const int side = Mg.side;
      const int r = static_cast<int>(Mg.r);
      const int64_t mnvec = Mg.nvec, ld = Mg.ld;
      const float* pm = reinterpret_cast<const float*>(Mg.param);   // the fp32 master
      const float* mup = Mg.mu;
      const float* vap = Mg.var;
      float* const zbase = Mg.z;
      char* const posbase = reinterpret_cast<char*>(Mg.pos);
      char* const negbase = reinterpret_cast<char*>(Mg.neg);
      const ModD& D = tb.mods[Mg.owner];
      const int KW = (side == 0) ? D.rca : D.rc;
      if (mi != cur) {
        // C of this module side (r x KW, row c), split into [C_hi | C_lo]: npad rows each
        const float* coef = reinterpret_cast<const float*>(tb.ws) + D.coef_off;
        const float* Cm = (side == 0) ? coef + static_cast<int64_t>(D.r) * D.rc : coef;
        const int cld = (side == 0) ? D.rca : D.rc;
        const int wdt = 32 * L.nbk, half = L.nbk * L.npad * 128;
        for (int e = gt; e < L.npad * wdt; e += 128) {
          const int c = e / wdt, k = e - c * wdt;
          const float x = (c < r && k < KW) ? Cm[c * cld + k] : 0.f;
          const float h = tc::tf32_hi(x);
          const int o = sk::swz_off(c, k, L.npad);
          *reinterpret_cast<float*>(cimg + o) = h;
          *reinterpret_cast<float*>(cimg + half + o) = x - h;
        }
        cur = mi;
      }
      // the tile's K rows: hi in place, lo into the group's buffer
      unsigned char* hi = smem + s * L.stage_bytes;
      for (int o = gt * 16; o < L.stage_bytes; o += 128 * 16) {
        const float4 x = *reinterpret_cast<const float4*>(hi + o);
        const float4 h = make_float4(tc::tf32_hi(x.x), tc::tf32_hi(x.y), tc::tf32_hi(x.z), tc::tf32_hi(x.w));
        *reinterpret_cast<float4*>(hi + o) = h;
        *reinterpret_cast<float4*>(lo + o) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
      }
      tc::fence_proxy_async_smem();
      named_sync(kBarGroup0 + grp, 128);
      if (gt == 0) {
        tc::tc_fence_after();
        const uint32_t ah = smem_u32(hi), al = smem_u32(lo), ch = smem_u32(cimg);
        const uint32_t cl = ch + static_cast<uint32_t>(L.nbk * L.npad * 128);
        const int nk = (KW + 7) / 8;
        for (int kk = 0; kk < nk; ++kk) {
          const uint32_t xo = static_cast<uint32_t>((kk >> 2) * kTile * 128 + (kk & 3) * 32);
          const uint32_t co = static_cast<uint32_t>((kk >> 2) * L.npad * 128 + (kk & 3) * 32);
          tc::mma_tf32(acc, tc::sdesc(ah + xo, 16, 1024), tc::sdesc(ch + co, 16, 1024), idesc, kk > 0 ? 1u : 0u);
          tc::mma_tf32(acc, tc::sdesc(ah + xo, 16, 1024), tc::sdesc(cl + co, 16, 1024), idesc, 1u);
          tc::mma_tf32(acc, tc::sdesc(al + xo, 16, 1024), tc::sdesc(ch + co, 16, 1024), idesc, 1u);
        }
        tc::mma_commit(mbar + grp);
      }
      // the tile's elements in memory order, four per unit (16 bytes): master, momentum and
      // variance in, z, pos, neg and the Kalman partials out. kU units per thread per batch;
      // the first batch's loads are issued while the MMAs run.
      const int64_t s0 = static_cast<int64_t>(t - ttab[mi]) * kTile;
      const int nv = static_cast<int>(min(static_cast<int64_t>(kTile), mnvec - s0));
      const int nch = L.npad / 4, sw = (nch < 8 ? nch : 8) - 1;
      const int upr = (side == 0) ? nch : kTile / 4;              // units per tile row (a power of 2)
      const int ush = 31 - __clz(upr);
      const int nunits = ((side == 0) ? nv : r) * upr;
      constexpr int kU = 8;
      float4 P[kU], Mu[kU], W[kU];
      auto unit = [&](int u, int& row, int& col, int64_t& g) {
        row = u >> ush;
        col = u & (upr - 1);
        g = (side == 0) ? (s0 + row) * ld + 4 * col : static_cast<int64_t>(row) * ld + s0 + 4 * col;
        return u < nunits && (side == 0 ? 4 * col < r : 4 * col < nv);
      };
      auto load = [&](int u0) {
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          int row, col;
          int64_t g;
          if (unit(u0 + k * 128, row, col, g)) {
            P[k] = __ldg(reinterpret_cast<const float4*>(pm + g));
            Mu[k] = __ldg(reinterpret_cast<const float4*>(mup + g));
            W[k] = __ldg(reinterpret_cast<const float4*>(vap + g));
          }
        }
      };
      load(gt);
      pending = true;
      const bool wm = mbar_wait(mbar + grp, mphase & 1u, err);
      dead = !sk::agree(kBarGroup0 + grp, 128, wm);
      if (dead) break;
      pending = false;
      ++mphase;
      tc::tc_fence_after();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);             // the MMAs have read the stage
      // z = eps D into the group's lo buffer (free now) in the matrix's memory order: side 0
      // row-major [v][c] with 16-byte chunks swizzled by the row, side 1 [c][v]
      float* zs = reinterpret_cast<float*>(lo);
      const uint32_t trow = acc + (static_cast<uint32_t>(32 * q) << 16);
      for (int c0 = 0; c0 < L.npad; c0 += 16) {
        float zz[16];
        tc::tmem_ld16(trow + c0, zz);
        if (side == 0) {
#pragma unroll
          for (int u = 0; u < 16; u += 4) {
            const int ch = (c0 + u) >> 2;
            *reinterpret_cast<float4*>(zs + v * L.npad + 4 * (ch ^ (v & sw))) =
                make_float4(zz[u] * eps, zz[u + 1] * eps, zz[u + 2] * eps, zz[u + 3] * eps);
          }
        } else {
#pragma unroll
          for (int u = 0; u < 16; ++u) zs[(c0 + u) * kTile + v] = zz[u] * eps;
        }
      }
      tc::tc_fence_before();
      named_sync(kBarGroup0 + grp, 128);
      float* zt = zbase + static_cast<int64_t>(tb.dir) * tb.dstride_z;
      const int64_t fo = static_cast<int64_t>(tb.dir) * tb.dstride_f * FES;
      char* posb = posbase + fo;
      char* negb = negbase + fo;
      for (int u0 = gt; u0 < nunits; u0 += 128 * kU) {
        if (u0 != gt) load(u0);
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          int row, col;
          int64_t g;
          if (!unit(u0 + k * 128, row, col, g)) continue;
          const float4 z4 = (side == 0)
              ? *reinterpret_cast<const float4*>(zs + row * L.npad + 4 * (col ^ (row & sw)))
              : *reinterpret_cast<const float4*>(zs + row * kTile + 4 * col);
          *reinterpret_cast<float4*>(zt + g) = z4;
          const float4 pv = make_float4(__fadd_rn(P[k].x, z4.x), __fadd_rn(P[k].y, z4.y),
                                        __fadd_rn(P[k].z, z4.z), __fadd_rn(P[k].w, z4.w));
          const float4 nv4 = make_float4(__fsub_rn(P[k].x, z4.x), __fsub_rn(P[k].y, z4.y),
                                         __fsub_rn(P[k].z, z4.z), __fsub_rn(P[k].w, z4.w));
          sk::st_fac4<FES>(posb, g, pv);
          sk::st_fac4<FES>(negb, g, nv4);
#pragma unroll
          for (int pp = 0; pp < kMaxPeers; ++pp) {     // the peers' copies of this shard
            if (pp >= gp.n) break;
            sk::st_fac4<FES>(posb + gp.dpos[pp], g, pv);
            sk::st_fac4<FES>(negb + gp.dneg[pp], g, nv4);
          }
          const float z[4] = {z4.x, z4.y, z4.z, z4.w};
          const float mv[4] = {Mu[k].x, Mu[k].y, Mu[k].z, Mu[k].w}, wv[4] = {W[k].x, W[k].y, W[k].z, W[k].w};
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const float mu1 = __fmul_rn(mv[qq], kin.beta);
            const float var1 = __fadd_rn(__fmul_rn(wv[qq], kin.beta2), kin.q);
            s_zmu = fmaf(z[qq], mu1, s_zmu);
            s_zzv = fmaf(__fmul_rn(z[qq], z[qq]), var1, s_zzv);
          }
        }
      }
      tc::tc_fence_before();
      named_sync(kBarGroup0 + grp, 128);                 // TMEM, lo and C are free again
    }
    if (pending && gt == 0) mbar_drain(mbar + grp, mphase & 1u);
    // the CTA's Kalman partials (fixed order): warps 2..9, then CTA 0 clears the slots past
    // the grid (the reduction sums every segment slot)
    double a = s_zmu, bb = s_zzv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      bb += __shfl_xor_sync(0xffffffffu, bb, o);
    }
    if (lane == 0) { red[2 * gw] = a; red[2 * gw + 1] = bb; }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (threadIdx.x == 0) {
    double sa = 0.0, sb = 0.0;
    for (int w = 0; w < 4 * kGroups; ++w) { sa += red[2 * w]; sb += red[2 * w + 1]; }
    double* out = reinterpret_cast<double*>(tb.ws) + tb.seg_kal_off;
    out[2 * b] = sa;
    out[2 * b + 1] = sb;
    if (b == 0)
      for (int i = static_cast<int>(G); i < nsegs; ++i) { out[2 * i] = 0.0; out[2 * i + 1] = 0.0; }
  }
  if (gp.n > 0) __threadfence_system();               // the peer stores precede this rank's next collective
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(static_cast<uint32_t>(ncols))
                 : "memory");
}

}  // namespace atc
}  // namespace dsmz
