// Perturbation of the adapter phase on the tensor cores (controller.py:178-193, 241-248,
// 262-270; ds_mezo/kernels.py:290-368, 399-412), for r <= 64 and a basis width <= 64.
//
// A tile is 128 vectors of one matrix (rows of a tall A, columns of a wide B). Its z^T /
// eps is a 128 x r product D = X C^T with K = the draw width: X the tile's K rows (Zc_A
// rows, or basis rows), C the module side's coefficient matrix (Q, or Zc_B * sqrt(var_B
// V^2)). Both are fp32; each is split into a tf32 pair (x = hi + lo, hi = tf32(x), lo
// exact) and D = X_hi C_hi^T + X_hi C_lo^T + X_lo C_hi^T on tcgen05 (kind::tf32, fp32
// accumulation in TMEM): the dropped X_lo C_lo^T and lo's own tf32 rounding are below 2^-21
// of each product term. TMEM lane v holds vector v, so the epilogue thread of vector v
// reads its r values of z and streams the vector's fp32 master, momentum and variance
// straight from global memory (a warp covers 32 consecutive vectors: consecutive columns
// of a wide B, coalesced; rows of a tall A, 16-byte vectors along the row) and writes z,
// pos, neg and the Kalman partials.
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
  L.lo_bytes = L.stage_bytes;
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
__host__ __device__ inline bool perturb_ok(int r, int KW) { return r >= 1 && r <= 64 && KW >= 1 && KW <= 64; }

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
                                                            int nsegs, PLayout L, float eps, KalmanIn kin, int* err) {
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
      const MatD& M = tb.mats[mi];
      const ModD& D = tb.mods[M.owner];
      const int r = static_cast<int>(M.r);
      const int KW = (M.side == 0) ? D.rca : D.rc;
      if (mi != cur) {
        // C of this module side (r x KW, row c), split into [C_hi | C_lo]: npad rows each
        const float* coef = reinterpret_cast<const float*>(tb.ws) + D.coef_off;
        const float* Cm = (M.side == 0) ? coef + static_cast<int64_t>(D.r) * D.rc : coef;
        const int cld = (M.side == 0) ? D.rca : D.rc;
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
      // the vector's master, momentum and variance, 16 components per chunk: each chunk's
      // loads are issued together one chunk ahead (the first while the MMAs run), so a
      // thread has up to 96 values in flight
      const int64_t s0 = static_cast<int64_t>(t - ttab[mi]) * kTile;
      const bool live = s0 + v < M.nvec;
      const int64_t ld = M.ld;
      const float* pm = reinterpret_cast<const float*>(M.param);   // the fp32 master
      const float* mup = M.mu;
      const float* vap = M.var;
      auto gidx = [&](int c) -> int64_t {
        return M.side == 0 ? (s0 + v) * ld + c : static_cast<int64_t>(c) * ld + s0 + v;
      };
      auto load = [&](int c0, float (&P)[16], float (&Mu)[16], float (&W)[16]) {
        if (!live) return;
        if (M.side == 0) {
#pragma unroll
          for (int u = 0; u < 16; u += 4) {
            if (c0 + u >= r) continue;
            const int64_t g = gidx(c0 + u);
            const float4 p4 = __ldg(reinterpret_cast<const float4*>(pm + g));
            const float4 m4 = __ldg(reinterpret_cast<const float4*>(mup + g));
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(vap + g));
            P[u] = p4.x; P[u + 1] = p4.y; P[u + 2] = p4.z; P[u + 3] = p4.w;
            Mu[u] = m4.x; Mu[u + 1] = m4.y; Mu[u + 2] = m4.z; Mu[u + 3] = m4.w;
            W[u] = w4.x; W[u + 1] = w4.y; W[u + 2] = w4.z; W[u + 3] = w4.w;
          }
        } else {
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            if (c0 + u >= r) continue;
            const int64_t g = gidx(c0 + u);
            P[u] = __ldg(pm + g);
            Mu[u] = __ldg(mup + g);
            W[u] = __ldg(vap + g);
          }
        }
      };
      float Pc[16], Mc[16], Wc[16];
      load(0, Pc, Mc, Wc);
      pending = true;
      const bool wm = mbar_wait(mbar + grp, mphase & 1u, err);
      dead = !sk::agree(kBarGroup0 + grp, 128, wm);
      if (dead) break;
      pending = false;
      ++mphase;
      tc::tc_fence_after();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);             // the MMAs have read the stage
      // epilogue: vector v of the tile
      float* zt = M.z + static_cast<int64_t>(tb.dir) * tb.dstride_z;
      const int64_t fo = static_cast<int64_t>(tb.dir) * tb.dstride_f * FES;
      char* posb = reinterpret_cast<char*>(M.pos) + fo;
      char* negb = reinterpret_cast<char*>(M.neg) + fo;
      const uint32_t trow = acc + (static_cast<uint32_t>(32 * q) << 16);
      for (int c0 = 0; c0 < L.npad; c0 += 16) {
        float Pn[16], Mn[16], Wn[16];
        if (c0 + 16 < r) load(c0 + 16, Pn, Mn, Wn);
        float zz[16];
        tc::tmem_ld16(trow + c0, zz);
        if (live) {
          if (M.side == 0) {
            const int64_t g0 = gidx(c0);
#pragma unroll
            for (int u = 0; u < 16; u += 4) {
              if (c0 + u >= r) continue;
              const int64_t g = g0 + u;
              const float z[4] = {zz[u] * eps, zz[u + 1] * eps, zz[u + 2] * eps, zz[u + 3] * eps};
              *reinterpret_cast<float4*>(zt + g) = make_float4(z[0], z[1], z[2], z[3]);
              sk::st_fac4<FES>(posb, g, make_float4(__fadd_rn(Pc[u], z[0]), __fadd_rn(Pc[u + 1], z[1]),
                                                    __fadd_rn(Pc[u + 2], z[2]), __fadd_rn(Pc[u + 3], z[3])));
              sk::st_fac4<FES>(negb, g, make_float4(__fsub_rn(Pc[u], z[0]), __fsub_rn(Pc[u + 1], z[1]),
                                                    __fsub_rn(Pc[u + 2], z[2]), __fsub_rn(Pc[u + 3], z[3])));
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                const float mu1 = __fmul_rn(Mc[u + qq], kin.beta);
                const float var1 = __fadd_rn(__fmul_rn(Wc[u + qq], kin.beta2), kin.q);
                s_zmu = fmaf(z[qq], mu1, s_zmu);
                s_zzv = fmaf(__fmul_rn(z[qq], z[qq]), var1, s_zzv);
              }
            }
          } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              if (c0 + u >= r) continue;
              const int64_t g = gidx(c0 + u);
              const float z = zz[u] * eps;
              zt[g] = z;
              sk::st_fac<FES>(posb, g, __fadd_rn(Pc[u], z));
              sk::st_fac<FES>(negb, g, __fsub_rn(Pc[u], z));
              const float mu1 = __fmul_rn(Mc[u], kin.beta);
              const float var1 = __fadd_rn(__fmul_rn(Wc[u], kin.beta2), kin.q);
              s_zmu = fmaf(z, mu1, s_zmu);
              s_zzv = fmaf(__fmul_rn(z, z), var1, s_zzv);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) { Pc[u] = Pn[u]; Mc[u] = Mn[u]; Wc[u] = Wn[u]; }
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
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(static_cast<uint32_t>(ncols))
                 : "memory");
}

}  // namespace atc
}  // namespace dsmz
