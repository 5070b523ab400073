// Single-pass tensor-core power iteration on sm_100a: W = H^T (H V) for every basis with
// each activation read from HBM once per iteration (ds_mezo/kernels.py:214-225 streams each
// token tile once per iteration and forms both products on it).
//
// Every CTA (one per SM) runs two independent pipelines, each with its own TMA producer,
// MMA issuer, epilogue warps, shared-memory ring and half of TMEM:
//   Y pipeline: items of the Y queue, Y(b, tile, [k0, k1)) = 256 tokens x 2R of H V over d
//       k-steps [k0, k1), H streamed from HBM (kept in L2 with an evict_last hint). A tile
//       split over several items writes fp32 partials into a ring of slots; the item that
//       completes the tile (last arrival on its counter) sums them in split order
//       (deterministic), writes the tile's [Y_hi | Y_lo]^T and raises the tile's flag.
//   W pipeline: items of the W queue, W(b, dtile) = 256 d-rows x 2R of H^T Y over all of the
//       basis's tokens; before each 256-token tile it waits for that tile's flag, then
//       re-reads the tile's activations from L2 (evict_first), and it ends with the W rows
//       and the tile's fused fp64 Gram.
// The Y queue interleaves the bases of a window token tile by token tile, so each basis's
// tiles complete at a pace its W items (fewer, longer) can follow while the tiles are in L2.
// A waiting W pipeline never holds up the Y pipeline: Y items wait only for earlier Y tiles
// (partial-slot reuse), W items only for Y tiles, so the kernel cannot deadlock. Every wait
// is bounded all the same (globaltimer, ~1 s, error word).
//
// Warps (384 threads): 0 Y producer, 1 W producer, 2 TMEM owner + Y MMA issuer, 3 W MMA
// issuer, 4-7 Y epilogue, 8-11 W epilogue. TMEM: Y accumulators (two 128-row halves, 2R
// columns each) in columns [0, 256), W accumulators in [256, 512); R <= 64.
#pragma once

#include "dsmz_tc.cuh"

namespace dsmz {
namespace tc {

struct PiItem {
  int32_t basis;
  int32_t tile;       // Y: 256-token tile of the basis; W: 256-row d tile of the basis
  int32_t k0, k1;     // Y: d k-steps [k0, k1); W: token k-steps [k0, k1) (64 each)
  int32_t ytile;      // Y: global id of its token tile; W: global id of the basis's token tile 0
  int32_t nsplit;     // Y: items the tile is split into (1: no partials)
  int32_t ks;         // Y: this item's split index
  int32_t slot;       // Y: this item's partial slot
  int32_t slot0;      // Y: partial slot of split 0 (split k uses (slot0 + k) mod the ring size)
  int32_t wait_tile;  // Y: global tile whose reduction frees this item's partial slot (-1: none)
  int32_t end;        // 1: no more items
  int32_t pad[5];
};

struct PiSync {       // launch-local state in the workspace (counters zeroed before every launch)
  int32_t* head;      // [2]: next index of the Y queue, the W queue
  int32_t* ycnt;      // per global token tile: split items arrived
  int32_t* ytdone;    // per global token tile: 1 once its [Y_hi | Y_lo]^T is written
  float* part;        // nslots partial slots of R x 256 fp32 (component-major)
  int32_t nslots;
};

constexpr int kFusedThreads = 384;
constexpr int kItemRing = 4;
constexpr int kBarY = 1, kBarW = 2;    // named barriers of the two epilogue groups (128 threads)

__host__ __device__ inline int fused_stage_bytes(int R) { return ring_stage_bytes(R, 2); }
// Fixed shared memory after the two rings: Gram staging, item rings, barriers, TMEM slot, flags.
__host__ __device__ inline int fused_fixed_bytes(int R) {
  return w_stage_bytes(R) + 2 * kItemRing * static_cast<int>(sizeof(PiItem)) + 512 + 256;
}

__device__ __forceinline__ bool group_agree(int bar_id, bool ok) {
  uint32_t all;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, %2, 128, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(all)
      : "r"(static_cast<uint32_t>(ok)), "r"(bar_id)
      : "memory");
  return all != 0;
}
__device__ __forceinline__ void group_sync(int bar_id) { asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory"); }

// [hi | lo] bf16 pair of the fp32 y into rows c and R + c of a 2R x ld buffer, column t.
__device__ __forceinline__ void put_y2t(__nv_bfloat16* y2t, int64_t ld, int R, int c, int64_t t, float y) {
  const __nv_bfloat16 yh = __float2bfloat16_rn(y);
  const __nv_bfloat16 yl = __float2bfloat16_rn(y - __bfloat162float(yh));
  y2t[static_cast<int64_t>(c) * ld + t] = yh;
  y2t[static_cast<int64_t>(R + c) * ld + t] = yl;
}

// One pipeline's shared-memory state.
struct Pipe {
  unsigned char* ring;     // stages x fused_stage_bytes
  int stages;
  uint64_t* full;          // [stages]
  uint64_t* empty;         // [stages]
  uint64_t* tfull;         // accumulator committed
  uint64_t* tempty;        // accumulator read by the four epilogue warps
  PiItem* items;           // [kItemRing]
  uint64_t* itfull;        // [kItemRing]
  uint64_t* itempty;       // [kItemRing]: MMA issuer + epilogue group
};

// Producer lane of a pipeline: takes items in queue order, hands each to the MMA issuer and
// the epilogue through the item ring, and fills the stage ring. W (Y = false) waits for each
// token tile's flag before its k-steps.
template <bool Y>
__device__ void pipe_producer(const Pipe& p, const TCBasis* __restrict__ bases, const PiItem* __restrict__ q, int n,
                              int32_t* head, const PiSync& sync, int R, int* err) {
  const int sbytes = fused_stage_bytes(R);
  const int a_bytes = 2 * kBM * kBK * 2;
  const uint64_t pol = Y ? l2_policy_evict_last() : l2_policy_evict_first();
  int g = 0, i = 0, cur = -1;
  bool ok = true;
  while (ok) {
    const int idx = atomicAdd(head, 1);
    PiItem it;
    if (idx < n) {
      it = q[idx];
    } else {
      it.end = 1;
    }
    const int s = i % kItemRing;
    if (i >= kItemRing && !mbar_wait(p.itempty + s, static_cast<uint32_t>((i / kItemRing) & 1) ^ 1u, err)) {
      ok = false;
      break;
    }
    p.items[s] = it;
    mbar_arrive(p.itfull + s);          // release: the consumers see the item
    ++i;
    if (it.end) break;
    const TCBasis* B = bases + it.basis;
    if (it.basis != cur) {
      if (Y) { tmap_acquire(&B->mapHy); tmap_acquire(&B->mapV2); }
      else { tmap_acquire(&B->mapHw); tmap_acquire(&B->mapY2); }
      cur = it.basis;
    }
    if (Y && it.wait_tile >= 0 && !spin_geq(sync.ytdone + it.wait_tile, 1, err)) { ok = false; break; }
    for (int k = it.k0; k < it.k1; ++k) {
      if (!Y && ((k - it.k0) & 3) == 0) {
        // the 256-token tile holding k-steps k .. k+3 has its [Y_hi | Y_lo]^T
        if (!spin_geq(sync.ytdone + it.ytile + k / 4, 1, err)) { ok = false; break; }
        fence_proxy_async_global();
      }
      const int st = g % p.stages;
      const uint32_t u = static_cast<uint32_t>(g / p.stages);
      if (g >= p.stages && !mbar_wait(p.empty + st, (u & 1u) ^ 1u, err)) { ok = false; break; }
      unsigned char* As = p.ring + st * sbytes;
      mbar_expect_tx(p.full + st, static_cast<uint32_t>(sbytes));
      if (Y) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_2d_hint(As + h * (kBM * kBK * 2), &B->mapHy, k * kBK, (it.tile * 2 + h) * kBM, p.full + st, pol);
        tma_load_2d(As + a_bytes, &B->mapV2, k * kBK, 0, p.full + st);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int x = (it.tile * 2 + h) * kBM;
          tma_load_2d_hint(As + h * (kBM * kBK * 2), &B->mapHw, x, k * kBK, p.full + st, pol);
          tma_load_2d_hint(As + h * (kBM * kBK * 2) + kBM * kBK, &B->mapHw, x + 64, k * kBK, p.full + st, pol);
        }
        tma_load_2d(As + a_bytes, &B->mapY2, k * kBK, 0, p.full + st);
      }
      ++g;
    }
  }
  if (!ok) {
    // the loads already issued land before the CTA can exit
    for (int j = (g > p.stages ? g - p.stages : 0); j < g; ++j)
      mbar_drain(p.full + (j % p.stages), static_cast<uint32_t>(j / p.stages) & 1u);
  }
}

// MMA issuer lane of a pipeline: one accumulator pair (two 128-row halves) at TMEM column dacc.
template <bool Y>
__device__ void pipe_mma(const Pipe& p, uint32_t dacc, int R, int* err) {
  const int N = 2 * R;
  const int acc_cols = tmem_cols(N);
  const int sbytes = fused_stage_bytes(R);
  const int a_bytes = 2 * kBM * kBK * 2;
  const uint32_t idesc = Y ? idesc_bf16(N, 0, 0) : idesc_bf16(N, 1, 0);
  int g = 0, i = 0, j = 0, last = -1;
  bool ok = true;
  while (ok) {
    const int s = i % kItemRing;
    if (!mbar_wait(p.itfull + s, static_cast<uint32_t>(i / kItemRing) & 1u, err)) { ok = false; break; }
    const PiItem it = p.items[s];
    mbar_arrive(p.itempty + s);
    ++i;
    if (it.end) break;
    if (j >= 1 && !mbar_wait(p.tempty, static_cast<uint32_t>(j - 1) & 1u, err)) { ok = false; break; }
    tc_fence_after();
    for (int k = it.k0; k < it.k1; ++k) {
      const int st = g % p.stages;
      if (!mbar_wait(p.full + st, static_cast<uint32_t>(g / p.stages) & 1u, err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a0 = smem_u32(p.ring + st * sbytes);
      const uint32_t b0 = a0 + static_cast<uint32_t>(a_bytes);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint32_t acc = (k > it.k0 || kk > 0) ? 1u : 0u;
          if (Y)   // A and B K-major rows of 128 B (half h 16 KB on)
            mma_bf16(dacc + static_cast<uint32_t>(h * acc_cols), sdesc(a0 + h * 16384 + kk * 32, 16, 1024),
                     sdesc(b0 + kk * 32, 16, 1024), idesc, acc);
          else     // A MN-major 64 x 8 atoms, two along MN 8 KB apart; B K-major
            mma_bf16(dacc + static_cast<uint32_t>(h * acc_cols), sdesc(a0 + h * 16384 + kk * 2048, 8192, 1024),
                     sdesc(b0 + kk * 32, 16, 1024), idesc, acc);
        }
      mma_commit(p.empty + st);
      ++g;
    }
    mma_commit(p.tfull);                // on an error too: it completes once the issued MMAs have
    last = j;
    ++j;
  }
  if (!ok && last >= 0) mbar_drain(p.tfull, static_cast<uint32_t>(last) & 1u);
}

__global__ void __launch_bounds__(kFusedThreads, 1)
    k_pi_fused(const TCBasis* __restrict__ bases, const PiItem* __restrict__ yq, int ny, const PiItem* __restrict__ wq,
               int nw, PiSync sync, int stages_y, int stages_w, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared pointer
  const int R = bases[0].R;
  const int N = 2 * R;
  const int sbytes = fused_stage_bytes(R);
  const int acc_cols = tmem_cols(N);      // 128 for R <= 64
  Pipe py, pw;
  py.ring = smem;
  py.stages = stages_y;
  pw.ring = smem + stages_y * sbytes;
  pw.stages = stages_w;
  unsigned char* fx = smem + (stages_y + stages_w) * sbytes;
  double* wt = reinterpret_cast<double*>(fx);
  py.items = reinterpret_cast<PiItem*>(fx + w_stage_bytes(R));
  pw.items = py.items + kItemRing;
  uint64_t* bars = reinterpret_cast<uint64_t*>(pw.items + kItemRing);
  py.full = bars;              bars += stages_y;
  py.empty = bars;             bars += stages_y;
  pw.full = bars;              bars += stages_w;
  pw.empty = bars;             bars += stages_w;
  py.tfull = bars++;           py.tempty = bars++;
  pw.tfull = bars++;           pw.tempty = bars++;
  py.itfull = bars;            bars += kItemRing;
  py.itempty = bars;           bars += kItemRing;
  pw.itfull = bars;            bars += kItemRing;
  pw.itempty = bars;           bars += kItemRing;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars);
  int* yflag = reinterpret_cast<int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (const Pipe* p : {&py, &pw}) {
      for (int s = 0; s < p->stages; ++s) { mbar_init(p->full + s, 1); mbar_init(p->empty + s, 1); }
      mbar_init(p->tfull, 1);
      mbar_init(p->tempty, 4);
      for (int s = 0; s < kItemRing; ++s) { mbar_init(p->itfull + s, 1); mbar_init(p->itempty + s, 2); }
    }
    mbar_init_fence();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t wcol0 = static_cast<uint32_t>(2 * acc_cols);

  if (warp == 0) {
    if (lane == 0) pipe_producer<true>(py, bases, yq, ny, sync.head, sync, R, err);
  } else if (warp == 1) {
    if (lane == 0) pipe_producer<false>(pw, bases, wq, nw, sync.head + 1, sync, R, err);
  } else if (warp == 2) {
    if (lane == 0) pipe_mma<true>(py, tmem, R, err);
  } else if (warp == 3) {
    if (lane == 0) pipe_mma<false>(pw, tmem + wcol0, R, err);
  } else if (warp < 8) {
    // ------------------------------------------------------------ Y epilogue (warps 4-7)
    const int q = warp & 3;
    const int row = q * 32 + lane;          // TMEM lane = token row of a half
    const int et = (warp - 4) * 32 + lane;  // 0..127
    int i = 0, jy = 0;
    while (true) {
      const int s = i % kItemRing;
      const bool got = mbar_wait(py.itfull + s, static_cast<uint32_t>(i / kItemRing) & 1u, err);
      if (!group_agree(kBarY, got)) break;
      const PiItem it = py.items[s];
      group_sync(kBarY);                    // every thread has its copy of the slot
      if (et == 0) mbar_arrive(py.itempty + s);
      ++i;
      if (it.end) break;
      const bool ready = mbar_wait(py.tfull, static_cast<uint32_t>(jy) & 1u, err);
      if (!group_agree(kBarY, ready)) break;
      tc_fence_after();
      ++jy;
      const TCBasis* B = bases + it.basis;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
      const bool split = it.nsplit > 1;
      float* pslot = sync.part + static_cast<int64_t>(it.slot) * R * 256;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int64_t t = (static_cast<int64_t>(it.tile) * 2 + h) * kBM + row;
        for (int c0 = 0; c0 < R; c0 += 16) {
          float hi[16], lo[16];
          tmem_ld16(tbase + static_cast<uint32_t>(h * acc_cols) + c0, hi);
          tmem_ld16(tbase + static_cast<uint32_t>(h * acc_cols) + R + c0, lo);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float yv = hi[c] + lo[c];
            if (split) pslot[(c0 + c) * 256 + h * kBM + row] = yv;
            else if (t < B->T) put_y2t(B->Y2T, B->ldy2, R, c0 + c, t, yv);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(py.tempty);   // this warp's lanes of the Y accumulator are read
      bool finish = !split;
      if (split) {
        __threadfence();                    // the partial is visible before the arrival
        group_sync(kBarY);
        if (et == 0) *yflag = (atomicAdd(sync.ycnt + it.ytile, 1) == it.nsplit - 1) ? 1 : 0;
        group_sync(kBarY);
        finish = *yflag != 0;
        if (finish) {
          __threadfence();                  // every split's partial is visible
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int tl = h * kBM + et;
            const int64_t t = static_cast<int64_t>(it.tile) * 256 + tl;
            if (t >= B->T) continue;
            // the splits in order; one token row (R <= 64 components) per split, so each
            // thread has a whole row of independent loads in flight
            float yv[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) yv[c] = 0.f;
#pragma unroll 1
            for (int k = 0; k < it.nsplit; ++k) {
              int sl = it.slot0 + k;
              if (sl >= sync.nslots) sl -= sync.nslots;
              const float* pk = sync.part + static_cast<int64_t>(sl) * R * 256 + tl;
#pragma unroll
              for (int c = 0; c < 64; ++c)
                if (c < R) yv[c] += __ldcg(pk + c * 256);
            }
#pragma unroll
            for (int c = 0; c < 64; ++c)
              if (c < R) put_y2t(B->Y2T, B->ldy2, R, c, t, yv[c]);
          }
        }
      }
      if (finish) {
        fence_proxy_async_global();         // Y2T is read by other CTAs' TMA
        __threadfence();
        group_sync(kBarY);
        if (et == 0) atomicExch(sync.ytdone + it.ytile, 1);
      }
    }
  } else {
    // ------------------------------------------------------------ W epilogue (warps 8-11)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int tld = w_stage_ld(R);
    int i = 0, jw = 0;
    while (true) {
      const int s = i % kItemRing;
      const bool got = mbar_wait(pw.itfull + s, static_cast<uint32_t>(i / kItemRing) & 1u, err);
      if (!group_agree(kBarW, got)) break;
      const PiItem it = pw.items[s];
      group_sync(kBarW);
      if ((warp - 8) * 32 + lane == 0) mbar_arrive(pw.itempty + s);
      ++i;
      if (it.end) break;
      const bool ready = mbar_wait(pw.tfull, static_cast<uint32_t>(jw) & 1u, err);
      if (!group_agree(kBarW, ready)) break;
      tc_fence_after();
      ++jw;
      const TCBasis* B = bases + it.basis;
      const uint32_t tbase = tmem + wcol0 + (static_cast<uint32_t>(q * 32) << 16);
      const bool gram = B->Gp != nullptr;
      TileGram gr(tld, R, B->nq, q, lane);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const uint32_t trow = tbase + static_cast<uint32_t>(h * acc_cols);
        const int64_t d = (static_cast<int64_t>(it.tile) * 2 + h) * kBM + row;
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
        if (h == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(pw.tempty);   // this warp's lanes of the W accumulator are read
        }
        if (gram) {
          // the tile's fp64 Gram on the fp64 MMA, one epilogue warp's 32 rows staged at a time
          // (rows past D are zero: the activation box there is zero filled)
#pragma unroll 1
          for (int r = 0; r < 4; ++r) {
            if (q == r) {
              double* stg = wt + lane * tld;
#pragma unroll
              for (int c = 0; c < 64; c += 2)
                if (c < R) *reinterpret_cast<double2*>(stg + c) = make_double2(w[c], w[c + 1]);
            }
            group_sync(kBarW);              // the quarter is staged
            gr.rows(wt, tld, 32);
            group_sync(kBarW);              // the staging region is free again
          }
        }
      }
      if (gram) gr.store(B->Gp + static_cast<int64_t>(it.tile) * B->nq * 64);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace tc
}  // namespace dsmz
