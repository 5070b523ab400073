// Internal device tables and helpers of libdsmezo (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <curand_kernel.h>
#include <stdint.h>

#include "dsmezo.h"

namespace dsmz {

constexpr int kThreads = 256;

// One matrix viewed as `nvec` r-vectors. Side A (d_out x r): vector v is row v, component k
// at v*ld + k. Side B (r x d_in): vector v is column v, component k at k*ld + v. Power
// iteration bases reuse the struct for W (D x R, side A).
struct MatD {
  void* param; void* pos; void* neg;
  float* mu; float* var; float* z; float* scratch;
  void* shadow;               // adapters: copy-dtype image of the updated master (NULL: none)
  int64_t nvec, r, ld, cs;    // element (v, k) at side A: v*ld + k*cs, side B: k*ld + v*cs
  int32_t side, owner;        // owner: module index (adapters) or basis index (power iteration)
  int32_t seg0, nseg;         // global index of the first vector segment, segment count
  int32_t segv, pad0;         // vectors per segment
  int64_t gram_off;           // doubles: nseg * r*r Gram partials
  int64_t p_off;              // floats: r*r apply matrix (fp32), then 4 floats of scalars
  int64_t dw_off;             // doubles: W matrices of the power iteration: 3 * r*r fp64 (Gram,
                              // R^{-1} for the QR apply, R^{-1}); 0 for adapter matrices
  __nv_bfloat16* v2t;         // power-iteration W only: [V_hi | V_lo]^T output (NULL: none)
  int64_t ldv2;
  // streaming kernels: the global tile space (TV-vector tiles of every matrix in order) is
  // cut into one contiguous chunk per CTA; a segment is a chunk's run within one matrix
  int32_t tile0, ntile;       // first global tile, tiles of this matrix
  int32_t chunk0;             // chunk (CTA) holding tile0; segment seg0 + c - chunk0 of chunk c
  int32_t tmap;               // side 1: first of four 2-D tensor maps (param, mu, var, z) in
                              // Tables::smaps, or -1
  int32_t kmap;               // 128-byte-swizzled row boxes (Tables::smaps) of the perturbation's
                              // K operand (Zc_A rows on side 0, basis rows on side 1), or -1
  int32_t rmap;               // the same for the matrix's own rows (side-0 mu; W), or -1
  int32_t pad1;
};

struct ModD {
  int32_t a, b, basis, r, rc, rca;
  int64_t d_out, d_in;
  uint64_t offB, offA;        // generator offsets of the two draws, relative to the step base
  int64_t thrB, thrA;         // torch launch width (threads) of each draw
  int32_t chunk0, nchunk;     // B-side sums: first CTA whose column range meets this module, and
                              // the number of such CTAs (one partial each)
  int64_t col0;               // first column of this module in the concatenated d_in columns
  int64_t coef_off;           // floats: Zc_B (r*rc) then Q (r*rca)
  int64_t bpart_off;          // floats: nchunk * 2 * r*rc partial sums (B V, var_B V^2)
  const float* zcB_ext;       // explicit Zc_B (R x RC) / Zc_A (d_out x RCA) for the drop-in op
  const float* zcA_ext;
  const float* Bp;            // B factor (R x d_in, fp32) and its variance, read by the B-side sums
  const float* varB;          // NULL: skip var_B V^2 (drop-in op)
  int64_t b_s0, b_s1;
  int64_t zca_off;            // floats: materialised Zc_A draw (d_out x RCA)
  int32_t dblk0, ndblk;       // blocks of the Zc_A draw kernel (one torch thread each)
  int64_t qrw_off;            // doubles: G and R^{-1} (rca x rca each) of the QR of B V when they do
                              // not fit beside it in shared memory (r or rca > 64), else 0
};

struct BasisD {
  const void* H; int32_t hdt; int32_t R;
  int64_t T, D, h_s0, h_s1;   // activation T x D with element strides
  const float* Vin; int64_t v_s0, v_s1;  // basis (strided); the grouped step updates it in place
  float* Vout;                // D x R contiguous result of the power iteration
  int64_t y_off, w_off;       // floats: Y (T x R) and W (D x R)
  int32_t ytile0, nytile;     // (T/64) x (R/64) output tiles of Y = H V
  int64_t ypart_off;          // floats: ysplit partial Y (T x R each) of the split-K Y product
  int32_t wtile0, nwtile;     // (D/64) x (R/64) output tiles of W = H^T Y
};

// Fused all-gathers (one process per GPU of a node): byte distances from this rank's gather
// buffers (+/- copies, and the factor shadow) to each peer's, mapped over NVLink; a kernel
// that stores an element of its shard also stores it at those distances, so every rank
// receives every shard while the kernel runs instead of in an all-gather after it.
constexpr int kMaxPeers = 7;
struct GatherPeers {
  int32_t n;
  int32_t pad;
  int64_t dpos[kMaxPeers], dneg[kMaxPeers];
};

// Everything a launch needs, passed by value.
struct Tables {
  const MatD* mats; int32_t nmats; int32_t nsegs;      // adapter matrices
  const ModD* mods; int32_t nmods; int32_t nchunks;
  const BasisD* bases; int32_t nbases; int32_t nytiles; int32_t nwtiles;
  int32_t ysplit;                                       // K splits of the CUDA-core Y product
  const MatD* wA; const MatD* wB;                       // W of each basis: CholeskyQR round 1, round 2 (-> V)
  int32_t nwsegsA; int32_t nwsegsB;
  int32_t copy_dtype; int32_t ndblk;                   // +/- copies and shadows; ndblk: blocks of the Zc_A draw
  char* ws;                                            // workspace base
  int64_t seg_kal_off;        // doubles: nsegs * 2 per-segment Kalman partials
  int64_t kal_sum_off;        // doubles: 2 summed Kalman scalars per direction
  const CUtensorMap* smaps;   // 2-D tensor maps of the side-1 matrices' arrays (tile boxes)
  int32_t ndir, dir;          // directions; the one a perturbation launch writes
  int64_t dstride_f;          // factor elements between directions' pos/neg copies
  int64_t dstride_z;          // fp32 elements between directions' z
};

// ------------------------------------------------------------------ dtype helpers
__device__ __forceinline__ float ldf(const void* p, int64_t i, int dt) {
  return dt == DSMZ_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                         : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void stf(void* p, int64_t i, float x, int dt) {
  if (dt == DSMZ_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}
__device__ __forceinline__ int64_t vaddr(int side, int64_t v, int64_t k, int64_t ld) {
  return side == 0 ? v * ld + k : k * ld + v;
}

// Index of the owner whose [start, start+count) range holds `item` (starts ascending).
template <typename T, typename F>
__device__ __forceinline__ int find_owner(const T* tab, int n, int item, F start_of) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (start_of(tab[mid]) <= item) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ------------------------------------------------------------------ torch Philox stream
// Element `li` of torch.randn(n) drawn from a CUDA generator at (seed, offset), where the
// draw ran `threads` = blockDim*gridDim threads (ATen DistributionTemplates.h
// distribution_elementwise_grid_stride_kernel): thread idx = li mod threads takes
// curand_init(seed, idx, offset) and calls curand_normal4 once per grid-stride round;
// round j component c covers li = idx + 4*threads*j + threads*c. The j-th call equals a
// fresh state at offset + 4*j (each call consumes one Philox block), so any element is
// reachable directly. Values come from the cuRAND device API itself.
__device__ __forceinline__ float torch_randn_at(uint64_t seed, uint64_t offset, int64_t threads, int64_t li) {
  const int64_t idx = li % threads;
  const int64_t q = li / threads;
  const int comp = static_cast<int>(q & 3);
  const unsigned long long round = static_cast<unsigned long long>(q >> 2);
  curandStatePhilox4_32_10_t st;
  curand_init(seed, static_cast<unsigned long long>(idx), offset + 4ull * round, &st);
  const float4 g = curand_normal4(&st);
  return comp == 0 ? g.x : (comp == 1 ? g.y : (comp == 2 ? g.z : g.w));
}

}  // namespace dsmz
