// Kernels of the DS-MeZO optimizer step (sm_100a). Exact-arithmetic path: fp32 FFMA for
// the streamed products, fp64 for cross-tile sums and for the r x r Newton-Schulz and
// Cholesky solves. Every launch covers all matrices (or bases, or modules) of a plan.
#pragma once

#include "dsmz_internal.cuh"
#include "dsmz_ptx.cuh"

namespace dsmz {

// Per-step Kalman inputs; rounding follows ds_mezo/controller.py:267-285 op by op, with
// every scalar cast to fp32 the way torch applies a Python float to an fp32 tensor.
struct KalmanIn {
  float beta;    // fp32(beta)
  float beta2;   // fp32(beta * beta), product taken in double as in the controller
  float q;       // fp32(eps^2 (1 - beta^2))
  float dd;      // fp32(dd)
  float floor_;  // norm_floor
};

struct KalScal { float beta, beta2, q, innov, inv_s; };

__device__ __forceinline__ KalScal kal_derive(const KalmanIn& k, const double* sums) {
  KalScal s;
  s.beta = k.beta; s.beta2 = k.beta2; s.q = k.q;
  const float y_hat = static_cast<float>(sums[0]);
  const float S = __fadd_rn(static_cast<float>(sums[1]), k.floor_);   // S = s_sum + norm_floor
  s.inv_s = __fdiv_rn(1.0f, S);                                       // inv_S = 1 / S
  s.innov = __fsub_rn(k.dd, y_hat);                                    // innovation = dd - y_hat
  return s;
}

// Kalman predict (controller.py:267-268): mu1 = mu*beta; var1 = var*beta^2 + q.
__device__ __forceinline__ void kal_predict(float mu0, float var0, const KalScal& s, float& mu1, float& var1) {
  mu1 = __fmul_rn(mu0, s.beta);
  var1 = __fadd_rn(__fmul_rn(var0, s.beta2), s.q);
}
// Kalman observation (controller.py:283-285): K = var*z*inv_S; mu += innov*K; var *= 1 - K*z.
__device__ __forceinline__ void kal_observe(float mu1, float var1, float z, const KalScal& s, float& mu2, float& var2) {
  const float K = __fmul_rn(__fmul_rn(var1, z), s.inv_s);
  mu2 = __fadd_rn(mu1, __fmul_rn(s.innov, K));
  var2 = __fmul_rn(var1, __fsub_rn(1.0f, __fmul_rn(K, z)));
}

// Vectors per shared-memory sub-tile: about 8192 elements, so the 4 x 8 register blocks of
// rows_x_mat cover all 256 threads at r = 64.
__host__ __device__ inline int tile_vectors(int r) {
  int tv = (8192 / (r < 1 ? 1 : r)) & ~3;   // a multiple of the 4-vector blocks
  return tv < 16 ? 16 : (tv > 1024 ? 1024 : tv);
}
__host__ __device__ inline int pad4(int r) { return (r + 3) & ~3; }
__host__ __device__ inline int pad8(int r) { return (r + 7) & ~7; }

// out[v][c] = sum_{a<K} X[v*xld + a] * P[a*pld + c] for v < nv, c < nc, both operands in
// shared memory. Each thread owns 4 vectors x 8 columns (32 fp32 accumulators): columns
// 4cb..4cb+3 and pld/2+4cb..+3, so the eight column blocks of a warp read one contiguous
// 128-byte run of a P row per float4 load (no bank conflicts). pld % 8 == 0 and columns
// padded with zeros to pld; X needs ceil(nv/4)*4 readable rows, and an odd xld keeps the
// four row reads of a warp on distinct banks. sink(v, c, value) takes each output.
template <typename Sink>
__device__ __forceinline__ void rows_x_mat(const float* __restrict__ X, int xld, const float* __restrict__ P, int pld,
                                           int nv, int K, int nc, Sink sink) {
  const int cbs = pld >> 3;
  const int half = pld >> 1;
  const int vbs = (nv + 3) >> 2;
  for (int blk = threadIdx.x; blk < vbs * cbs; blk += kThreads) {
    const int vb = blk / cbs, cb = blk - vb * cbs;
    const int v0 = vb * 4, c0 = cb * 4;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    const float* x0 = X + v0 * xld;
#pragma unroll 4
    for (int a = 0; a < K; ++a) {
      const float4 p0 = *reinterpret_cast<const float4*>(P + a * pld + c0);
      const float4 p1 = *reinterpret_cast<const float4*>(P + a * pld + half + c0);
      const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = x0[i * xld + a];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(x, pv[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (v0 + i >= nv) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = (j < 4) ? c0 + j : half + c0 + j - 4;
        if (c < nc) sink(v0 + i, c, acc[i][j]);
      }
    }
  }
}

// Element e of a sub-tile of nv vectors in coalesced memory order: side A walks each row
// (vector) along its r components, side B walks each of the r rows along the vectors.
__device__ __forceinline__ void elem_vk(int side, int e, int r, int nv, int& v, int& k) {
  if (side == 0) { v = e / r; k = e - v * r; } else { k = e / nv; v = e - k * nv; }
}
constexpr int kUnroll = 8;   // elements in flight per thread in the streaming loops

// Sum of n values spaced `stride` apart, four independent chains to overlap the loads.
__device__ __forceinline__ double strided_sum(const double* p, int n, int64_t stride) {
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  int g = 0;
  for (; g + 4 <= n; g += 4) {
    s0 += p[(g + 0) * stride];
    s1 += p[(g + 1) * stride];
    s2 += p[(g + 2) * stride];
    s3 += p[(g + 3) * stride];
  }
  for (; g < n; ++g) s0 += p[g * stride];
  return (s0 + s1) + (s2 + s3);
}

__device__ __forceinline__ int64_t vaddr2(const MatD& M, int64_t v, int64_t k) {
  return M.side == 0 ? v * M.ld + k * M.cs : k * M.ld + v * M.cs;
}

// =====================================================================================
// Gram partials: for each segment of each matrix, G_seg = sum_v x_v x_v^T (r x r).
// SRC 0: x = mu (plain). SRC 1: x = Kalman-updated momentum mu2 (controller.py:283-284).
// ACC double: fp64 products and sums. The Gram squares the condition number, and the
// Newton-Schulz polynomial of an ill-conditioned momentum (a fresh start, where
// mu_B ~ Zc_B V^T with a square Gaussian Zc_B) and the CholeskyQR of the power-iteration
// W need its small eigenvalues intact. ACC float is the fp32-accumulate variant.
// =====================================================================================
template <int SRC, int RB, typename ACC>
__global__ void __launch_bounds__(kThreads) k_gram(Tables tb, const MatD* __restrict__ mats, int nmats,
                                                   KalmanIn kin) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int seg = blockIdx.x;
  const int mi = find_owner(mats, nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = mats[mi];
  const int r = static_cast<int>(M.r);
  const int tpr = (r + RB - 1) / RB;
  const int tpg = tpr * tpr;
  const int ngroups = kThreads / tpg;
  const int rp = tpr * RB;
  const int TV = tile_vectors(r);
  const int xld = rp + 4;                                   // 16-byte rows for the float4 Gram loads
  float* xs = reinterpret_cast<float*>(smem_raw);          // TV x xld
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  const int tid = threadIdx.x;
  const int grp = tid / tpg, lt = tid % tpg;
  const int bi = lt / tpr, bj = lt % tpr;
  const bool active = grp < ngroups;
  KalScal ks{};
  if (SRC == 1) ks = kal_derive(kin, reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off);

  ACC acc[RB][RB];
#pragma unroll
  for (int i = 0; i < RB; ++i)
#pragma unroll
    for (int j = 0; j < RB; ++j) acc[i][j] = ACC(0);

  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    {
      const int n = nv * r;
      for (int base = tid; base < n; base += kThreads * kUnroll) {
        float m0[kUnroll], w0[kUnroll], z0[kUnroll];
        int vv[kUnroll], kk[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {          // issue every load before using any
          const int e = base + u * kThreads;
          elem_vk(M.side, e, r, nv, vv[u], kk[u]);
          if (e < n) {
            const int64_t a = vaddr2(M, s0 + vv[u], kk[u]);
            m0[u] = M.mu[a];
            if (SRC == 1) { w0[u] = M.var[a]; z0[u] = M.z[a]; }
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          if (base + u * kThreads < n) {
            float x = m0[u];
            if (SRC == 1) {
              float mu1, var1, mu2, var2;
              kal_predict(m0[u], w0[u], ks, mu1, var1);
              kal_observe(mu1, var1, z0[u], ks, mu2, var2);
              x = mu2;
            }
            xs[vv[u] * xld + kk[u]] = x;
          }
        }
      }
      if (rp > r || nv < TV) {                        // zero padding columns and rows past nv
        for (int e = tid; e < TV * rp; e += kThreads) {
          const int v = e / rp, k = e - v * rp;
          if (v >= nv || k >= r) xs[v * xld + k] = 0.f;
        }
      }
    }
    __syncthreads();
    if (active) {
      for (int v = grp; v < nv; v += ngroups) {
        const float* row = xs + v * xld;
        ACC xa[RB], xb[RB];
#pragma unroll
        for (int i = 0; i < RB; i += 4) {
          const float4 fa = *reinterpret_cast<const float4*>(row + bi * RB + i);
          const float4 fb = *reinterpret_cast<const float4*>(row + bj * RB + i);
          xa[i] = static_cast<ACC>(fa.x); xa[i + 1] = static_cast<ACC>(fa.y);
          xa[i + 2] = static_cast<ACC>(fa.z); xa[i + 3] = static_cast<ACC>(fa.w);
          xb[i] = static_cast<ACC>(fb.x); xb[i + 1] = static_cast<ACC>(fb.y);
          xb[i + 2] = static_cast<ACC>(fb.z); xb[i + 3] = static_cast<ACC>(fb.w);
        }
#pragma unroll
        for (int i = 0; i < RB; ++i)
#pragma unroll
          for (int j = 0; j < RB; ++j) acc[i][j] = fma(xa[i], xb[j], acc[i][j]);
      }
    }
    __syncthreads();
  }

  double* out = reinterpret_cast<double*>(tb.ws) + M.gram_off + static_cast<int64_t>(seg - M.seg0) * r * r;
  if (ngroups == 1) {
    if (active) {
#pragma unroll
      for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          const int a = bi * RB + i, b = bj * RB + j;
          if (a < r && b < r) out[a * r + b] = static_cast<double>(acc[i][j]);
        }
    }
  } else {
    double* red = reinterpret_cast<double*>(smem_raw);   // ngroups * rp * rp
    if (active) {
#pragma unroll
      for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int j = 0; j < RB; ++j)
          red[(grp * rp + bi * RB + i) * rp + bj * RB + j] = static_cast<double>(acc[i][j]);
    }
    __syncthreads();
    for (int e = tid; e < r * r; e += kThreads) {
      const int a = e / r, b = e - a * r;
      double sum = 0.0;
      for (int g = 0; g < ngroups; ++g) sum += red[(g * rp + a) * rp + b];
      out[e] = sum;
    }
  }
}

// C = A B for r x r fp64 matrices that are symmetric and commute (polynomials of one
// Gram matrix), so C is symmetric: only the upper 8 x 8 blocks are formed, with the fp64
// MMA (m8n8k4), and mirrored. Up to kSymmU blocks per warp per pass (one pass for r <= 64).
// The products are held in registers across a barrier before C is written, so with one
// pass (r <= 64) C may be A or B (in place); with several, C must be distinct. Pitch ld (= rp + 4: a warp's fragment loads fall in two wavefronts);
// rows and columns r..rp-1 are zero and stay zero. Every position is written by exactly one
// thread. Ends with a barrier.
constexpr int kSymmU = 5;
__device__ void cta_symm_mm(double* C, const double* A, const double* B, int rp, int ld) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nw = kThreads / 32;
  const int nb = rp >> 3, nq = nb * (nb + 1) / 2;
  for (int q0 = warp; q0 < ((nq + nw - 1) / nw + kSymmU - 1) / kSymmU * kSymmU * nw; q0 += kSymmU * nw) {
    int bi[kSymmU], bj[kSymmU];
    double acc[kSymmU][2];
#pragma unroll
    for (int u = 0; u < kSymmU; ++u) {
      int q = q0 + u * nw;
      bi[u] = -1; bj[u] = 0;
      acc[u][0] = 0.0; acc[u][1] = 0.0;
      if (q < nq) {
        int row = 0;
        while (q >= nb - row) { q -= nb - row; ++row; }
        bi[u] = row; bj[u] = row + q;
      }
    }
    for (int k0 = 0; k0 < rp; k0 += 4) {
#pragma unroll
      for (int u = 0; u < kSymmU; ++u)
        if (bi[u] >= 0)
          dmma8x8x4(acc[u][0], acc[u][1], A[(8 * bi[u] + g) * ld + k0 + t], B[(k0 + t) * ld + 8 * bj[u] + g]);
    }
    __syncthreads();                                   // every read of A and B is done
#pragma unroll
    for (int u = 0; u < kSymmU; ++u) {
      if (bi[u] < 0) continue;
      const int row = 8 * bi[u] + g;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = 8 * bj[u] + 2 * t + h;
        if (bi[u] == bj[u] && col < row) continue;        // the mirror of the upper half
        C[row * ld + col] = acc[u][h];
        if (col != row) C[col * ld + row] = acc[u][h];
      }
    }
    __syncthreads();
  }
}

__device__ double cta_sum(double v, double* red) {
  const int tid = threadIdx.x;
  red[tid] = v;
  __syncthreads();
  for (int s = kThreads / 2; s > 0; s >>= 1) {
    if (tid < s) red[tid] += red[tid + s];
    __syncthreads();
  }
  const double out = red[0];
  __syncthreads();
  return out;
}

struct NSArgs {
  int iters;
  double c[DSMZ_MAX_NS_ITERS][3];
  float norm_floor;
};

// Pitch (doubles) of the r x r solve matrices: rows of pad8(r) + 4.
__host__ __device__ inline int ns_ld(int r) { return pad8(r) + 4; }

// =====================================================================================
// Newton-Schulz in Gram space, one CTA per matrix (ds_mezo/kernels.py:26-164 rewritten):
// X_k = X_0 P_k with P_k a polynomial of G_0 = X_0^T X_0, so the 12 X-space passes become
// G <- S G S, P <- P S on r x r (fp64), S = c0 I + c1 G + c2 G^2. Stores the fp32 apply
// matrix Pm with X[v,:] = x_v^T Pm for every vector x_v of the matrix (P is symmetric, so
// tall and wide matrices use it alike). r <= 64: three matrices in shared memory (two CTAs
// per SM), products in place (one pass of cta_symm_mm); k_ns_solve_packed takes larger r.
// =====================================================================================
__global__ void __launch_bounds__(kThreads, 2) k_ns_solve(Tables tb, const MatD* __restrict__ mats, NSArgs ns) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[kThreads];
  const MatD M = mats[blockIdx.x];
  const int r = static_cast<int>(M.r);
  const int rr = r * r;
  const int rp = pad8(r), ld = ns_ld(r), mm = rp * ld;
  const int tid = threadIdx.x;
  double* dw = reinterpret_cast<double*>(smem_raw);
  double* G = dw;
  double* P = dw + mm;
  double* S = dw + 2 * mm;
  const double* part = reinterpret_cast<const double*>(tb.ws) + M.gram_off;
  for (int e = tid; e < 3 * mm; e += kThreads) dw[e] = 0.0;
  __syncthreads();
  double tr = 0.0;
  constexpr int kSumU = 8;                             // independent partial loads in flight
  for (int e0 = tid; e0 < rr; e0 += kSumU * kThreads) {
    double v[kSumU];
#pragma unroll
    for (int u = 0; u < kSumU; ++u) v[u] = 0.0;
    for (int sg = 0; sg < M.nseg; ++sg) {
#pragma unroll
      for (int u = 0; u < kSumU; ++u) {
        const int e = e0 + u * kThreads;
        if (e < rr) v[u] += part[static_cast<int64_t>(sg) * rr + e];
      }
    }
#pragma unroll
    for (int u = 0; u < kSumU; ++u) {
      const int e = e0 + u * kThreads;
      if (e >= rr) continue;
      const int a = e / r, b = e - a * r;
      G[a * ld + b] = v[u];
      if (a == b) tr += v[u];
    }
  }
  const double norm_sq = cta_sum(tr, red);
  const double inv = 1.0 / sqrt(fmax(norm_sq, static_cast<double>(ns.norm_floor)));
  const double inv2 = inv * inv;
  for (int e = tid; e < rr; e += kThreads) {
    const int a = e / r, b = e - a * r;
    G[a * ld + b] *= inv2;
    P[a * ld + b] = (a == b) ? 1.0 : 0.0;
  }
  __syncthreads();
  for (int it = 0; it < ns.iters; ++it) {
    const double c0 = ns.c[it][0], c1 = ns.c[it][1], c2 = ns.c[it][2];
    if (c2 != 0.0) cta_symm_mm(S, G, G, rp, ld);
    for (int e = tid; e < rr; e += kThreads) {
      const int a = e / r, b = e - a * r;
      const double g2 = (c2 != 0.0) ? S[a * ld + b] : 0.0;
      S[a * ld + b] = ((a == b) ? c0 : 0.0) + c1 * G[a * ld + b] + c2 * g2;
    }
    __syncthreads();
    cta_symm_mm(P, P, S, rp, ld);            // P <- P S
    cta_symm_mm(G, S, G, rp, ld);            // G <- S G S
    cta_symm_mm(G, G, S, rp, ld);
  }
  float* Pm = reinterpret_cast<float*>(tb.ws) + M.p_off;
  for (int e = tid; e < rr; e += kThreads) {
    const int a = e / r, b = e - a * r;
    Pm[e] = static_cast<float>(P[a * ld + b] * inv);
  }
}

// =====================================================================================
// Newton-Schulz solve with the three matrices in shared memory. They are symmetric, so only
// their upper 8 x 8 blocks are stored (packed row by row: 136 blocks, 204 KB for r = 128);
// a block holds all 64 entries, XOR-swizzled (column j of row i
// at i*8 + (j ^ 4*((i>>1)&1))) so that the MMA fragments of a block or of its transpose are
// two wavefronts. NT / 32 warps, up to nine output blocks each: every product is one pass,
// held in registers across a barrier and written in place. Launched for 64 < r <= 128
// with sixteen warps.
// =====================================================================================
constexpr int kNsPThreads = 512, kNsPU = 9;
__host__ __device__ inline int ns_packed_blocks(int r) { const int nb = pad8(r) >> 3; return nb * (nb + 1) / 2; }

// Shared-memory index of element (row, col) of a packed symmetric matrix with nb block rows.
__device__ __forceinline__ int nsp_idx(int row, int col, int nb) {
  int bi = row >> 3, bj = col >> 3, i = row & 7, j = col & 7;
  if (bi > bj) { const int t = bi; bi = bj; bj = t; const int u = i; i = j; j = u; }
  const int q = bi * nb - ((bi * (bi - 1)) >> 1) + (bj - bi);
  return q * 64 + i * 8 + (j ^ (((i >> 1) & 1) << 2));
}

// C = A B (symmetric, commuting, packed); C may be A or B. Per k block kb a warp reads, for
// each of its output blocks (bi, bj), block (bi, kb) of A and (kb, bj) of B, each stored
// as itself or as its transpose: in-block offsets dir (row g, column k) and tr (row k,
// column g) are fixed per thread, so a k step costs a few integer adds per block.
__device__ __forceinline__ int nsp_row0(int b, int nb) { return b * nb - ((b * (b - 1)) >> 1); }
template <int NT>
__device__ void nsp_mm(double* C, const double* A, const double* B, int nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  constexpr int nw = NT / 32;
  const int nq = nb * (nb + 1) / 2;
  int bi[kNsPU], bj[kNsPU], rsi[kNsPU], rsj[kNsPU];
  double acc[kNsPU][2];
#pragma unroll
  for (int u = 0; u < kNsPU; ++u) {
    int q = warp + u * nw;
    bi[u] = -1; bj[u] = 0;
    acc[u][0] = 0.0; acc[u][1] = 0.0;
    if (q < nq) {
      int row = 0;
      while (q >= nb - row) { q -= nb - row; ++row; }
      bi[u] = row; bj[u] = row + q;
    }
    rsi[u] = nsp_row0(bi[u] < 0 ? 0 : bi[u], nb);
    rsj[u] = nsp_row0(bj[u], nb);
  }
  int dir[2], tr[2];                                   // k half kh: columns / rows 4kh + t
#pragma unroll
  for (int kh = 0; kh < 2; ++kh) {
    const int k = 4 * kh + t;
    dir[kh] = g * 8 + (k ^ (((g >> 1) & 1) << 2));
    tr[kh] = k * 8 + (g ^ (((k >> 1) & 1) << 2));
  }
  for (int kb = 0; kb < nb; ++kb) {
    const int rsk = nsp_row0(kb, nb);
#pragma unroll
    for (int u = 0; u < kNsPU; ++u) {
      if (bi[u] < 0) continue;
      const bool at = bi[u] <= kb, bt = kb <= bj[u];
      const double* a = A + 64 * (at ? rsi[u] + kb - bi[u] : rsk + bi[u] - kb);
      const double* b = B + 64 * (bt ? rsk + bj[u] - kb : rsj[u] + kb - bj[u]);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh)
        dmma8x8x4(acc[u][0], acc[u][1], a[at ? dir[kh] : tr[kh]], b[bt ? tr[kh] : dir[kh]]);
    }
  }
  __syncthreads();                                     // every read of A and B is done
#pragma unroll
  for (int u = 0; u < kNsPU; ++u) {
    if (bi[u] < 0) continue;
    const int row = 8 * bi[u] + g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = 8 * bj[u] + 2 * t + h;
      if (bi[u] == bj[u] && col < row) continue;          // the mirror of the upper half
      C[nsp_idx(row, col, nb)] = acc[u][h];
      if (bi[u] == bj[u] && col != row) C[nsp_idx(col, row, nb)] = acc[u][h];
    }
  }
  __syncthreads();
}

template <int NT>
__global__ void __launch_bounds__(NT, 1) k_ns_solve_packed(Tables tb, const MatD* __restrict__ mats,
                                                                                 NSArgs ns) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[NT];
  const MatD M = mats[blockIdx.x];
  const int r = static_cast<int>(M.r);
  const int rr = r * r;
  const int nb = pad8(r) >> 3, mm = ns_packed_blocks(r) * 64;
  const int tid = threadIdx.x;
  double* G = reinterpret_cast<double*>(smem_raw);
  double* P = G + mm;
  double* S = P + mm;
  for (int e = tid; e < 3 * mm; e += NT) G[e] = 0.0;   // padding rows and columns stay zero
  __syncthreads();
  double tr = 0.0;
  const double* part = reinterpret_cast<const double*>(tb.ws) + M.gram_off;
  constexpr int kSumU = 4;                             // independent partial loads in flight
  for (int e0 = tid; e0 < rr; e0 += kSumU * NT) {
    double v[kSumU];
#pragma unroll
    for (int u = 0; u < kSumU; ++u) v[u] = 0.0;
    for (int sg = 0; sg < M.nseg; ++sg) {
#pragma unroll
      for (int u = 0; u < kSumU; ++u) {
        const int e = e0 + u * NT;
        if (e < rr) v[u] += part[static_cast<int64_t>(sg) * rr + e];
      }
    }
#pragma unroll
    for (int u = 0; u < kSumU; ++u) {
      const int e = e0 + u * NT;
      if (e >= rr) continue;
      const int a = e / r, b = e - a * r;
      if ((a >> 3) > (b >> 3)) continue;               // the lower blocks are the upper ones
      G[nsp_idx(a, b, nb)] = v[u];
      if (a == b) tr += v[u];
    }
  }
  red[tid] = tr;
  __syncthreads();
  for (int w = NT / 2; w > 0; w >>= 1) {
    if (tid < w) red[tid] += red[tid + w];
    __syncthreads();
  }
  const double norm_sq = red[0];
  const double inv = 1.0 / sqrt(fmax(norm_sq, static_cast<double>(ns.norm_floor)));
  const double inv2 = inv * inv;
  // every stored element: block q, entry (i, j) -> matrix element (8bi+i, 8bj+j')
  auto each = [&](auto&& f) {
    for (int e = tid; e < mm; e += NT) {
      int q = e >> 6, row = 0;
      while (q >= nb - row) { q -= nb - row; ++row; }
      const int i = (e >> 3) & 7, js = e & 7;
      const int a = 8 * row + i, b = 8 * (row + q) + (js ^ (((i >> 1) & 1) << 2));
      if (a < r && b < r) f(e, a, b);
    }
  };
  each([&](int e, int a, int b) {
    G[e] *= inv2;
    P[e] = (a == b) ? 1.0 : 0.0;
  });
  __syncthreads();
  for (int it = 0; it < ns.iters; ++it) {
    const double c0 = ns.c[it][0], c1 = ns.c[it][1], c2 = ns.c[it][2];
    if (c2 != 0.0) nsp_mm<NT>(S, G, G, nb);
    each([&](int e, int a, int b) {
      const double g2 = (c2 != 0.0) ? S[e] : 0.0;
      S[e] = ((a == b) ? c0 : 0.0) + c1 * G[e] + c2 * g2;
    });
    __syncthreads();
    nsp_mm<NT>(P, P, S, nb);                               // P <- P S
    nsp_mm<NT>(G, S, G, nb);                               // G <- S G S
    nsp_mm<NT>(G, G, S, nb);
  }
  float* Pm = reinterpret_cast<float*>(tb.ws) + M.p_off;
  for (int e = tid; e < rr; e += NT) {
    const int a = e / r, b = e - a * r;
    Pm[e] = static_cast<float>(P[nsp_idx(a, b, nb)] * inv);
  }
}

// Cholesky of the r x r symmetric matrix A (row-major, pitch r) in place and the inverse
// of its upper factor: afterwards A's upper triangle holds R (G = R^T R, pivots
// sqrt(max(d, fl)), the clamp of the reference MGS norms) and Ri holds R^{-1} (zero below
// the diagonal). Right-looking on the upper triangle with one barrier per column (row j of
// R is scaled one step later, when nothing reads it; piv carries the pivots across the
// barrier), then R^{-1} row by row from the bottom with four threads per column
// (shuffle-reduced). piv: r doubles of shared memory. Ends with a barrier.
__device__ void cta_chol_rinv(double* A, double* Ri, double* piv, int r, double fl) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int j = 0; j < r; ++j) {
    const double dd = fmax(A[j * r + j], fl);          // nothing writes A[j][j] in step j
    if (tid == 0) piv[j] = sqrt(dd);
    if (j > 0) {                                       // row j - 1 of R (no longer read)
      const double dp = piv[j - 1], idp = 1.0 / dp;
      for (int i = j - 1 + tid; i < r; i += kThreads) A[(j - 1) * r + i] = (i == j - 1) ? dp : A[(j - 1) * r + i] * idp;
    }
    const double idd = 1.0 / dd;                       // (x / d)(y / d) = x y / d^2
    for (int a = j + 1 + warp; a < r; a += kThreads / 32) {
      const double sa = A[j * r + a] * idd;
      for (int b = a + lane; b < r; b += 32) A[a * r + b] = fma(-sa, A[j * r + b], A[a * r + b]);
    }
    __syncthreads();
  }
  if (tid == 0) A[(r - 1) * r + r - 1] = piv[r - 1];
  __syncthreads();
  // R^{-1}, rows from the bottom: Ri[i][c] = -(sum_{i<k<=c} R[i][k] Ri[k][c]) / R[i][i]
  for (int i = r - 1; i >= 0; --i) {
    const double irii = 1.0 / A[i * r + i];
    for (int c0 = 0; c0 < r; c0 += kThreads / 4) {
      const int c = c0 + (tid >> 2), sl = tid & 3;
      double acc = 0.0;
      if (c > i && c < r)
        for (int k = i + 1 + sl; k <= c; k += 4) acc += A[i * r + k] * Ri[k * r + c];
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (sl == 0 && c < r) Ri[i * r + c] = (c == i) ? irii : (c > i ? -acc * irii : 0.0);
    }
    __syncthreads();
  }
}

// Blocked form of cta_chol_rinv for r % 8 == 0 (same factor and inverse up to rounding),
// with look-ahead: one barrier per 8-wide block column J. In phase J the warps apply the
// trailing update of every upper block (K, L), J < K <= L, each recomputing the row-panel
// products it needs, P_K = R_JJ^{-T} A_JK, from the unmodified row J (two fp64 MMAs per
// block, transposed into operand layout by shuffles); warp 0 updates (J+1, J+1) first and
// then factors it (scalar steps, the same pivot clamp) and inverts it into Ri's diagonal
// block while the other warps finish; the others also write row J-1's panel R_{J-1,K} in
// place (nobody reads row J-1 in phase J). R^{-1}'s off-diagonal blocks follow by block
// back-substitution, X_IJ = -R_II^{-1} sum_{I<K<=J} R_IK X_KJ, block rows from the bottom.
// A's lower triangle is left as it was.
__device__ void cta_chol_rinv8(double* A, double* Ri, int r, double fl) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, kq = lane & 3;
  const int nb = r >> 3, nw = kThreads / 32;
  for (int e = tid; e < r * r; e += kThreads) Ri[e] = 0.0;
  __syncthreads();
  // warp 0: factor the 8 x 8 diagonal block J in place and write its inverse into Ri
  auto diag = [&](int J) {
    double* AJJ = A + 8 * J * r + 8 * J;
    double* RJJ = Ri + 8 * J * r + 8 * J;
    double idj = 0.0;                                // lane jj keeps 1 / R_jj of this block
    for (int jj = 0; jj < 8; ++jj) {
      // one reciprocal square root per column (the chain of divisions and square roots is
      // the serial path of the factorisation): 1/d, d = dd/d and 1/dd = (1/d)^2
      const double dd = fmax(AJJ[jj * r + jj], fl);
      const double id = rsqrt(dd), d = dd * id, idd = id * id;
      if (lane == jj) idj = id;
      int p = lane, a = jj + 1;                      // pair (a, b), jj < a <= b < 8, per lane
      while (a < 8 && p >= 8 - a) { p -= 8 - a; ++a; }
      const int b = a + p;
      double upd = 0.0, rowv = 0.0;
      if (a < 8) upd = fma(-AJJ[jj * r + a] * idd, AJJ[jj * r + b], AJJ[a * r + b]);
      if (lane > jj && lane < 8) rowv = AJJ[jj * r + lane] * id;
      __syncwarp();
      if (a < 8) AJJ[a * r + b] = upd;
      if (lane == jj) AJJ[jj * r + jj] = d;
      if (lane > jj && lane < 8) AJJ[jj * r + lane] = rowv;
      __syncwarp();
    }
    for (int i = 7; i >= 0; --i) {                   // its inverse, rows from the bottom
      const double irii = __shfl_sync(0xffffffffu, idj, i);
      const int c = lane >> 2, sl = lane & 3;
      double acc = 0.0;
      if (c > i)
        for (int k = i + 1 + sl; k <= c; k += 4) acc += AJJ[i * r + k] * RJJ[k * r + c];
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (sl == 0 && c >= i) RJJ[i * r + c] = (c == i) ? irii : -acc * irii;
      __syncwarp();
    }
  };
  // operand fragment of column c of a transposed panel product held as an MMA result
  // (lane (g, kq) holds P^T[g][2kq], P^T[g][2kq + 1]): P^T[g][c] for this lane's c
  auto frag = [&](double p0, double p1, int c) {
    const int src = (lane & ~3) | (c >> 1);
    const double v0 = __shfl_sync(0xffffffffu, p0, src), v1 = __shfl_sync(0xffffffffu, p1, src);
    return (c & 1) ? v1 : v0;
  };
  if (warp == 0) diag(0);
  __syncthreads();
  for (int J = 0; J < nb; ++J) {
    const double* RJJ = Ri + 8 * J * r + 8 * J;      // R_JJ^{-1}
    const int m = nb - 1 - J, np = m * (m + 1) / 2;
    // P_K^T = A_JK^T R_JJ^{-1} (lane (g, kq): P_K^T[g][2kq..2kq+1])
    auto panelT = [&](int K, double& p0, double& p1) {
      const double* AJK = A + 8 * J * r + 8 * K;
      p0 = 0.0; p1 = 0.0;
#pragma unroll
      for (int k0 = 0; k0 < 8; k0 += 4) dmma8x8x4(p0, p1, AJK[(k0 + kq) * r + g], RJJ[(k0 + kq) * r + g]);
    };
    auto trailing = [&](int q) {                     // A_KL -= P_K^T P_L for upper block q
      int p = q, K = J + 1;
      while (p >= nb - K) { p -= nb - K; ++K; }
      const int L = K + p;
      double pk0, pk1, pl0, pl1;
      panelT(K, pk0, pk1);
      if (L == K) { pl0 = pk0; pl1 = pk1; } else panelT(L, pl0, pl1);
      double* AKL = A + 8 * K * r + 8 * L;
      double c0 = AKL[g * r + 2 * kq], c1 = AKL[g * r + 2 * kq + 1];
#pragma unroll
      for (int k0 = 0; k0 < 8; k0 += 4)
        dmma8x8x4(c0, c1, -frag(pk0, pk1, k0 + kq), frag(pl0, pl1, k0 + kq));
      AKL[g * r + 2 * kq] = c0;
      AKL[g * r + 2 * kq + 1] = c1;
    };
    if (warp == 0) {
      if (np > 0) {                                  // (J+1, J+1), then factor it
        trailing(0);
        __syncwarp();
        diag(J + 1);
      }
    } else {
      for (int q = warp; q < np; q += nw - 1) trailing(q);
      if (J > 0) {                                   // row J-1's panel: R_{J-1,K} in place
        const double* RPP = Ri + 8 * (J - 1) * r + 8 * (J - 1);
        for (int K = J + warp - 1; K < nb; K += nw - 1) {
          double* APK = A + 8 * (J - 1) * r + 8 * K;
          double c0 = 0.0, c1 = 0.0;
#pragma unroll
          for (int k0 = 0; k0 < 8; k0 += 4) dmma8x8x4(c0, c1, RPP[(k0 + kq) * r + g], APK[(k0 + kq) * r + g]);
          __syncwarp();
          APK[g * r + 2 * kq] = c0;
          APK[g * r + 2 * kq + 1] = c1;
        }
      }
    }
    __syncthreads();
  }
  for (int I = nb - 2; I >= 0; --I) {                // off-diagonal blocks of R^{-1}
    for (int J = I + 1 + warp; J < nb; J += nw) {
      double t0 = 0.0, t1 = 0.0;
      for (int K = I + 1; K <= J; ++K) {
        const double* RIK = A + 8 * I * r + 8 * K;
        const double* XKJ = Ri + 8 * K * r + 8 * J;
#pragma unroll
        for (int k0 = 0; k0 < 8; k0 += 4) dmma8x8x4(t0, t1, RIK[g * r + k0 + kq], XKJ[(k0 + kq) * r + g]);
      }
      double* XIJ = Ri + 8 * I * r + 8 * J;          // stage T there, then X = -R_II^{-1} T
      XIJ[g * r + 2 * kq] = t0;
      XIJ[g * r + 2 * kq + 1] = t1;
      __syncwarp();
      const double* RII = Ri + 8 * I * r + 8 * I;
      double x0 = 0.0, x1 = 0.0;
#pragma unroll
      for (int k0 = 0; k0 < 8; k0 += 4) dmma8x8x4(x0, x1, -RII[g * r + k0 + kq], XIJ[(k0 + kq) * r + g]);
      __syncwarp();
      XIJ[g * r + 2 * kq] = x0;
      XIJ[g * r + 2 * kq + 1] = x1;
    }
    __syncthreads();
  }
}

// =====================================================================================
// CholeskyQR step for the power-iteration bases, one CTA per W matrix: G = W^T W (the
// Gram partials, one per segment, summed here), G = R^T R with pivots
// sqrt(max(d, norm_floor)) (the clamp of the reference MGS, ds_mezo/kernels.py:238), and
// R^{-1}. The factorization is right-looking with one barrier per column on the upper
// triangle (row j of A ends as row j of R; it is scaled one step later, when nothing reads
// it any more); R^{-1} is formed row by row from the bottom with four threads per column
// (shuffle-reduced). Exports R^{-1} in fp32 (apply matrix) and fp64 (after the
// workspace's first r*r doubles).
// =====================================================================================
__global__ void __launch_bounds__(kThreads) k_chol(Tables tb, const MatD* __restrict__ mats, float norm_floor,
                                                   int summed) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const MatD M = mats[blockIdx.x];
  const int r = static_cast<int>(M.r);
  const int rr = r * r;
  const int tid = threadIdx.x;
  const double fl = static_cast<double>(norm_floor);
  // r <= 64: factor and inverse in shared memory; larger r works on the fp64 workspace
  const bool in_smem = r <= 64;
  double* dw = reinterpret_cast<double*>(tb.ws) + M.dw_off;
  double* A = in_smem ? reinterpret_cast<double*>(smem_raw) : dw;
  double* Ri = in_smem ? A + rr : dw + 2 * rr;
  const double* part = reinterpret_cast<const double*>(tb.ws) + M.gram_off;
  const int nsg = summed ? 1 : M.nseg;              // summed: the Gram is in the first slot already
  constexpr int kSumU = 8;                             // independent partial loads in flight
  for (int e0 = tid; e0 < rr; e0 += kSumU * kThreads) {
    double v[kSumU];
#pragma unroll
    for (int u = 0; u < kSumU; ++u) v[u] = 0.0;
    for (int sg = 0; sg < nsg; ++sg) {
#pragma unroll
      for (int u = 0; u < kSumU; ++u) {
        const int e = e0 + u * kThreads;
        if (e < rr) v[u] += part[static_cast<int64_t>(sg) * rr + e];
      }
    }
#pragma unroll
    for (int u = 0; u < kSumU; ++u) {
      const int e = e0 + u * kThreads;
      if (e < rr) { A[e] = v[u]; Ri[e] = 0.0; }
    }
  }
  __syncthreads();
  __shared__ double piv[DSMZ_MAX_RANK];
  if ((r & 7) == 0) cta_chol_rinv8(A, Ri, r, fl);
  else cta_chol_rinv(A, Ri, piv, r, fl);
  float* Pm = reinterpret_cast<float*>(tb.ws) + M.p_off;
  double* Rd = dw + rr;                       // fp64 copy for the fp64-accumulated apply
  for (int e = tid; e < rr; e += kThreads) {
    Pm[e] = static_cast<float>(Ri[e]);
    Rd[e] = Ri[e];
  }
}

// out[v][c] = sum_{a<K} X[v*xld + a] * P[a*pld + c] with fp32 X, fp64 P and fp64 sums,
// 4 vectors x 8 columns per thread: column pairs 2cb + g*pld/4 (g < 4), so a warp's double2
// loads of a P row are one contiguous run (pld % 8 == 0, columns zero-padded to pld).
// =====================================================================================
// Apply: X[v,:] = x_v^T Pm for every vector of every matrix segment.
// OUT 0: param -= eta * X (factor dtype), optional scratch = X  (ds_mezo/kernels.py:84-92).
// OUT 1: param (fp32) = X (CholeskyQR: V = Q1 R2^-1).
// SRC 1 recomputes the Kalman update and writes mu, var (controller.py:283-285).
// Loads and stores run in coalesced element order; the r x r product in between runs
// from shared memory with rows_x_mat.
// =====================================================================================
template <int SRC, int OUT>
__global__ void __launch_bounds__(kThreads) k_apply(Tables tb, const MatD* __restrict__ mats, int nmats,
                                                    KalmanIn kin, float eta, int pdt) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int seg = blockIdx.x;
  const int mi = find_owner(mats, nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = mats[mi];
  const int r = static_cast<int>(M.r);
  const int r8 = pad8(r);
  const int TV = tile_vectors(r);
  const int xld = r8 + 1;
  float* Ps = reinterpret_cast<float*>(smem_raw);  // r x r8
  float* xs = Ps + r * r8;                         // TV x xld
  float* os = xs + TV * xld;                       // TV x xld
  const int tid = threadIdx.x;
  const float* Pm = reinterpret_cast<const float*>(tb.ws) + M.p_off;
  for (int e = tid; e < r * r8; e += kThreads) {
    const int a = e / r8, c = e - a * r8;
    Ps[e] = (c < r) ? Pm[a * r + c] : 0.f;
  }
  KalScal ks{};
  if (SRC == 1) ks = kal_derive(kin, reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off);
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  __syncthreads();
  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    const int n = nv * r;
    for (int base = tid; base < n; base += kThreads * kUnroll) {
      float m0[kUnroll], w0[kUnroll], z0[kUnroll];
      int vv[kUnroll], kk[kUnroll];
      int64_t ad[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {            // issue every load before using any
        const int e = base + u * kThreads;
        elem_vk(M.side, e, r, nv, vv[u], kk[u]);
        ad[u] = vaddr2(M, s0 + vv[u], kk[u]);
        if (e < n) {
          m0[u] = M.mu[ad[u]];
          if (SRC == 1) { w0[u] = M.var[ad[u]]; z0[u] = M.z[ad[u]]; }
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (base + u * kThreads >= n) continue;
        float x = m0[u];
        if (SRC == 1) {
          float mu1, var1, mu2, var2;
          kal_predict(m0[u], w0[u], ks, mu1, var1);
          kal_observe(mu1, var1, z0[u], ks, mu2, var2);
          M.mu[ad[u]] = mu2;
          M.var[ad[u]] = var2;
          x = mu2;
        }
        xs[vv[u] * xld + kk[u]] = x;
      }
    }
    __syncthreads();
    rows_x_mat(xs, xld, Ps, r8, nv, r, r, [&](int v, int c, float x) { os[v * xld + c] = x; });
    __syncthreads();
    for (int base = tid; base < n; base += kThreads * kUnroll) {
      float p0[kUnroll];
      int vv[kUnroll], kk[kUnroll];
      int64_t ad[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int e = base + u * kThreads;
        elem_vk(M.side, e, r, nv, vv[u], kk[u]);
        ad[u] = vaddr2(M, s0 + vv[u], kk[u]);
        if (OUT == 0 && e < n) p0[u] = ldf(M.param, ad[u], pdt);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (base + u * kThreads >= n) continue;
        const float X = os[vv[u] * xld + kk[u]];
        if (OUT == 0) {
          stf(M.param, ad[u], __fsub_rn(p0[u], __fmul_rn(eta, X)), pdt);
          if (M.scratch) M.scratch[ad[u]] = X;
        } else {
          reinterpret_cast<float*>(M.param)[ad[u]] = X;
        }
      }
    }
    __syncthreads();
  }
}

// =====================================================================================
// B-side reductions per (module, chunk of d_in): B V and var_B (V*V), both R x RC
// (ds_mezo/kernels.py:325-326 and controller.py:183). Partials summed by k_coef.
// 64 x 64 output blocks; a thread holds 4 x 4 of each product. The chunk is walked 32
// columns of d_in at a time: the next 32 columns' global loads are in flight while the
// current ones are multiplied, and the shared tiles are stored transposed (j-major, V*V
// formed once per element) so that a thread's four rows or four columns are one 16-byte
// load: per j, four 16-byte loads feed 32 FMAs.
// =====================================================================================
constexpr int kBsJ = 32, kBsP = 68;
// Read-only loads with a 256-byte L2 fill: a CTA walks each row 32 columns at a time, so
// the next steps' columns are already in L2.
__device__ __forceinline__ float ldg_l2pf(const float* p) {
  float v;
  asm("ld.global.nc.L2::256B.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__global__ void __launch_bounds__(kThreads, 2) k_bside(Tables tb, int64_t ncols) {
  __shared__ __align__(16) float sh[4][kBsJ][kBsP];
  float (*Bs)[kBsP] = sh[0];
  float (*Ws)[kBsP] = sh[1];
  float (*Vs)[kBsP] = sh[2];
  float (*Qs)[kBsP] = sh[3];
  static_assert(4 * kBsJ * kBsP >= 2 * 64 * 64, "the parity reduction reuses the operand tiles");
  const int tid = threadIdx.x;
  // Four groups of 64 threads: group g forms product g & 1 (B V, or var_B V^2) over the
  // columns jj of parity g >> 1. A thread holds rows {4bi..4bi+3, 32+4bi..} x columns
  // {4bj..4bj+3, 32+4bj..} of the 64 x 64 block: per jj, four 16-byte shared loads (each
  // quarter-warp reads 128 contiguous bytes) feed 64 FMAs.
  const int grp = tid >> 6, lt = tid & 63;
  const int pr = grp & 1, hp = grp >> 1;
  const int bi = lt >> 3, bj = lt & 7;
  // this CTA's range of the concatenated d_in columns, and the modules it meets
  const int64_t G = gridDim.x, cb = blockIdx.x;
  const int64_t g0 = cb * ncols / G, g1 = (cb + 1) * ncols / G;
  int mi = 0;
  for (int lo = 0, hi = tb.nmods - 1; lo <= hi;) {   // last module with col0 <= g0
    const int mid = (lo + hi) >> 1;
    if (tb.mods[mid].col0 <= g0) { mi = mid; lo = mid + 1; } else { hi = mid - 1; }
  }
  for (; mi < tb.nmods && tb.mods[mi].col0 < g1; ++mi) {
  const ModD D = tb.mods[mi];
  const BasisD Bd = tb.bases[D.basis];
  const int chunk = static_cast<int>(cb) - D.chunk0;  // this CTA's partial slot of the module
  const int R = D.r, RC = D.rc;
  const int64_t j0 = max(g0, D.col0) - D.col0;
  const int64_t j1 = min(g1, D.col0 + D.d_in) - D.col0;
  const bool with_var = (D.varB != nullptr);
  const float* V = Bd.Vin;
  const int64_t vs0 = Bd.v_s0, vs1 = Bd.v_s1;
  float* outp = reinterpret_cast<float*>(tb.ws) + D.bpart_off + static_cast<int64_t>(chunk) * 2 * R * RC;
  for (int rt = 0; rt < R; rt += 64) {
    for (int ct = 0; ct < RC; ct += 64) {
      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
      float lb[8], lw[8], lv[8];
      auto gload = [&](int64_t jb) {                // 24 independent loads per thread
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int e = tid + u * kThreads;
          const int rr = e >> 5, jj = e & 31;
          const int64_t j = jb + jj;
          const bool ok = (rt + rr < R) && (j < j1);
          const int64_t a = static_cast<int64_t>(rt + rr) * D.b_s0 + j * D.b_s1;
          // out-of-range elements load element 0 (always valid) and are replaced by zero
          const int64_t ac = ok ? a : 0;
          const float b0 = ldg_l2pf(D.Bp + ac);
          const float w0 = with_var ? ldg_l2pf(D.varB + ac) : 0.f;
          lb[u] = ok ? b0 : 0.f;
          lw[u] = ok ? w0 : 0.f;
          const int jv = e >> 6, cc = e & 63;
          const int64_t jv_g = jb + jv;
          const bool vok = jv_g < j1 && ct + cc < RC;
          const float v0 = ldg_l2pf(V + (vok ? jv_g * vs0 + static_cast<int64_t>(ct + cc) * vs1 : 0));
          lv[u] = vok ? v0 : 0.f;
        }
      };
      gload(j0);
      for (int64_t jb = j0; jb < j1; jb += kBsJ) {
        __syncthreads();                            // the previous columns are consumed
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int e = tid + u * kThreads;
          Bs[e & 31][e >> 5] = lb[u];
          Ws[e & 31][e >> 5] = lw[u];
          Vs[e >> 6][e & 63] = lv[u];
          Qs[e >> 6][e & 63] = lv[u] * lv[u];
        }
        __syncthreads();
        if (jb + kBsJ < j1) gload(jb + kBsJ);
        const float (*As)[kBsP] = pr ? Ws : Bs;
        const float (*Cs)[kBsP] = pr ? Qs : Vs;
#pragma unroll 4
        for (int jj = hp; jj < kBsJ; jj += 2) {
          const float4 a0 = *reinterpret_cast<const float4*>(&As[jj][4 * bi]);
          const float4 a1 = *reinterpret_cast<const float4*>(&As[jj][32 + 4 * bi]);
          const float4 c0 = *reinterpret_cast<const float4*>(&Cs[jj][4 * bj]);
          const float4 c1 = *reinterpret_cast<const float4*>(&Cs[jj][32 + 4 * bj]);
          const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; j += 2) {   // packed fp32x2 FMA, each component as fmaf
              asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %2};\n mov.b64 rb, {%3, %4};\n mov.b64 rc, {%0, %1};\n"
                  " fma.rn.f32x2 rc, ra, rb, rc;\n mov.b64 {%0, %1}, rc;\n}"
                  : "+f"(acc[i][j]), "+f"(acc[i][j + 1])
                  : "f"(av[i]), "f"(cv[j]), "f"(cv[j + 1]));
            }
        }
      }
      // the odd-column groups hand their sums to the even-column groups, which write
      float* red = &sh[0][0][0];
      __syncthreads();
      if (hp == 1) {
#pragma unroll
        for (int e = 0; e < 64; ++e) red[pr * 4096 + e * 64 + lt] = acc[e >> 3][e & 7];
      }
      __syncthreads();
      if (hp == 0) {
        float* o = outp + pr * R * RC;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int rr = rt + (i < 4 ? 4 * bi + i : 28 + 4 * bi + i);
            const int cc = ct + (j < 4 ? 4 * bj + j : 28 + 4 * bj + j);
            if (rr < R && cc < RC) o[rr * RC + cc] = acc[i][j] + red[pr * 4096 + (i * 8 + j) * 64 + lt];
          }
      }
      __syncthreads();                              // the tiles are rewritten by the next block
    }
  }
  }
}

// Per module: sum the chunk partials (fp64), Zc_B = randn(R,RC) * sqrt(var_B V^2)
// (controller.py:183-186), and Q = MGS(B V)[:, :RCA] (ds_mezo/kernels.py:328-340) in fp64
// by one warp. MODE 0 draws Zc_B from the torch Philox stream, MODE 1 copies it.
// =====================================================================================
constexpr int kQBlocks = 8;    // output blocks per warp per pass of the Q update (64 x 64: one pass)
// The QR of B V keeps G and R^{-1} in shared memory beside B V up to 64 x 64; beyond that
// they live in the module's fp64 workspace (qrw_off) and B V alone stays on chip.
__host__ __device__ inline bool coef_qr_in_smem(int R, int RCA) { return RCA <= 64 && R <= 64; }
template <int MODE>
__global__ void __launch_bounds__(kThreads) k_coef(Tables tb, uint64_t seed, uint64_t base_off, float norm_floor,
                                                   int with_qr) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const ModD D = tb.mods[blockIdx.x];
  const int R = D.r, RC = D.rc, RCA = D.rca;
  const int tid = threadIdx.x;
  const int bld = R + 4;                              // padded column stride: the MMA fragments
                                                      // half-warp rows on distinct banks
  double* BVt = reinterpret_cast<double*>(smem_raw);  // RC x bld (column-major B V)
  const float* part = reinterpret_cast<const float*>(tb.ws) + D.bpart_off;
  float* ZcB = reinterpret_cast<float*>(tb.ws) + D.coef_off;
  float* Qo = ZcB + static_cast<int64_t>(R) * RC;
  for (int e = tid; e < R * RC; e += kThreads) {
    double sbv = 0.0, svb = 0.0;
    for (int c = 0; c < D.nchunk; ++c) {
      sbv += part[static_cast<int64_t>(c) * 2 * R * RC + e];
      svb += part[static_cast<int64_t>(c) * 2 * R * RC + R * RC + e];
    }
    const int i = e / RC, c = e - i * RC;
    BVt[c * bld + i] = sbv;
    if (MODE == 0) {
      const float g = torch_randn_at(seed, base_off + D.offB, D.thrB, e);
      ZcB[e] = __fmul_rn(g, sqrtf(static_cast<float>(svb)));
    } else {
      ZcB[e] = D.zcB_ext[e];
    }
  }
  // Later directions of a many-direction step reuse the Q of direction 0 (B V is the same).
  if (!with_qr) return;
  __syncthreads();
  // Q = QR(B V)[:, :RCA] with a positive diagonal, the factor the reference's modified
  // Gram-Schmidt produces (ds_mezo/kernels.py:328-340), as CholeskyQR2 in fp64: two rounds of
  // G = Q^T Q, G = R^T R, Q <- Q R^{-1}, every step parallel over the CTA. Up to 64 x 64 any
  // shape; beyond, blocks of 8 (G and R^{-1} in the workspace).
  const bool in_smem = coef_qr_in_smem(R, RCA);
  if (in_smem || ((R & 7) == 0 && (RCA & 7) == 0)) {
  __shared__ double piv[DSMZ_MAX_RANK];
  double* G = in_smem ? BVt + RC * bld : reinterpret_cast<double*>(tb.ws) + D.qrw_off;   // RCA x RCA
  double* Rm = G + RCA * RCA;               // inverse of the upper factor
  for (int round = 0; round < 2; ++round) {
    if ((R & 3) == 0 && (RCA & 7) == 0) {
      // G = Q^T Q on the fp64 MMA: the upper 8 x 8 blocks, mirrored; Q^T is BVt row-major
      // (pitch bld), so both fragments are BVt rows: A[g][k] = BVt[(8bi+g)*bld + k],
      // B[k][g] = BVt[(8bj+g)*bld + k].
      const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, kq = lane & 3;
      const int nb = RCA >> 3, nq = nb * (nb + 1) / 2;
      for (int q0 = warp; q0 < nq; q0 += kThreads / 32) {
        int qq = q0, rb = 0;
        while (qq >= nb - rb) { qq -= nb - rb; ++rb; }
        const int bi = rb, bj = rb + qq;
        double c0 = 0.0, c1 = 0.0;
        const double* ar = BVt + (8 * bi + g) * bld + kq;
        const double* br = BVt + (8 * bj + g) * bld + kq;
        for (int k0 = 0; k0 < R; k0 += 4) dmma8x8x4(c0, c1, ar[k0], br[k0]);
        const int row = 8 * bi + g;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = 8 * bj + 2 * kq + h;
          const double v = h ? c1 : c0;
          G[row * RCA + col] = v;
          G[col * RCA + row] = v;
        }
      }
    } else {
      for (int e = tid; e < RCA * RCA; e += kThreads) {
        const int a = e / RCA, b = e - a * RCA;
        const double* qa = BVt + a * bld;
        const double* qb = BVt + b * bld;
        double sacc = 0.0;
        for (int i = 0; i < R; ++i) sacc = fma(qa[i], qb[i], sacc);
        G[e] = sacc;
      }
    }
    __syncthreads();
    // Second round: after an fp64 first round, G = Q1^T Q1 = I + E with |E| ~ u cond(B V)^2,
    // and R = I + U + O(E^2), R^{-1} = I - U + O(E^2) with U = E's upper triangle, its
    // diagonal halved. For max|E| <= 1e-6 the dropped terms are below 1e-10 of Q's entries,
    // far under the fp32 Q written here, so the second factorisation (the serial part of this
    // kernel) is skipped; a larger or non-finite E factors G in full.
    bool near_identity = false;
    if (round == 1) {
      __shared__ double s_emax[kThreads / 32];
      double e = 0.0;
      for (int idx = tid; idx < RCA * RCA; idx += kThreads) {
        const int a = idx / RCA, c = idx - a * RCA;
        const double x = fabs(G[idx] - (a == c ? 1.0 : 0.0));
        if (!(x <= e)) e = x;                          // NaN propagates
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const double y = __shfl_xor_sync(0xffffffffu, e, o);
        if (!(y <= e)) e = y;
      }
      if ((tid & 31) == 0) s_emax[tid >> 5] = e;
      __syncthreads();
      e = 0.0;
      for (int w = 0; w < kThreads / 32; ++w) if (!(s_emax[w] <= e)) e = s_emax[w];
      near_identity = e <= 1e-6;
      if (near_identity) {
        for (int idx = tid; idx < RCA * RCA; idx += kThreads) {
          const int a = idx / RCA, c = idx - a * RCA;
          Rm[idx] = (a == c) ? 1.0 - 0.5 * (G[idx] - 1.0) : (a < c ? -G[idx] : 0.0);
        }
        __syncthreads();
      }
    }
    if (!near_identity) {
      if ((RCA & 7) == 0) cta_chol_rinv8(G, Rm, RCA, static_cast<double>(norm_floor));
      else cta_chol_rinv(G, Rm, piv, RCA, static_cast<double>(norm_floor));
    }
    if ((R & 7) == 0 && (RCA & 7) == 0) {
      // Q <- Q R^{-1} on the fp64 MMA, as Q^T <- R^{-T} Q^T on BVt (Q^T row-major): output
      // block (column block cb of Q, row block ib of Q) = sum_{a < 8cb+8} R^{-1}[a][8cb+..]
      // Q^T[a][8ib+..] (R^{-1} upper), held in registers across a barrier, then in place.
      // Passes take column blocks from the last: a pass writes only rows of Q^T that later
      // passes (lower column blocks) no longer read. 64 x 64 is one pass, 128 x 128 four.
      const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, kq = lane & 3;
      const int ncb = RCA >> 3, nib = R >> 3;
      const int cpp = (kQBlocks * (kThreads / 32)) / nib;     // column blocks per pass (>= 4)
      for (int chi = ncb - 1; chi >= 0; chi -= cpp) {
        const int clo = chi - cpp + 1 > 0 ? chi - cpp + 1 : 0;
        const int nblk = (chi - clo + 1) * nib;
        double o[kQBlocks][2];
        int cbq[kQBlocks], ibq[kQBlocks];
#pragma unroll
        for (int u = 0; u < kQBlocks; ++u) {
          const int q = warp + u * (kThreads / 32);
          cbq[u] = q < nblk ? clo + q / nib : -1;
          ibq[u] = q < nblk ? q - (q / nib) * nib : 0;
          o[u][0] = 0.0; o[u][1] = 0.0;
          if (cbq[u] < 0) continue;
          const double* ra = Rm + kq * RCA + 8 * cbq[u] + g;
          const double* qb = BVt + kq * bld + 8 * ibq[u] + g;
          for (int k0 = 0; k0 < 8 * cbq[u] + 8; k0 += 4)
            dmma8x8x4(o[u][0], o[u][1], ra[k0 * RCA], qb[k0 * bld]);
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < kQBlocks; ++u) {
          if (cbq[u] < 0) continue;
          double* dst = BVt + (8 * cbq[u] + g) * bld + 8 * ibq[u] + 2 * kq;
          dst[0] = o[u][0];
          dst[1] = o[u][1];
        }
        __syncthreads();
      }
    } else {
    // Q <- Q R^{-1}: every output (i, c) = sum_{a<=c} Q[i][a] R^{-1}[a][c] held in registers
    // across a barrier, then written in place. Thread: row i = tid % R, columns
    // c = cg, cg + ncg, ... with cg = tid / R.
    {
      constexpr int kQc = 16;
      double out[kQc];
      const int i = tid % R, cg = tid / R, ncg = kThreads / R;
      const bool act = R <= kThreads && cg < ncg && i < R;
#pragma unroll
      for (int j = 0; j < kQc; ++j) out[j] = 0.0;
      if (act) {
        for (int a = 0; a < RCA; ++a) {
          const double qa = BVt[a * bld + i];
#pragma unroll
          for (int j = 0; j < kQc; ++j) {
            const int c = cg + j * ncg;
            if (c < RCA && a <= c) out[j] = fma(qa, Rm[a * RCA + c], out[j]);
          }
        }
      }
      __syncthreads();
      if (act) {
#pragma unroll
        for (int j = 0; j < kQc; ++j) {
          const int c = cg + j * ncg;
          if (c < RCA) BVt[c * bld + i] = out[j];
        }
      }
    }
    }
    __syncthreads();
  }
  } else if (tid < 32) {
    // RCA > 64: modified Gram-Schmidt by one warp (column-major, conflict-free lanes)
    const int lane = tid;
    for (int col = 0; col < RCA; ++col) {
      double* vc = BVt + col * bld;
      for (int prev = 0; prev < col; ++prev) {
        const double* qp = BVt + prev * bld;
        double d = 0.0;
        for (int i = lane; i < R; i += 32) d += vc[i] * qp[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        for (int i = lane; i < R; i += 32) vc[i] -= d * qp[i];
        __syncwarp();
      }
      double n2 = 0.0;
      for (int i = lane; i < R; i += 32) n2 += vc[i] * vc[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
      const double inv = 1.0 / sqrt(fmax(n2, static_cast<double>(norm_floor)));
      for (int i = lane; i < R; i += 32) vc[i] *= inv;
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = tid; e < R * RCA; e += kThreads) {
    const int i = e / RCA, k = e - i * RCA;
    Qo[e] = static_cast<float>(BVt[k * bld + i]);
  }
}

// =====================================================================================
// The AGZO perturbation of one module for the drop-in op (ds_mezo/kernels.py:290-368):
//   side A: z[i,:] = eps * Zc_A[i,:] Q^T  (Zc_A from the caller)
//   side B: z[:,j] = eps * Zc_B V[j,:]^T
// One CTA per vector segment; the grouped step uses the streaming sk::k_sperturb.
// =====================================================================================
__global__ void __launch_bounds__(kThreads) k_perturb(Tables tb, float eps) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int seg = blockIdx.x;
  const int mi = find_owner(tb.mats, tb.nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = tb.mats[mi];
  const ModD D = tb.mods[M.owner];
  const int r = static_cast<int>(M.r);
  const int R = D.r, RC = D.rc, RCA = D.rca;
  const int TV = tile_vectors(r);
  const int tid = threadIdx.x;
  const int KW = (M.side == 0) ? RCA : RC;     // inner width of the z product
  const int R8 = pad8(R);
  float* Cs = reinterpret_cast<float*>(smem_raw);        // KW x R8 : Q^T (side A) or Zc_B^T (side B)
  float* Ks = Cs + KW * R8;                              // TV x (KW+1): Zc_A rows or V rows
  float* zs = Ks + TV * (KW + 1);                        // TV x (r+1)
  const float* coef = reinterpret_cast<const float*>(tb.ws) + D.coef_off;
  if (M.side == 0) {
    const float* Q = coef + static_cast<int64_t>(R) * RC;   // R x RCA
    for (int e = tid; e < KW * R8; e += kThreads) {
      const int k = e / R8, c = e - k * R8;
      Cs[e] = (c < R) ? Q[c * RCA + k] : 0.f;
    }
  } else {
    for (int e = tid; e < KW * R8; e += kThreads) {
      const int k = e / R8, c = e - k * R8;
      Cs[e] = (c < R) ? coef[c * RC + k] : 0.f;
    }
  }
  const BasisD Bd = tb.bases[D.basis];
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  __syncthreads();
  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    for (int e = tid; e < nv * KW; e += kThreads) {
      const int v = e / KW, k = e - v * KW;
      const float x = (M.side == 0) ? D.zcA_ext[(s0 + v) * RCA + k]
                                    : Bd.Vin[(s0 + v) * Bd.v_s0 + static_cast<int64_t>(k) * Bd.v_s1];
      Ks[v * (KW + 1) + k] = x;
    }
    __syncthreads();
    rows_x_mat(Ks, KW + 1, Cs, R8, nv, KW, R, [&](int v, int c, float x) { zs[v * (r + 1) + c] = x * eps; });
    __syncthreads();
    const int n = nv * r;
    for (int e = tid; e < n; e += kThreads) {
      int v, k;
      elem_vk(M.side, e, r, nv, v, k);
      M.z[vaddr2(M, s0 + v, k)] = zs[v * (r + 1) + k];
    }
    __syncthreads();
  }
}

// =====================================================================================
// Frobenius norms of the fp32 master factors (ds_mezo/controller.py:78-82 takes their
// median for eps). Block (m, s) sums the squares of slice s of matrix m's elements in fp64;
// k_norm_finish adds the kNormSlices partials of each matrix in order (deterministic).
// =====================================================================================
constexpr int kNormSlices = 16;
__global__ void __launch_bounds__(kThreads) k_norm_partial(Tables tb, double* part) {
  __shared__ double red[kThreads / 32];
  const int m = blockIdx.x, sl = blockIdx.y;
  const MatD M = tb.mats[m];
  const int64_t n = M.nvec * M.r;
  const int64_t e0 = n * sl / kNormSlices, e1 = n * (sl + 1) / kNormSlices;
  const float* p = reinterpret_cast<const float*>(M.param);
  double acc = 0.0;
  for (int64_t e = e0 + threadIdx.x; e < e1; e += kThreads) {
    int64_t v, k;
    if (M.side == 0) { v = e / M.r; k = e - v * M.r; } else { k = e / M.nvec; v = e - k * M.nvec; }
    const double x = p[M.side == 0 ? v * M.ld + k * M.cs : k * M.ld + v * M.cs];
    acc = fma(x, x, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    part[m * kNormSlices + sl] = t;
  }
}
__global__ void __launch_bounds__(kThreads) k_norm_finish(const double* part, int nmats, float* norms) {
  const int m = blockIdx.x * kThreads + threadIdx.x;
  if (m >= nmats) return;
  double t = 0.0;
  for (int s = 0; s < kNormSlices; ++s) t += part[m * kNormSlices + s];
  norms[m] = static_cast<float>(sqrt(t));
}

// Sums the per-segment Kalman partials in a fixed order (deterministic).
__global__ void __launch_bounds__(kThreads) k_kalman_reduce(Tables tb) {
  __shared__ double red[2][kThreads];
  const double* p = reinterpret_cast<const double*>(tb.ws) + tb.seg_kal_off;
  double a = 0.0, b = 0.0;
  for (int s = threadIdx.x; s < tb.nsegs; s += kThreads) { a += p[2 * s]; b += p[2 * s + 1]; }
  red[0][threadIdx.x] = a;
  red[1][threadIdx.x] = b;
  __syncthreads();
  for (int s = kThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) { red[0][threadIdx.x] += red[0][threadIdx.x + s]; red[1][threadIdx.x] += red[1][threadIdx.x + s]; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double* out = reinterpret_cast<double*>(tb.ws) + tb.kal_sum_off + 2 * tb.dir;
    out[0] = red[0][0];
    out[1] = red[1][0];
  }
}

// =====================================================================================
// Power-iteration products (ds_mezo/kernels.py:215-225), grouped over bases, 64 x 64
// output tiles, fp32 FFMA:  MODE 0: Y = H V (T x R);  MODE 1: W = H^T Y (D x R).
// `first` reads V from the caller's strided basis; later iterations read Vout.
// =====================================================================================
template <int MODE>
__global__ void __launch_bounds__(kThreads) k_pi_gemm(Tables tb, int first) {
  __shared__ __align__(16) float As[16][64 + 4];
  __shared__ __align__(16) float Bs[16][64 + 4];
  const int item = blockIdx.x;
  const int bi = (MODE == 0) ? find_owner(tb.bases, tb.nbases, item, [](const BasisD& b) { return b.ytile0; })
                             : find_owner(tb.bases, tb.nbases, item, [](const BasisD& b) { return b.wtile0; });
  const BasisD Bd = tb.bases[bi];
  const int R = Bd.R;
  const int ntn = (R + 63) / 64;
  const int local = item - ((MODE == 0) ? Bd.ytile0 : Bd.wtile0);
  const int mt = local / ntn, nt = local - mt * ntn;
  const int64_t m0 = static_cast<int64_t>(mt) * 64;
  const int n0 = nt * 64;
  const int64_t Mdim = (MODE == 0) ? Bd.T : Bd.D;
  int64_t Kdim = (MODE == 0) ? Bd.D : Bd.T;
  // Y = H V with K = D split over blockIdx.y (tb.ysplit chunks of a multiple of 16):
  // chunk s writes its partial product into slot s, summed in order by k_pi_ysum
  int64_t kbeg = 0;
  const bool split = MODE == 0 && tb.ysplit > 1;
  if (split) {
    const int64_t kc = ((Kdim + tb.ysplit - 1) / tb.ysplit + 15) & ~static_cast<int64_t>(15);
    kbeg = static_cast<int64_t>(blockIdx.y) * kc;
    Kdim = min(Kdim, kbeg + kc);
  }
  float* Y = reinterpret_cast<float*>(tb.ws) + Bd.y_off;
  float* W = reinterpret_cast<float*>(tb.ws) + Bd.w_off;
  const float* Vsrc = first ? Bd.Vin : Bd.Vout;
  const int64_t vs0 = first ? Bd.v_s0 : R, vs1 = first ? Bd.v_s1 : 1;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  // the next 16 K-columns' operands are loaded into registers while the current ones are
  // multiplied from shared memory (four A and four B values per thread)
  float ra[4], rb[4];
  auto gload = [&](int64_t k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = tid + u * kThreads;
      int mm, kk;
      if (MODE == 0) { mm = e >> 4; kk = e & 15; } else { kk = e >> 6; mm = e & 63; }
      const int64_t m = m0 + mm, k = k0 + kk;
      float a = 0.f;
      if (m < Mdim && k < Kdim) {
        const int64_t ad = (MODE == 0) ? (m * Bd.h_s0 + k * Bd.h_s1) : (k * Bd.h_s0 + m * Bd.h_s1);
        a = ldf(Bd.H, ad, Bd.hdt);
      }
      ra[u] = a;
      const int kb = e >> 6, nn = e & 63;
      const int64_t kg = k0 + kb;
      float bval = 0.f;
      if (kg < Kdim && n0 + nn < R) {
        bval = (MODE == 0) ? Vsrc[kg * vs0 + static_cast<int64_t>(n0 + nn) * vs1] : Y[kg * R + n0 + nn];
      }
      rb[u] = bval;
    }
  };
  static_assert(4 * kThreads == 1024, "four operand values per thread per K-step");
  if (kbeg < Kdim) gload(kbeg);
  for (int64_t k0 = kbeg; k0 < Kdim; k0 += 16) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = tid + u * kThreads;
      if (MODE == 0) As[e & 15][e >> 4] = ra[u]; else As[e >> 6][e & 63] = ra[u];
      Bs[e >> 6][e & 63] = rb[u];
    }
    __syncthreads();
    if (k0 + 16 < Kdim) gload(k0 + 16);
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ti * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tj * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* C = (MODE == 0) ? (split ? reinterpret_cast<float*>(tb.ws) + Bd.ypart_off + blockIdx.y * Bd.T * R : Y) : W;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ti * 4 + i;
      const int n = n0 + tj * 4 + j;
      if (m < Mdim && n < R) C[m * R + n] = acc[i][j];
    }
}

// Y = sum of the split-K partials of every basis, in slot order (grid-stride over all
// bases' T x R elements; each basis's elements are a contiguous run of the launch).
__global__ void __launch_bounds__(kThreads) k_pi_ysum(Tables tb, int64_t total) {
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * kThreads) {
    int b = 0;
    int64_t base = 0;
    for (; b < tb.nbases; ++b) {              // a handful of bases on this path
      const int64_t n = tb.bases[b].T * tb.bases[b].R;
      if (e < base + n) break;
      base += n;
    }
    const BasisD& B = tb.bases[b];
    const int64_t li = e - base, n = B.T * B.R;
    const float* part = reinterpret_cast<const float*>(tb.ws) + B.ypart_off + li;
    float s = 0.f;
    for (int k = 0; k < tb.ysplit; ++k) s += part[k * n];
    reinterpret_cast<float*>(tb.ws)[B.y_off + li] = s;
  }
}

// pos = base + z, neg = base - z (ds_mezo/kernels.py:399-412).
__global__ void __launch_bounds__(kThreads) k_dual(const void* base, const float* z, void* pos, void* neg, int64_t n,
                                                   int dt) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const float b = ldf(base, i, dt), zz = z[i];
    stf(pos, i, __fadd_rn(b, zz), dt);
    stf(neg, i, __fsub_rn(b, zz), dt);
  }
}

// n normals in torch.randn order for a generator at (seed, offset).
__global__ void __launch_bounds__(kThreads) k_randn(float* out, int64_t n, uint64_t seed, uint64_t offset,
                                                    int64_t threads) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads)
    out[i] = torch_randn_at(seed, offset, threads, i);
}

// Copies descriptor tables given by value into device memory (single-op entry points).
template <typename T, int N>
struct Pack { T v[N]; };
template <typename T, int N>
__global__ void k_write_pack(Pack<T, N> p, T* dst, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = p.v[i];
}

}  // namespace dsmz
