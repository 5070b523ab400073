// Kernels of the DS-MeZO optimizer step (sm_100a). Exact-arithmetic path: fp32 FFMA for
// the streamed products, fp64 for cross-tile sums and for the r x r Newton-Schulz and
// Cholesky solves. Every launch covers all matrices (or bases, or modules) of a plan.
#pragma once

#include "dsmz_internal.cuh"

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

__host__ __device__ inline int tile_vectors(int r) {
  int tv = 2048 / (r < 1 ? 1 : r);
  return tv < 16 ? 16 : (tv > 256 ? 256 : tv);
}
__host__ __device__ inline int pad4(int r) { return (r + 3) & ~3; }

__device__ __forceinline__ int64_t vaddr2(const MatD& M, int64_t v, int64_t k) {
  return M.side == 0 ? v * M.ld + k * M.cs : k * M.ld + v * M.cs;
}

// =====================================================================================
// Gram partials: for each segment of each matrix, G_seg = sum_v x_v x_v^T (r x r), fp64
// products and sums of the fp32 vectors.
// SRC 0: x = mu (plain). SRC 1: x = Kalman-updated momentum mu2 (controller.py:283-284).
// =====================================================================================
template <int SRC, int RB>
__global__ void __launch_bounds__(kThreads) k_gram(Tables tb, const MatD* __restrict__ mats, int nmats,
                                                   KalmanIn kin) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);
  const int seg = blockIdx.x;
  const int mi = find_owner(mats, nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = mats[mi];
  const int r = static_cast<int>(M.r);
  const int tpr = (r + RB - 1) / RB;
  const int tpg = tpr * tpr;
  const int ngroups = kThreads / tpg;
  const int rp = tpr * RB;
  const int TV = tile_vectors(r);
  const int xld = rp + 1;
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  const int tid = threadIdx.x;
  const int grp = tid / tpg, lt = tid % tpg;
  const int bi = lt / tpr, bj = lt % tpr;
  const bool active = grp < ngroups;
  KalScal ks{};
  if (SRC == 1) ks = kal_derive(kin, reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off);

  double acc[RB][RB];
#pragma unroll
  for (int i = 0; i < RB; ++i)
#pragma unroll
    for (int j = 0; j < RB; ++j) acc[i][j] = 0.0;

  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    for (int e = tid; e < TV * rp; e += kThreads) {
      int v, k;
      if (M.side == 0) { v = e / rp; k = e - v * rp; } else { k = e / TV; v = e - k * TV; }
      float x = 0.f;
      if (v < nv && k < r) {
        const int64_t a = vaddr2(M, s0 + v, k);
        if (SRC == 0) {
          x = M.mu[a];
        } else {
          float mu1, var1, mu2, var2;
          kal_predict(M.mu[a], M.var[a], ks, mu1, var1);
          kal_observe(mu1, var1, M.z[a], ks, mu2, var2);
          x = mu2;
        }
      }
      xs[v * xld + k] = x;
    }
    __syncthreads();
    if (active) {
      // fp64 products and sums: the Gram squares the condition number, and the
      // Newton-Schulz polynomial of an ill-conditioned momentum (a fresh start, where
      // mu_B ~ Zc_B V^T with a square Gaussian Zc_B) needs its small eigenvalues intact.
      for (int v = grp; v < nv; v += ngroups) {
        const float* row = xs + v * xld;
        double xa[RB], xb[RB];
#pragma unroll
        for (int i = 0; i < RB; ++i) {
          xa[i] = static_cast<double>(row[bi * RB + i]);
          xb[i] = static_cast<double>(row[bj * RB + i]);
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
          if (a < r && b < r) out[a * r + b] = acc[i][j];
        }
    }
  } else {
    double* red = reinterpret_cast<double*>(smem_raw);   // ngroups * rp * rp
    if (active) {
#pragma unroll
      for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int j = 0; j < RB; ++j)
          red[(grp * rp + bi * RB + i) * rp + bj * RB + j] = acc[i][j];
    }
    __syncthreads();
    for (int e = tid; e < r * r; e += kThreads) {
      const int a = e / r, b = e - a * r;
      double s = 0.0;
      for (int g = 0; g < ngroups; ++g) s += red[(g * rp + a) * rp + b];
      out[e] = s;
    }
  }
}

// C = A B for r x r fp64 matrices in global memory, one CTA, 64 x 64 output tiles.
// C must not alias A or B. Ends with a barrier so C is visible to the whole CTA.
__device__ void cta_dgemm(double* __restrict__ C, const double* __restrict__ A, const double* __restrict__ B,
                          int r, double* sh) {
  double* As = sh;            // [16][64]
  double* Bs = sh + 16 * 64;  // [16][64]
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  for (int m0 = 0; m0 < r; m0 += 64) {
    for (int n0 = 0; n0 < r; n0 += 64) {
      double acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
      for (int k0 = 0; k0 < r; k0 += 16) {
        for (int e = tid; e < 1024; e += kThreads) {
          const int mm = e >> 4, kk = e & 15;
          As[kk * 64 + mm] = (m0 + mm < r && k0 + kk < r) ? A[(m0 + mm) * r + k0 + kk] : 0.0;
          const int kb = e >> 6, nn = e & 63;
          Bs[kb * 64 + nn] = (k0 + kb < r && n0 + nn < r) ? B[(k0 + kb) * r + n0 + nn] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          double a[4], b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) { a[i] = As[kk * 64 + ti * 4 + i]; b[i] = Bs[kk * 64 + tj * 4 + i]; }
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = m0 + ti * 4 + i, n = n0 + tj * 4 + j;
          if (m < r && n < r) C[m * r + n] = acc[i][j];
        }
    }
  }
  __syncthreads();
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

// =====================================================================================
// Newton-Schulz in Gram space, one CTA per matrix (ds_mezo/kernels.py:26-164 rewritten):
// X_k = X_0 P_k with P_k a polynomial of G_0 = X_0^T X_0, so the 12 X-space passes become
// G <- S G S, P <- P S on r x r (fp64), S = c0 I + c1 G + c2 G^2. Stores the fp32 apply
// matrix Pm with X[v,:] = x_v^T Pm for every vector x_v of the matrix.
// =====================================================================================
__global__ void __launch_bounds__(kThreads) k_ns_solve(Tables tb, const MatD* __restrict__ mats, NSArgs ns) {
  __shared__ double sh[2 * 16 * 64];
  __shared__ double red[kThreads];
  const MatD M = mats[blockIdx.x];
  const int r = static_cast<int>(M.r);
  const int rr = r * r;
  const int tid = threadIdx.x;
  double* dw = reinterpret_cast<double*>(tb.ws) + M.dw_off;
  double* G = dw;
  double* P = dw + rr;
  double* S = dw + 2 * rr;
  double* U = dw + 3 * rr;
  const double* part = reinterpret_cast<const double*>(tb.ws) + M.gram_off;
  double tr = 0.0;
  for (int e = tid; e < rr; e += kThreads) {
    double s = 0.0;
    for (int g = 0; g < M.nseg; ++g) s += part[static_cast<int64_t>(g) * rr + e];
    G[e] = s;
    const int a = e / r;
    if (a * r + a == e) tr += s;
  }
  const double norm_sq = cta_sum(tr, red);
  const double inv = 1.0 / sqrt(fmax(norm_sq, static_cast<double>(ns.norm_floor)));
  const double inv2 = inv * inv;
  for (int e = tid; e < rr; e += kThreads) {
    G[e] *= inv2;
    const int a = e / r;
    P[e] = (a * r + a == e) ? 1.0 : 0.0;
  }
  __syncthreads();
  for (int it = 0; it < ns.iters; ++it) {
    const double c0 = ns.c[it][0], c1 = ns.c[it][1], c2 = ns.c[it][2];
    if (c2 != 0.0) cta_dgemm(S, G, G, r, sh);
    for (int e = tid; e < rr; e += kThreads) {
      const int a = e / r;
      const double g2 = (c2 != 0.0) ? S[e] : 0.0;
      S[e] = ((a * r + a == e) ? c0 : 0.0) + c1 * G[e] + c2 * g2;
    }
    __syncthreads();
    cta_dgemm(U, P, S, r, sh);
    double* t = P; P = U; U = t;
    cta_dgemm(U, S, G, r, sh);
    cta_dgemm(G, U, S, r, sh);
  }
  float* Pm = reinterpret_cast<float*>(tb.ws) + M.p_off;
  for (int e = tid; e < rr; e += kThreads) {
    const int a = e / r, b = e - a * r;
    // tall (side A): X = X0 P -> row x^T P ; wide (side B): X = P X0 -> column P x = x^T P^T
    const double pv = (M.side == 0) ? P[a * r + b] : P[b * r + a];
    Pm[e] = static_cast<float>(pv * inv);
  }
}

// =====================================================================================
// CholeskyQR step for the power-iteration bases, one CTA per W matrix: G = W^T W (from
// the Gram partials), G = R^T R with pivots sqrt(max(d, norm_floor)) (the clamp of the
// reference MGS, ds_mezo/kernels.py:238), and the fp32 apply matrix R^{-1}.
// =====================================================================================
__global__ void __launch_bounds__(kThreads) k_chol(Tables tb, const MatD* __restrict__ mats, float norm_floor) {
  const MatD M = mats[blockIdx.x];
  const int r = static_cast<int>(M.r);
  const int rr = r * r;
  const int tid = threadIdx.x;
  double* dw = reinterpret_cast<double*>(tb.ws) + M.dw_off;
  double* G = dw;
  double* Rm = dw + rr;   // upper triangular factor
  double* Ri = dw + 2 * rr;
  const double* part = reinterpret_cast<const double*>(tb.ws) + M.gram_off;
  for (int e = tid; e < rr; e += kThreads) {
    double s = 0.0;
    for (int g = 0; g < M.nseg; ++g) s += part[static_cast<int64_t>(g) * rr + e];
    G[e] = s;
    Rm[e] = 0.0;
    Ri[e] = 0.0;
  }
  __syncthreads();
  __shared__ double diag;
  for (int j = 0; j < r; ++j) {
    if (tid == 0) {
      double d = G[j * r + j];
      for (int k = 0; k < j; ++k) d -= Rm[k * r + j] * Rm[k * r + j];
      diag = sqrt(fmax(d, static_cast<double>(norm_floor)));
      Rm[j * r + j] = diag;
    }
    __syncthreads();
    const double dj = diag;
    for (int i = j + 1 + tid; i < r; i += kThreads) {
      double s = G[j * r + i];
      for (int k = 0; k < j; ++k) s -= Rm[k * r + j] * Rm[k * r + i];
      Rm[j * r + i] = s / dj;
    }
    __syncthreads();
  }
  // R^{-1}: column j solves R x = e_j by back substitution.
  for (int j = tid; j < r; j += kThreads) {
    Ri[j * r + j] = 1.0 / Rm[j * r + j];
    for (int i = j - 1; i >= 0; --i) {
      double s = 0.0;
      for (int k = i + 1; k <= j; ++k) s += Rm[i * r + k] * Ri[k * r + j];
      Ri[i * r + j] = -s / Rm[i * r + i];
    }
  }
  __syncthreads();
  float* Pm = reinterpret_cast<float*>(tb.ws) + M.p_off;
  for (int e = tid; e < rr; e += kThreads) Pm[e] = static_cast<float>(Ri[e]);
}

// =====================================================================================
// Apply: X[v,:] = x_v^T Pm for every vector of every matrix segment.
// OUT 0: param -= eta * X (factor dtype), optional scratch = X  (ds_mezo/kernels.py:84-92).
// OUT 1: param (fp32) = X (CholeskyQR: Q = W R^{-1}).
// SRC 1 recomputes the Kalman update and writes mu, var (controller.py:283-285).
// =====================================================================================
template <int SRC, int OUT>
__global__ void __launch_bounds__(kThreads) k_apply(Tables tb, const MatD* __restrict__ mats, int nmats,
                                                    KalmanIn kin, float eta, int pdt) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int seg = blockIdx.x;
  const int mi = find_owner(mats, nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = mats[mi];
  const int r = static_cast<int>(M.r);
  const int rp = pad4(r);
  const int TV = tile_vectors(r);
  const int xld = rp + 1;
  float* Ps = reinterpret_cast<float*>(smem_raw);  // r x rp
  float* xs = Ps + r * rp;                         // TV x xld
  const int tid = threadIdx.x;
  const float* Pm = reinterpret_cast<const float*>(tb.ws) + M.p_off;
  for (int e = tid; e < r * rp; e += kThreads) {
    const int a = e / rp, c = e - a * rp;
    Ps[e] = (c < r) ? Pm[a * r + c] : 0.f;
  }
  KalScal ks{};
  if (SRC == 1) ks = kal_derive(kin, reinterpret_cast<const double*>(tb.ws) + tb.kal_sum_off);
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  const int ncb = rp / 4;
  __syncthreads();
  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    for (int e = tid; e < TV * r; e += kThreads) {
      int v, k;
      if (M.side == 0) { v = e / r; k = e - v * r; } else { k = e / TV; v = e - k * TV; }
      if (v >= nv) continue;
      const int64_t a = vaddr2(M, s0 + v, k);
      float x;
      if (SRC == 0) {
        x = M.mu[a];
      } else {
        float mu1, var1, mu2, var2;
        kal_predict(M.mu[a], M.var[a], ks, mu1, var1);
        kal_observe(mu1, var1, M.z[a], ks, mu2, var2);
        M.mu[a] = mu2;
        M.var[a] = var2;
        x = mu2;
      }
      xs[v * xld + k] = x;
    }
    __syncthreads();
    for (int it = tid; it < nv * ncb; it += kThreads) {
      int v, cb;
      if (M.side == 0) { v = it / ncb; cb = it - v * ncb; } else { cb = it / nv; v = it - cb * nv; }
      const float* xr = xs + v * xld;
      float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
      for (int a = 0; a < r; ++a) {
        const float xa = xr[a];
        const float4 p = *reinterpret_cast<const float4*>(Ps + a * rp + cb * 4);
        acc0 = fmaf(xa, p.x, acc0); acc1 = fmaf(xa, p.y, acc1);
        acc2 = fmaf(xa, p.z, acc2); acc3 = fmaf(xa, p.w, acc3);
      }
      const float accs[4] = {acc0, acc1, acc2, acc3};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cb * 4 + j;
        if (c >= r) break;
        const int64_t ad = vaddr2(M, s0 + v, c);
        const float X = accs[j];
        if (OUT == 0) {
          const float p = ldf(M.param, ad, pdt);
          stf(M.param, ad, __fsub_rn(p, __fmul_rn(eta, X)), pdt);
          if (M.scratch) M.scratch[ad] = X;
        } else {
          reinterpret_cast<float*>(M.param)[ad] = X;
        }
      }
    }
    __syncthreads();
  }
}

// =====================================================================================
// B-side reductions per (module, chunk of d_in): B V and var_B (V*V), both R x RC
// (ds_mezo/kernels.py:325-326 and controller.py:183). Partials summed by k_coef.
// =====================================================================================
__global__ void __launch_bounds__(kThreads) k_bside(Tables tb) {
  __shared__ float Bs[64][33];
  __shared__ float Ws[64][33];
  __shared__ float Vs[32][65];
  const int item = blockIdx.x;
  const int mi = find_owner(tb.mods, tb.nmods, item, [](const ModD& d) { return d.chunk0; });
  const ModD D = tb.mods[mi];
  const BasisD Bd = tb.bases[D.basis];
  const int chunk = item - D.chunk0;
  const int R = D.r, RC = D.rc;
  const int64_t j0 = static_cast<int64_t>(chunk) * D.chunkw;
  const int64_t j1 = min(j0 + static_cast<int64_t>(D.chunkw), D.d_in);
  const bool with_var = (D.varB != nullptr);
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  const float* V = Bd.Vin;
  const int64_t vs0 = Bd.v_s0, vs1 = Bd.v_s1;
  float* outp = reinterpret_cast<float*>(tb.ws) + D.bpart_off + static_cast<int64_t>(chunk) * 2 * R * RC;
  for (int rt = 0; rt < R; rt += 64) {
    for (int ct = 0; ct < RC; ct += 64) {
      float abv[4][4], avb[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) { abv[i][j] = 0.f; avb[i][j] = 0.f; }
      for (int64_t jb = j0; jb < j1; jb += 32) {
        for (int e = tid; e < 64 * 32; e += kThreads) {
          const int rr = e >> 5, jj = e & 31;
          const int64_t j = jb + jj;
          const bool ok = (rt + rr < R) && (j < j1);
          const int64_t a = static_cast<int64_t>(rt + rr) * D.b_s0 + j * D.b_s1;
          Bs[rr][jj] = ok ? ldf(D.Bp, a, D.bdt) : 0.f;
          Ws[rr][jj] = (ok && with_var) ? D.varB[a] : 0.f;
          const int jv = e >> 6, cc = e & 63;
          const int64_t jv_g = jb + jv;
          Vs[jv][cc] = (jv_g < j1 && ct + cc < RC) ? V[jv_g * vs0 + static_cast<int64_t>(ct + cc) * vs1] : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int jj = 0; jj < 32; ++jj) {
          float b[4], w[4], v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) { b[i] = Bs[ti * 4 + i][jj]; w[i] = Ws[ti * 4 + i][jj]; v[i] = Vs[jj][tj * 4 + i]; }
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              abv[i][j] = fmaf(b[i], v[j], abv[i][j]);
              avb[i][j] = fmaf(w[i], v[j] * v[j], avb[i][j]);
            }
        }
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int rr = rt + ti * 4 + i, cc = ct + tj * 4 + j;
          if (rr < R && cc < RC) {
            outp[rr * RC + cc] = abv[i][j];
            outp[R * RC + rr * RC + cc] = avb[i][j];
          }
        }
    }
  }
}

// =====================================================================================
// Per module: sum the chunk partials (fp64), Zc_B = randn(R,RC) * sqrt(var_B V^2)
// (controller.py:183-186), and Q = MGS(B V)[:, :RCA] (ds_mezo/kernels.py:328-340) in fp64
// by one warp. MODE 0 draws Zc_B from the torch Philox stream, MODE 1 copies it.
// =====================================================================================
template <int MODE>
__global__ void __launch_bounds__(kThreads) k_coef(Tables tb, uint64_t seed, uint64_t base_off, float norm_floor) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const ModD D = tb.mods[blockIdx.x];
  const int R = D.r, RC = D.rc, RCA = D.rca;
  const int tid = threadIdx.x;
  double* BV = reinterpret_cast<double*>(smem_raw);   // R x RC
  const float* part = reinterpret_cast<const float*>(tb.ws) + D.bpart_off;
  float* ZcB = reinterpret_cast<float*>(tb.ws) + D.coef_off;
  float* Qo = ZcB + static_cast<int64_t>(R) * RC;
  for (int e = tid; e < R * RC; e += kThreads) {
    double sbv = 0.0, svb = 0.0;
    for (int c = 0; c < D.nchunk; ++c) {
      sbv += part[static_cast<int64_t>(c) * 2 * R * RC + e];
      svb += part[static_cast<int64_t>(c) * 2 * R * RC + R * RC + e];
    }
    BV[e] = sbv;
    if (MODE == 0) {
      const float g = torch_randn_at(seed, base_off + D.offB, D.thrB, e);
      ZcB[e] = __fmul_rn(g, sqrtf(static_cast<float>(svb)));
    } else {
      ZcB[e] = D.zcB_ext[e];
    }
  }
  __syncthreads();
  if (tid < 32) {
    const int lane = tid;
    for (int col = 0; col < RCA; ++col) {
      for (int prev = 0; prev < col; ++prev) {
        double d = 0.0;
        for (int i = lane; i < R; i += 32) d += BV[i * RC + col] * BV[i * RC + prev];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        for (int i = lane; i < R; i += 32) BV[i * RC + col] -= d * BV[i * RC + prev];
        __syncwarp();
      }
      double n2 = 0.0;
      for (int i = lane; i < R; i += 32) n2 += BV[i * RC + col] * BV[i * RC + col];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
      const double inv = 1.0 / sqrt(fmax(n2, static_cast<double>(norm_floor)));
      for (int i = lane; i < R; i += 32) BV[i * RC + col] *= inv;
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = tid; e < R * RCA; e += kThreads) {
    const int i = e / RCA, k = e - i * RCA;
    Qo[e] = static_cast<float>(BV[i * RC + k]);
  }
}

// =====================================================================================
// Perturbation pass over every adapter matrix segment (controller.py:178-193, 241-248,
// 262-270; ds_mezo/kernels.py:290-368, 399-412):
//   side A: z[i,:] = eps * Zc_A[i,:] Q^T  with Zc_A[i,k] = randn draw A element i*RCA+k
//   side B: z[:,j] = eps * Zc_B V[j,:]^T
// MODE 0 (step): z stored, pos = p + z, neg = p - z, Kalman sums of this segment
//                (sum z*beta*mu, sum z*z*(beta^2 var + q)).
// MODE 1 (drop-in op): z stored only, Zc_A read from the caller's tensor.
// =====================================================================================
template <int MODE>
__global__ void __launch_bounds__(kThreads) k_perturb(Tables tb, uint64_t seed, uint64_t base_off, float eps,
                                                      KalmanIn kin) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[2][kThreads / 32];
  const int seg = blockIdx.x;
  const int mi = find_owner(tb.mats, tb.nmats, seg, [](const MatD& m) { return m.seg0; });
  const MatD M = tb.mats[mi];
  const ModD D = tb.mods[M.owner];
  const int r = static_cast<int>(M.r);
  const int R = D.r, RC = D.rc, RCA = D.rca;
  const int TV = tile_vectors(r);
  const int tid = threadIdx.x;
  const int KW = (M.side == 0) ? RCA : RC;     // inner width of the z product
  float* Cs = reinterpret_cast<float*>(smem_raw);        // KW x R : Q^T (side A) or Zc_B^T (side B)
  float* Ks = Cs + KW * R;                               // TV x (KW+1): Zc_A rows or V rows
  float* zs = Ks + TV * (KW + 1);                        // TV x (r+1)
  const float* coef = reinterpret_cast<const float*>(tb.ws) + D.coef_off;
  if (M.side == 0) {
    const float* Q = coef + static_cast<int64_t>(R) * RC;   // R x RCA
    for (int e = tid; e < KW * R; e += kThreads) { const int k = e / R, c = e - k * R; Cs[e] = Q[c * RCA + k]; }
  } else {
    for (int e = tid; e < KW * R; e += kThreads) { const int k = e / R, c = e - k * R; Cs[e] = coef[c * RC + k]; }
  }
  const BasisD Bd = tb.bases[D.basis];
  float s_zmu = 0.f, s_zzv = 0.f;
  const int64_t v0 = static_cast<int64_t>(seg - M.seg0) * M.segv;
  const int64_t v1 = min(v0 + static_cast<int64_t>(M.segv), M.nvec);
  __syncthreads();
  for (int64_t s0 = v0; s0 < v1; s0 += TV) {
    const int nv = static_cast<int>(min(static_cast<int64_t>(TV), v1 - s0));
    for (int e = tid; e < nv * KW; e += kThreads) {
      const int v = e / KW, k = e - v * KW;
      float x;
      if (M.side == 0) {
        const int64_t li = (s0 + v) * RCA + k;
        x = (MODE == 0) ? torch_randn_at(seed, base_off + D.offA, D.thrA, li) : D.zcA_ext[li];
      } else {
        x = Bd.Vin[(s0 + v) * Bd.v_s0 + static_cast<int64_t>(k) * Bd.v_s1];
      }
      Ks[v * (KW + 1) + k] = x;
    }
    __syncthreads();
    for (int e = tid; e < nv * r; e += kThreads) {
      const int v = e / r, c = e - v * r;
      const float* kr = Ks + v * (KW + 1);
      float acc = 0.f;
      for (int k = 0; k < KW; ++k) acc = fmaf(kr[k], Cs[k * R + c], acc);
      zs[v * (r + 1) + c] = acc * eps;
    }
    __syncthreads();
    for (int e = tid; e < nv * r; e += kThreads) {
      int v, k;
      if (M.side == 0) { v = e / r; k = e - v * r; } else { k = e / nv; v = e - k * nv; }
      const int64_t a = vaddr2(M, s0 + v, k);
      const float z = zs[v * (r + 1) + k];
      M.z[a] = z;
      if (MODE == 0) {
        const float p = ldf(M.param, a, tb.factor_dtype);
        stf(M.pos, a, __fadd_rn(p, z), tb.factor_dtype);
        stf(M.neg, a, __fsub_rn(p, z), tb.factor_dtype);
        const float mu1 = __fmul_rn(M.mu[a], kin.beta);
        const float var1 = __fadd_rn(__fmul_rn(M.var[a], kin.beta2), kin.q);
        s_zmu = fmaf(z, mu1, s_zmu);
        s_zzv = fmaf(__fmul_rn(z, z), var1, s_zzv);
      }
    }
    __syncthreads();
  }
  if (MODE == 0) {
    double a = s_zmu, b = s_zzv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if ((tid & 31) == 0) { red[0][tid >> 5] = a; red[1][tid >> 5] = b; }
    __syncthreads();
    if (tid == 0) {
      double sa = 0.0, sb = 0.0;
      for (int w = 0; w < kThreads / 32; ++w) { sa += red[0][w]; sb += red[1][w]; }
      double* out = reinterpret_cast<double*>(tb.ws) + tb.seg_kal_off + 2 * static_cast<int64_t>(seg);
      out[0] = sa;
      out[1] = sb;
    }
  }
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
    double* out = reinterpret_cast<double*>(tb.ws) + tb.kal_sum_off;
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
  const int64_t Kdim = (MODE == 0) ? Bd.D : Bd.T;
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
  for (int64_t k0 = 0; k0 < Kdim; k0 += 16) {
    for (int e = tid; e < 1024; e += kThreads) {
      int mm, kk;
      if (MODE == 0) { mm = e >> 4; kk = e & 15; } else { kk = e >> 6; mm = e & 63; }
      const int64_t m = m0 + mm, k = k0 + kk;
      float a = 0.f;
      if (m < Mdim && k < Kdim) {
        const int64_t ad = (MODE == 0) ? (m * Bd.h_s0 + k * Bd.h_s1) : (k * Bd.h_s0 + m * Bd.h_s1);
        a = ldf(Bd.H, ad, Bd.hdt);
      }
      As[kk][mm] = a;
      const int kb = e >> 6, nn = e & 63;
      const int64_t kg = k0 + kb;
      float b = 0.f;
      if (kg < Kdim && n0 + nn < R) {
        b = (MODE == 0) ? Vsrc[kg * vs0 + static_cast<int64_t>(n0 + nn) * vs1] : Y[kg * R + n0 + nn];
      }
      Bs[kb][nn] = b;
    }
    __syncthreads();
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
  float* C = (MODE == 0) ? Y : W;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ti * 4 + i;
      const int n = n0 + tj * 4 + j;
      if (m < Mdim && n < R) C[m * R + n] = acc[i][j];
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
