// First-step calibration of the activation bases (ds_mezo/controller.py:156-163): per unique
// activation H (T x D) the reference takes V of torch.svd_lowrank(H, q=R, niter), a
// randomized range finder (Halko et al. 2009, Algorithm 4.4) followed by the SVD of the
// projected matrix (their Algorithm 5.1; torch/_lowrank.py). svd_lowrank works on H when
// T >= D and on H^T when T < D, which gives, with the plan's power iteration
// (Y = H V, W = H^T Y, V = W R_W^-1 by CholeskyQR):
//   T >= D: sketch R_D (D x R) into V; niter iterations leave P, spanning (H^T H)^niter R_D.
//           The reference's Q = orth(H P) and V_ref = left singular vectors of H^T Q. With
//           Y = H P, G_Y = Y^T Y and one more iteration (P' = W R_W^-1, W = H^T Y):
//           H^T Q = P' R_W R_Y^-1, so V_ref = P' C with C the eigenvectors of
//           R_W^-T G_Y R_W^-1 = (R_W G_Y^-1 R_W^T)^-1, eigenvalues 1 / s^2 ascending.
//   T <  D: sketch R_T (T x R) into Y; W = H^T R_T, its CholeskyQR and niter iterations leave
//           P', spanning (H^T H)^niter H^T R_T; V_ref = P' C with C the eigenvectors of
//           G_Y = Y^T Y, Y = H P' (the Ritz vectors), eigenvalues s^2 descending.
// The rotation V <- V C is applied in place; s are the singular values svd_lowrank returns.
#pragma once

#include "dsmz_tc.cuh"

namespace dsmz {

// Per basis: its sketch and where its calibration state lives (doubles, from the
// calibration workspace).
struct CalibD {
  int64_t e0;          // first element of this basis's draw in the launch's element space
  int64_t n;           // draw elements: rows x R (rows = D when T >= D, else T)
  int64_t threads;     // torch launch width of a draw of n normals (DistributionTemplates.h)
  uint64_t offset;     // generator offset of the draw, relative to the calibration's start
  int32_t into_y;      // 0: the sketch is V (T >= D); 1: the sketch is Y (T < D)
  int32_t pad;
  int64_t gpart_off;   // kCalibGroups partial Grams of Y, R x R each
  int64_t u_off;       // R x R rotation (column j: the j-th singular vector), then R values
  int64_t uw_off;      // n x n Jacobi rotation when it does not fit in shared memory
};

// Order of the Jacobi matrices (R rounded up to even) and whether the working rotation
// stays in shared memory beside the matrix (two 96 x 96 fp64 matrices at most).
__host__ __device__ inline int jacobi_n(int R) { return R + (R & 1); }
__host__ __device__ inline bool jacobi_u_in_smem(int R) { return jacobi_n(R) <= 96; }
__host__ __device__ inline size_t jacobi_smem(int R) {
  const size_t n = jacobi_n(R);
  return (n * n * (jacobi_u_in_smem(R) ? 2 : 1) + n) * sizeof(double) + n * sizeof(int);
}

constexpr int kCalibGroups = 8;       // token groups (CTAs) per basis of the Gram of Y
constexpr int kCalibChunk = 32;       // tokens staged per pass of the Gram of Y
__host__ __device__ inline size_t ygram_smem(int R) { return static_cast<size_t>(kCalibChunk) * R * sizeof(double); }

// Writes the sketch of every basis whose into_y equals `which`: element li of
// torch.randn(rows, R) (row li / R, column li % R) into V (row-major D x R) or into Y
// (the tensor-core path's [Y_hi | Y_lo]^T bf16 pair, 2R x ldy2, or the CUDA-core path's
// fp32 T x R Y).
__global__ void __launch_bounds__(kThreads) k_calib_draw(Tables tb, const CalibD* __restrict__ cd,
                                                         const tc::TCBasis* __restrict__ tcb, int64_t total,
                                                         uint64_t seed, uint64_t base_off, int which) {
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * kThreads) {
    int lo = 0, hi = tb.nbases - 1;             // the basis whose element range holds e
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cd[mid].e0 <= e) lo = mid; else hi = mid - 1;
    }
    const CalibD& C = cd[lo];
    if (C.into_y != which) continue;
    const int64_t li = e - C.e0;
    if (li >= C.n) continue;
    const BasisD& B = tb.bases[lo];
    const int R = B.R;
    const float x = torch_randn_at(seed, base_off + C.offset, C.threads, li);
    const int64_t row = li / R;
    const int c = static_cast<int>(li - row * R);
    if (which == 0) {
      B.Vout[row * R + c] = x;
    } else if (tcb != nullptr) {
      const tc::TCBasis& T = tcb[lo];
      const __nv_bfloat16 xh = __float2bfloat16_rn(x);
      T.Y2T[static_cast<int64_t>(c) * T.ldy2 + row] = xh;
      T.Y2T[static_cast<int64_t>(R + c) * T.ldy2 + row] = __float2bfloat16_rn(x - __bfloat162float(xh));
    } else {
      reinterpret_cast<float*>(tb.ws)[B.y_off + row * R + c] = x;
    }
  }
}

// Partial Grams of Y = H V: block (b, g) sums y_t y_t^T in fp64 over the token chunks
// g, g + kCalibGroups, ... (kCalibChunk tokens each, a fixed order), y_t from the bf16 pair
// (hi + lo, exact in fp64) or the fp32 Y. Thread (ty, tx) of a 16 x 16 grid owns the entries
// (ty + 16a, tx + 16c), a, c < NB, of the R x R Gram (R <= 16 NB).
template <int NB>
__global__ void __launch_bounds__(kThreads) k_calib_ygram(Tables tb, const CalibD* __restrict__ cd,
                                                          const tc::TCBasis* __restrict__ tcb, char* cws) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* ys = reinterpret_cast<double*>(smem_raw);         // kCalibChunk tokens x R
  const int b = blockIdx.x / kCalibGroups, g = blockIdx.x - b * kCalibGroups;
  const BasisD& B = tb.bases[b];
  const int R = B.R;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  double acc[NB][NB];
#pragma unroll
  for (int a = 0; a < NB; ++a)
#pragma unroll
    for (int c = 0; c < NB; ++c) acc[a][c] = 0.0;
  const int64_t nchunk = (B.T + kCalibChunk - 1) / kCalibChunk;
  for (int64_t ch = g; ch < nchunk; ch += kCalibGroups) {
    const int64_t t0 = ch * kCalibChunk;
    __syncthreads();
    for (int e = threadIdx.x; e < kCalibChunk * R; e += kThreads) {
      const int c = e / kCalibChunk, tl = e - c * kCalibChunk;    // consecutive threads: consecutive tokens
      const int64_t t = t0 + tl;
      double y = 0.0;
      if (t < B.T) {
        if (tcb != nullptr) {
          const tc::TCBasis& T = tcb[b];
          y = static_cast<double>(__bfloat162float(T.Y2T[static_cast<int64_t>(c) * T.ldy2 + t])) +
              static_cast<double>(__bfloat162float(T.Y2T[static_cast<int64_t>(R + c) * T.ldy2 + t]));
        } else {
          y = reinterpret_cast<const float*>(tb.ws)[B.y_off + t * R + c];
        }
      }
      ys[tl * R + c] = y;
    }
    __syncthreads();
    for (int tl = 0; tl < kCalibChunk; ++tl) {
      const double* yr = ys + tl * R;
      double yi[NB], yj[NB];
#pragma unroll
      for (int a = 0; a < NB; ++a) {
        const int i = ty + 16 * a, j = tx + 16 * a;
        yi[a] = i < R ? yr[i] : 0.0;
        yj[a] = j < R ? yr[j] : 0.0;
      }
#pragma unroll
      for (int a = 0; a < NB; ++a)
#pragma unroll
        for (int c = 0; c < NB; ++c) acc[a][c] = fma(yi[a], yj[c], acc[a][c]);
    }
  }
  double* gp = reinterpret_cast<double*>(cws) + cd[b].gpart_off + static_cast<int64_t>(g) * R * R;
#pragma unroll
  for (int a = 0; a < NB; ++a)
#pragma unroll
    for (int c = 0; c < NB; ++c) {
      const int i = ty + 16 * a, j = tx + 16 * c;
      if (i < R && j < R) gp[i * R + j] = acc[a][c];
    }
}

// One CTA per basis with into_y == which. The R x R matrix M (G_Y for which 1;
// R_W^-T G_Y R_W^-1 for which 0, with R_W^-1 the fp64 inverse Cholesky factor that the last
// CholeskyQR of the basis left in its workspace) is eigen-decomposed by the cyclic Jacobi
// method in fp64 (round-robin pairing: n/2 disjoint rotations per round, n - 1 rounds per
// sweep). The eigenvectors are ordered by descending singular value (s = sqrt(lambda) for
// which 1, 1/sqrt(lambda) for which 0) and each is signed so that its largest-magnitude
// entry is positive. Writes the rotation and the singular values at u_off, and the values
// as floats into sv (R per basis) when given.
constexpr int kJacobiSweeps = 20;
__global__ void __launch_bounds__(kThreads) k_calib_eig(Tables tb, const CalibD* __restrict__ cd, char* cws,
                                                        int which, float* sv) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  if (cd[b].into_y != which) return;
  const BasisD& B = tb.bases[b];
  const int R = B.R;
  const int n = jacobi_n(R);                 // even order for the pairing (a padded zero row)
  const bool u_smem = jacobi_u_in_smem(R);
  double* A = reinterpret_cast<double*>(smem_raw);   // n x n
  double* U = u_smem ? A + n * n : reinterpret_cast<double*>(cws) + cd[b].uw_off;   // n x n
  double* cs = A + n * n * (u_smem ? 2 : 1); // n/2 (c, s) pairs
  int* pr = reinterpret_cast<int*>(cs + n);  // n/2 pairs (p, q)
  __shared__ double red[kThreads];
  const double* gp = reinterpret_cast<const double*>(cws) + cd[b].gpart_off;
  for (int e = threadIdx.x; e < n * n; e += kThreads) {
    const int i = e / n, j = e - i * n;
    double s = 0.0;
    if (i < R && j < R)
      for (int g = 0; g < kCalibGroups; ++g) s += gp[static_cast<int64_t>(g) * R * R + i * R + j];
    A[e] = s;
  }
  __syncthreads();
  if (which == 0) {
    // M = Ri^T G Ri (V = W Ri): U <- G Ri, then A <- Ri^T U
    const MatD& W = tb.wA[b];
    const double* Ri = reinterpret_cast<const double*>(tb.ws) + W.dw_off + static_cast<int64_t>(R) * R;
    for (int e = threadIdx.x; e < n * n; e += kThreads) {
      const int i = e / n, j = e - i * n;
      double s = 0.0;
      if (i < R && j < R)
        for (int k = 0; k < R; ++k) s = fma(A[i * n + k], Ri[k * R + j], s);
      U[e] = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n * n; e += kThreads) {
      const int i = e / n, j = e - i * n;
      double s = 0.0;
      if (i < R && j < R)
        for (int k = 0; k < R; ++k) s = fma(Ri[k * R + i], U[k * n + j], s);
      A[e] = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n * n; e += kThreads) {   // symmetrise (rounding)
      const int i = e / n, j = e - i * n;
      if (i < j) {
        const double m = 0.5 * (A[e] + A[j * n + i]);
        A[e] = m;
        A[j * n + i] = m;
      }
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < n * n; e += kThreads) U[e] = (e / n == e % n) ? 1.0 : 0.0;
  // scale of the stopping test
  double fro = 0.0;
  for (int e = threadIdx.x; e < n * n; e += kThreads) fro += A[e] * A[e];
  const double tol2 = cta_sum(fro, red) * 1e-32;
  const int half = n / 2;
  for (int sweep = 0; sweep < kJacobiSweeps; ++sweep) {
    double off = 0.0;
    for (int e = threadIdx.x; e < n * n; e += kThreads) {
      const int i = e / n, j = e - i * n;
      if (i != j) off += A[e] * A[e];
    }
    if (cta_sum(off, red) <= tol2) break;
    for (int round = 0; round < n - 1; ++round) {
      // round-robin pairing: element 0 fixed, the others rotate
      for (int k = threadIdx.x; k < half; k += kThreads) {
        const int a = (k == 0) ? 0 : 1 + (k - 1 + round) % (n - 1);
        const int c = 1 + (n - 2 - k + round) % (n - 1);
        const int p = a < c ? a : c, q = a < c ? c : a;
        pr[2 * k] = p;
        pr[2 * k + 1] = q;
        const double apq = A[p * n + q];
        double cc = 1.0, ss = 0.0;
        if (apq != 0.0) {
          const double theta = (A[q * n + q] - A[p * n + p]) / (2.0 * apq);
          const double t = (theta >= 0.0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
          cc = 1.0 / sqrt(t * t + 1.0);
          ss = t * cc;
        }
        cs[2 * k] = cc;
        cs[2 * k + 1] = ss;
      }
      __syncthreads();
      // columns p, q of A and U (disjoint pairs)
      for (int e = threadIdx.x; e < half * n; e += kThreads) {
        const int k = e / n, i = e - k * n;
        const int p = pr[2 * k], q = pr[2 * k + 1];
        const double cc = cs[2 * k], ss = cs[2 * k + 1];
        const double aip = A[i * n + p], aiq = A[i * n + q];
        A[i * n + p] = cc * aip - ss * aiq;
        A[i * n + q] = ss * aip + cc * aiq;
        const double uip = U[i * n + p], uiq = U[i * n + q];
        U[i * n + p] = cc * uip - ss * uiq;
        U[i * n + q] = ss * uip + cc * uiq;
      }
      __syncthreads();
      // rows p, q of A
      for (int e = threadIdx.x; e < half * n; e += kThreads) {
        const int k = e / n, j = e - k * n;
        const int p = pr[2 * k], q = pr[2 * k + 1];
        const double cc = cs[2 * k], ss = cs[2 * k + 1];
        const double apj = A[p * n + j], aqj = A[q * n + j];
        A[p * n + j] = cc * apj - ss * aqj;
        A[q * n + j] = ss * apj + cc * aqj;
      }
      __syncthreads();
    }
  }
  // order by singular value, sign, write out
  double* out = reinterpret_cast<double*>(cws) + cd[b].u_off;
  for (int j = threadIdx.x; j < R; j += kThreads) {
    auto key = [&](int i) {          // descending key of eigenvalue i
      const double l = A[i * n + i];
      return which ? l : (l > 0.0 ? -l : -INFINITY);
    };
    const double kj = key(j);
    int rank = 0;
    for (int i = 0; i < R; ++i) {
      const double ki = key(i);
      rank += (ki > kj || (ki == kj && i < j)) ? 1 : 0;
    }
    int imax = 0;
    double vmax = -1.0;
    for (int i = 0; i < R; ++i)
      if (fabs(U[i * n + j]) > vmax) { vmax = fabs(U[i * n + j]); imax = i; }
    const double sgn = U[imax * n + j] < 0.0 ? -1.0 : 1.0;
    for (int i = 0; i < R; ++i) out[i * R + rank] = sgn * U[i * n + j];
    const double l = A[j * n + j];
    const double s = which ? sqrt(l > 0.0 ? l : 0.0) : (l > 0.0 ? 1.0 / sqrt(l) : 0.0);
    out[R * R + rank] = s;
    if (sv) sv[static_cast<int64_t>(b) * R + rank] = static_cast<float>(s);
  }
}

// V <- V U for every basis: block (b, tile) takes kRotRows rows of V into shared memory with
// U (fp64 products of fp32 V and the fp64 rotation, rounded once), and writes the rotated
// rows back in place.
constexpr int kRotRows = 32;
__host__ __device__ inline size_t rotate_smem(int R) {
  return static_cast<size_t>(R) * R * sizeof(double) + static_cast<size_t>(kRotRows) * R * sizeof(float);
}
__global__ void __launch_bounds__(kThreads) k_calib_rotate(Tables tb, const CalibD* __restrict__ cd,
                                                           const int32_t* __restrict__ tile0, char* cws) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int lo = 0, hi = tb.nbases - 1;
  const int item = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile0[mid] <= item) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const BasisD& B = tb.bases[b];
  const int R = B.R;
  double* Us = reinterpret_cast<double*>(smem_raw);         // R x R
  float* Vs = reinterpret_cast<float*>(Us + R * R);         // kRotRows x R
  const double* U = reinterpret_cast<const double*>(cws) + cd[b].u_off;
  const int64_t r0 = static_cast<int64_t>(item - tile0[b]) * kRotRows;
  const int nr = static_cast<int>(min(static_cast<int64_t>(kRotRows), B.D - r0));
  for (int e = threadIdx.x; e < R * R; e += kThreads) Us[e] = U[e];
  for (int e = threadIdx.x; e < nr * R; e += kThreads) Vs[e] = B.Vout[r0 * R + e];
  __syncthreads();
  for (int e = threadIdx.x; e < nr * R; e += kThreads) {
    const int i = e / R, c = e - i * R;
    double s = 0.0;
    for (int k = 0; k < R; ++k) s = fma(static_cast<double>(Vs[i * R + k]), Us[k * R + c], s);
    B.Vout[r0 * R + e] = static_cast<float>(s);
  }
}

}  // namespace dsmz
