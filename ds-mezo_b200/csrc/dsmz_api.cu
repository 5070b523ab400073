// C ABI of libdsmezo: plans, launch sequences and the per-op drop-ins declared in dsmezo.h.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "dsmz_handoff.cuh"
#include "dsmz_kernels.cuh"
#include "dsmz_pi_fused.cuh"
#include "dsmz_calib.cuh"
#include "dsmz_adapter_tc.cuh"
#include "dsmz_score.cuh"
#include "dsmz_stream.cuh"
#include "dsmz_tc.cuh"

using namespace dsmz;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(const char* what, cudaError_t e) {
  return fail(DSMZ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define DSMZ_LAUNCHED(what)                                  \
  do {                                                        \
    cudaError_t e_ = cudaGetLastError();                      \
    if (e_ != cudaSuccess) return cuda_fail((what), e_);      \
  } while (0)

// ------------------------------------------------------------------ workspace layout
struct Layout {
  size_t bytes = 0;
  size_t take(size_t n, size_t align = 256) {
    bytes = (bytes + align - 1) & ~(align - 1);
    const size_t off = bytes;
    bytes += n;
    return off;
  }
};

int seg_vectors(int r) {
  // ~128K elements per segment keeps the Gram partials small; a multiple of the sub-tile.
  const int tv = tile_vectors(r);
  int segv = (131072 / (r < 1 ? 1 : r)) / tv * tv;
  return segv < tv ? tv : segv;
}

int gram_rb(int r) { return r <= 64 ? 4 : 8; }

size_t gram_smem(int r) {
  const int RB = gram_rb(r);
  const int tpr = (r + RB - 1) / RB;
  const int rp = tpr * RB;
  const int ngroups = kThreads / (tpr * tpr);
  const size_t tv = static_cast<size_t>(tile_vectors(r));
  const size_t xs = tv * (rp + 4) * sizeof(float);
  const size_t red = ngroups > 1 ? static_cast<size_t>(ngroups) * rp * rp * sizeof(double) : 0;
  return xs > red ? xs : red;
}
size_t apply_smem(int r) {
  const int r8 = pad8(r);
  return (static_cast<size_t>(r) * r8 + 2 * static_cast<size_t>(tile_vectors(r)) * (r8 + 1)) * sizeof(float);
}
size_t perturb_smem(int r, int R, int RC) {
  const int KW = RC;  // side B width; side A uses RCA <= RC
  const int TV = tile_vectors(r);
  return (static_cast<size_t>(KW) * pad8(R) + static_cast<size_t>(TV) * (KW + 1) + static_cast<size_t>(TV) * (r + 1)) *
         sizeof(float);
}
size_t coef_smem(int R, int RC) {
  const int rca = R < RC ? R : RC;
  return (static_cast<size_t>(R + 4) * RC +
          (coef_qr_in_smem(R, rca) ? 2 * static_cast<size_t>(rca) * rca : 0)) * sizeof(double);
}
size_t ns_smem(int r) {
  return r <= 64 ? 3 * static_cast<size_t>(pad8(r)) * ns_ld(r) * sizeof(double)
                 : 3 * static_cast<size_t>(ns_packed_blocks(r)) * 64 * sizeof(double);
}
size_t chol_smem(int R) { return R <= 64 ? 2 * static_cast<size_t>(R) * R * sizeof(double) : 0; }

// Dynamic shared memory of a streaming-kernel CTA (one CTA per SM).
constexpr int kStreamSmem = 220 * 1024;

template <typename K>
int set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute", e);
  }
  return 0;
}

// Newton-Schulz solve of nm matrices of rank r: r <= 64 two CTAs per SM with the full
// matrices in shared memory (k_ns_solve); larger r the packed-symmetric kernel (one CTA per
// SM). The packed kernel at r <= 64 (four warps, four CTAs per SM) took 291 us per matrix
// against ~150 us: its per-block addressing makes it issue-bound at that size.
int launch_ns_solve(const Tables& tb, const MatD* mats, int nm, int r, const NSArgs& ns, cudaStream_t s) {
  int rc;
  if (r <= 64) {
    if ((rc = set_smem(k_ns_solve, ns_smem(r)))) return rc;
    k_ns_solve<<<nm, kThreads, ns_smem(r), s>>>(tb, mats, ns);
  } else {
    if ((rc = set_smem(k_ns_solve_packed<kNsPThreads>, ns_smem(r)))) return rc;
    k_ns_solve_packed<kNsPThreads><<<nm, kNsPThreads, ns_smem(r), s>>>(tb, mats, ns);
  }
  return 0;
}

// One adapter matrix (or W basis matrix) with its segment and workspace slots. Without
// alloc_gram the Gram partials are placed later by chunk_matrices.
void add_matrix(std::vector<MatD>& mats, Layout& L, MatD m, int& seg_counter, bool alloc_gram = true) {
  m.segv = seg_vectors(static_cast<int>(m.r));
  m.nseg = static_cast<int32_t>((m.nvec + m.segv - 1) / m.segv);
  if (m.nseg < 1) m.nseg = 1;
  m.seg0 = seg_counter;
  seg_counter += m.nseg;
  const size_t rr = static_cast<size_t>(m.r) * m.r;
  m.gram_off = alloc_gram ? static_cast<int64_t>(L.take(m.nseg * rr * sizeof(double)) / sizeof(double)) : 0;
  m.tmap = -1;
  m.kmap = -1;
  m.rmap = -1;
  m.p_off = static_cast<int64_t>(L.take((rr + 4) * sizeof(float)) / sizeof(float));
  m.dw_off = 0;                                  // the Newton-Schulz solve works in shared memory
  mats.push_back(m);
}

// B-side sums: the modules' d_in columns, concatenated in module order, are cut into G
// equal contiguous ranges, one per CTA (G no larger than the column count, so none is
// empty). Each module gets its first column col0, the first CTA whose range meets it
// (chunk0), the number of such CTAs (nchunk, one partial each, summed in order by
// k_coef) and room for those partials.
void plan_bside(std::vector<ModD>& mods, int G, Layout& ws, int* grid, int64_t* ncols) {
  int64_t total = 0;
  for (ModD& m : mods) { m.col0 = total; total += m.d_in; }
  if (G > total) G = static_cast<int>(total);
  if (G < 1) G = 1;
  auto start = [&](int64_t b) { return b * total / G; };   // first column of CTA b
  int b = 0;
  for (ModD& m : mods) {
    while (b + 1 < G && start(b + 1) <= m.col0) ++b;     // the CTA holding column col0
    int e = b;
    while (e + 1 < G && start(e + 1) < m.col0 + m.d_in) ++e;   // the CTA holding the last column
    m.chunk0 = b;
    m.nchunk = e - b + 1;
    const size_t nB = static_cast<size_t>(m.r) * m.rc;
    m.bpart_off = static_cast<int64_t>(ws.take(static_cast<size_t>(m.nchunk) * 2 * nB * sizeof(float)) / sizeof(float));
  }
  *grid = G;
  *ncols = total;
}

// Streaming-kernel schedule of a matrix list: TV-vector tiles numbered across the list,
// cut into G = min(max_ctas, T) contiguous chunks (one per CTA, [c*T/G, (c+1)*T/G)), so no
// chunk is empty and every chunk between two that touch a matrix lies inside it; a segment
// is a chunk's run within one matrix. Sets tile0/ntile/chunk0/seg0/nseg and, with L, places
// the Gram partials (one r x r block per segment). Returns the number of segments; *grid
// receives G, the grid every streaming kernel over this list must be launched with.
int chunk_matrices(std::vector<MatD>& mats, int TV, int max_ctas, Layout* L, int* grid) {
  int64_t T = 0;
  for (MatD& m : mats) {
    m.tile0 = static_cast<int32_t>(T);
    m.ntile = static_cast<int32_t>((m.nvec + TV - 1) / TV);
    T += m.ntile;
  }
  const int G = static_cast<int>(T < max_ctas ? T : max_ctas);
  *grid = G;
  auto chunk_of = [&](int64_t t) {   // largest c with c*T/G <= t
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if ((static_cast<int64_t>(mid) * T) / G <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
  };
  int nseg = 0;
  for (MatD& m : mats) {
    m.chunk0 = chunk_of(m.tile0);
    const int c1 = chunk_of(static_cast<int64_t>(m.tile0) + m.ntile - 1);
    m.nseg = c1 - m.chunk0 + 1;
    m.seg0 = nseg;
    nseg += m.nseg;
    if (L) {
      const size_t rr = static_cast<size_t>(m.r) * m.r;
      m.gram_off = static_cast<int64_t>(L->take(m.nseg * rr * sizeof(double)) / sizeof(double));
    }
  }
  return nseg;
}

void fill_basis_tiles(BasisD& b, int& ytiles, int& wtiles) {
  const int ntn = (b.R + 63) / 64;
  b.ytile0 = ytiles;
  b.nytile = static_cast<int32_t>(((b.T + 63) / 64) * ntn);
  ytiles += b.nytile;
  b.wtile0 = wtiles;
  b.nwtile = static_cast<int32_t>(((b.D + 63) / 64) * ntn);
  wtiles += b.nwtile;
}

NSArgs make_ns(const dsmz_ns_schedule* s, float floor_) {
  NSArgs a{};
  dsmz_ns_schedule cub;
  if (!s) { dsmz_ns_schedule_cubic(&cub); s = &cub; }
  a.iters = s->iters;
  for (int i = 0; i < s->iters && i < DSMZ_MAX_NS_ITERS; ++i)
    for (int j = 0; j < 3; ++j) a.c[i][j] = s->c[i][j];
  a.norm_floor = floor_;
  return a;
}

// ------------------------------------------------------------------ tensor-core power iteration
// cuTensorMapEncodeTiled from the driver, looked up once per process.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D tensor map of fp32 or bf16 rows (inner dimension contiguous), no swizzle, zero fill
// outside: the tile boxes of the streaming kernels' side-1 arrays.
bool encode_rows_2d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, dtype == DSMZ_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
            const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp32 tensor map over rows of `cols` floats with boxes of 32 columns x TV rows and the
// 128-byte swizzle (the streaming kernels' swizzled row image), zero fill outside.
bool encode_rows_swz(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes,
                     uint32_t TV) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {32, TV};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D bf16 tensor map (inner dimension contiguous), 128-byte swizzle, zero fill outside.
bool encode_bf16_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


int pw_stages(int R);

// Shapes the tcgen05 products take: bf16 H with 16-byte rows, R a multiple of 16 (N = 2R),
// and room for a ring of at least two stages beside the persistent W kernel's fp64 staging.
bool tc_shape_ok(int hdt, int64_t D, int64_t ld_H, int64_t h_s1, int64_t R, const void* H) {
  return hdt == DSMZ_BF16 && h_s1 == 1 && D % 8 == 0 && ld_H % 8 == 0 && R % 16 == 0 && R <= DSMZ_MAX_RANK &&
         (reinterpret_cast<uintptr_t>(H) & 15) == 0 && pw_stages(static_cast<int>(R)) >= 2;
}

// Persistent Y kernel (one CTA per SM): ring of up to six stages of w_halves(R) x 128 rows.
int py_stages(int R) {
  const int n = (227 * 1024 - 2048) / tc::ring_stage_bytes(R, tc::w_halves(R));
  return n > 6 ? 6 : n;
}
size_t py_smem(int R) { return static_cast<size_t>(py_stages(R)) * tc::ring_stage_bytes(R, tc::w_halves(R)) + 1024 + 512; }
// Persistent W kernel (one CTA per SM): the ring takes what the fp64 staging region leaves.
int pw_stages(int R) {
  const int n = (227 * 1024 - 2048 - tc::w_stage_bytes(R)) / tc::ring_stage_bytes(R, tc::w_halves(R));
  return n > 6 ? 6 : n;
}
size_t pw_smem(int R) {
  return static_cast<size_t>(pw_stages(R)) * tc::ring_stage_bytes(R, tc::w_halves(R)) + tc::w_stage_bytes(R) + 1024 +
         512;
}

// Single-pass power iteration: stages of 2 x 128 rows plus the shared B operand, shared by
// the Y ring (the larger half) and the W ring.
int pf_stages(int R) {
  const int n = (227 * 1024 - 2048 - tc::fused_fixed_bytes(R)) / tc::fused_stage_bytes(R);
  return n > 8 ? 8 : n;
}
int pf_stages_y(int R) { return (pf_stages(R) + 1) / 2; }
int pf_stages_w(int R) { return pf_stages(R) / 2; }
size_t pf_smem(int R) {
  return static_cast<size_t>(pf_stages(R)) * tc::fused_stage_bytes(R) + tc::fused_fixed_bytes(R) + 1024;
}

struct TCSlots {             // workspace byte offsets of one basis
  size_t v2t = 0, y2t = 0;
  size_t gp = 0;             // fused W Gram partials (R <= 64), 0: none
  int64_t ldv2 = 0, ldy2 = 0;
};

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

}  // namespace

// ====================================================================== plan
struct dsmz_plan {
  std::vector<MatD> mats, w1, w2;
  std::vector<ModD> mods;
  std::vector<BasisD> bases;
  Layout ws;                        // workspace layout
  size_t off_mats = 0, off_w1 = 0, off_w2 = 0, off_mods = 0, off_bases = 0, table_bytes = 0;
  std::vector<unsigned char> blob;  // host copy of the tables
  char* dev_tables = nullptr;
  char* workspace = nullptr;
  int nsegs = 0, nwsegsA = 0, nwsegsB = 0, nchunks = 0, nytiles = 0, nwtiles = 0, ndblk = 0;
  int ysplit = 1;                   // K splits of the CUDA-core Y product (few output tiles)
  int64_t ytotal = 0;               // elements of every basis's Y
  int64_t bside_cols = 0;   // concatenated d_in columns of the B-side sums (nchunks CTAs over them)
  int sm_count = 0;
  int grid_m = 0, grid_w = 0, grid_w1 = 0;   // streaming-kernel grids (chunks) of mats, w2, w1
  int ndir = 1;                      // SPSA directions per step
  int64_t dstride_f = 0, dstride_z = 0;
  uint64_t rng_inc1 = 0, rng_dir_stride = 0;   // one direction's generator advance (this plan / all ranks)
  sk::Layout Lp{}, Lg{}, La{}, Lq{};   // streaming kernels: perturb, Kalman Gram, apply, QR apply
  sk::Layout Lw{};                     // Gram of the power-iteration W
  int copy_dtype = DSMZ_F32;          // +/- copies and shadows (the masters are fp32)
  bool ptc = false;                   // perturbation on the tensor cores (atc::k_perturb_tc)
  atc::PLayout Lpt{};                 // its shared-memory layout
  std::vector<int32_t> ptiles;        // its tiles: first 128-vector tile of each matrix, then the total
  GatherPeers gpeers{};               // fused +/- all-gather: byte distances to the peers' buffers
  GatherPeers speers{};               // fused factor all-gather: distances to the peers' shadows (dpos)
  size_t off_ptiles = 0;
  int r = 0, R = 0, RC = 0;
  int64_t seg_kal_off = 0, kal_sum_off = 0;
  size_t norm_off = 0;                // fp64 partials of the factor norms (kNormSlices per matrix)
  uint64_t rng_increment = 0;
  // tensor-core power iteration
  bool tc = false;
  std::vector<CUtensorMap> smaps;     // side-1 tile boxes of the adapter arrays (4 per matrix)
  size_t off_smaps = 0;
  std::vector<tc::TCBasis> tcb;
  std::vector<int32_t> ysched;       // Y tiles per CTA of the persistent Y kernel (empty: round-robin)
  int ysched_G = 0;
  size_t off_ysched = 0;
  std::vector<TCSlots> tcs;
  size_t off_tcb = 0, err_off = 0;
  int ntc_y = 0, ntc_w = 0, ntc_vt = 0;
  // single-pass (fused) power iteration, R <= 64: work queue and launch-local counters
  bool fused = false;
  std::vector<tc::PiItem> pitems_y, pitems_w;   // the Y and W queues
  size_t off_pitems_y = 0, off_pitems_w = 0;
  size_t fsync_off = 0, fsync_bytes = 0, fpart_off = 0;
  int f_ytiles = 0, f_nslots = 0;
  mutable bool split_current = false;   // [V_hi | V_lo]^T matches V (set by a power iteration)
  // Zc_A draws of direction 0 issued ahead (dsmz_step_draw) for the perturbation at this key
  mutable bool pre_drawn = false;
  mutable uint64_t pre_seed = 0, pre_off = 0;
  // first-step calibration: per-basis sketches and state, rotation tiles
  std::vector<CalibD> calib;
  std::vector<int32_t> rot_tile0;
  size_t off_calib = 0, off_rot = 0, calib_ws_bytes = 0;
  int rot_tiles = 0;
  int64_t calib_total = 0;
  uint64_t calib_inc = 0;
  struct Probe {
    std::vector<cudaEvent_t> start, stop;
    int count = 0;
  };
  mutable Probe probes[DSMZ_NUM_KIDS];

  void probe_begin(int kid, cudaStream_t s) const {
    Probe& p = probes[kid];
    if (p.count < static_cast<int>(p.start.size())) cudaEventRecord(p.start[p.count], s);
  }
  void probe_end(int kid, cudaStream_t s) const {
    Probe& p = probes[kid];
    if (p.count < static_cast<int>(p.stop.size())) cudaEventRecord(p.stop[p.count++], s);
  }

  Tables tables() const {
    Tables t{};
    t.mats = reinterpret_cast<const MatD*>(dev_tables + off_mats);
    t.nmats = static_cast<int32_t>(mats.size());
    t.nsegs = nsegs;
    t.mods = reinterpret_cast<const ModD*>(dev_tables + off_mods);
    t.nmods = static_cast<int32_t>(mods.size());
    t.nchunks = nchunks;
    t.bases = reinterpret_cast<const BasisD*>(dev_tables + off_bases);
    t.nbases = static_cast<int32_t>(bases.size());
    t.nytiles = nytiles;
    t.ysplit = ysplit;
    t.nwtiles = nwtiles;
    t.wA = reinterpret_cast<const MatD*>(dev_tables + off_w1);
    t.wB = reinterpret_cast<const MatD*>(dev_tables + off_w2);
    t.nwsegsA = nwsegsA;
    t.nwsegsB = nwsegsB;
    t.copy_dtype = copy_dtype;
    t.ndblk = ndblk;
    t.ws = workspace;
    t.seg_kal_off = seg_kal_off;
    t.kal_sum_off = kal_sum_off;
    t.smaps = smaps.empty() ? nullptr : reinterpret_cast<const CUtensorMap*>(dev_tables + off_smaps);
    t.ndir = ndir;
    t.dir = 0;
    t.dstride_f = dstride_f;
    t.dstride_z = dstride_z;
    return t;
  }

  // Lays the tables out in one blob; pointers into the workspace are patched at bind.
  void pack() {
    Layout T;
    off_mats = T.take(mats.size() * sizeof(MatD), 64);
    off_w1 = T.take(w1.size() * sizeof(MatD), 64);
    off_w2 = T.take(w2.size() * sizeof(MatD), 64);
    off_mods = T.take(mods.size() * sizeof(ModD), 64);
    off_bases = T.take(bases.size() * sizeof(BasisD), 64);
    off_tcb = T.take(tcb.size() * sizeof(tc::TCBasis), 64);
    off_smaps = T.take(smaps.size() * sizeof(CUtensorMap), 64);
    off_ysched = T.take(ysched.size() * sizeof(int32_t), 64);
    off_pitems_y = T.take(pitems_y.size() * sizeof(tc::PiItem), 64);
    off_pitems_w = T.take(pitems_w.size() * sizeof(tc::PiItem), 64);
    off_calib = T.take(calib.size() * sizeof(CalibD), 64);
    off_rot = T.take(rot_tile0.size() * sizeof(int32_t), 64);
    off_ptiles = T.take(ptiles.size() * sizeof(int32_t), 64);
    table_bytes = T.bytes < 64 ? 64 : T.bytes;
  }
  void write_blob() {
    blob.assign(table_bytes, 0);
    if (!mats.empty()) std::memcpy(blob.data() + off_mats, mats.data(), mats.size() * sizeof(MatD));
    if (!w1.empty()) std::memcpy(blob.data() + off_w1, w1.data(), w1.size() * sizeof(MatD));
    if (!w2.empty()) std::memcpy(blob.data() + off_w2, w2.data(), w2.size() * sizeof(MatD));
    if (!mods.empty()) std::memcpy(blob.data() + off_mods, mods.data(), mods.size() * sizeof(ModD));
    if (!bases.empty()) std::memcpy(blob.data() + off_bases, bases.data(), bases.size() * sizeof(BasisD));
    if (!tcb.empty()) std::memcpy(blob.data() + off_tcb, tcb.data(), tcb.size() * sizeof(tc::TCBasis));
    if (!smaps.empty()) std::memcpy(blob.data() + off_smaps, smaps.data(), smaps.size() * sizeof(CUtensorMap));
    if (!ysched.empty()) std::memcpy(blob.data() + off_ysched, ysched.data(), ysched.size() * sizeof(int32_t));
    if (!pitems_y.empty()) std::memcpy(blob.data() + off_pitems_y, pitems_y.data(), pitems_y.size() * sizeof(tc::PiItem));
    if (!pitems_w.empty()) std::memcpy(blob.data() + off_pitems_w, pitems_w.data(), pitems_w.size() * sizeof(tc::PiItem));
    if (!calib.empty()) std::memcpy(blob.data() + off_calib, calib.data(), calib.size() * sizeof(CalibD));
    if (!rot_tile0.empty()) std::memcpy(blob.data() + off_rot, rot_tile0.data(), rot_tile0.size() * sizeof(int32_t));
    if (!ptiles.empty()) std::memcpy(blob.data() + off_ptiles, ptiles.data(), ptiles.size() * sizeof(int32_t));
  }
};

namespace {

// The CUDA-core Y product has (T/64) x (R/64) output tiles per basis: when that is well
// under two CTAs per SM (small sets), K = D is split so each split's CTAs stream their own
// chunk of H, and k_pi_ysum adds the partials in slot order (deterministic).
void plan_ysplit(dsmz_plan* P) {
  P->ysplit = 1;
  if (P->tc || P->bases.empty()) return;
  int64_t mind = P->bases[0].D;
  P->ytotal = 0;
  for (const BasisD& b : P->bases) {
    mind = std::min(mind, b.D);
    P->ytotal += b.T * b.R;
  }
  int sp = std::max(1, std::min(8, 296 / std::max(1, P->nytiles)));
  while (sp > 1 && mind / sp < 128) --sp;
  P->ysplit = sp;
  if (sp > 1)
    for (BasisD& b : P->bases)
      b.ypart_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(sp) * b.T * b.R * sizeof(float)) / sizeof(float));
}

// First-step calibration: each basis draws torch.randn(rows, R), rows = D when T >= D, else T
// (torch.svd_lowrank transposes H when T < D), in basis order from one generator; its
// calibration state takes 8 partial Grams, the rotation and, for R > 96, the Jacobi rotation.
void plan_calibration(dsmz_plan* P, int sm_count, int mtps) {
  Layout L;
  int64_t e0 = 0;
  uint64_t off = 0;
  int tiles = 0;
  for (const BasisD& b : P->bases) {
    CalibD c{};
    c.into_y = b.T < b.D ? 1 : 0;
    const int64_t rows = c.into_y ? b.T : b.D;
    c.e0 = e0;
    c.n = rows * b.R;
    c.threads = dsmz_randn_threads(c.n, sm_count, mtps);
    c.offset = off;
    e0 += c.n;
    off += dsmz_randn_offset_increment(c.n, sm_count, mtps);
    const size_t rr = static_cast<size_t>(b.R) * b.R;
    c.gpart_off = static_cast<int64_t>(L.take(kCalibGroups * rr * sizeof(double), 256) / sizeof(double));
    c.u_off = static_cast<int64_t>(L.take((rr + b.R) * sizeof(double), 256) / sizeof(double));
    const size_t jn = static_cast<size_t>(jacobi_n(b.R));
    c.uw_off = jacobi_u_in_smem(b.R) ? 0 : static_cast<int64_t>(L.take(jn * jn * sizeof(double), 256) / sizeof(double));
    P->calib.push_back(c);
    P->rot_tile0.push_back(tiles);
    tiles += static_cast<int>((b.D + kRotRows - 1) / kRotRows);
  }
  P->calib_total = e0;
  P->calib_inc = off;
  P->rot_tiles = tiles;
  P->calib_ws_bytes = L.bytes < 256 ? 256 : L.bytes;
}

// Workspace-relative slots that hold device pointers (W, Y) are stored as offsets during
// planning and turned into addresses once the workspace is known.
void patch_ws_pointers(dsmz_plan* P) {
  for (size_t i = 0; i < P->bases.size(); ++i) {
    const BasisD& b = P->bases[i];
    float* W = reinterpret_cast<float*>(P->workspace) + b.w_off;
    P->w1[i].mu = W;
    P->w1[i].param = W;
    P->w2[i].mu = W;
    P->w2[i].param = b.Vout;
    if (P->tc && i < P->tcs.size()) {
      P->w2[i].v2t = reinterpret_cast<__nv_bfloat16*>(P->workspace + P->tcs[i].v2t);
      P->w2[i].ldv2 = P->tcs[i].ldv2;
    } else {
      P->w2[i].v2t = nullptr;
    }
  }
}

// CholeskyQR tables of every basis W (D x R): the Gram pass (its segments and partials are
// placed by chunk_matrices) and the apply segments of V = W R^{-1}.
void add_w_tables(dsmz_plan* P) {
  for (size_t i = 0; i < P->bases.size(); ++i) {
    const BasisD& b = P->bases[i];
    const size_t rr = static_cast<size_t>(b.R) * b.R;
    MatD a{};
    a.nvec = b.D; a.r = b.R; a.ld = b.R; a.cs = 1; a.side = 0; a.owner = static_cast<int32_t>(i);
    a.tmap = -1;
    a.kmap = -1;
    a.rmap = -1;
    a.segv = seg_vectors(b.R);
    a.nseg = static_cast<int32_t>((b.D + a.segv - 1) / a.segv);
    a.p_off = static_cast<int64_t>(P->ws.take((rr + 4) * sizeof(float)) / sizeof(float));
    a.dw_off = static_cast<int64_t>(P->ws.take(3 * rr * sizeof(double)) / sizeof(double));
    MatD m = a;                 // apply segments: V = W R^{-1} (fp64 R^{-1} in a's workspace)
    m.segv = seg_vectors(b.R);
    m.nseg = static_cast<int32_t>((b.D + m.segv - 1) / m.segv);
    m.seg0 = P->nwsegsB;
    P->nwsegsB += m.nseg;
    P->w1.push_back(a);
    P->w2.push_back(m);
  }
}

// Reserves the tensor-core slots of every basis (host only, no CUDA calls).
void plan_tc_layout(dsmz_plan* P) {
  P->tcb.assign(P->bases.size(), tc::TCBasis{});
  P->tcs.assign(P->bases.size(), TCSlots{});
  for (size_t i = 0; i < P->bases.size(); ++i) {
    const BasisD& b = P->bases[i];
    TCSlots& t = P->tcs[i];
    t.ldv2 = round_up(b.D, 64);
    t.ldy2 = round_up(b.T, 64);
    t.v2t = P->ws.take(static_cast<size_t>(2 * b.R) * t.ldv2 * 2, 1024);
    t.y2t = P->ws.take(static_cast<size_t>(2 * b.R) * t.ldy2 * 2, 1024);
    tc::TCBasis& c = P->tcb[i];
    c.T = b.T; c.D = b.D; c.R = b.R; c.ldv2 = t.ldv2; c.ldy2 = t.ldy2;
    const int64_t wrows = static_cast<int64_t>(tc::w_halves(static_cast<int>(b.R))) * tc::kBM;   // rows per tile
    c.ytile0 = P->ntc_y; c.nytile = static_cast<int32_t>((b.T + wrows - 1) / wrows); P->ntc_y += c.nytile;
    c.wtile0 = P->ntc_w; c.nwtile = static_cast<int32_t>((b.D + wrows - 1) / wrows); P->ntc_w += c.nwtile;
    c.vt0 = P->ntc_vt; c.nvt = static_cast<int32_t>((b.D + tc::kSplitD - 1) / tc::kSplitD); P->ntc_vt += c.nvt;
    if (b.R <= 64) {           // the W epilogue forms the Gram: one block-major partial per W tile
      const int nb = b.R / 8;
      c.nq = nb * (nb + 1) / 2;
      t.gp = P->ws.take(static_cast<size_t>(c.nwtile) * c.nq * 64 * sizeof(double));
    }
  }
  // Persistent Y kernel: tiles cost ceil(D / 64) k-steps (plus the epilogue), so with the
  // SM count known the tiles are dealt longest first, each to the least-loaded CTA.
  P->ysched.clear();
  P->ysched_G = 0;
  if (P->sm_count > 0 && P->ntc_y > 0) {
    const int G = std::min(P->ntc_y, P->sm_count);
    std::vector<std::pair<int64_t, int>> items;           // (cost, item)
    for (const tc::TCBasis& c : P->tcb)
      for (int t = 0; t < c.nytile; ++t) items.push_back({(c.D + tc::kBK - 1) / tc::kBK + 4, c.ytile0 + t});
    std::stable_sort(items.begin(), items.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    std::vector<int64_t> load(G, 0);
    std::vector<std::vector<int32_t>> lists(G);
    for (const auto& it : items) {
      const int c = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
      load[c] += it.first;
      lists[c].push_back(it.second);
    }
    P->ysched.assign(G + 1, 0);
    for (int c = 0; c < G; ++c) P->ysched[c + 1] = P->ysched[c] + static_cast<int32_t>(lists[c].size());
    for (int c = 0; c < G; ++c) P->ysched.insert(P->ysched.end(), lists[c].begin(), lists[c].end());
    P->ysched_G = G;
  }
}

// Work queues of the single-pass power iteration (R <= 64, see dsmz_pi_fused.cuh).
// Y queue: bases in windows of kWindowBases (one decoder layer's four module inputs); within
// a window the bases' 256-token tiles go row by row (tile t of every basis, then t + 1), each
// tile split over d into items of about kYSplitSteps k-steps, its splits consecutive. Split
// items write partials into a ring of kPartSlots slots by queue position; an item whose slot
// was last written by another tile waits for that tile to be reduced first.
// W queue: the same windows; one item per 256-row d tile of a basis over all of its tokens,
// the bases of a window dealt in proportion to their tile counts.
constexpr int kYSplitSteps = 20;
constexpr int kPartSlots = 512;
constexpr int kWindowBases = 4;

void plan_pi_fused(dsmz_plan* P) {
  const int nb = static_cast<int>(P->bases.size());
  std::vector<int> tile0(nb), ntile(nb), nsplit(nb), kper(nb), nkd(nb);
  int nt = 0;
  for (int b = 0; b < nb; ++b) {
    const BasisD& B = P->bases[b];
    tile0[b] = nt;
    ntile[b] = static_cast<int>((B.T + 255) / 256);
    nt += ntile[b];
    nkd[b] = static_cast<int>((B.D + tc::kBK - 1) / tc::kBK);
    int ns = (nkd[b] + kYSplitSteps - 1) / kYSplitSteps;
    kper[b] = (nkd[b] + ns - 1) / ns;
    nsplit[b] = (nkd[b] + kper[b] - 1) / kper[b];
  }
  P->f_ytiles = nt;
  P->pitems_y.clear();
  P->pitems_w.clear();
  int nslots = 0, nyitems = 0;
  for (int b = 0; b < nb; ++b) {
    nyitems += ntile[b] * nsplit[b];
    if (nsplit[b] > 1) nslots = kPartSlots;
  }
  int max_split = 1;
  for (int b = 0; b < nb; ++b) max_split = std::max(max_split, nsplit[b]);
  if (nslots) nslots = std::max(nslots, 2 * max_split);   // a tile's own splits never share a slot
  nslots = std::min(nslots, nyitems);
  std::vector<int> last_user(std::max(nslots, 1), -1);    // tile whose split last wrote each slot
  int qpos = 0;
  for (int w0 = 0; w0 < nb; w0 += kWindowBases) {
    const int w1 = std::min(nb, w0 + kWindowBases);
    int rows = 0;
    for (int b = w0; b < w1; ++b) rows = std::max(rows, ntile[b]);
    for (int t = 0; t < rows; ++t) {
      for (int b = w0; b < w1; ++b) {
        if (t >= ntile[b]) continue;
        const int slot0 = nslots ? qpos % nslots : 0;
        for (int ks = 0; ks < nsplit[b]; ++ks, ++qpos) {
          tc::PiItem it{};
          it.basis = b;
          it.tile = t;
          it.k0 = ks * kper[b];
          it.k1 = std::min(nkd[b], it.k0 + kper[b]);
          it.ytile = tile0[b] + t;
          it.nsplit = nsplit[b];
          it.ks = ks;
          it.slot0 = slot0;
          it.slot = nslots ? qpos % nslots : 0;
          it.wait_tile = -1;
          if (nsplit[b] > 1) {
            const int prev = last_user[it.slot];
            if (prev >= 0 && prev != it.ytile) it.wait_tile = prev;
            last_user[it.slot] = it.ytile;
          }
          P->pitems_y.push_back(it);
        }
      }
    }
    // W items of the window, bases dealt in proportion to their d tiles
    std::vector<int> nwt(w1 - w0), done(w1 - w0, 0);
    int total = 0;
    for (int b = w0; b < w1; ++b) { nwt[b - w0] = static_cast<int>((P->bases[b].D + 255) / 256); total += nwt[b - w0]; }
    for (int e = 0; e < total; ++e) {
      int best = -1;
      for (int j = 0; j < w1 - w0; ++j)
        if (done[j] < nwt[j] && (best < 0 || static_cast<int64_t>(done[j]) * nwt[best] < static_cast<int64_t>(done[best]) * nwt[j]))
          best = j;
      const int b = w0 + best;
      tc::PiItem it{};
      it.basis = b;
      it.tile = done[best]++;
      it.k0 = 0;
      it.k1 = static_cast<int>((P->bases[b].T + tc::kBK - 1) / tc::kBK);
      it.ytile = tile0[b];
      it.wait_tile = -1;
      P->pitems_w.push_back(it);
    }
  }
  P->f_nslots = nslots;
  // launch-local counters (zeroed before each launch) and the partial slots
  P->fsync_bytes = static_cast<size_t>(2 + 2 * nt) * sizeof(int32_t);
  P->fsync_off = P->ws.take(P->fsync_bytes);
  P->fpart_off = P->ws.take(static_cast<size_t>(std::max(nslots, 1)) * P->R * 256 * sizeof(float));
  P->fused = true;
}

// The four tile-box maps (param, mu, var, z) of every side-1 adapter matrix; a matrix whose
// arrays the driver refuses (alignment) keeps the copy-engine path (tmap = -1).
void bind_side1_maps(dsmz_plan* P) {
  const int TV = P->Lg.TV;
  for (MatD& m : P->mats) {
    if (m.tmap < 0) continue;
    bool ok = TV <= 256 && m.r <= 256 && m.cs == 1;
    const void* arr[4] = {m.param, m.mu, m.var, m.z};
    const int dt[4] = {DSMZ_F32, DSMZ_F32, DSMZ_F32, DSMZ_F32};
    for (int j = 0; j < 4 && ok; ++j) {
      const int es = (dt[j] == DSMZ_BF16) ? 2 : 4;
      ok = ((reinterpret_cast<uintptr_t>(arr[j]) & 15) == 0) && ((m.ld * es) % 16 == 0) &&
           encode_rows_2d(&P->smaps[m.tmap + j], dt[j], arr[j], static_cast<uint64_t>(m.nvec),
                          static_cast<uint64_t>(m.r), static_cast<uint64_t>(m.ld) * es, static_cast<uint32_t>(TV),
                          static_cast<uint32_t>(m.r));
    }
    if (!ok) m.tmap = -1;
  }
}

// Swizzled row boxes (32 fp32 columns x TV rows) of the perturbation's K operand (Zc_A rows
// in the workspace, or the basis rows), of side-0 mu and of W; a slot the driver refuses
// (alignment, strides) falls back to element copies into the same image (slot = -1).
void bind_swz_maps(dsmz_plan* P) {
  // K-operand rows of the perturbation: 128-row boxes for the tensor-core kernel, which needs
  // every one of them (else the plan keeps the CUDA-core perturbation)
  if (P->ptc) {
    for (const MatD& m : P->mats) {
      const ModD& D = P->mods[m.owner];
      CUtensorMap tmp;
      const void* base = m.side == 0 ? static_cast<const void*>(reinterpret_cast<const float*>(P->workspace) + D.zca_off)
                                      : static_cast<const void*>(P->bases[D.basis].Vin);
      const int64_t cols = m.side == 0 ? D.rca : D.rc;
      const int64_t rows = m.side == 0 ? m.nvec : P->bases[D.basis].D;
      const int64_t ld = m.side == 0 ? D.rca : P->bases[D.basis].v_s0;
      const int64_t cs = m.side == 0 ? 1 : P->bases[D.basis].v_s1;
      const bool ok = m.kmap >= 0 && cs == 1 && (reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 4) % 16 == 0 &&
                      encode_rows_swz(&tmp, base, static_cast<uint64_t>(cols), static_cast<uint64_t>(rows),
                                      static_cast<uint64_t>(ld) * 4, static_cast<uint32_t>(atc::kTile));
      if (!ok) { P->ptc = false; break; }
    }
  }
  const int krows = P->ptc ? atc::kTile : P->Lp.TV;
  auto enc = [&](int32_t& slot, const void* base, int64_t cols, int64_t rows, int64_t ld, int64_t cs, int TV) {
    if (slot < 0) return;
    const bool ok = base != nullptr && cs == 1 && TV <= 256 && TV % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 4) % 16 == 0 &&
                    encode_rows_swz(&P->smaps[slot], base, static_cast<uint64_t>(cols), static_cast<uint64_t>(rows),
                                    static_cast<uint64_t>(ld) * 4, static_cast<uint32_t>(TV));
    if (!ok) slot = -1;
  };
  for (MatD& m : P->mats) {
    const ModD& D = P->mods[m.owner];
    if (m.side == 0) {
      enc(m.kmap, reinterpret_cast<const float*>(P->workspace) + D.zca_off, D.rca, m.nvec, D.rca, 1, krows);
      enc(m.rmap, m.mu, m.r, m.nvec, m.ld, m.cs, P->La.TV);
    } else {
      const BasisD& Bd = P->bases[D.basis];
      enc(m.kmap, Bd.Vin, D.rc, Bd.D, Bd.v_s0, Bd.v_s1, krows);
    }
  }
  for (MatD& m : P->w2) enc(m.rmap, m.mu, m.r, m.nvec, m.ld, m.cs, P->Lq.TV);
}

// Fills pointers and tensor maps once the workspace is known; false if the driver refuses
// a tensor map (the plan then keeps the CUDA-core path).
bool bind_tc(dsmz_plan* P) {
  for (size_t i = 0; i < P->bases.size(); ++i) {
    const BasisD& b = P->bases[i];
    const TCSlots& t = P->tcs[i];
    tc::TCBasis& c = P->tcb[i];
    c.V2T = reinterpret_cast<__nv_bfloat16*>(P->workspace + t.v2t);
    c.Y2T = reinterpret_cast<__nv_bfloat16*>(P->workspace + t.y2t);
    c.W = reinterpret_cast<float*>(P->workspace) + b.w_off;
    c.Gp = t.gp ? reinterpret_cast<double*>(P->workspace + t.gp) : nullptr;
    c.Vsrc = b.Vin; c.v_s0 = b.v_s0; c.v_s1 = b.v_s1; c.Vout = b.Vout;
    const uint32_t n2 = static_cast<uint32_t>(2 * b.R);
    if (!encode_bf16_2d(&c.mapHy, b.H, b.D, b.T, b.h_s0 * 2, 64, 128) ||
        !encode_bf16_2d(&c.mapHw, b.H, b.D, b.T, b.h_s0 * 2, 64, 64) ||
        !encode_bf16_2d(&c.mapV2, c.V2T, b.D, n2, t.ldv2 * 2, 64, n2) ||
        !encode_bf16_2d(&c.mapY2, c.Y2T, b.T, n2, t.ldy2 * 2, 64, n2))
      return false;
  }
  return true;
}


// Tile width of the adapter matrices' streaming kernels: the widest (a multiple of 8, at
// most sk::stream_tv(r)) whose perturbation, Gram and apply layouts all fit with a ring
// of at least kTeams stages for the team kernels (two for the Gram). One width for all of
// them: their segments (Kalman and Gram partials) follow the same tile chunks.
// The tensor-core perturbation's epilogue moves the tile's elements in 16-byte units: unit
// component strides, leading dimensions, row lengths (tall matrices) or column counts (wide
// ones) and the arrays' alignment multiples of four elements.
bool ptc_strides_ok(const dsmz_plan* P) {
  const int fes = P->copy_dtype == DSMZ_BF16 ? 2 : 4;
  auto al = [](const void* p, int b) { return (reinterpret_cast<uintptr_t>(p) % b) == 0; };
  if ((P->dstride_f % 4) != 0 || (P->dstride_z % 4) != 0) return false;
  for (const MatD& m : P->mats) {
    if (m.cs != 1 || (m.ld % 4) != 0 || !al(m.param, 16) || !al(m.mu, 16) || !al(m.var, 16) || !al(m.z, 16) ||
        !al(m.pos, 4 * fes) || !al(m.neg, 4 * fes))
      return false;
    if (m.side == 0 ? (m.r % 4) != 0 : (m.nvec % 4) != 0) return false;
  }
  return true;
}

bool choose_adapter_layouts(dsmz_plan* P) {
  const int r = P->r, rca = P->r < P->RC ? P->r : P->RC;
  for (int tv = sk::stream_tv(r); tv >= 8; tv = (tv / 2) & ~7) {
    P->Lp = sk::perturb_layout(r, r, P->RC, rca, kStreamSmem, tv);
    P->Lg = sk::gram_layout(r, 1, kStreamSmem, tv);
    P->La = sk::apply_layout(r, kStreamSmem, tv);
    const bool ok = P->Lp.S >= sk::kTeams && P->La.S >= sk::kTeams && P->Lg.S >= 2 &&
                    P->Lp.total <= kStreamSmem + 2048 && P->La.total <= kStreamSmem + 2048 &&
                    P->Lg.total <= kStreamSmem + 2048;
    if (ok) {
      // the tensor-core perturbation when its shapes, strides and shared memory allow
      const int kw = P->RC > rca ? P->RC : rca;
      if (P->ptc && atc::perturb_ok(r, kw) && ptc_strides_ok(P)) {
        P->Lpt = atc::perturb_layout(r, kw, kStreamSmem);
        P->ptc = P->Lpt.S >= 2 && P->Lpt.total <= kStreamSmem + 2048;
      } else {
        P->ptc = false;
      }
      if (P->ptc) {
        P->ptiles.clear();
        int32_t t = 0;
        for (const MatD& m : P->mats) {
          P->ptiles.push_back(t);
          t += static_cast<int32_t>((m.nvec + atc::kTile - 1) / atc::kTile);
        }
        P->ptiles.push_back(t);
      }
      return true;
    }
    if (tv == 8) break;
  }
  return false;
}

bool choose_qr_layout(dsmz_plan* P) {
  bool ok = false;
  for (int tv = sk::stream_tv(P->R); tv >= 8 && !ok; tv -= 8) {    // QR apply: widest tile that fits
    if (sk::qr_variant(tv, P->R) < 0) continue;
    P->Lq = sk::qr_layout(P->R, kStreamSmem, tv);
    ok = P->Lq.S >= sk::kQrGroups && P->Lq.total <= kStreamSmem + 2048;
  }
  if (!ok) return false;
  for (int tv = sk::stream_tv(P->R); tv >= 8; tv = (tv / 2) & ~7) {    // Gram of W (plain)
    P->Lw = sk::gram_layout(P->R, 0, kStreamSmem, tv);
    if (P->Lw.S >= 2 && P->Lw.total <= kStreamSmem + 2048) return true;
    if (tv == 8) break;
  }
  return false;
}

// Streaming schedule of the power-iteration tables once the SM count is known: the W Gram
// (with its per-segment partials, placed here when alloc, else reserved beforehand by
// reserve_w_gram) and the QR apply.
void chunk_w_tables(dsmz_plan* P, bool alloc) {
  if (P->w1.empty()) return;
  P->nwsegsA = chunk_matrices(P->w1, P->Lw.TV, P->sm_count, alloc ? &P->ws : nullptr, &P->grid_w1);
  chunk_matrices(P->w2, P->Lq.TV, P->sm_count, nullptr, &P->grid_w);
}

// One-basis plans are laid out before the device is known: room for the Gram partials of
// up to kMaxChunks segments (one per CTA of a grid no wider than that).
constexpr int kMaxChunks = 1024;
void reserve_w_gram(dsmz_plan* P) {
  for (MatD& a : P->w1) {
    const int64_t tiles = (a.nvec + P->Lw.TV - 1) / P->Lw.TV;
    const int64_t n = tiles < kMaxChunks ? tiles : kMaxChunks;
    a.gram_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(n) * a.r * a.r * sizeof(double)) / sizeof(double));
  }
}

// ---------------------------------------------------------------- launch sequences
// Launch helpers of the power iteration: set-up (shared-memory limits, tables), the Y
// product, and the rest of an iteration (W product, CholeskyQR of W, V = W R^-1).
struct PiCtx {
  Tables tb;
  int R = 0, nb = 0, gpb = 0;
  const tc::TCBasis* dtcb = nullptr;
  int* err = nullptr;
  bool gram_fused = false;   // the tensor-core W epilogue forms the fp64 W Gram (R <= 64)
  bool small = false;
};

int pi_setup(const dsmz_plan* P, PiCtx& c) {
  c.tb = P->tables();
  c.R = P->R;
  c.nb = static_cast<int>(P->bases.size());
  c.dtcb = reinterpret_cast<const tc::TCBasis*>(P->dev_tables + P->off_tcb);
  c.err = reinterpret_cast<int*>(P->workspace + P->err_off);
  c.gram_fused = P->tc && c.R <= 64;
  c.gpb = (c.R * c.R / 2 + c.R * 4 + kThreads - 1) / kThreads;   // k_gsum CTAs per basis
  c.small = sk::gram_maxb(c.R) <= 5;
  int rc;
  if ((rc = set_smem(sk::k_sgram<0, 5>, P->Lw.total))) return rc;
  if ((rc = set_smem(sk::k_sgram<0, 17>, P->Lw.total))) return rc;
  if ((rc = set_smem(sk::k_sqr_apply<2, 4>, P->Lq.total))) return rc;
  if ((rc = set_smem(sk::k_sqr_apply<4, 2>, P->Lq.total))) return rc;
  if ((rc = set_smem(sk::k_sqr_apply<1, 8>, P->Lq.total))) return rc;
  if ((rc = set_smem(sk::k_sqr_apply<8, 1>, P->Lq.total))) return rc;
  if ((rc = set_smem(k_chol, chol_smem(c.R)))) return rc;
  if (P->tc) {
    if ((rc = set_smem(tc::k_pi_yp<1>, py_smem(c.R)))) return rc;
    if ((rc = set_smem(tc::k_pi_yp<2>, py_smem(c.R)))) return rc;
    if ((rc = set_smem(tc::k_pi_w<1>, pw_smem(c.R)))) return rc;
    if ((rc = set_smem(tc::k_pi_w<2>, pw_smem(c.R)))) return rc;
  }
  if (P->fused) {
    if ((rc = set_smem(tc::k_pi_fused, pf_smem(c.R)))) return rc;
  }
  return 0;
}

// [V_hi | V_lo]^T of the bases as they stand (tensor-core path), from the caller's strided
// basis when `first`, else from the contiguous result buffer.
int pi_split(const dsmz_plan* P, const PiCtx& c, cudaStream_t s, int first = 1) {
  if (!P->tc) return 0;
  P->probe_begin(DSMZ_KID_PI_SPLIT, s);
  tc::k_split_vt<<<P->ntc_vt, kThreads, 0, s>>>(c.dtcb, c.nb, first);
  P->probe_end(DSMZ_KID_PI_SPLIT, s);
  DSMZ_LAUNCHED("power iteration basis split");
  return 0;
}

// Y = H V of every basis: the tensor-core path writes [Y_hi | Y_lo]^T, the CUDA-core path
// the fp32 Y (from the caller's strided basis when `first`).
int pi_y(const dsmz_plan* P, const PiCtx& c, cudaStream_t s, int first) {
  const int R = c.R;
  P->probe_begin(DSMZ_KID_PI_Y, s);
  if (P->tc) {
    const int32_t* ys = P->ysched.empty() ? nullptr : reinterpret_cast<const int32_t*>(P->dev_tables + P->off_ysched);
    const int gy = ys ? P->ysched_G : std::min(P->ntc_y, P->sm_count);
    if (tc::w_halves(R) == 2)
      tc::k_pi_yp<2><<<gy, tc::kThreadsTC, py_smem(R), s>>>(c.dtcb, c.nb, P->ntc_y, ys, py_stages(R), c.err);
    else
      tc::k_pi_yp<1><<<gy, tc::kThreadsTC, py_smem(R), s>>>(c.dtcb, c.nb, P->ntc_y, ys, py_stages(R), c.err);
  } else {
    k_pi_gemm<0><<<dim3(P->nytiles, P->ysplit), kThreads, 0, s>>>(c.tb, first);
    if (P->ysplit > 1) {
      DSMZ_LAUNCHED("power iteration Y = H V (split)");
      const int g = static_cast<int>(std::min<int64_t>((P->ytotal + kThreads - 1) / kThreads, 1184));
      k_pi_ysum<<<g, kThreads, 0, s>>>(c.tb, P->ytotal);
    }
  }
  P->probe_end(DSMZ_KID_PI_Y, s);
  DSMZ_LAUNCHED(P->tc ? "power iteration Y = H V (tcgen05)" : "power iteration Y = H V");
  return 0;
}

int pi_qr_tail(const dsmz_plan* P, const PiCtx& c, float floor_, cudaStream_t s);

// W = H^T Y, the Gram of W, its Cholesky factor and V = W R^-1 (with the bf16 pair of V for
// the next tensor-core Y product).
int pi_w_tail(const dsmz_plan* P, const PiCtx& c, float floor_, cudaStream_t s) {
  const int R = c.R, nb = c.nb;
  const Tables& tb = c.tb;
  P->probe_begin(DSMZ_KID_PI_W, s);
  if (P->tc) {
    if (tc::w_halves(R) == 2)
      tc::k_pi_w<2><<<std::min(P->ntc_w, P->sm_count), tc::kThreadsTC, pw_smem(R), s>>>(c.dtcb, nb, P->ntc_w,
                                                                                      pw_stages(R), c.err);
    else
      tc::k_pi_w<1><<<std::min(P->ntc_w, P->sm_count), tc::kThreadsTC, pw_smem(R), s>>>(c.dtcb, nb, P->ntc_w,
                                                                                      pw_stages(R), c.err);
  } else {
    k_pi_gemm<1><<<P->nwtiles, kThreads, 0, s>>>(tb, 0);
  }
  P->probe_end(DSMZ_KID_PI_W, s);
  DSMZ_LAUNCHED(P->tc ? "power iteration W = H^T Y (tcgen05)" : "power iteration W = H^T Y");
  return pi_qr_tail(P, c, floor_, s);
}

// CholeskyQR of W from its exact fp64 Gram (fp64 MMA: fused into the tensor-core W epilogue
// for R <= 64, else streamed); V = W R^{-1} accumulated in fp64, with the bf16 pair for the
// next tensor-core Y.
int pi_qr_tail(const dsmz_plan* P, const PiCtx& c, float floor_, cudaStream_t s) {
  const int R = c.R, nb = c.nb;
  const Tables& tb = c.tb;
  const KalmanIn kin{};
  P->probe_begin(DSMZ_KID_PI_GRAM, s);
  if (c.gram_fused) {
    tc::k_gsum<<<nb * c.gpb, kThreads, 0, s>>>(c.dtcb, tb, tb.wA, c.gpb);
  } else if (c.small) {
    sk::k_sgram<0, 5><<<P->grid_w1, sk::kSTG, P->Lw.total, s>>>(tb, tb.wA, nb, P->nwsegsA, P->Lw, kin, c.err);
  } else {
    sk::k_sgram<0, 17><<<P->grid_w1, sk::kSTG, P->Lw.total, s>>>(tb, tb.wA, nb, P->nwsegsA, P->Lw, kin, c.err);
  }
  P->probe_end(DSMZ_KID_PI_GRAM, s);
  DSMZ_LAUNCHED("power iteration Gram of W");
  P->probe_begin(DSMZ_KID_PI_CHOL, s);
  k_chol<<<nb, kThreads, chol_smem(R), s>>>(tb, tb.wA, floor_, c.gram_fused ? 1 : 0);
  P->probe_end(DSMZ_KID_PI_CHOL, s);
  DSMZ_LAUNCHED("power iteration Cholesky");
  P->probe_begin(DSMZ_KID_PI_APPLY, s);
  switch (sk::qr_variant(P->Lq.TV, P->R)) {
    case 0: sk::k_sqr_apply<2, 4><<<P->grid_w, sk::kQrThreads, P->Lq.total, s>>>(tb, tb.wB, nb, P->nwsegsB, P->Lq, c.err); break;
    case 1: sk::k_sqr_apply<4, 2><<<P->grid_w, sk::kQrThreads, P->Lq.total, s>>>(tb, tb.wB, nb, P->nwsegsB, P->Lq, c.err); break;
    case 2: sk::k_sqr_apply<1, 8><<<P->grid_w, sk::kQrThreads, P->Lq.total, s>>>(tb, tb.wB, nb, P->nwsegsB, P->Lq, c.err); break;
    default: sk::k_sqr_apply<8, 1><<<P->grid_w, sk::kQrThreads, P->Lq.total, s>>>(tb, tb.wB, nb, P->nwsegsB, P->Lq, c.err); break;
  }
  P->probe_end(DSMZ_KID_PI_APPLY, s);
  DSMZ_LAUNCHED("power iteration V = W R^-1");
  return 0;
}

int run_power_iteration(const dsmz_plan* P, int iters, float floor_, cudaStream_t s, uint32_t flags = 0u) {
  if (P->bases.empty() || iters <= 0) return 0;
  PiCtx c;
  int rc;
  if ((rc = pi_setup(P, c))) return rc;
  if (P->tc) {
    if (!((flags & DSMZ_PI_BASIS_UNCHANGED) && P->split_current) && (rc = pi_split(P, c, s))) return rc;
    P->split_current = true;            // the last QR apply writes [V_hi | V_lo]^T of V
  }
  for (int it = 0; it < iters; ++it) {
    if (P->fused) {
      // one launch: Y tiles stream H from HBM, W tiles re-read it from L2
      cudaError_t ez = cudaMemsetAsync(P->workspace + P->fsync_off, 0, P->fsync_bytes, s);
      if (ez != cudaSuccess) return cuda_fail("power iteration counters", ez);
      tc::PiSync sy;
      sy.head = reinterpret_cast<int32_t*>(P->workspace + P->fsync_off);
      sy.ycnt = sy.head + 2;
      sy.ytdone = sy.ycnt + P->f_ytiles;
      sy.part = reinterpret_cast<float*>(P->workspace + P->fpart_off);
      sy.nslots = P->f_nslots;
      const tc::PiItem* yq = reinterpret_cast<const tc::PiItem*>(P->dev_tables + P->off_pitems_y);
      const tc::PiItem* wq = reinterpret_cast<const tc::PiItem*>(P->dev_tables + P->off_pitems_w);
      const int ny = static_cast<int>(P->pitems_y.size()), nw = static_cast<int>(P->pitems_w.size());
      P->probe_begin(DSMZ_KID_PI_FUSED, s);
      tc::k_pi_fused<<<std::min(P->sm_count, std::max(ny, nw)), tc::kFusedThreads, pf_smem(c.R), s>>>(
          c.dtcb, yq, ny, wq, nw, sy, pf_stages_y(c.R), pf_stages_w(c.R), c.err);
      P->probe_end(DSMZ_KID_PI_FUSED, s);
      DSMZ_LAUNCHED("power iteration W = H^T (H V) (single pass, tcgen05)");
      if ((rc = pi_qr_tail(P, c, floor_, s))) return rc;
    } else {
      if ((rc = pi_y(P, c, s, it == 0 ? 1 : 0))) return rc;
      if ((rc = pi_w_tail(P, c, floor_, s))) return rc;
    }
  }
  return 0;
}

// First-step calibration (the sequence is derived at the top of dsmz_calib.cuh): sketches,
// niter power iterations, the Ritz stage of the T >= D bases (Gram of Y, one more iteration,
// eigenvectors of R_W^-T G_Y R_W^-1), that of the T < D bases (Y of the new basis, its Gram,
// eigenvectors), then V <- V C.
int run_calibration(const dsmz_plan* P, uint64_t seed, uint64_t offset, int niter, float floor_, char* cws,
                    float* sv, cudaStream_t s) {
  if (P->bases.empty()) return 0;
  PiCtx c;
  int rc;
  if ((rc = pi_setup(P, c))) return rc;
  const int R = c.R, nb = c.nb;
  if ((rc = set_smem(k_calib_eig, jacobi_smem(R)))) return rc;
  if ((rc = set_smem(k_calib_rotate, rotate_smem(R)))) return rc;
  const CalibD* dcd = reinterpret_cast<const CalibD*>(P->dev_tables + P->off_calib);
  const int32_t* dt0 = reinterpret_cast<const int32_t*>(P->dev_tables + P->off_rot);
  const tc::TCBasis* ytcb = P->tc ? c.dtcb : nullptr;
  const int gdraw = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((P->calib_total + kThreads - 1) / kThreads,
                                                                            static_cast<int64_t>(P->sm_count) * 8)));
  auto ygram = [&]() {
    const size_t sm = ygram_smem(R);
    if (R <= 16) k_calib_ygram<1><<<nb * kCalibGroups, kThreads, sm, s>>>(c.tb, dcd, ytcb, cws);
    else if (R <= 32) k_calib_ygram<2><<<nb * kCalibGroups, kThreads, sm, s>>>(c.tb, dcd, ytcb, cws);
    else if (R <= 64) k_calib_ygram<4><<<nb * kCalibGroups, kThreads, sm, s>>>(c.tb, dcd, ytcb, cws);
    else k_calib_ygram<8><<<nb * kCalibGroups, kThreads, sm, s>>>(c.tb, dcd, ytcb, cws);
    DSMZ_LAUNCHED("calibration Gram of Y");
    return 0;
  };
  // sketches: V = R_D (T >= D); Y = H V for all bases, then Y = R_T (T < D)
  k_calib_draw<<<gdraw, kThreads, 0, s>>>(c.tb, dcd, nullptr, P->calib_total, seed, offset, 0);
  DSMZ_LAUNCHED("calibration sketch (V)");
  if ((rc = pi_split(P, c, s, 0))) return rc;
  if ((rc = pi_y(P, c, s, 0))) return rc;
  k_calib_draw<<<gdraw, kThreads, 0, s>>>(c.tb, dcd, ytcb, P->calib_total, seed, offset, 1);
  DSMZ_LAUNCHED("calibration sketch (Y)");
  if (niter >= 1) {
    if ((rc = pi_w_tail(P, c, floor_, s))) return rc;
    for (int it = 1; it < niter; ++it) {
      if ((rc = pi_y(P, c, s, 0))) return rc;
      if ((rc = pi_w_tail(P, c, floor_, s))) return rc;
    }
    if ((rc = pi_y(P, c, s, 0))) return rc;
  }
  // T >= D: G_Y, one more iteration (R_W^-1 in the Cholesky workspace), eigenvectors
  if ((rc = ygram())) return rc;
  if ((rc = pi_w_tail(P, c, floor_, s))) return rc;
  k_calib_eig<<<nb, kThreads, jacobi_smem(R), s>>>(c.tb, dcd, cws, 0, sv);
  DSMZ_LAUNCHED("calibration eigenvectors (T >= D)");
  // T < D: Y of the new basis, its Gram, eigenvectors
  if ((rc = pi_y(P, c, s, 0))) return rc;
  if ((rc = ygram())) return rc;
  k_calib_eig<<<nb, kThreads, jacobi_smem(R), s>>>(c.tb, dcd, cws, 1, sv);
  DSMZ_LAUNCHED("calibration eigenvectors (T < D)");
  k_calib_rotate<<<P->rot_tiles, kThreads, rotate_smem(R), s>>>(c.tb, dcd, dt0, cws);
  DSMZ_LAUNCHED("calibration rotation");
  P->split_current = false;
  return 0;
}

// K directions: joint Kalman observation (k_kalman_dirs) writes mu2 / var2, then the plain
int run_update_dirs(const dsmz_plan* P, const sk::KalmanDirs& kd, float eta, const NSArgs& ns, cudaStream_t s) {
  if (P->mats.empty()) return 0;
  const Tables tb = P->tables();
  const int r = P->r;
  const int nm = static_cast<int>(P->mats.size());
  int rc;
  int* err = reinterpret_cast<int*>(P->workspace + P->err_off);
  const bool small = sk::gram_maxb(r) <= 5;
  if ((rc = set_smem(sk::k_sgram<0, 5>, P->Lg.total))) return rc;
  if ((rc = set_smem(sk::k_sgram<0, 17>, P->Lg.total))) return rc;
  if ((rc = set_smem(sk::k_sapply<2>, P->La.total))) return rc;
  if ((rc = set_smem(sk::k_sapply<4>, P->La.total))) return rc;
  P->probe_begin(DSMZ_KID_KALMAN_DIRS, s);
  sk::k_kalman_dirs<<<8 * P->sm_count, 256, 0, s>>>(tb, kd, P->Lg.TV);   // plain stream: many CTAs per SM
  P->probe_end(DSMZ_KID_KALMAN_DIRS, s);
  DSMZ_LAUNCHED("K-direction Kalman update");
  const KalmanIn none{};
  P->probe_begin(DSMZ_KID_GRAM, s);
  if (small) sk::k_sgram<0, 5><<<P->grid_m, sk::kSTG, P->Lg.total, s>>>(tb, tb.mats, nm, P->nsegs, P->Lg, none, err);
  else sk::k_sgram<0, 17><<<P->grid_m, sk::kSTG, P->Lg.total, s>>>(tb, tb.mats, nm, P->nsegs, P->Lg, none, err);
  P->probe_end(DSMZ_KID_GRAM, s);
  DSMZ_LAUNCHED("Gram of the updated momentum");
  P->probe_begin(DSMZ_KID_NS_SOLVE, s);
  if ((rc = launch_ns_solve(tb, tb.mats, nm, r, ns, s))) return rc;
  P->probe_end(DSMZ_KID_NS_SOLVE, s);
  DSMZ_LAUNCHED("Newton-Schulz solve");
  P->probe_begin(DSMZ_KID_APPLY, s);
  if (P->copy_dtype == DSMZ_BF16)
    sk::k_sapply<2><<<P->grid_m, sk::kSTP, P->La.total, s>>>(tb, tb.mats, nm, P->nsegs, P->La, eta, P->speers, err);
  else
    sk::k_sapply<4><<<P->grid_m, sk::kSTP, P->La.total, s>>>(tb, tb.mats, nm, P->nsegs, P->La, eta, P->speers, err);
  P->probe_end(DSMZ_KID_APPLY, s);
  DSMZ_LAUNCHED("Kalman + ZO-Muon apply");
  return 0;
}

KalmanIn make_kin(float beta, float q, float dd, float floor_) {
  KalmanIn k;
  k.beta = beta;
  k.beta2 = static_cast<float>(static_cast<double>(beta) * static_cast<double>(beta));
  k.q = q;
  k.dd = dd;
  k.floor_ = floor_;
  return k;
}

int run_perturb(const dsmz_plan* P, uint64_t seed, uint64_t offset, float eps, KalmanIn kin, float floor_,
                cudaStream_t s) {
  if (P->mods.empty()) return 0;
  const Tables tb = P->tables();
  int rc;
  const size_t cs = coef_smem(P->r, P->RC);
  int* err = reinterpret_cast<int*>(P->workspace + P->err_off);
  if ((rc = set_smem(k_coef<0>, cs))) return rc;
  const bool bf = P->copy_dtype == DSMZ_BF16;
  if (P->ptc) {
    if ((rc = set_smem(atc::k_perturb_tc<2>, P->Lpt.total))) return rc;
    if ((rc = set_smem(atc::k_perturb_tc<4>, P->Lpt.total))) return rc;
  } else {
    if ((rc = set_smem(sk::k_sperturb<2>, P->Lp.total))) return rc;
    if ((rc = set_smem(sk::k_sperturb<4>, P->Lp.total))) return rc;
  }
  P->probe_begin(DSMZ_KID_BSIDE, s);
  k_bside<<<P->nchunks, kThreads, 0, s>>>(tb, P->bside_cols);     // B V and var_B V^2: the same for every direction
  P->probe_end(DSMZ_KID_BSIDE, s);
  DSMZ_LAUNCHED("B-side sums");
  for (int k = 0; k < P->ndir; ++k) {
    Tables td = tb;
    td.dir = k;
    const uint64_t off = offset + static_cast<uint64_t>(k) * P->rng_dir_stride;
    if (!(k == 0 && P->pre_drawn && P->pre_seed == seed && P->pre_off == offset)) {
      P->probe_begin(DSMZ_KID_DRAW, s);
      sk::k_draw_zca<<<std::min(P->ndblk, 16 * P->sm_count), 256, 0, s>>>(td, seed, off);
      P->probe_end(DSMZ_KID_DRAW, s);
      DSMZ_LAUNCHED("Zc_A draws");
    }
    if (k == 0) P->pre_drawn = false;   // consumed (or superseded by this launch's own draws)
    P->probe_begin(DSMZ_KID_COEF, s);
    k_coef<0><<<static_cast<int>(P->mods.size()), kThreads, cs, s>>>(td, seed, off, floor_, k == 0 ? 1 : 0);
    P->probe_end(DSMZ_KID_COEF, s);
    DSMZ_LAUNCHED("AGZO coefficients");
    P->probe_begin(DSMZ_KID_PERTURB, s);
    if (P->ptc) {
      const int32_t* tt = reinterpret_cast<const int32_t*>(P->dev_tables + P->off_ptiles);
      const int nt = P->ptiles.back();
      const int g = std::max(1, std::min(std::min(P->sm_count, P->nsegs), nt));
      if (bf) atc::k_perturb_tc<2><<<g, atc::kThreads, P->Lpt.total, s>>>(td, tt, nt, P->nsegs, P->Lpt, eps, kin,
                                                                          P->gpeers, err);
      else atc::k_perturb_tc<4><<<g, atc::kThreads, P->Lpt.total, s>>>(td, tt, nt, P->nsegs, P->Lpt, eps, kin,
                                                                       P->gpeers, err);
    } else {
      if (bf) sk::k_sperturb<2><<<P->grid_m, sk::kSTP, P->Lp.total, s>>>(td, P->Lp, seed, off, eps, kin, P->gpeers, err);
      else sk::k_sperturb<4><<<P->grid_m, sk::kSTP, P->Lp.total, s>>>(td, P->Lp, seed, off, eps, kin, P->gpeers, err);
    }
    P->probe_end(DSMZ_KID_PERTURB, s);
    DSMZ_LAUNCHED("perturbation");
    P->probe_begin(DSMZ_KID_KALMAN_SUM, s);
    k_kalman_reduce<<<1, kThreads, 0, s>>>(td);
    P->probe_end(DSMZ_KID_KALMAN_SUM, s);
    DSMZ_LAUNCHED("Kalman sums");
  }
  return 0;
}

int run_update(const dsmz_plan* P, KalmanIn kin, float eta, const NSArgs& ns, cudaStream_t s) {
  if (P->mats.empty()) return 0;
  const Tables tb = P->tables();
  const int r = P->r;
  const int nm = static_cast<int>(P->mats.size());
  int rc;
  int* err = reinterpret_cast<int*>(P->workspace + P->err_off);
  const bool small = sk::gram_maxb(r) <= 5;
  if ((rc = set_smem(sk::k_sgram<1, 5>, P->Lg.total))) return rc;
  if ((rc = set_smem(sk::k_sgram<1, 17>, P->Lg.total))) return rc;
  if ((rc = set_smem(sk::k_sapply<2>, P->La.total))) return rc;
  if ((rc = set_smem(sk::k_sapply<4>, P->La.total))) return rc;
  P->probe_begin(DSMZ_KID_GRAM, s);
  if (small) sk::k_sgram<1, 5><<<P->grid_m, sk::kSTG, P->Lg.total, s>>>(tb, tb.mats, nm, P->nsegs, P->Lg, kin, err);
  else sk::k_sgram<1, 17><<<P->grid_m, sk::kSTG, P->Lg.total, s>>>(tb, tb.mats, nm, P->nsegs, P->Lg, kin, err);
  P->probe_end(DSMZ_KID_GRAM, s);
  DSMZ_LAUNCHED("Kalman Gram");
  P->probe_begin(DSMZ_KID_NS_SOLVE, s);
  if ((rc = launch_ns_solve(tb, tb.mats, nm, r, ns, s))) return rc;
  P->probe_end(DSMZ_KID_NS_SOLVE, s);
  DSMZ_LAUNCHED("Newton-Schulz solve");
  P->probe_begin(DSMZ_KID_APPLY, s);
  if (P->copy_dtype == DSMZ_BF16)
    sk::k_sapply<2><<<P->grid_m, sk::kSTP, P->La.total, s>>>(tb, tb.mats, nm, P->nsegs, P->La, eta, P->speers, err);
  else
    sk::k_sapply<4><<<P->grid_m, sk::kSTP, P->La.total, s>>>(tb, tb.mats, nm, P->nsegs, P->La, eta, P->speers, err);
  P->probe_end(DSMZ_KID_APPLY, s);
  DSMZ_LAUNCHED("Kalman + ZO-Muon apply");
  return 0;
}

}  // namespace

// Context lookups of the allocation-free ZO-Muon entry (its scratch array is defined with it).
namespace {
struct NoallocSlot {
  unsigned long long ctx_id = 0;   // 0: no lookup yet
  void* addr = nullptr;
};
std::mutex g_noalloc_mutex;
NoallocSlot g_noalloc_slot[256];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique ID (never reused in the process) of the calling thread's current context, or 0
// when there is none yet or the driver cannot say.
unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_cur || !get_id) return 0;
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}
}  // namespace

// ====================================================================== C ABI
extern "C" {

const char* dsmz_last_error(void) { return g_err.c_str(); }
int dsmz_abi_version(void) { return DSMZ_ABI_VERSION; }

int dsmz_ns_schedule_cubic(dsmz_ns_schedule* out) {
  if (!out) return fail(DSMZ_ERR_INVALID, "dsmz_ns_schedule_cubic: null output");
  std::memset(out, 0, sizeof(*out));
  const double eps = static_cast<double>(1.1920928955078125e-07f);  // FLT_EPSILON
  double lo = std::sqrt(eps), up = 1.0;
  int n = 0;
  while (1.0 - lo >= eps && n < DSMZ_MAX_NS_ITERS) {
    const double s = up * up + lo * up + lo * lo;
    const double alpha = std::sqrt(3.0 / s);
    const double alpha3 = alpha * alpha * alpha;
    const double beta = 4.0 / (2.0 + lo * up * (lo + up) * alpha3);
    const double c1 = 1.5 * beta * alpha;
    const double c3 = -0.5 * beta * alpha3;
    out->c[n][0] = c1;
    out->c[n][1] = c3;
    out->c[n][2] = 0.0;
    ++n;
    lo = c1 * lo + c3 * lo * lo * lo;
    up = 2.0 - lo;
  }
  out->iters = n;
  return DSMZ_OK;
}

int dsmz_ns_schedule_quintic(dsmz_ns_schedule* out) {
  if (!out) return fail(DSMZ_ERR_INVALID, "dsmz_ns_schedule_quintic: null output");
  std::memset(out, 0, sizeof(*out));
  out->iters = 5;
  for (int i = 0; i < 5; ++i) {
    out->c[i][0] = 3.4445;
    out->c[i][1] = -4.7750;
    out->c[i][2] = 2.0315;
  }
  return DSMZ_OK;
}

int64_t dsmz_randn_threads(int64_t n, int32_t sm_count, int32_t max_threads_per_sm) {
  if (n <= 0) return 0;
  const int64_t blocks = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count) * (max_threads_per_sm / 256);
  return 256 * (blocks < cap ? blocks : cap);
}

uint64_t dsmz_randn_offset_increment(int64_t n, int32_t sm_count, int32_t max_threads_per_sm) {
  if (n <= 0) return 0;
  const int64_t thr = dsmz_randn_threads(n, sm_count, max_threads_per_sm);
  return static_cast<uint64_t>(((n - 1) / (thr * 4) + 1) * 4);
}

int dsmz_randn(float* out, int64_t n, uint64_t seed, uint64_t offset, int32_t sm_count, int32_t max_threads_per_sm,
               dsmz_stream_t stream) {
  if (n <= 0) return DSMZ_OK;
  if (!out || sm_count <= 0 || max_threads_per_sm < 256) return fail(DSMZ_ERR_INVALID, "dsmz_randn: bad arguments");
  const int64_t thr = dsmz_randn_threads(n, sm_count, max_threads_per_sm);
  int64_t blocks = (n + kThreads - 1) / kThreads;
  if (blocks > 65535) blocks = 65535;
  k_randn<<<static_cast<int>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, offset, thr);
  DSMZ_LAUNCHED("dsmz_randn");
  return DSMZ_OK;
}

// ------------------------------------------------------------ activation handoff
int dsmz_activation_load(int32_t dst_dtype, void* dst, int64_t T, int64_t D, int64_t ld_dst, int32_t src_dtype,
                         const void* src, int64_t n, int64_t src_s0, int64_t src_s1, dsmz_stream_t stream) {
  if (!dst || (n > 0 && !src)) return fail(DSMZ_ERR_INVALID, "dsmz_activation_load: null pointer");
  if ((dst_dtype != DSMZ_F32 && dst_dtype != DSMZ_BF16) || (src_dtype != DSMZ_F32 && src_dtype != DSMZ_BF16))
    return fail(DSMZ_ERR_INVALID, "dsmz_activation_load: dtypes must be DSMZ_F32 or DSMZ_BF16");
  if (T <= 0 || D <= 0 || ld_dst < D || n < 0 || n > T || src_s0 < 0 || src_s1 < 0)
    return fail(DSMZ_ERR_INVALID,
                "dsmz_activation_load: need T > 0, D > 0, ld_dst >= D, 0 <= n <= T and non-negative strides");
  const int ses = src_dtype == DSMZ_F32 ? 4 : 2, des = dst_dtype == DSMZ_F32 ? 4 : 2;
  const bool vec = D % 8 == 0 && (n == 0 || src_s1 == 1) && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                   (src_s0 * ses) % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0 && (ld_dst * des) % 16 == 0;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail("dsmz_activation_load: device query", e);
  const int64_t work = vec ? T * (D / 8) : T * D;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sms) * 8;      // grid-stride beyond eight CTAs per SM
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = static_cast<int>(blocks), v = vec ? 1 : 0;
  if (src_dtype == DSMZ_F32 && dst_dtype == DSMZ_BF16) k_act_load<0, 1><<<g, 256, 0, s>>>(dst, T, D, ld_dst, src, n, src_s0, src_s1, v);
  else if (src_dtype == DSMZ_BF16 && dst_dtype == DSMZ_BF16) k_act_load<1, 1><<<g, 256, 0, s>>>(dst, T, D, ld_dst, src, n, src_s0, src_s1, v);
  else if (src_dtype == DSMZ_F32) k_act_load<0, 0><<<g, 256, 0, s>>>(dst, T, D, ld_dst, src, n, src_s0, src_s1, v);
  else k_act_load<1, 0><<<g, 256, 0, s>>>(dst, T, D, ld_dst, src, n, src_s0, src_s1, v);
  DSMZ_LAUNCHED("dsmz_activation_load");
  return DSMZ_OK;
}

// ------------------------------------------------------------ contrastive scoring loss
size_t dsmz_contrastive_loss_workspace_bytes(int64_t ntok) {
  return ntok > 0 ? static_cast<size_t>(ntok) * sizeof(double) + 256 : 256;
}

int dsmz_contrastive_loss(int32_t kind, const void* src, int64_t V, int64_t ld, const int32_t* targets, int64_t ntok,
                          const int64_t* seq_start, const double* advantages, int32_t nseq, double* out,
                          void* workspace, size_t workspace_bytes, dsmz_stream_t stream) {
  if (!src || !out || !workspace || (kind != DSMZ_SCORE_LOGPROBS_F32 && !targets))
    return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: null pointer");
  if (kind != DSMZ_SCORE_LOGITS_F32 && kind != DSMZ_SCORE_LOGITS_BF16 && kind != DSMZ_SCORE_LOGPROBS_F32)
    return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: kind must be a DSMZ_SCORE_* value");
  if (nseq < 1 || nseq > kMaxScoreSeqs || !seq_start || !advantages)
    return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: 1 <= nseq <= " + std::to_string(kMaxScoreSeqs) +
                                      " with host arrays seq_start[nseq + 1] and advantages[nseq]");
  if (kind != DSMZ_SCORE_LOGPROBS_F32 && (V < 1 || ld < V))
    return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: need V >= 1 and ld >= V");
  if (seq_start[0] != 0 || seq_start[nseq] != ntok || ntok < 1)
    return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: seq_start must run from 0 to ntok >= 1");
  ScoreSeqs q{};
  q.n = nseq;
  for (int i = 0; i < nseq; ++i) {
    const int64_t len = seq_start[i + 1] - seq_start[i];
    // the reference's mean over a sequence (ds_mezo/controller.py:14-15) has no empty case
    if (len < 1) return fail(DSMZ_ERR_INVALID, "dsmz_contrastive_loss: every sequence needs a scored token");
    q.start[i] = seq_start[i];
    q.w[i] = advantages[i] / static_cast<double>(len);
  }
  q.start[nseq] = ntok;
  if (workspace_bytes < dsmz_contrastive_loss_workspace_bytes(ntok) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(DSMZ_ERR_WORKSPACE, "dsmz_contrastive_loss: workspace too small or not 16-byte aligned");
  double* term = static_cast<double*>(workspace);
  int* err = reinterpret_cast<int*>(static_cast<char*>(workspace) + static_cast<size_t>(ntok) * sizeof(double));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail("dsmz_contrastive_loss: error word", e);
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail("dsmz_contrastive_loss: device query", e);
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  const int g = static_cast<int>(ntok < cap ? ntok : cap);
  const int es = kind == DSMZ_SCORE_LOGITS_BF16 ? 2 : 4;
  const int per = 16 / es;                              // elements per 16-byte load
  const int vec = (V % per == 0 && (ld * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) ? 1 : 0;
  if (kind == DSMZ_SCORE_LOGITS_F32) k_token_nll<0><<<g, 256, 0, s>>>(src, ld, V, targets, ntok, q, vec, term, err);
  else if (kind == DSMZ_SCORE_LOGITS_BF16) k_token_nll<1><<<g, 256, 0, s>>>(src, ld, V, targets, ntok, q, vec, term, err);
  else k_token_nll<2><<<g, 256, 0, s>>>(src, ld, V, targets, ntok, q, vec, term, err);
  DSMZ_LAUNCHED("dsmz_contrastive_loss: token terms");
  k_seq_sum<<<1, 256, 0, s>>>(term, ntok, err, out);
  DSMZ_LAUNCHED("dsmz_contrastive_loss: sum");
  return DSMZ_OK;
}

// ---------------------------------------------------------------------- plan
int dsmz_plan_create(const dsmz_plan_desc* d, dsmz_plan** out) {
  if (!d || !out) return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: null argument");
  *out = nullptr;
  if (d->copy_dtype != DSMZ_F32 && d->copy_dtype != DSMZ_BF16)
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: copy_dtype must be DSMZ_F32 or DSMZ_BF16");
  if (d->num_modules < 0 || d->num_bases < 0 || (d->num_modules > 0 && !d->modules) ||
      (d->num_bases > 0 && !d->bases))
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: bad module/basis arrays");
  if (d->sm_count <= 0 || d->max_threads_per_sm < 256)
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: sm_count / max_threads_per_sm describe the device");
  if (d->directions < 0 || d->directions > DSMZ_MAX_DIRECTIONS)
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: directions must be in [0, DSMZ_MAX_DIRECTIONS]");
  if (d->directions > 1 && (d->dir_stride_factor <= 0 || d->dir_stride_z <= 0))
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: several directions need positive direction strides");
  auto* P = new dsmz_plan();
  P->copy_dtype = d->copy_dtype;
  P->sm_count = d->sm_count;
  P->ndir = d->directions > 1 ? d->directions : 1;
  P->dstride_f = P->ndir > 1 ? d->dir_stride_factor : 0;
  P->dstride_z = P->ndir > 1 ? d->dir_stride_z : 0;
  P->err_off = P->ws.take(256);      // device error word of the bounded waits
  // bases
  for (int i = 0; i < d->num_bases; ++i) {
    const dsmz_basis_spec& b = d->bases[i];
    if (!b.H || !b.V || b.T <= 0 || b.D <= 0 || b.R <= 0 || b.R > DSMZ_MAX_RANK || b.ld_H < b.D ||
        (b.h_dtype != DSMZ_F32 && b.h_dtype != DSMZ_BF16)) {
      delete P;
      return fail(DSMZ_ERR_INVALID, "dsmz_plan_create: basis " + std::to_string(i) + " is invalid");
    }
    if (i > 0 && b.R != P->R) {
      delete P;
      return fail(DSMZ_ERR_UNSUPPORTED, "dsmz_plan_create: all bases must share one width R");
    }
    P->R = static_cast<int>(b.R);
    BasisD bd{};
    bd.H = b.H; bd.hdt = b.h_dtype; bd.R = static_cast<int32_t>(b.R);
    bd.T = b.T; bd.D = b.D; bd.h_s0 = b.ld_H; bd.h_s1 = 1;
    bd.Vin = b.V; bd.v_s0 = b.R; bd.v_s1 = 1; bd.Vout = b.V;
    bd.y_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(b.T) * b.R * sizeof(float)) / sizeof(float));
    bd.w_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(b.D) * b.R * sizeof(float)) / sizeof(float));
    fill_basis_tiles(bd, P->nytiles, P->nwtiles);
    P->bases.push_back(bd);
  }
  plan_calibration(P, d->sm_count, d->max_threads_per_sm);
  if (!P->bases.empty() && !(d->flags & DSMZ_PLAN_SIMT_POWER_ITER)) {
    bool ok = true;
    for (int i = 0; i < d->num_bases; ++i) {
      const dsmz_basis_spec& b = d->bases[i];
      ok = ok && tc_shape_ok(b.h_dtype, b.D, b.ld_H, 1, b.R, b.H);
    }
    if (ok) {
      P->tc = true;
      plan_tc_layout(P);
      if (P->R <= 64 && pf_stages(P->R) >= 4 && (d->flags & DSMZ_PLAN_SINGLE_PASS_POWER_ITER)) plan_pi_fused(P);
    }
  }
  plan_ysplit(P);
  add_w_tables(P);
  // modules
  uint64_t off = d->rng_offset_before;   // draws are placed relative to the step's base offset
  uint64_t own = 0;                      // this plan's one-direction generator advance
  for (int i = 0; i < d->num_modules; ++i) {
    const dsmz_module_spec& m = d->modules[i];
    const std::string who = "dsmz_plan_create: module " + std::to_string(i);
    if (!m.A || !m.B || !m.pos_A || !m.pos_B || !m.neg_A || !m.neg_B || !m.mu_A || !m.mu_B || !m.var_A ||
        !m.var_B || !m.z_A || !m.z_B) {
      delete P;
      return fail(DSMZ_ERR_INVALID, who + " has a null tensor pointer");
    }
    if (m.r <= 0 || m.r > DSMZ_MAX_RANK || m.d_out <= 0 || m.d_in <= 0 || m.ld_A < m.r || m.ld_B < m.d_in) {
      delete P;
      return fail(DSMZ_ERR_INVALID, who + " has an invalid shape or stride");
    }
    if (m.ld_B * m.r > INT32_MAX || m.ld_A * 4096 > INT32_MAX) {   // 32-bit offsets within a streamed tile
      delete P;
      return fail(DSMZ_ERR_UNSUPPORTED, who + ": leading dimension too large");
    }
    if (m.basis < 0 || m.basis >= d->num_bases || d->bases[m.basis].D != m.d_in) {
      delete P;
      return fail(DSMZ_ERR_INVALID, who + ": basis index out of range or basis D != d_in");
    }
    if (i > 0 && m.r != P->r) {
      delete P;
      return fail(DSMZ_ERR_UNSUPPORTED, "dsmz_plan_create: all modules must share one adapter rank r");
    }
    P->r = static_cast<int>(m.r);
    const int RC = static_cast<int>(d->bases[m.basis].R);
    P->RC = RC;
    ModD md{};
    md.r = static_cast<int32_t>(m.r); md.rc = RC; md.rca = md.r < RC ? md.r : RC;
    md.d_out = m.d_out; md.d_in = m.d_in; md.basis = m.basis;
    const int64_t nB = static_cast<int64_t>(md.r) * RC, nA = m.d_out * md.rca;
    md.thrB = dsmz_randn_threads(nB, d->sm_count, d->max_threads_per_sm);
    md.thrA = dsmz_randn_threads(nA, d->sm_count, d->max_threads_per_sm);
    const uint64_t incB = dsmz_randn_offset_increment(nB, d->sm_count, d->max_threads_per_sm);
    const uint64_t incA = dsmz_randn_offset_increment(nA, d->sm_count, d->max_threads_per_sm);
    if (d->module_rng_offsets) off = d->module_rng_offsets[i];   // the module's place in the whole model's draws
    md.offB = off;
    off += incB;
    md.offA = off;
    off += incA;
    own += incB + incA;
    md.coef_off = static_cast<int64_t>(P->ws.take((nB + static_cast<size_t>(md.r) * md.rca) * sizeof(float)) / sizeof(float));
    md.qrw_off = coef_qr_in_smem(md.r, md.rca) ? 0 : static_cast<int64_t>(
        P->ws.take(2 * static_cast<size_t>(md.rca) * md.rca * sizeof(double)) / sizeof(double));
    md.Bp = m.B; md.varB = m.var_B; md.b_s0 = m.ld_B; md.b_s1 = 1;
    md.zca_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(nA) * sizeof(float)) / sizeof(float));
    md.dblk0 = P->ndblk;
    md.ndblk = static_cast<int32_t>(md.thrA / 256);
    P->ndblk += md.ndblk;
    md.a = static_cast<int32_t>(P->mats.size());
    md.b = md.a + 1;
    MatD a{};
    a.param = m.A; a.pos = m.pos_A; a.neg = m.neg_A; a.mu = m.mu_A; a.var = m.var_A; a.z = m.z_A;
    a.shadow = m.shadow_A;
    a.scratch = m.scratch_A; a.nvec = m.d_out; a.r = m.r; a.ld = m.ld_A; a.cs = 1; a.side = 0; a.owner = i;
    add_matrix(P->mats, P->ws, a, P->nsegs, false);
    MatD b{};
    b.param = m.B; b.pos = m.pos_B; b.neg = m.neg_B; b.mu = m.mu_B; b.var = m.var_B; b.z = m.z_B;
    b.shadow = m.shadow_B;
    b.scratch = m.scratch_B; b.nvec = m.d_in; b.r = m.r; b.ld = m.ld_B; b.cs = 1; b.side = 1; b.owner = i;
    add_matrix(P->mats, P->ws, b, P->nsegs, false);
    P->mods.push_back(md);
  }
  // B-side sums: two CTAs per SM over the modules' concatenated d_in columns
  plan_bside(P->mods, 2 * P->sm_count, P->ws, &P->nchunks, &P->bside_cols);
  P->rng_inc1 = own;
  P->rng_dir_stride = d->rng_direction_stride ? d->rng_direction_stride : P->rng_inc1;
  P->rng_increment = P->rng_inc1 * static_cast<uint64_t>(P->ndir);
  // streaming layouts, then the tile chunks they imply, then the per-segment buffers
  P->ptc = (d->flags & DSMZ_PLAN_CUDA_CORE_PERTURB) == 0;
  if (P->r > 0 && !choose_adapter_layouts(P)) {
    delete P;
    return fail(DSMZ_ERR_UNSUPPORTED, "dsmz_plan_create: rank too large for the streaming kernels' shared memory");
  }
  if (P->R > 0 && !choose_qr_layout(P)) {
    delete P;
    return fail(DSMZ_ERR_UNSUPPORTED, "dsmz_plan_create: basis width too large for the streaming kernels");
  }
  if (!P->mats.empty()) P->nsegs = chunk_matrices(P->mats, P->Lg.TV, P->sm_count, &P->ws, &P->grid_m);
  chunk_w_tables(P, true);
  for (MatD& m : P->mats) {           // tile-box tensor maps, encoded at bind
    if (m.side != 1) continue;
    m.tmap = static_cast<int32_t>(P->smaps.size());
    P->smaps.resize(P->smaps.size() + 4);
  }
  for (MatD& m : P->mats) {           // swizzled row boxes: K operand, side-0 own rows
    m.kmap = static_cast<int32_t>(P->smaps.size());
    P->smaps.resize(P->smaps.size() + 1);
    if (m.side != 0) continue;
    m.rmap = static_cast<int32_t>(P->smaps.size());
    P->smaps.resize(P->smaps.size() + 1);
  }
  for (MatD& m : P->w2) {             // W rows of the QR apply
    m.rmap = static_cast<int32_t>(P->smaps.size());
    P->smaps.resize(P->smaps.size() + 1);
  }
  P->seg_kal_off = static_cast<int64_t>(P->ws.take(static_cast<size_t>(P->nsegs > 0 ? P->nsegs : 1) * 2 * sizeof(double)) / sizeof(double));
  P->kal_sum_off = static_cast<int64_t>(P->ws.take(2 * static_cast<size_t>(P->ndir) * sizeof(double)) / sizeof(double));
  P->norm_off = P->ws.take((P->mats.empty() ? 1 : P->mats.size()) * kNormSlices * sizeof(double));
  P->pack();
  *out = P;
  return DSMZ_OK;
}

void dsmz_plan_destroy(dsmz_plan* plan) { delete plan; }
size_t dsmz_plan_table_bytes(const dsmz_plan* p) { return p ? p->table_bytes : 0; }
size_t dsmz_plan_workspace_bytes(const dsmz_plan* p) { return p ? (p->ws.bytes < 256 ? 256 : p->ws.bytes) : 0; }
uint64_t dsmz_plan_rng_increment(const dsmz_plan* p) { return p ? p->rng_increment : 0; }

int32_t dsmz_plan_launch_count(const dsmz_plan* p, int32_t num_iters) {
  if (!p) return 0;
  int32_t n = 0;
  // per iteration: Y, W (one fused launch on the single-pass path), Gram of W, Cholesky, V;
  // plus the first bf16 split of the caller's basis on the tensor-core path
  if (!p->bases.empty() && num_iters > 0)
    n += num_iters * ((p->fused ? 4 : 5) + (p->ysplit > 1 ? 1 : 0)) + (p->tc ? 1 : 0);
  if (!p->mods.empty()) n += 1 + 4 * p->ndir + (p->ndir > 1 ? 4 : 3);   // B-side, per direction 4, update
  return n;
}

int dsmz_plan_bind(dsmz_plan* P, void* device_tables, size_t table_bytes, void* workspace, size_t workspace_bytes,
                   dsmz_stream_t stream) {
  if (!P || !device_tables || !workspace) return fail(DSMZ_ERR_INVALID, "dsmz_plan_bind: null argument");
  if (table_bytes < P->table_bytes) return fail(DSMZ_ERR_WORKSPACE, "dsmz_plan_bind: table buffer too small");
  if (workspace_bytes < dsmz_plan_workspace_bytes(P))
    return fail(DSMZ_ERR_WORKSPACE, "dsmz_plan_bind: workspace too small (need " +
                                        std::to_string(dsmz_plan_workspace_bytes(P)) + " bytes)");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0 || (reinterpret_cast<uintptr_t>(device_tables) & 63) != 0)
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_bind: workspace must be 256-byte and tables 64-byte aligned");
  P->dev_tables = static_cast<char*>(device_tables);
  P->workspace = static_cast<char*>(workspace);
  P->split_current = false;
  patch_ws_pointers(P);
  if (P->tc && !bind_tc(P)) { P->tc = false; P->fused = false; }   // keep the CUDA-core power iteration
  bind_side1_maps(P);
  bind_swz_maps(P);
  {
    cudaError_t ez = cudaMemsetAsync(P->workspace + P->err_off, 0, sizeof(int), static_cast<cudaStream_t>(stream));
    if (ez != cudaSuccess) return cuda_fail("dsmz_plan_bind: error word", ez);
  }
  P->write_blob();
  cudaError_t e = cudaMemcpyAsync(device_tables, P->blob.data(), P->table_bytes, cudaMemcpyHostToDevice,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("dsmz_plan_bind: table upload", e);
  return DSMZ_OK;
}

int32_t dsmz_plan_perturb_on_tensor_cores(const dsmz_plan* P) { return (P && P->ptc) ? 1 : 0; }

int32_t dsmz_plan_uses_tensor_cores(const dsmz_plan* P) { return (P && P->tc) ? (P->fused ? 2 : 1) : 0; }

int32_t dsmz_plan_device_error(const dsmz_plan* P, dsmz_stream_t stream) {
  if (!P || !P->workspace) return 0;
  int v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&v, P->workspace + P->err_off, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(s) != cudaSuccess) return -1;
  if (v) cudaMemsetAsync(P->workspace + P->err_off, 0, sizeof(int), s);
  return v;
}

static int plan_ready(const dsmz_plan* P, const char* who) {
  if (!P) return fail(DSMZ_ERR_INVALID, std::string(who) + ": null plan");
  if (!P->dev_tables || !P->workspace) return fail(DSMZ_ERR_INVALID, std::string(who) + ": plan is not bound");
  return DSMZ_OK;
}

int dsmz_step_power_iteration(const dsmz_plan* P, int32_t num_iters, float norm_floor, dsmz_stream_t stream) {
  return dsmz_step_power_iteration_ex(P, num_iters, norm_floor, 0u, stream);
}

int dsmz_step_power_iteration_ex(const dsmz_plan* P, int32_t num_iters, float norm_floor, uint32_t flags,
                                 dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_step_power_iteration");
  if (rc) return rc;
  return run_power_iteration(P, num_iters, norm_floor, static_cast<cudaStream_t>(stream), flags);
}

int dsmz_step_perturb(const dsmz_plan* P, uint64_t seed, uint64_t offset, float eps, float beta, float q,
                      float norm_floor, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_step_perturb");
  if (rc) return rc;
  return run_perturb(P, seed, offset, eps, make_kin(beta, q, 0.f, norm_floor), norm_floor,
                     static_cast<cudaStream_t>(stream));
}

int dsmz_plan_set_gather_peers(dsmz_plan* P, int32_t npeers, const int64_t* pos_delta, const int64_t* neg_delta,
                               const int64_t* shadow_delta) {
  if (!P) return fail(DSMZ_ERR_INVALID, "dsmz_plan_set_gather_peers: null plan");
  if (npeers < 0 || npeers > kMaxPeers || (npeers > 0 && (!pos_delta || !neg_delta)))
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_set_gather_peers: 0 to " + std::to_string(kMaxPeers) + " peers");
  if (npeers > 0 && shadow_delta && P->copy_dtype == DSMZ_F32)
    return fail(DSMZ_ERR_UNSUPPORTED, "dsmz_plan_set_gather_peers: fp32 copies have no factor shadow");
  for (int i = 0; i < npeers; ++i)
    if ((pos_delta[i] % 16) != 0 || (neg_delta[i] % 16) != 0 || (shadow_delta && (shadow_delta[i] % 16) != 0))
      return fail(DSMZ_ERR_INVALID, "dsmz_plan_set_gather_peers: distances must be multiples of 16 bytes");
  P->gpeers = GatherPeers{};
  P->speers = GatherPeers{};
  P->gpeers.n = npeers;
  for (int i = 0; i < npeers; ++i) { P->gpeers.dpos[i] = pos_delta[i]; P->gpeers.dneg[i] = neg_delta[i]; }
  if (shadow_delta) {
    P->speers.n = npeers;
    for (int i = 0; i < npeers; ++i) P->speers.dpos[i] = shadow_delta[i];
  }
  return DSMZ_OK;
}

// CUDA IPC of a device buffer: the handle of the allocation that holds `ptr`, and ptr's
// offset in it; a peer process opens the handle and adds the offset.
int dsmz_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail(DSMZ_ERR_INVALID, "dsmz_ipc_export: null argument");
  CUdeviceptr base = 0;
  size_t size = 0;
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
      return fail(DSMZ_ERR_CUDA, "dsmz_ipc_export: cuMemGetAddressRange unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(DSMZ_ERR_CUDA, "dsmz_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail("dsmz_ipc_export", e);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return DSMZ_OK;
}

int dsmz_ipc_import(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return fail(DSMZ_ERR_INVALID, "dsmz_ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail("dsmz_ipc_import", e);
  *ptr = static_cast<char*>(base) + offset;
  return DSMZ_OK;
}

int dsmz_ipc_close(void* ptr, int64_t offset) {
  if (!ptr) return DSMZ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  return e == cudaSuccess ? DSMZ_OK : cuda_fail("dsmz_ipc_close", e);
}

// One device-to-device copy on `stream` (a copy engine moves it; between this GPU's memory
// and a peer's mapped buffer it crosses NVLink without taking an SM).
int dsmz_peer_copy(void* dst, const void* src, int64_t bytes, dsmz_stream_t stream) {
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(DSMZ_ERR_INVALID, "dsmz_peer_copy: bad argument");
  if (bytes == 0) return DSMZ_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice,
                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? DSMZ_OK : cuda_fail("dsmz_peer_copy", e);
}

int dsmz_step_draw(const dsmz_plan* P, uint64_t seed, uint64_t offset, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_step_draw");
  if (rc) return rc;
  if (P->mods.empty()) return DSMZ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Tables tb = P->tables();
  P->probe_begin(DSMZ_KID_DRAW, s);
  sk::k_draw_zca<<<std::min(P->ndblk, 16 * P->sm_count), 256, 0, s>>>(tb, seed, offset);
  P->probe_end(DSMZ_KID_DRAW, s);
  DSMZ_LAUNCHED("Zc_A draws");
  P->pre_drawn = true;
  P->pre_seed = seed;
  P->pre_off = offset;
  return DSMZ_OK;
}

double* dsmz_step_kalman_sums(const dsmz_plan* P) {
  if (!P || !P->workspace) return nullptr;
  return reinterpret_cast<double*>(P->workspace) + P->kal_sum_off;
}

int32_t dsmz_plan_directions(const dsmz_plan* P) { return P ? P->ndir : 0; }

size_t dsmz_plan_calibration_workspace_bytes(const dsmz_plan* P) { return P ? P->calib_ws_bytes : 0; }

int32_t dsmz_plan_calibration_launch_count(const dsmz_plan* P, int32_t niter) {
  if (!P || P->bases.empty() || niter < 0) return 0;
  // sketches 2, Y products niter + 2 (niter 0: 2), W tails niter + 1 of four launches,
  // Grams of Y 2, eigen-solves 2, rotation 1, the first bf16 split on the tensor-core path
  const int ny = niter >= 1 ? niter + 2 : 2;
  return 2 + ny * (1 + (P->ysplit > 1 ? 1 : 0)) + 4 * (niter + 1) + 5 + (P->tc ? 1 : 0);
}
uint64_t dsmz_plan_calibration_rng_increment(const dsmz_plan* P) { return P ? P->calib_inc : 0; }

int dsmz_plan_calibrate(const dsmz_plan* P, uint64_t seed, uint64_t offset, int32_t niter, float norm_floor,
                        void* workspace, size_t workspace_bytes, float* singular_values, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_plan_calibrate");
  if (rc) return rc;
  if (niter < 0) return fail(DSMZ_ERR_INVALID, "dsmz_plan_calibrate: niter must be >= 0");
  if (!workspace || workspace_bytes < P->calib_ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(DSMZ_ERR_WORKSPACE, "dsmz_plan_calibrate: workspace must be 256-byte aligned and hold " +
                                        std::to_string(P->calib_ws_bytes) + " bytes");
  for (const BasisD& b : P->bases)
    if (b.R > b.T || b.R > b.D)
      return fail(DSMZ_ERR_INVALID, "dsmz_plan_calibrate: the basis width exceeds min(T, D) of a basis");
  return run_calibration(P, seed, offset, niter, norm_floor, static_cast<char*>(workspace), singular_values,
                         static_cast<cudaStream_t>(stream));
}

int dsmz_plan_factor_norms(const dsmz_plan* P, float* norms, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_plan_factor_norms");
  if (rc) return rc;
  if (!norms) return fail(DSMZ_ERR_INVALID, "dsmz_plan_factor_norms: null output");
  if (P->mats.empty()) return DSMZ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nm = static_cast<int>(P->mats.size());
  double* part = reinterpret_cast<double*>(P->workspace + P->norm_off);
  k_norm_partial<<<dim3(nm, kNormSlices), kThreads, 0, s>>>(P->tables(), part);
  DSMZ_LAUNCHED("factor norms");
  k_norm_finish<<<(nm + kThreads - 1) / kThreads, kThreads, 0, s>>>(part, nm, norms);
  DSMZ_LAUNCHED("factor norms (sum)");
  return DSMZ_OK;
}

int dsmz_step_update_directions(const dsmz_plan* P, const float* dd, int32_t n, float beta, float q, float eta,
                                float norm_floor, const dsmz_ns_schedule* schedule, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_step_update_directions");
  if (rc) return rc;
  if (!dd || n != P->ndir) return fail(DSMZ_ERR_INVALID, "dsmz_step_update_directions: need one dd per direction");
  if (schedule && (schedule->iters < 0 || schedule->iters > DSMZ_MAX_NS_ITERS))
    return fail(DSMZ_ERR_INVALID, "dsmz_step_update_directions: schedule iters out of range");
  if (n == 1) return dsmz_step_update(P, dd[0], beta, q, eta, norm_floor, schedule, stream);
  sk::KalmanDirs kd{};
  kd.beta = beta;
  kd.beta2 = static_cast<float>(static_cast<double>(beta) * static_cast<double>(beta));
  kd.q = q;
  kd.floor_ = norm_floor;
  kd.n = n;
  for (int k = 0; k < n; ++k) kd.dd[k] = dd[k];
  return run_update_dirs(P, kd, eta, make_ns(schedule, norm_floor), static_cast<cudaStream_t>(stream));
}

int dsmz_step_update(const dsmz_plan* P, float dd, float beta, float q, float eta, float norm_floor,
                     const dsmz_ns_schedule* schedule, dsmz_stream_t stream) {
  int rc = plan_ready(P, "dsmz_step_update");
  if (rc) return rc;
  if (P->ndir != 1) return fail(DSMZ_ERR_INVALID, "dsmz_step_update: the plan has several directions");
  if (schedule && (schedule->iters < 0 || schedule->iters > DSMZ_MAX_NS_ITERS))
    return fail(DSMZ_ERR_INVALID, "dsmz_step_update: schedule iters out of range");
  return run_update(P, make_kin(beta, q, dd, norm_floor), eta, make_ns(schedule, norm_floor),
                    static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------- per-op drop-ins
// Each builds a one-matrix (or one-basis, one-module) plan whose tables live at the head
// of the caller's workspace, written by a kernel that takes them by value.
static size_t table_head_bytes() { return 4096; }

static int upload_small(dsmz_plan* P, char* ws, cudaStream_t s) {
  P->dev_tables = ws;
  if (P->table_bytes > table_head_bytes()) return fail(DSMZ_ERR_INVALID, "internal: table head overflow");
  auto put_mats = [&](const std::vector<MatD>& v, size_t off) {
    if (v.empty()) return;
    Pack<MatD, 2> pk{};
    for (size_t i = 0; i < v.size() && i < 2; ++i) pk.v[i] = v[i];
    k_write_pack<MatD, 2><<<1, 32, 0, s>>>(pk, reinterpret_cast<MatD*>(ws + off), static_cast<int>(v.size()));
  };
  put_mats(P->mats, P->off_mats);
  put_mats(P->w1, P->off_w1);
  put_mats(P->w2, P->off_w2);
  if (!P->mods.empty()) {
    Pack<ModD, 1> pk{};
    pk.v[0] = P->mods[0];
    k_write_pack<ModD, 1><<<1, 32, 0, s>>>(pk, reinterpret_cast<ModD*>(ws + P->off_mods), 1);
  }
  if (!P->bases.empty()) {
    Pack<BasisD, 1> pk{};
    pk.v[0] = P->bases[0];
    k_write_pack<BasisD, 1><<<1, 32, 0, s>>>(pk, reinterpret_cast<BasisD*>(ws + P->off_bases), 1);
  }
  if (P->tc && !P->tcb.empty()) {
    Pack<tc::TCBasis, 1> pk{};
    pk.v[0] = P->tcb[0];
    k_write_pack<tc::TCBasis, 1><<<1, 32, 0, s>>>(pk, reinterpret_cast<tc::TCBasis*>(ws + P->off_tcb), 1);
  }
  DSMZ_LAUNCHED("table upload");
  return 0;
}

static dsmz_plan muon_plan(int64_t M, int64_t N, Layout* L_out) {
  dsmz_plan P;
  P.ws.take(table_head_bytes());
  MatD m{};
  const bool tall = M >= N;
  m.nvec = tall ? M : N;
  m.r = tall ? N : M;
  m.side = tall ? 0 : 1;
  add_matrix(P.mats, P.ws, m, P.nsegs);
  P.r = static_cast<int>(m.r);
  P.pack();
  if (L_out) *L_out = P.ws;
  return P;
}

size_t dsmz_zo_muon_update_workspace_bytes(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  Layout L;
  muon_plan(M, N, &L);
  return L.bytes;
}

int dsmz_zo_muon_update(int32_t param_dtype, void* param, int64_t ps0, int64_t ps1, const float* buf, int64_t bs0,
                        int64_t bs1, float* scratch, int64_t ss0, int64_t ss1, int64_t M, int64_t N, float eta,
                        float norm_floor, const dsmz_ns_schedule* schedule, void* workspace, size_t workspace_bytes,
                        dsmz_stream_t stream) {
  if (M <= 0 || N <= 0) return DSMZ_OK;
  if (!param || !buf || !workspace) return fail(DSMZ_ERR_INVALID, "zo_muon_update: null pointer");
  if (param_dtype != DSMZ_F32 && param_dtype != DSMZ_BF16) return fail(DSMZ_ERR_INVALID, "zo_muon_update: bad dtype");
  if ((M < N ? M : N) > DSMZ_MAX_RANK)
    return fail(DSMZ_ERR_UNSUPPORTED, "zo_muon_update: min(M, N) must be <= " + std::to_string(DSMZ_MAX_RANK));
  if (bs0 != ps0 || bs1 != ps1 || (scratch && (ss0 != ps0 || ss1 != ps1)))
    return fail(DSMZ_ERR_INVALID,
                "zo_muon_update: buf and scratch must have param's strides (the reference indexes all three "
                "with param.stride())");
  if (schedule && (schedule->iters < 0 || schedule->iters > DSMZ_MAX_NS_ITERS))
    return fail(DSMZ_ERR_INVALID, "zo_muon_update: schedule iters out of range");
  Layout L;
  dsmz_plan P = muon_plan(M, N, &L);
  if (workspace_bytes < L.bytes) return fail(DSMZ_ERR_WORKSPACE, "zo_muon_update: workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(DSMZ_ERR_INVALID, "zo_muon_update: workspace must be 256-byte aligned");
  MatD& m = P.mats[0];
  m.param = param; m.mu = const_cast<float*>(buf); m.scratch = scratch;
  m.ld = ps0; m.cs = ps1;   // side B (wide) swaps roles inside vaddr2: element (k=row, v=col)
  P.workspace = static_cast<char*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = upload_small(&P, static_cast<char*>(workspace), s);
  if (rc) return rc;
  const Tables tb = P.tables();
  const int r = P.r;
  const size_t gs = gram_smem(r), as = apply_smem(r);
  const KalmanIn kin{};
  if (gram_rb(r) == 4) {
    if ((rc = set_smem(k_gram<0, 4, double>, gs))) return rc;
    k_gram<0, 4, double><<<P.nsegs, kThreads, gs, s>>>(tb, tb.mats, 1, kin);
  } else {
    if ((rc = set_smem(k_gram<0, 8, double>, gs))) return rc;
    k_gram<0, 8, double><<<P.nsegs, kThreads, gs, s>>>(tb, tb.mats, 1, kin);
  }
  DSMZ_LAUNCHED("zo_muon_update Gram");
  if ((rc = launch_ns_solve(tb, tb.mats, 1, r, make_ns(schedule, norm_floor), s))) return rc;
  DSMZ_LAUNCHED("zo_muon_update solve");
  if ((rc = set_smem(k_apply<0, 0>, as))) return rc;
  k_apply<0, 0><<<P.nsegs, kThreads, as, s>>>(tb, tb.mats, 1, kin, eta, param_dtype);
  DSMZ_LAUNCHED("zo_muon_update apply");
  return DSMZ_OK;
}

static dsmz_plan pi_plan(int64_t T, int64_t D, int64_t R, bool tc) {
  dsmz_plan P;
  P.ws.take(table_head_bytes());
  P.err_off = P.ws.take(256);
  P.R = static_cast<int>(R);
  choose_qr_layout(&P);
  BasisD bd{};
  bd.R = static_cast<int32_t>(R); bd.T = T; bd.D = D;
  bd.y_off = static_cast<int64_t>(P.ws.take(static_cast<size_t>(T) * R * sizeof(float)) / sizeof(float));
  bd.w_off = static_cast<int64_t>(P.ws.take(static_cast<size_t>(D) * R * sizeof(float)) / sizeof(float));
  fill_basis_tiles(bd, P.nytiles, P.nwtiles);
  P.bases.push_back(bd);
  P.R = static_cast<int>(R);
  if (tc) plan_tc_layout(&P);
  P.tc = tc;
  plan_ysplit(&P);
  add_w_tables(&P);
  reserve_w_gram(&P);
  P.pack();
  return P;
}

size_t dsmz_power_iter_workspace_bytes(int64_t T, int64_t D, int64_t R) {
  if (T <= 0 || D <= 0 || R <= 0) return 0;
  const size_t a = pi_plan(T, D, R, false).ws.bytes, b = pi_plan(T, D, R, true).ws.bytes;
  return a > b ? a : b;   // either path fits
}

int dsmz_power_iter(int32_t h_dtype, const void* H, int64_t T, int64_t D, int64_t hs0, int64_t hs1, const float* V,
                    int64_t R, int64_t vs0, int64_t vs1, float* out, int32_t num_iters, float norm_floor,
                    void* workspace, size_t workspace_bytes, dsmz_stream_t stream) {
  if (!H || !V || !out || !workspace) return fail(DSMZ_ERR_INVALID, "power_iter: null pointer");
  if (T <= 0 || D <= 0 || R <= 0) return fail(DSMZ_ERR_INVALID, "power_iter: empty shape");
  if (R > DSMZ_MAX_RANK) return fail(DSMZ_ERR_UNSUPPORTED, "power_iter: R must be <= " + std::to_string(DSMZ_MAX_RANK));
  if (h_dtype != DSMZ_F32 && h_dtype != DSMZ_BF16) return fail(DSMZ_ERR_INVALID, "power_iter: bad dtype");
  const bool want_tc = tc_shape_ok(h_dtype, D, hs0, hs1, R, H);
  dsmz_plan P = pi_plan(T, D, R, want_tc);
  if (workspace_bytes < P.ws.bytes) return fail(DSMZ_ERR_WORKSPACE, "power_iter: workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(DSMZ_ERR_INVALID, "power_iter: workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_iters <= 0) {
    // zero iterations return the basis unchanged (contiguous copy)
    if (vs1 != 1) return fail(DSMZ_ERR_UNSUPPORTED, "power_iter: num_iters == 0 needs unit column stride");
    cudaError_t e = cudaMemcpy2DAsync(out, R * sizeof(float), V, vs0 * sizeof(float), R * sizeof(float), D,
                                      cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_fail("power_iter copy", e);
    return DSMZ_OK;
  }
  BasisD& b = P.bases[0];
  b.H = H; b.hdt = h_dtype; b.h_s0 = hs0; b.h_s1 = hs1;
  b.Vin = V; b.v_s0 = vs0; b.v_s1 = vs1; b.Vout = out;
  P.workspace = static_cast<char*>(workspace);
  patch_ws_pointers(&P);
  if (P.tc && !bind_tc(&P)) {   // driver refused a tensor map: rebuild for the CUDA-core path
    P = pi_plan(T, D, R, false);
    BasisD& b2 = P.bases[0];
    b2.H = H; b2.hdt = h_dtype; b2.h_s0 = hs0; b2.h_s1 = hs1;
    b2.Vin = V; b2.v_s0 = vs0; b2.v_s1 = vs1; b2.Vout = out;
    P.workspace = static_cast<char*>(workspace);
    patch_ws_pointers(&P);
  }
  {
    int dev = 0;
    cudaError_t ed = cudaGetDevice(&dev);
    if (ed == cudaSuccess) ed = cudaDeviceGetAttribute(&P.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (ed != cudaSuccess) return cuda_fail("power_iter: device query", ed);
    cudaError_t ez = cudaMemsetAsync(P.workspace + P.err_off, 0, sizeof(int), s);
    if (ez != cudaSuccess) return cuda_fail("power_iter: error word", ez);
  }
  if (P.sm_count > kMaxChunks) return fail(DSMZ_ERR_UNSUPPORTED, "power_iter: too many SMs");
  chunk_w_tables(&P, false);
  int rc = upload_small(&P, static_cast<char*>(workspace), s);
  if (rc) return rc;
  return run_power_iteration(&P, num_iters, norm_floor, s);
}

static dsmz_plan agzo_plan(int64_t R, int64_t d_in, int64_t RC, int64_t d_out) {
  dsmz_plan P;
  P.ws.take(table_head_bytes());
  const int rca = static_cast<int>(R < RC ? R : RC);
  ModD md{};
  md.r = static_cast<int32_t>(R); md.rc = static_cast<int32_t>(RC); md.rca = rca;
  md.d_out = d_out; md.d_in = d_in; md.basis = 0;
  const size_t nB = static_cast<size_t>(R) * RC;
  md.coef_off = static_cast<int64_t>(P.ws.take((nB + static_cast<size_t>(R) * rca) * sizeof(float)) / sizeof(float));
  md.qrw_off = coef_qr_in_smem(md.r, rca) ? 0 : static_cast<int64_t>(
      P.ws.take(2 * static_cast<size_t>(rca) * rca * sizeof(double)) / sizeof(double));
  md.a = 0; md.b = 1;
  P.mods.push_back(md);
  // one CTA per 2048 columns (the device is not known yet)
  plan_bside(P.mods, static_cast<int>((d_in + 2047) / 2048), P.ws, &P.nchunks, &P.bside_cols);
  MatD a{};
  a.nvec = d_out; a.r = R; a.ld = R; a.cs = 1; a.side = 0; a.owner = 0;
  add_matrix(P.mats, P.ws, a, P.nsegs);
  MatD b{};
  b.nvec = d_in; b.r = R; b.ld = d_in; b.cs = 1; b.side = 1; b.owner = 0;
  add_matrix(P.mats, P.ws, b, P.nsegs);
  BasisD bd{};
  bd.R = static_cast<int32_t>(RC); bd.D = d_in;
  P.bases.push_back(bd);
  P.r = static_cast<int>(R);
  P.RC = static_cast<int>(RC);
  P.pack();
  return P;
}

size_t dsmz_agzo_perturbation_workspace_bytes(int64_t R, int64_t d_in, int64_t RC, int64_t d_out) {
  if (R <= 0 || d_in <= 0 || RC <= 0 || d_out <= 0) return 0;
  return agzo_plan(R, d_in, RC, d_out).ws.bytes;
}

int dsmz_agzo_perturbation(const float* B, int64_t R, int64_t d_in, int64_t bs0, int64_t bs1, const float* V,
                           int64_t RC, int64_t vs0, int64_t vs1, const float* zcB, const float* zcA, int64_t d_out,
                           float* z_A, float* z_B, float eps, float norm_floor, void* workspace,
                           size_t workspace_bytes, dsmz_stream_t stream) {
  if (!B || !V || !zcB || !zcA || !z_A || !z_B || !workspace)
    return fail(DSMZ_ERR_INVALID, "agzo_perturbation: null pointer");
  if (R <= 0 || d_in <= 0 || RC <= 0 || d_out <= 0) return fail(DSMZ_ERR_INVALID, "agzo_perturbation: empty shape");
  if (R > DSMZ_MAX_RANK || RC > DSMZ_MAX_RANK)
    return fail(DSMZ_ERR_UNSUPPORTED, "agzo_perturbation: R and RC must be <= " + std::to_string(DSMZ_MAX_RANK));
  dsmz_plan P = agzo_plan(R, d_in, RC, d_out);
  if (workspace_bytes < P.ws.bytes) return fail(DSMZ_ERR_WORKSPACE, "agzo_perturbation: workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(DSMZ_ERR_INVALID, "agzo_perturbation: workspace must be 256-byte aligned");
  ModD& md = P.mods[0];
  md.zcB_ext = zcB; md.zcA_ext = zcA; md.Bp = B; md.varB = nullptr; md.b_s0 = bs0; md.b_s1 = bs1;
  P.mats[0].z = z_A;
  P.mats[1].z = z_B;
  BasisD& bd = P.bases[0];
  bd.Vin = V; bd.v_s0 = vs0; bd.v_s1 = vs1;
  P.workspace = static_cast<char*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = upload_small(&P, static_cast<char*>(workspace), s);
  if (rc) return rc;
  const Tables tb = P.tables();
  const size_t cs = coef_smem(static_cast<int>(R), static_cast<int>(RC));
  const size_t ps = perturb_smem(static_cast<int>(R), static_cast<int>(R), static_cast<int>(RC));
  if ((rc = set_smem(k_coef<1>, cs))) return rc;
  if ((rc = set_smem(k_perturb, ps))) return rc;
  k_bside<<<P.nchunks, kThreads, 0, s>>>(tb, P.bside_cols);
  DSMZ_LAUNCHED("agzo B V");
  k_coef<1><<<1, kThreads, cs, s>>>(tb, 0, 0, norm_floor, 1);
  DSMZ_LAUNCHED("agzo QR");
  k_perturb<<<P.nsegs, kThreads, ps, s>>>(tb, eps);
  DSMZ_LAUNCHED("agzo z");
  return DSMZ_OK;
}

int dsmz_perturb_dual(int32_t dtype, const void* base, const float* z, void* pos, void* neg, int64_t n,
                      dsmz_stream_t stream) {
  if (n <= 0) return DSMZ_OK;
  if (!base || !z || !pos || !neg) return fail(DSMZ_ERR_INVALID, "perturb_dual: null pointer");
  if (dtype != DSMZ_F32 && dtype != DSMZ_BF16) return fail(DSMZ_ERR_INVALID, "perturb_dual: bad dtype");
  int64_t blocks = (n + kThreads - 1) / kThreads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_dual<<<static_cast<int>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(base, z, pos, neg, n, dtype);
  DSMZ_LAUNCHED("perturb_dual");
  return DSMZ_OK;
}

// ---------------------------------------------------------------------- allocation-free ZO-Muon
// Scratch of dsmz_zo_muon_update_noalloc: a fixed array in this library, held by every GPU
// that loads it until the process exits. Host code must not use the symbol's host-side
// address; its device address is looked up with the device current and cached per device
// together with the unique ID of the context the lookup ran in. A different current context
// on that device (a context the caller made current, or the primary context created again
// after cudaDeviceReset) has its own copy of the array, so the lookup is repeated for it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[DSMZ_NOALLOC_SCRATCH_BYTES];


int dsmz_zo_muon_update_noalloc(int32_t param_dtype, void* param, int64_t ps0, int64_t ps1, const float* buf,
                                int64_t bs0, int64_t bs1, float* scratch, int64_t ss0, int64_t ss1, int64_t M,
                                int64_t N, float eta, float norm_floor, const dsmz_ns_schedule* schedule,
                                dsmz_stream_t stream) {
  if (M <= 0 || N <= 0) return DSMZ_OK;
  const size_t need = dsmz_zo_muon_update_workspace_bytes(M, N);
  if (need > DSMZ_NOALLOC_SCRATCH_BYTES)
    return fail(DSMZ_ERR_UNSUPPORTED, "zo_muon_update_noalloc: a " + std::to_string(M) + " x " + std::to_string(N) +
                                          " update needs " + std::to_string(need) + " scratch bytes, above the " +
                                          std::to_string(DSMZ_NOALLOC_SCRATCH_BYTES) +
                                          " built in; use dsmz_zo_muon_update with a workspace");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("zo_muon_update_noalloc: cudaGetDevice", e);
  if (dev < 0 || dev >= 256) return fail(DSMZ_ERR_UNSUPPORTED, "zo_muon_update_noalloc: device index above 255");
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoallocSlot& slot = g_noalloc_slot[dev];
    const unsigned long long id = current_ctx_id();
    if (id == 0 || slot.ctx_id != id || !slot.addr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // with this device (and context) current
      if (e != cudaSuccess) return cuda_fail("zo_muon_update_noalloc: cudaGetSymbolAddress", e);
      slot.addr = p;
      slot.ctx_id = current_ctx_id();   // the lookup has created the primary context if there was none
    }
    ws = slot.addr;
  }
  // Every slot the kernels read (tables, Gram partials, solve workspace, apply matrix) is
  // written earlier in the same call, so nothing has to be cleared between calls.
  return dsmz_zo_muon_update(param_dtype, param, ps0, ps1, buf, bs0, bs1, scratch, ss0, ss1, M, N, eta, norm_floor,
                             schedule, ws, DSMZ_NOALLOC_SCRATCH_BYTES, stream);
}

int dsmz_plan_set_probe(dsmz_plan* P, int32_t kernel, void** start_events, void** stop_events, int32_t capacity) {
  if (!P || kernel < 0 || kernel >= DSMZ_NUM_KIDS || capacity < 0 || (capacity > 0 && (!start_events || !stop_events)))
    return fail(DSMZ_ERR_INVALID, "dsmz_plan_set_probe: bad arguments");
  auto& p = P->probes[kernel];
  p.start.assign(reinterpret_cast<cudaEvent_t*>(start_events), reinterpret_cast<cudaEvent_t*>(start_events) + capacity);
  p.stop.assign(reinterpret_cast<cudaEvent_t*>(stop_events), reinterpret_cast<cudaEvent_t*>(stop_events) + capacity);
  p.count = 0;
  return DSMZ_OK;
}

int32_t dsmz_plan_probe_count(const dsmz_plan* P, int32_t kernel) {
  if (!P || kernel < 0 || kernel >= DSMZ_NUM_KIDS) return 0;
  return P->probes[kernel].count;
}

}  // extern "C"
