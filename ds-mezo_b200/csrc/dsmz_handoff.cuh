// Device-resident activation handoff (ds_mezo/backend.py:55-93 and ds_mezo/controller.py:171
// move each captured module input GPU -> pinned host -> GPU in fp32 every step): the forward
// hook's tensor is converted on the device straight into the T x D activation buffer that
// the power iteration reads.
//
// k_act_load writes every row of the destination: rows t < n come from the source, rows
// n..T-1 are zero (zero rows leave H^T H unchanged, so a capture shorter than the buffer
// is exact). fp32 -> bf16 rounds to nearest even with CUDA's conversion, as torch's
// .to(torch.bfloat16) does; bf16 -> fp32 is exact and bf16 -> bf16 copies the bits. The vector path moves eight elements
// per thread (16-byte bf16 stores, two 16-byte fp32 loads) when rows are unit-stride,
// D % 8 == 0 and both row starts are 16-byte aligned; otherwise one element per thread.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace dsmz {

__device__ __forceinline__ uint16_t bf16_bits_rne(float x) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<const uint16_t*>(&h);
}

// SRC / DST: 0 = fp32, 1 = bf16 (the dsmz_dtype codes)
template <int SRC>
__device__ __forceinline__ float act_in(const void* src, int64_t i) {
  if (SRC == 0) return reinterpret_cast<const float*>(src)[i];
  const uint32_t b = reinterpret_cast<const uint16_t*>(src)[i];
  return __uint_as_float(b << 16);
}
template <int DST>
__device__ __forceinline__ void act_out(void* dst, int64_t i, float x) {
  if (DST == 0) reinterpret_cast<float*>(dst)[i] = x;
  else reinterpret_cast<uint16_t*>(dst)[i] = bf16_bits_rne(x);
}

template <int SRC, int DST>
__global__ void __launch_bounds__(256) k_act_load(void* __restrict__ dst, int64_t T, int64_t D, int64_t ld,
                                                  const void* __restrict__ src, int64_t n, int64_t s0, int64_t s1,
                                                  int vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t gpr = D >> 3;                        // groups of eight per row
    const int64_t total = T * gpr;
    for (int64_t g = first; g < total; g += stride) {
      const int64_t t = g / gpr;
      const int64_t c = (g - t * gpr) << 3;
      if (SRC == 1 && DST == 1) {                       // bf16 -> bf16: the bits as they are
        const uint4 u = (t < n) ? *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + t * s0 + c)
                                : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + t * ld + c) = u;
        continue;
      }
      float x[8];
      if (t < n) {
        if (SRC == 0) {
          const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + t * s0 + c);
          const float4 a = p[0], b = p[1];
          x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
          const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + t * s0 + c);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) { x[2 * q] = __uint_as_float(w[q] << 16); x[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u); }
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) x[q] = 0.f;
      }
      if (DST == 0) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(dst) + t * ld + c);
        o[0] = make_float4(x[0], x[1], x[2], x[3]);
        o[1] = make_float4(x[4], x[5], x[6], x[7]);
      } else {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          w[q] = static_cast<uint32_t>(bf16_bits_rne(x[2 * q])) | (static_cast<uint32_t>(bf16_bits_rne(x[2 * q + 1])) << 16);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + t * ld + c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  } else {
    const int64_t total = T * D;
    for (int64_t e = first; e < total; e += stride) {
      const int64_t t = e / D, c = e - t * D;
      if (SRC == 1 && DST == 1) {
        reinterpret_cast<uint16_t*>(dst)[t * ld + c] =
            (t < n) ? reinterpret_cast<const uint16_t*>(src)[t * s0 + c * s1] : static_cast<uint16_t>(0);
        continue;
      }
      const float x = (t < n) ? act_in<SRC>(src, t * s0 + c * s1) : 0.f;
      act_out<DST>(dst, t * ld + c, x);
    }
  }
}

}  // namespace dsmz
