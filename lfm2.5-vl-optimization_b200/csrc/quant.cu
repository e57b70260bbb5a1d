// Dynamic activation quantizers: bf16 [rows, K] -> int8 [rows, K] + fp32 absmax scales.
//
//   quant_rows:   one scale per row (token):            s[row]        = max(|x[row, :]|, 1e-8) / 127
//   quant_groups: one scale per row and 64-wide group:  sT[g][row]    = max(|x[row, 64g:64g+64]|, 1e-8) / 127
//   codes:        q = clamp(rint(x / s), -127, 127), the quotient an IEEE fp32 division, ties to even (computed
//                 as x * (1 / s) with an exact fallback near rounding boundaries: q8r in common.cuh).
//
// Semantics follow kernels/int8_gemm.cu:393-432 (quant_rows_kernel) and :435-474 (quant_groups_kernel) of the
// reference; the reference's per-row limit K <= 2048 (kernels/int8_gemm.cpp:93) is lifted here (K <= 16384,
// K % 8 == 0), and the grouped path needs K % 64 == 0 instead of K % 128 == 0.
//
// B200 layout: HBM-bound (reads 2 B, writes 1 B per element). RW warps own one row; every lane streams 16-byte
// chunks (8 bf16) at lane-contiguous addresses, keeps them in registers while the absmax is reduced with warp
// shuffles (and shared memory across the RW warps), then writes 8-byte int8 chunks, so each element crosses HBM
// exactly once in each direction.
#include "common.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

constexpr int QT = 256;  // threads per block (8 warps)

// QC: 16-byte chunks each lane holds (a row covers RW * 32 * QC chunks); fewer for short rows keeps registers, and
// with them the rows in flight per SM, up
template <int RW, bool GROUPED, int QC>
__global__ void __launch_bounds__(QT) quant_kernel(const bf16 *__restrict__ x, int8_t *__restrict__ q,
                                                   float *__restrict__ s, int rows, int K, int pdl) {
  // launched with programmatic serialization: let the next kernel (the GEMV / GEMM that reads q, s) start its own
  // weight streaming, and wait for the producer of x before reading it
  if (pdl) {
    pdl_trigger();
    pdl_wait();
  }
  constexpr int ROWS_PER_BLOCK = (QT / 32) / RW;
  __shared__ float red[QT / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * ROWS_PER_BLOCK + warp / RW, sub = warp % RW;
  const bool live = row < rows;
  const int K8 = K >> 3;  // 16-byte chunks per row
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + (size_t)(live ? row : 0) * K);

  uint4 v[QC];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < QC; ++i) {
    const int c = sub * 32 + lane + i * 32 * RW;
    if (live && c < K8) {
      v[i] = ld_cg16(xr + c);
    } else {
      v[i] = make_uint4(0, 0, 0, 0);
    }
  }
  if (!GROUPED) {
    {
      // |x| of bf16 pairs is the word with both sign bits cleared; the max of two non-negative bf16 values is their
      // larger 16-bit pattern, so the row maximum is a packed unsigned max over the words
      uint32_t m2 = 0;
#pragma unroll
      for (int i = 0; i < QC; ++i) {
        m2 = __vmaxu2(m2, __vmaxu2(v[i].x & 0x7FFF7FFFu, v[i].y & 0x7FFF7FFFu));
        m2 = __vmaxu2(m2, __vmaxu2(v[i].z & 0x7FFF7FFFu, v[i].w & 0x7FFF7FFFu));
      }
      amax = fmaxf(bf_lo(m2), bf_hi(m2));
    }
    amax = warp_max(amax);
    if (RW > 1) {
      if (lane == 0) red[warp] = amax;
      __syncthreads();
      amax = 0.f;
#pragma unroll
      for (int r = 0; r < RW; ++r) amax = fmaxf(amax, red[(warp / RW) * RW + r]);
    }
    if (!live) return;
    const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
    const float rinv = __frcp_rn(sc);
    if (sub == 0 && lane == 0) s[row] = sc;
    uint2 *qr = reinterpret_cast<uint2 *>(q + (size_t)row * K);
#pragma unroll
    for (int i = 0; i < QC; ++i) {
      const int c = sub * 32 + lane + i * 32 * RW;
      if (c < K8) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        uint32_t o[2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
          o[h] = pack_sums4(q8r2(make_float2(bf_lo(w[2 * h]), bf_hi(w[2 * h])), sc, rinv),
                            q8r2(make_float2(bf_lo(w[2 * h + 1]), bf_hi(w[2 * h + 1])), sc, rinv));
        qr[c] = make_uint2(o[0], o[1]);
      }
    }
  } else {
    // chunk c covers elements 8c..8c+7: group c / 8; the 8 chunks of a group sit on 8 consecutive lanes
    if (!live) return;
    uint2 *qr = reinterpret_cast<uint2 *>(q + (size_t)row * K);
#pragma unroll
    for (int i = 0; i < QC; ++i) {
      const int c = sub * 32 + lane + i * 32 * RW;
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf_lo(w[j])), fabsf(bf_hi(w[j]))));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      if (c < K8) {
        const float sc = __fdiv_rn(fmaxf(m, 1e-8f), 127.f);
        const float rinv = __frcp_rn(sc);
        if ((lane & 7) == 0) s[(size_t)(c >> 3) * rows + row] = sc;
        uint32_t o[2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
          o[h] = pack_sums4(q8r2(make_float2(bf_lo(w[2 * h]), bf_hi(w[2 * h])), sc, rinv),
                            q8r2(make_float2(bf_lo(w[2 * h + 1]), bf_hi(w[2 * h + 1])), sc, rinv));
        qr[c] = make_uint2(o[0], o[1]);
      }
    }
  }
}

template <bool GROUPED>
cudaError_t run_quant(const void *x, int8_t *q, float *s, int rows, int K, bool pdl, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int K8 = K / 8;
  // smallest RW whose RW * 32 lanes * 8 chunks cover the row
  int rw = 1;
  while (rw * 32 * 8 < K8) rw *= 2;
  const bf16 *xx = (const bf16 *)x;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(QT);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const int p = pdl ? 1 : 0;
  switch (rw) {
    case 1:
      cfg.gridDim = dim3((rows + 7) / 8);
      if (K8 <= 32 * 5) return cudaLaunchKernelEx(&cfg, quant_kernel<1, GROUPED, 5>, xx, q, s, rows, K, p);
      return cudaLaunchKernelEx(&cfg, quant_kernel<1, GROUPED, 8>, xx, q, s, rows, K, p);
    case 2: cfg.gridDim = dim3((rows + 3) / 4); return cudaLaunchKernelEx(&cfg, quant_kernel<2, GROUPED, 8>, xx, q, s, rows, K, p);
    case 4:
      cfg.gridDim = dim3((rows + 1) / 2);
      if (K8 <= 4 * 32 * 5) return cudaLaunchKernelEx(&cfg, quant_kernel<4, GROUPED, 5>, xx, q, s, rows, K, p);
      return cudaLaunchKernelEx(&cfg, quant_kernel<4, GROUPED, 8>, xx, q, s, rows, K, p);
    case 8: cfg.gridDim = dim3(rows); return cudaLaunchKernelEx(&cfg, quant_kernel<8, GROUPED, 8>, xx, q, s, rows, K, p);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_quant_rows(const void *x, int8_t *q, float *s, int rows, int K, bool pdl, cudaStream_t st) {
  return run_quant<false>(x, q, s, rows, K, pdl, st);
}

cudaError_t launch_quant_groups(const void *x, int8_t *q, float *sT, int rows, int K, bool pdl, cudaStream_t st) {
  return run_quant<true>(x, q, sT, rows, K, pdl, st);
}

}  // namespace lfm2q
