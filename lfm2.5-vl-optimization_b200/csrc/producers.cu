// Producers that write the next W8A8 GEMM's int8 input (+ per-row or per-64-group scales) directly:
//
//   add_layernorm_q  (vision)  h += y (bf16-rounded, in place); x = bf16(LayerNorm(h) * w + b); quantize x
//   add_rmsnorm_q    (LM)      h += y (bf16-rounded, in place); x = bf16(w * bf16(h * rsqrt(mean(h^2) + eps)))
//   silu_mul_q       (LM)      g = [rows, 2I] (w1 | w3 outputs); a = bf16(bf16(silu(g1)) * g3); quantize a
//
// Reference: kernels/int8_gemm.cu:529-585 (add_layernorm_q_kernel), :589-642 (add_rmsnorm_q_kernel), :646-682
// (silu_mul_q_kernel), launchers :787-820; bindings kernels/int8_gemm.cpp:107-141.
//
// Bit-exact with the reference: every fp32 value is produced by the same operations in the same order, so the
// reductions keep the reference's partition of a row over threads and its combining tree (a different tree gives a
// different fp32 sum, hence different codes):
//   - layernorm: one warp per row; lane l owns the 4-element chunks l, l + 32, l + 64, ... and adds each chunk's
//     ((v0 + v1) + v2) + v3 to its running sum in chunk order; the 32 lane sums meet in an xor butterfly
//     (16, 8, 4, 2, 1); the squared deviations accumulate per lane with fused multiply-adds in the same element order.
//   - rmsnorm: one 256-thread block per row; thread t accumulates fma(v, v, ss) over t, t + 256, ...; xor butterfly
//     per warp; the 8 warp sums are combined by a second 32-lane xor butterfly with zeros in lanes 8..31.
//   - the bf16 rounding points, rsqrtf and __expf are the reference's; fmaf where the reference's expressions
//     a * b + c are contracted by nvcc (its default -fmad=true build).
// Maxima (the quantization scales) do not depend on order.
//
// B200 layout: the rows are streamed once from HBM with coalesced loads; the fp32 row lives in shared memory between
// the passes (layernorm: per warp, 8 rows per 256-thread block; rms / silu: per block).
#include "common.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

constexpr int PT = 256;  // threads per block

// The reference's block_sum (kernels/lfm2_decode.cu:79-90): xor butterfly per warp, then the warp sums combined by a
// second butterfly over lanes (lane w < 8 holds warp w's sum, the rest 0). Every thread returns the total.
__device__ __forceinline__ float block_sum_ref(float v, float *red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_sum(lane < PT / 32 ? red[lane] : 0.f);
}
__device__ __forceinline__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < PT / 32; ++w) t = fmaxf(t, red[w]);
  return t;
}

// Quantize the bf16-exact fp32 row xs[0..K) held in shared memory into q[row], s (per row or per 64-group).
template <bool GROUPED>
__device__ __forceinline__ void quant_row_smem(const float *xs, int K, int8_t *__restrict__ q, float *__restrict__ s,
                                               int row, int rows, float *red) {
  int8_t *qr = q + (size_t)row * K;
  if (!GROUPED) {
    float m = 0.f;
    for (int i = threadIdx.x; i < K; i += PT) m = fmaxf(m, fabsf(xs[i]));
    const float sc = __fdiv_rn(fmaxf(block_max(m, red), 1e-8f), 127.f);
    const float rinv = __frcp_rn(sc);
    if (threadIdx.x == 0) s[row] = sc;
    for (int i = threadIdx.x; i < K; i += PT) qr[i] = (int8_t)q8r(xs[i], sc, rinv);
  } else {
    // one warp per 64-wide group: lane holds elements lane and lane + 32
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int g = warp; g < K / 64; g += PT / 32) {
      const float a = xs[g * 64 + lane], b = xs[g * 64 + 32 + lane];
      const float sc = __fdiv_rn(fmaxf(warp_max(fmaxf(fabsf(a), fabsf(b))), 1e-8f), 127.f);
      const float rinv = __frcp_rn(sc);
      qr[g * 64 + lane] = (int8_t)q8r(a, sc, rinv);
      qr[g * 64 + 32 + lane] = (int8_t)q8r(b, sc, rinv);
      if (lane == 0) s[(size_t)g * rows + row] = sc;
    }
  }
}

// Load row r of h (+ y) into xs as fp32 (16-byte chunks), writing h back when y is given.
__device__ __forceinline__ void load_residual(bf16 *__restrict__ h, const bf16 *__restrict__ y, int D, int row,
                                              float *xs) {
  uint4 *hr = reinterpret_cast<uint4 *>(h + (size_t)row * D);
  const uint4 *yr = y ? reinterpret_cast<const uint4 *>(y + (size_t)row * D) : nullptr;
  for (int c = threadIdx.x; c < D / 8; c += PT) {
    uint4 hv = hr[c];
    uint32_t *hw = &hv.x;
    if (yr) {
      const uint4 yv = yr[c];
      const uint32_t *yw = &yv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        hw[j] = pack_bf16x2(__fadd_rn(bf_lo(hw[j]), bf_lo(yw[j])), __fadd_rn(bf_hi(hw[j]), bf_hi(yw[j])));
      hr[c] = hv;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      xs[8 * c + 2 * j] = bf_lo(hw[j]);
      xs[8 * c + 2 * j + 1] = bf_hi(hw[j]);
    }
  }
  __syncthreads();
}

// Four bf16 (8 bytes) -> fp32
__device__ __forceinline__ float4 bf4(uint2 u) { return make_float4(bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y)); }

// One warp per row (blockDim.x / 32 rows per block: 8, fewer for rows wider than 6144). Chunk ci (elements 4ci .. 4ci + 3) belongs to lane ci % 32, as in the
// reference; the warp's fp32 row is kept in shared memory (D / 4 float4, lane-strided: conflict-free) between passes.
template <bool GROUPED>
__global__ void __launch_bounds__(PT) add_layernorm_q_kernel(bf16 *__restrict__ h, const bf16 *__restrict__ y,
                                                             const bf16 *__restrict__ w, const bf16 *__restrict__ b,
                                                             int8_t *__restrict__ q, float *__restrict__ s, int rows,
                                                             int D, float eps) {
  extern __shared__ float4 ln_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (int)(blockDim.x >> 5) + warp;
  if (row >= rows) return;  // warp-uniform; no block-wide barrier follows
  const int NC = D / 4;
  const int rounds = (NC + 31) / 32;  // warp-uniform loop count (the last round may leave lanes idle)
  float4 *xr = ln_smem + (size_t)warp * NC;
  uint2 *hr = reinterpret_cast<uint2 *>(h + (size_t)row * D);
  const uint2 *yr = y ? reinterpret_cast<const uint2 *>(y + (size_t)row * D) : nullptr;

  // pass 1: residual (h written back), fp32 row to shared memory, per-lane sum in the reference's order
  float sum = 0.f;
  constexpr int U = 4;  // chunks in flight per lane
  for (int r0 = 0; r0 < rounds; r0 += U) {
    uint2 hv[U], yv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ci = (r0 + u) * 32 + lane;
      if (r0 + u < rounds && ci < NC) {
        hv[u] = hr[ci];
        if (yr) yv[u] = yr[ci];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ci = (r0 + u) * 32 + lane;
      if (r0 + u < rounds && ci < NC) {
        float4 v = bf4(hv[u]);
        if (yr) {
          const float4 t = bf4(yv[u]);
          v = make_float4(rbf(__fadd_rn(v.x, t.x)), rbf(__fadd_rn(v.y, t.y)), rbf(__fadd_rn(v.z, t.z)),
                          rbf(__fadd_rn(v.w, t.w)));
          hr[ci] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        }
        xr[ci] = v;
        sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(__fadd_rn(v.x, v.y), v.z), v.w));
      }
    }
  }
  const float mean = __fdiv_rn(warp_sum(sum), (float)D);
  // pass 2: sum of squared deviations, element order, fused multiply-adds
  float qs = 0.f;
  for (int ci = lane; ci < NC; ci += 32) {
    const float4 v = xr[ci];
    const float d0 = __fsub_rn(v.x, mean), d1 = __fsub_rn(v.y, mean), d2 = __fsub_rn(v.z, mean),
                d3 = __fsub_rn(v.w, mean);
    qs = __fmaf_rn(d0, d0, qs);
    qs = __fmaf_rn(d1, d1, qs);
    qs = __fmaf_rn(d2, d2, qs);
    qs = __fmaf_rn(d3, d3, qs);
  }
  const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(warp_sum(qs), (float)D), eps));
  // pass 3: x = bf16(fma((v - mean) * rstd, w, b)); row absmax
  const uint2 *wr = reinterpret_cast<const uint2 *>(w), *br = reinterpret_cast<const uint2 *>(b);
  float amax = 0.f;
  for (int ci = lane; ci < NC; ci += 32) {
    const float4 v = xr[ci], wf = bf4(__ldg(wr + ci)), bf = bf4(__ldg(br + ci));
    const float4 x = make_float4(rbf(__fmaf_rn(__fmul_rn(__fsub_rn(v.x, mean), rstd), wf.x, bf.x)),
                                 rbf(__fmaf_rn(__fmul_rn(__fsub_rn(v.y, mean), rstd), wf.y, bf.y)),
                                 rbf(__fmaf_rn(__fmul_rn(__fsub_rn(v.z, mean), rstd), wf.z, bf.z)),
                                 rbf(__fmaf_rn(__fmul_rn(__fsub_rn(v.w, mean), rstd), wf.w, bf.w)));
    xr[ci] = x;
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
  }
  // pass 4: quantize. Per row: one scale. Grouped: a 64-wide group is 16 chunks, held by one half-warp in each round
  // (lanes 0-15: group 2r, lanes 16-31: group 2r + 1), its maximum reduced over those 16 lanes.
  uint32_t *qr = reinterpret_cast<uint32_t *>(q + (size_t)row * D);
  if (!GROUPED) {
    const float sc = __fdiv_rn(fmaxf(warp_max(amax), 1e-8f), 127.f);
    const float rinv = __frcp_rn(sc);
    if (lane == 0) s[row] = sc;
    for (int ci = lane; ci < NC; ci += 32) {
      const float4 x = xr[ci];
      qr[ci] = pack_sums4(q8r2(make_float2(x.x, x.y), sc, rinv), q8r2(make_float2(x.z, x.w), sc, rinv));
    }
  } else {
    for (int r = 0; r < rounds; ++r) {
      const int ci = r * 32 + lane;
      const bool ok = ci < NC;  // D % 64 == 0: a half-warp is either all in or all out
      const float4 x = ok ? xr[ci] : make_float4(0.f, 0.f, 0.f, 0.f);
      float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (ok) {
        const float sc = __fdiv_rn(fmaxf(m, 1e-8f), 127.f);
        const float rinv = __frcp_rn(sc);
        if ((lane & 15) == 0) s[(size_t)(ci >> 4) * rows + row] = sc;
        qr[ci] = pack_sums4(q8r2(make_float2(x.x, x.y), sc, rinv), q8r2(make_float2(x.z, x.w), sc, rinv));
      }
    }
  }
}

template <bool GROUPED>
__global__ void __launch_bounds__(PT) add_rmsnorm_q_kernel(bf16 *__restrict__ h, const bf16 *__restrict__ y,
                                                           const bf16 *__restrict__ w, int8_t *__restrict__ q,
                                                           float *__restrict__ s, int rows, int H, float eps) {
  extern __shared__ float xs[];
  __shared__ float red[PT / 32];
  const int row = blockIdx.x;
  load_residual(h, y, H, row, xs);
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += PT) ss = __fmaf_rn(xs[i], xs[i], ss);
  const float rs = rsqrtf(__fadd_rn(__fdiv_rn(block_sum_ref(ss, red), (float)H), eps));
  for (int i = threadIdx.x; i < H; i += PT) xs[i] = rbf(__fmul_rn(bf2f(w[i]), rbf(__fmul_rn(xs[i], rs))));
  __syncthreads();
  quant_row_smem<GROUPED>(xs, H, q, s, row, rows, red);
}

template <bool GROUPED>
__global__ void __launch_bounds__(PT) silu_mul_q_kernel(const bf16 *__restrict__ g, int8_t *__restrict__ q,
                                                        float *__restrict__ s, int rows, int I) {
  extern __shared__ float xs[];
  __shared__ float red[PT / 32];
  const int row = blockIdx.x;
  const uint4 *ga = reinterpret_cast<const uint4 *>(g + (size_t)row * 2 * I);
  const uint4 *gu = reinterpret_cast<const uint4 *>(g + (size_t)row * 2 * I + I);
  for (int c = threadIdx.x; c < I / 8; c += PT) {
    const uint4 av = ga[c], uv = gu[c];
    const uint32_t *aw = &av.x, *uw = &uv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = bf_lo(aw[j]), a1 = bf_hi(aw[j]);
      xs[8 * c + 2 * j] = rbf(__fmul_rn(rbf(__fdiv_rn(a0, 1.f + __expf(-a0))), bf_lo(uw[j])));
      xs[8 * c + 2 * j + 1] = rbf(__fmul_rn(rbf(__fdiv_rn(a1, 1.f + __expf(-a1))), bf_hi(uw[j])));
    }
  }
  __syncthreads();
  quant_row_smem<GROUPED>(xs, I, q, s, row, rows, red);
}

template <typename K>
cudaError_t set_smem(K kern, size_t bytes) {
  return bytes > 48 * 1024 ? cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes)
                           : cudaSuccess;
}

}  // namespace

cudaError_t launch_add_layernorm_q(void *h, const void *y, const void *w, const void *b, int8_t *q, float *s, int rows,
                                   int D, float eps, bool grouped, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  // rows per block: 8 while their fp32 rows fit in 192 KB of shared memory (D <= 6144), else fewer (D = 16384: 3)
  int rpb = (int)((192 * 1024) / ((size_t)D * sizeof(float)));
  rpb = rpb < 1 ? 1 : (rpb > PT / 32 ? PT / 32 : rpb);
  const size_t sm = (size_t)rpb * D * sizeof(float);
  const int blocks = (rows + rpb - 1) / rpb;
  if (grouped) {
    cudaError_t e = set_smem(add_layernorm_q_kernel<true>, 192 * 1024);
    if (e != cudaSuccess) return e;
    add_layernorm_q_kernel<true><<<blocks, 32 * rpb, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w,
                                                               (const bf16 *)b, q, s, rows, D, eps);
  } else {
    cudaError_t e = set_smem(add_layernorm_q_kernel<false>, 192 * 1024);
    if (e != cudaSuccess) return e;
    add_layernorm_q_kernel<false><<<blocks, 32 * rpb, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w,
                                                                (const bf16 *)b, q, s, rows, D, eps);
  }
  return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm_q(void *h, const void *y, const void *w, int8_t *q, float *s, int rows, int H, float eps,
                                 bool grouped, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const size_t sm = (size_t)H * sizeof(float);
  if (grouped) {
    cudaError_t e = set_smem(add_rmsnorm_q_kernel<true>, sm);
    if (e != cudaSuccess) return e;
    add_rmsnorm_q_kernel<true><<<rows, PT, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w, q, s, rows, H, eps);
  } else {
    cudaError_t e = set_smem(add_rmsnorm_q_kernel<false>, sm);
    if (e != cudaSuccess) return e;
    add_rmsnorm_q_kernel<false><<<rows, PT, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w, q, s, rows, H, eps);
  }
  return cudaGetLastError();
}

cudaError_t launch_silu_mul_q(const void *g, int8_t *q, float *s, int rows, int I, bool grouped, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const size_t sm = (size_t)I * sizeof(float);
  if (grouped) {
    cudaError_t e = set_smem(silu_mul_q_kernel<true>, sm);
    if (e != cudaSuccess) return e;
    silu_mul_q_kernel<true><<<rows, PT, sm, st>>>((const bf16 *)g, q, s, rows, I);
  } else {
    cudaError_t e = set_smem(silu_mul_q_kernel<false>, sm);
    if (e != cudaSuccess) return e;
    silu_mul_q_kernel<false><<<rows, PT, sm, st>>>((const bf16 *)g, q, s, rows, I);
  }
  return cudaGetLastError();
}

}  // namespace lfm2q
