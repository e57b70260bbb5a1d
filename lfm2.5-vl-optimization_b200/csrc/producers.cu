// Producers that write the next W8A8 GEMM's int8 input (+ per-row or per-64-group scales) directly:
//
//   add_layernorm_q  (vision)  h += y (bf16-rounded, in place); x = bf16(LayerNorm(h) * w + b); quantize x
//   add_rmsnorm_q    (LM)      h += y (bf16-rounded, in place); x = bf16(w * bf16(h * rsqrt(mean(h^2) + eps)))
//   silu_mul_q       (LM)      g = [rows, 2I] (w1 | w3 outputs); a = bf16(bf16(silu(g1)) * g3); quantize a
//
// Reference: kernels/int8_gemm.cu:529-585 (add_layernorm_q_kernel), :589-642 (add_rmsnorm_q_kernel), :646-682
// (silu_mul_q_kernel), launchers :787-820; bindings kernels/int8_gemm.cpp:107-141. The bf16 rounding points are the
// reference's; rsqrtf and __expf are the same intrinsics the reference calls.
//
// B200 layout: one 256-thread block per row; the row is read once with 16-byte loads into shared memory as fp32,
// reduced in a fixed order (per-thread sequential partial sums over the thread's elements in increasing index,
// xor-butterfly inside each warp, then the 8 warp sums in warp order), transformed, and quantized from shared
// memory. Rows up to 16384 wide fit (64 KB of fp32).
#include "common.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

constexpr int PT = 256;  // threads per row block

__device__ __forceinline__ float block_sum_fixed(float v, float *red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < PT / 32; ++w) t += red[w];
  return t;
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

template <bool GROUPED>
__global__ void __launch_bounds__(PT) add_layernorm_q_kernel(bf16 *__restrict__ h, const bf16 *__restrict__ y,
                                                             const bf16 *__restrict__ w, const bf16 *__restrict__ b,
                                                             int8_t *__restrict__ q, float *__restrict__ s, int rows,
                                                             int D, float eps) {
  extern __shared__ float xs[];
  __shared__ float red[PT / 32];
  const int row = blockIdx.x;
  load_residual(h, y, D, row, xs);
  float sum = 0.f;
  for (int i = threadIdx.x; i < D; i += PT) sum = __fadd_rn(sum, xs[i]);
  const float mean = __fdiv_rn(block_sum_fixed(sum, red), (float)D);
  float qs = 0.f;
  for (int i = threadIdx.x; i < D; i += PT) {
    const float d = __fsub_rn(xs[i], mean);
    qs = __fmaf_rn(d, d, qs);
  }
  const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(block_sum_fixed(qs, red), (float)D), eps));
  for (int i = threadIdx.x; i < D; i += PT)
    xs[i] = rbf(__fmaf_rn(__fmul_rn(__fsub_rn(xs[i], mean), rstd), bf2f(w[i]), bf2f(b[i])));
  __syncthreads();
  quant_row_smem<GROUPED>(xs, D, q, s, row, rows, red);
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
  const float rs = rsqrtf(__fadd_rn(__fdiv_rn(block_sum_fixed(ss, red), (float)H), eps));
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
      xs[8 * c + 2 * j] = rbf(__fmul_rn(rbf(a0 / (1.f + __expf(-a0))), bf_lo(uw[j])));
      xs[8 * c + 2 * j + 1] = rbf(__fmul_rn(rbf(a1 / (1.f + __expf(-a1))), bf_hi(uw[j])));
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
  const size_t sm = (size_t)D * sizeof(float);
  if (grouped) {
    cudaError_t e = set_smem(add_layernorm_q_kernel<true>, sm);
    if (e != cudaSuccess) return e;
    add_layernorm_q_kernel<true><<<rows, PT, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w, (const bf16 *)b,
                                                       q, s, rows, D, eps);
  } else {
    cudaError_t e = set_smem(add_layernorm_q_kernel<false>, sm);
    if (e != cudaSuccess) return e;
    add_layernorm_q_kernel<false><<<rows, PT, sm, st>>>((bf16 *)h, (const bf16 *)y, (const bf16 *)w, (const bf16 *)b,
                                                        q, s, rows, D, eps);
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
