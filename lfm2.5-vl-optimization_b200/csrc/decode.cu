// The small kernels of one LFM2 decode step around the GEMVs and the attention: residual add + RMSNorm, the
// short-convolution step, and the q/k norm + RoPE + KV-cache write.
//
// Reference: add_rmsnorm_kernel (kernels/lfm2_decode.cu:92-127), shortconv_step_kernel (:129-161),
// qk_norm_rope_kv_kernel (:163-213); bindings add_rmsnorm / shortconv_step / qk_norm_rope_kv
// (kernels/lfm2_decode.cpp:32-55); caller: the fused decode step (src/lfm2opt/runtime.py:247-282).
//
// The values are the reference kernels' bit for bit: every element goes through the same fp32 expressions in the
// same order (HF's bf16 rounding points), and every sum of squares through the same partition and shuffle tree.
// The B200 side: every kernel is a programmatic dependent (it starts while its predecessor drains and reads the
// predecessor's outputs through L2, ld.global.cg, after griddepcontrol.wait), reads weights through the read-only
// path, and keeps rows in registers. The q/k norm + RoPE runs one warp per head (a lane holds dims d and d + 32, the
// pair that RoPE rotates, so the rotation is a register swap and cos / sin are evaluated once per pair) instead of a
// 64-thread block with a shared-memory exchange; the value heads are 128-byte copies into the cache.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

__device__ __forceinline__ float ldcg_bf(const bf16 *p) {
  return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short *>(p)) << 16);
}
__device__ __forceinline__ float ldg_bf(const bf16 *p) {
  return __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(p)) << 16);
}

// ------------------------------------------------------------------ add_rmsnorm
// One block of NT = 256 threads per row. Thread t owns elements t, t + 256, ... (the reference's partition: its
// partial sum of squares is accumulated in that order), kept in registers (H <= 8192: at most 32 per thread).
// HF: h = bf16(h + y); x = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))).
constexpr int NT = 256;
constexpr int NORM_MAX_PER_THREAD = 32;

// GATHER (embed_rmsnorm): the row is read from embed[tok[row]] instead of h and copied into h (bits unchanged), the
// reference step's embedding lookup and first norm in one launch.
template <bool ADD, bool GATHER = false>
__global__ void __launch_bounds__(NT) add_rmsnorm_kernel(bf16 *__restrict__ h, const bf16 *__restrict__ y,
                                                         const bf16 *__restrict__ w, bf16 *__restrict__ x, int H,
                                                         float eps, const bf16 *__restrict__ embed,
                                                         const int64_t *__restrict__ tok) {
  __shared__ float red[NT / 32];
  const int t = threadIdx.x, lane = t & 31, wp = t >> 5;
  const size_t off = (size_t)blockIdx.x * H;
  float hv[NORM_MAX_PER_THREAD], yv[NORM_MAX_PER_THREAD], wv[NORM_MAX_PER_THREAD];
  // the norm weights are immutable: read before the dependency wait, off the critical path
#pragma unroll
  for (int k = 0; k < NORM_MAX_PER_THREAD; ++k)
    if (t + NT * k < H) wv[k] = ldg_bf(w + t + NT * k);
  pdl_trigger();
  pdl_wait();
  const bf16 *src = h + off;
  if (GATHER) src = embed + (size_t)__ldcg(reinterpret_cast<const long long *>(tok) + blockIdx.x) * H;
  // every load of the row first (all in flight together), then the arithmetic and the stores of h
#pragma unroll
  for (int k = 0; k < NORM_MAX_PER_THREAD; ++k) {
    const int i = t + NT * k;
    if (i < H) {
      hv[k] = GATHER ? ldg_bf(src + i) : ldcg_bf(src + i);
      if (ADD) yv[k] = ldcg_bf(y + off + i);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NORM_MAX_PER_THREAD; ++k) {
    const int i = t + NT * k;
    if (i < H) {
      float v = hv[k];
      if (ADD) {
        v = rbf(v + yv[k]);
        h[off + i] = f2bf(v);
      } else if (GATHER) {
        h[off + i] = f2bf(v);  // the embedding row, bits unchanged
      }
      hv[k] = v;
      ss += v * v;
    }
  }
  // block sum: butterfly in each warp, then the eight warp totals (padded with zeros) through one more butterfly
  ss = warp_sum(ss);
  if (lane == 0) red[wp] = ss;
  __syncthreads();
  ss = warp_sum(lane < NT / 32 ? red[lane] : 0.f);
  const float rs = rsqrtf(ss / H + eps);
#pragma unroll
  for (int k = 0; k < NORM_MAX_PER_THREAD; ++k) {
    const int i = t + NT * k;
    if (i < H) x[off + i] = f2bf(wv[k] * rbf(hv[k] * rs));
  }
}

// ------------------------------------------------------------------ shortconv_step
// bcx [B, 3H] = (B | C | x) of the in_proj GEMV. bx = bf16(B x); the state window (s1, s2, bx) shifts in;
// y = bf16(C * bf16(w0 s1 + w1 s2 + w2 bx (+ bias))). One thread per (sequence, channel); the three state values of
// a channel (6 bytes) are read and written by that thread only.
__global__ void __launch_bounds__(NT) shortconv_step_kernel(const bf16 *__restrict__ bcx, bf16 *__restrict__ state,
                                                            const bf16 *__restrict__ w, const bf16 *__restrict__ bias,
                                                            bf16 *__restrict__ y, int H) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y, i = blockIdx.x * NT + threadIdx.x;
  if (i >= H) return;
  const bf16 *row = bcx + (size_t)b * 3 * H;
  const float bx = rbf(ldcg_bf(row + i) * ldcg_bf(row + 2 * H + i));
  bf16 *st = state + ((size_t)b * H + i) * 3;
  const float s1 = ldcg_bf(st + 1), s2 = ldcg_bf(st + 2);
  st[0] = f2bf(s1);  // exact: s1, s2 are bf16 values
  st[1] = f2bf(s2);
  st[2] = f2bf(bx);
  float acc = ldg_bf(w + i * 3 + 0) * s1 + ldg_bf(w + i * 3 + 1) * s2 + ldg_bf(w + i * 3 + 2) * bx;
  if (bias) acc += ldg_bf(bias + i);
  y[(size_t)b * H + i] = f2bf(ldcg_bf(row + H + i) * rbf(acc));
}

// ------------------------------------------------------------------ qk_norm_rope_kv
// qkv [B, (NQ + 2 NKV) * 64] = q heads | k heads | v heads. One warp per (sequence, head), lane l holding dims l and
// l + 32. q / k heads: n = bf16(x * rsqrt(mean(x^2) + eps)), x = bf16(w * n); RoPE in bf16 as HF:
// c, s = bf16(cos / sin(pos * inv_freq[l]) * scaling) (the same for dims l and l + 32), out_d = bf16(bf16(x_d c) +
// bf16(rot_d s)), rot_l = -x_{l+32}, rot_{l+32} = x_l. q -> q_out[b, head]; k -> kc[b, kv head, pos]; v heads are
// copied to vc[b, kv head, pos] unchanged. The sum of squares is the reference's 64-thread block sum: the butterfly
// over dims 0..31 plus the butterfly over dims 32..63.
constexpr int QK_WARPS = 8;
__global__ void __launch_bounds__(32 * QK_WARPS) qk_norm_rope_kv_kernel(
    const bf16 *__restrict__ qkv, const bf16 *__restrict__ qw, const bf16 *__restrict__ kw,
    const float *__restrict__ inv_freq, float scaling, const int64_t *__restrict__ pos_p, bf16 *__restrict__ q_out,
    bf16 *__restrict__ kc, bf16 *__restrict__ vc, int B, int NQ, int NKV, int max_len, float eps) {
  pdl_trigger();
  pdl_wait();
  const int NH = NQ + 2 * NKV;
  const int unit = blockIdx.x * QK_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (unit >= B * NH) return;
  const int b = unit / NH, head = unit % NH;
  const long long pos = __ldcg(reinterpret_cast<const long long *>(pos_p));
  const bf16 *src = qkv + ((size_t)b * NH + head) * 64;
  if (head >= NQ + NKV) {  // value head: 128 bytes into the cache, bits unchanged
    if (lane < 8) {
      const uint4 v = ld_cg16(reinterpret_cast<const uint4 *>(src) + lane);
      reinterpret_cast<uint4 *>(vc + (((size_t)b * NKV + (head - NQ - NKV)) * max_len + pos) * 64)[lane] = v;
    }
    return;
  }
  const bool is_q = head < NQ;
  float x0 = ldcg_bf(src + lane), x1 = ldcg_bf(src + lane + 32);
  const float ss = warp_sum(x0 * x0) + warp_sum(x1 * x1);
  const float rs = rsqrtf(ss / 64 + eps);
  const bf16 *nw = is_q ? qw : kw;
  x0 = rbf(ldg_bf(nw + lane) * rbf(x0 * rs));
  x1 = rbf(ldg_bf(nw + lane + 32) * rbf(x1 * rs));
  const float f = (float)pos * __ldg(inv_freq + lane);
  const float c = rbf(cosf(f) * scaling), s = rbf(sinf(f) * scaling);
  const bf16 o0 = f2bf(rbf(x0 * c) + rbf(-x1 * s));
  const bf16 o1 = f2bf(rbf(x1 * c) + rbf(x0 * s));
  bf16 *dst = is_q ? q_out + ((size_t)b * NQ + head) * 64
                   : kc + (((size_t)b * NKV + (head - NQ)) * max_len + pos) * 64;
  dst[lane] = o0;
  dst[lane + 32] = o1;
}

// ------------------------------------------------------------------ argmax_next
// One block of AM = 1024 threads per sequence: tok[b] = the first index of the largest logit of row b (NaN counts as
// the largest, as torch.argmax), then pos[0] += 1 by block 0 (the reference step's argmax, token copy and position
// increment, src/lfm2opt/runtime.py:286-294, in one launch). Each thread scans 16-byte chunks c = tid, tid + 1024, ...
// in order, keeping the first maximum it meets; (value, index) pairs then meet in a warp butterfly and across warps,
// larger value first, smaller index on ties.
constexpr int AM = 1024;
__device__ __forceinline__ bool am_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}
__global__ void __launch_bounds__(AM) argmax_next_kernel(const bf16 *__restrict__ logits, int V,
                                                         int64_t *__restrict__ tok, int64_t *__restrict__ pos) {
  __shared__ float sv[AM / 32];
  __shared__ int si[AM / 32];
  pdl_trigger();
  pdl_wait();
  const bf16 *row = logits + (size_t)blockIdx.x * V;
  const int t = threadIdx.x, lane = t & 31, wp = t >> 5;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int chunks = V / 8;
  for (int c = t; c < chunks; c += AM) {
    const uint4 u = ld_cg16(reinterpret_cast<const uint4 *>(row) + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = (e & 1) ? bf_hi(w[e >> 1]) : bf_lo(w[e >> 1]);
      if (am_better(v, 8 * c + e, best, bi)) {
        best = v;
        bi = 8 * c + e;
      }
    }
  }
  for (int i = chunks * 8 + t; i < V; i += AM) {  // tail of a row whose length is not a multiple of 8
    const float v = ldcg_bf(row + i);
    if (am_better(v, i, best, bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(v2, i2, best, bi)) {
      best = v2;
      bi = i2;
    }
  }
  if (lane == 0) {
    sv[wp] = best;
    si[wp] = bi;
  }
  __syncthreads();
  if (wp == 0) {
    best = sv[lane];
    bi = si[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(v2, i2, best, bi)) {
        best = v2;
        bi = i2;
      }
    }
    if (lane == 0) {
      tok[blockIdx.x] = bi;
      if (pos && blockIdx.x == 0) pos[0] = __ldcg(reinterpret_cast<const long long *>(pos)) + 1;
    }
  }
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, bool pdl, cudaStream_t st, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  attr->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr->val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

}  // namespace

cudaError_t launch_add_rmsnorm(void *h, const void *y, const void *w, void *x, int rows, int H, float eps, bool pdl,
                               cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(NT), pdl, st, &attr);
  if (y)
    return cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<true>, (bf16 *)h, (const bf16 *)y, (const bf16 *)w, (bf16 *)x,
                              H, eps, (const bf16 *)nullptr, (const int64_t *)nullptr);
  return cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<false>, (bf16 *)h, (const bf16 *)nullptr, (const bf16 *)w,
                            (bf16 *)x, H, eps, (const bf16 *)nullptr, (const int64_t *)nullptr);
}

cudaError_t launch_embed_rmsnorm(const int64_t *tok, const void *embed, const void *w, void *h, void *x, int rows,
                                 int H, float eps, bool pdl, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(NT), pdl, st, &attr);
  return cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<false, true>, (bf16 *)h, (const bf16 *)nullptr, (const bf16 *)w,
                            (bf16 *)x, H, eps, (const bf16 *)embed, tok);
}

cudaError_t launch_argmax_next(const void *logits, int64_t *tok, int64_t *pos, int B, int V, bool pdl,
                               cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg = pdl_cfg(dim3(B), dim3(AM), pdl, st, &attr);
  return cudaLaunchKernelEx(&cfg, argmax_next_kernel, (const bf16 *)logits, V, tok, pos);
}

cudaError_t launch_shortconv_step(const void *bcx, void *state, const void *w, const void *bias, void *y, int B, int H,
                                  bool pdl, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg = pdl_cfg(dim3((H + NT - 1) / NT, B), dim3(NT), pdl, st, &attr);
  return cudaLaunchKernelEx(&cfg, shortconv_step_kernel, (const bf16 *)bcx, (bf16 *)state, (const bf16 *)w,
                            (const bf16 *)bias, (bf16 *)y, H);
}

cudaError_t launch_qk_norm_rope_kv(const void *qkv, const void *qw, const void *kw, const float *inv_freq,
                                   float scaling, const int64_t *pos, void *q_out, void *kc, void *vc, int B, int NQ,
                                   int NKV, int max_len, float eps, bool pdl, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  const long long units = (long long)B * (NQ + 2 * NKV);
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg =
      pdl_cfg(dim3((unsigned)((units + QK_WARPS - 1) / QK_WARPS)), dim3(32 * QK_WARPS), pdl, st, &attr);
  return cudaLaunchKernelEx(&cfg, qk_norm_rope_kv_kernel, (const bf16 *)qkv, (const bf16 *)qw, (const bf16 *)kw,
                            inv_freq, scaling, pos, (bf16 *)q_out, (bf16 *)kc, (bf16 *)vc, B, NQ, NKV, max_len, eps);
}

}  // namespace lfm2q
