// INT4 weight-only decode GEMV: y[b, n] = bf16( sum_g s[n, g] * sum_{k in g} q[n, k] x[b, k] ), q in [-8, 7] with one
// fp32 scale per group of `group` inputs along K.
//
// Reference: gemv_w4_kernel / launch_gemv_w4 (kernels/lfm2_decode.cu:829-945), binding gemv_w4
// (kernels/lfm2_decode.cpp:87-98), packing quantize_int4 (src/lfm2opt/quant.py:22-40): Wp [N, K/2] bytes, element 2j
// in the low nibble and 2j + 1 in the high nibble of byte j, each stored as q + 8; S [N, K / group] fp32.
//
// B200 design: the int8 tensor path of the x-sliced weight-only GEMV (gemv.cu), fed with nibbles. The tokens are
// written once per block into shared memory as exact 3-byte fixed point (x = q_x * 2^E, q_x = sum_s q_s 256^s),
// so every partial sum is an exact int32 and the weights go to the MMA without any conversion to floating point:
//   - a warp step is 16 weight rows x 128 inputs = 64 packed bytes per row (the same 1 KB cp.async ring slots as the
//     int8 GEMV), lane (g, t) holding 16 packed bytes = 32 inputs of rows g and g + 8;
//   - a word of 4 packed bytes (8 inputs) becomes two MMA words with two masks: the low nibbles (the even inputs)
//     as bytes u = q + 8 in 0..15, and the high nibbles (the odd inputs) left in place as bytes 16 u (unsigned
//     int8 MMA operands), accumulated separately and divided by 16 (exactly) at the group's end. The token slices
//     are stored in the matching order (slice_tokens<3, EO = true>), so each MMA pairs every u with its own x;
//   - sum_k q x = sum_k u x - 8 sum_k x: the group sums of every token slice are computed once per block while the
//     tokens are sliced (half-warp reductions), so the
//     +8 is removed exactly from each group's int32 partial, which then folds into the fp32 result with the group's
//     scale: f += (float)(A - 8 C) * s[n, g]. |A - 8 C| < 2^19, so the conversion is exact.
// One 128-input step is one group-128 block; groups of 256, 384, ... fold every group / 128 steps (group must be a
// multiple of 128: one MMA spans inputs from all four 32-input blocks of a step).
#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

constexpr int W4_RING = 6;  // K steps (1 KB of packed weights each) a warp keeps in flight

// unsigned int8 A (the weights' nibbles as bytes) x signed int8 B (the token slices) -> exact int32
__device__ __forceinline__ void mma_u8s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// NT MMA column groups of 8: the 3 slices of 1..2 tokens (NT = 1) or 3..4 tokens (NT = 2)
template <int KS, int NT>
__global__ void __launch_bounds__(GV_THREADS) gemv_w4_kernel(const uint8_t *__restrict__ Wp, const float *__restrict__ S,
                                                             const bf16 *__restrict__ x, bf16 *__restrict__ y, int N,
                                                             int K, int B, int group, int pdl) {
  constexpr int RG = 8 / KS, NSL = 3;
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x W4_RING x 1 KB, sliced tokens, group sums
  __shared__ float red[8 * 16 * 8 * NT];
  __shared__ int e_s[4];
  __shared__ float red_max[4][8];
  if (pdl == 2) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rg = warp / KS, ks = warp % KS;
  const int cols = B * NSL;                 // MMA columns: NSL slices per token
  const int kslice = K / KS;                // inputs per K-slice (a multiple of group)
  const int steps = kslice / 128;
  const int sets = ((N + 15) / 16 + RG - 1) / RG;
  const int xstride = K + 64;
  const int groups = K / group, gsteps = group / 128;
  int8_t *xs = reinterpret_cast<int8_t *>(rings + 8 * W4_RING * 1024);
  int *csum = reinterpret_cast<int *>(xs + (size_t)cols * xstride);  // [K / 128][16]: slice sums per 128 inputs
  const uint32_t slot0 = (uint32_t)__cvta_generic_to_shared(rings + warp * W4_RING * 1024) + g * 64 + t * 16;

  // the weight stream of one set: rows r0 + g and r0 + g + 8, this warp's K-slice, 64 packed bytes per step
  int r0 = (blockIdx.x * RG + rg) * 16;
  const uint8_t *row0 = nullptr, *row1 = nullptr;
  auto set_rows = [&]() {
    row0 = Wp + (size_t)min(r0 + g, N - 1) * (K / 2) + (size_t)ks * (kslice / 2) + t * 16;
    row1 = Wp + (size_t)min(r0 + g + 8, N - 1) * (K / 2) + (size_t)ks * (kslice / 2) + t * 16;
  };
  auto issue = [&](int st) {
    if (st < steps) {
      const uint32_t d = slot0 + (st % W4_RING) * 1024;
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d), "l"(row0 + st * 64) : "memory");
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d + 512), "l"(row1 + st * 64) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // this lane's rows' scales of the K-slice's first group (immutable, like the weights)
  const int g_first = (ks * kslice) / group, g_count = kslice / group;
  auto scales = [&](int gi, float &a, float &b) {
    a = __ldg(S + (size_t)min(r0 + g, N - 1) * groups + gi);
    b = __ldg(S + (size_t)min(r0 + g + 8, N - 1) * groups + gi);
  };
  float sa_n, sb_n;  // the next group's scales, loaded one group ahead of their use
  set_rows();
#pragma unroll
  for (int st = 0; st < W4_RING; ++st) issue(st);  // weights are immutable: stream before the dependency wait
  scales(g_first, sa_n, sb_n);
  if (pdl) pdl_wait();
  slice_tokens<NSL, true>(x, K, B, xs, xstride, e_s, red_max, csum);
  __syncthreads();

  for (int set = blockIdx.x; set < sets; set += gridDim.x) {
    if (set != (int)blockIdx.x) {
      r0 = (set * RG + rg) * 16;
      set_rows();
#pragma unroll
      for (int st = 0; st < W4_RING; ++st) issue(st);
      scales(g_first, sa_n, sb_n);
    }
    const int8_t *xrow = xs + ks * kslice + t * 32;
    const int *cs_col = csum + ((ks * kslice) / 128) * 16;  // this K-slice's first block of slice sums
    // per column group j: (row g, column 8j + 2t), (g, 8j + 2t + 1), (g + 8, 8j + 2t), (g + 8, 8j + 2t + 1)
    float f[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) f[j][e] = 0.f;
    int st = 0, slot = 0;  // step of the K-slice, and its ring slot (st mod W4_RING, kept incrementally)
    for (int gl = 0; gl < g_count; ++gl) {
      const float sa = sa_n, sb = sb_n;  // this group's scales of rows r0 + g, r0 + g + 8 (loaded a group ago)
      if (gl + 1 < g_count) scales(g_first + gl + 1, sa_n, sb_n);
      int acc[NT][4], acc_h[NT][4];  // low nibbles (even inputs): sum u x; high nibbles in place (odd): sum 16 u x
      int cs0[NT], cs1[NT];          // this group's slice sums of the lane's two columns of every group
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        cs0[j] = cs1[j] = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = acc_h[j][e] = 0;
      }
      for (int sg = 0; sg < gsteps; ++sg, ++st) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          if (8 * j + 2 * t < cols) cs0[j] += cs_col[st * 16 + 8 * j + 2 * t];
          if (8 * j + 2 * t + 1 < cols) cs1[j] += cs_col[st * 16 + 8 * j + 2 * t + 1];
        }
        asm volatile("cp.async.wait_group %0;" ::"n"(W4_RING - 1) : "memory");
        const uint32_t d = slot0 + slot * 1024;
        uint4 wa, wb;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(wa.x), "=r"(wa.y), "=r"(wa.z), "=r"(wa.w) : "r"(d)
                     : "memory");
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(wb.x), "=r"(wb.y), "=r"(wb.z), "=r"(wb.w)
                     : "r"(d + 512)
                     : "memory");
        uint4 xv0[NT], xv1[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          xv0[j] = xv1[j] = make_uint4(0u, 0u, 0u, 0u);
          if (g + 8 * j < cols) {
            const int8_t *xr = xrow + (size_t)(g + 8 * j) * xstride + st * 128;
            xv0[j] = *reinterpret_cast<const uint4 *>(xr);
            xv1[j] = *reinterpret_cast<const uint4 *>(xr + 16);
          }
        }
        // the slot just read refills with the step W4_RING ahead
        if (st + W4_RING < steps) {
          asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d), "l"(row0 + (st + W4_RING) * 64)
                       : "memory");
          asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d + 512),
                       "l"(row1 + (st + W4_RING) * 64)
                       : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        slot = slot + 1 == W4_RING ? 0 : slot + 1;
        const uint32_t pa[4] = {wa.x, wa.y, wa.z, wa.w}, pb[4] = {wb.x, wb.y, wb.z, wb.w};
        // packed words j, j + 1 (inputs 8j .. 8j + 15 of the lane's 32): one MMA over their low nibbles with the even
        // inputs' slices, one over their high nibbles (as 16 u, unsigned, no shift) with the odd inputs' slices
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          const uint32_t lo[4] = {pa[j] & 0x0F0F0F0Fu, pb[j] & 0x0F0F0F0Fu, pa[j + 1] & 0x0F0F0F0Fu,
                                  pb[j + 1] & 0x0F0F0F0Fu};
          const uint32_t hi[4] = {pa[j] & 0xF0F0F0F0u, pb[j] & 0xF0F0F0F0u, pa[j + 1] & 0xF0F0F0F0u,
                                  pb[j + 1] & 0xF0F0F0F0u};
#pragma unroll
          for (int c = 0; c < NT; ++c) {
            const uint32_t xw[8] = {xv0[c].x, xv0[c].y, xv0[c].z, xv0[c].w, xv1[c].x, xv1[c].y, xv1[c].z, xv1[c].w};
            mma_u8s8_16832(acc[c], lo, xw[2 * j], xw[2 * j + 2]);
            mma_u8s8_16832(acc_h[c], hi, xw[2 * j + 1], xw[2 * j + 3]);
          }
        }
      }
      // the group ends: sum u x = acc + acc_h / 16 (exact), remove the +8, fold with the group's scales
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        f[j][0] = __fmaf_rn((float)(acc[j][0] + (acc_h[j][0] >> 4) - 8 * cs0[j]), sa, f[j][0]);
        f[j][1] = __fmaf_rn((float)(acc[j][1] + (acc_h[j][1] >> 4) - 8 * cs1[j]), sa, f[j][1]);
        f[j][2] = __fmaf_rn((float)(acc[j][2] + (acc_h[j][2] >> 4) - 8 * cs0[j]), sb, f[j][2]);
        f[j][3] = __fmaf_rn((float)(acc[j][3] + (acc_h[j][3] >> 4) - 8 * cs1[j]), sb, f[j][3]);
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (pdl == 1 && set + (int)gridDim.x >= sets) pdl_trigger();
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[((rg * KS + ks) * 16 + frag_row(lane, e)) * 8 * NT + frag_tok(lane, j, e)] = f[j][e];
    __syncthreads();
    for (int i = threadIdx.x; i < RG * 16 * B; i += GV_THREADS) {
      const int b = i % B, rr = (i / B) % 16, g2 = i / (16 * B);
      const int n = (set * RG + g2) * 16 + rr;
      if (n >= N) continue;
      float v = 0.f;
#pragma unroll
      for (int sl = NSL - 1; sl >= 0; --sl) {
        float a = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < KS; ++s2) a += red[((g2 * KS + s2) * 16 + rr) * 8 * NT + b * NSL + sl];
        v = __fmaf_rn(v, 256.f, a);
      }
      y[(size_t)b * N + n] = f2bf(ldexpf(v, e_s[b]));
    }
    __syncthreads();
  }
}

// dynamic shared memory: rings, the sliced tokens (3 slices per token), the slice sums
size_t w4_smem(int K, int B) {
  return (size_t)8 * W4_RING * 1024 + (size_t)B * 3 * (K + 64) + (size_t)(K / 128) * 16 * sizeof(int);
}

std::mutex g_w4_mu;
std::set<std::pair<const void *, int>> g_w4_attr;

template <int KS, int NT>
cudaError_t w4_launch(const uint8_t *Wp, const float *S, const bf16 *x, bf16 *y, int N, int K, int B, int group,
                      bool pdl, int trigger, cudaStream_t st) {
  auto kern = gemv_w4_kernel<KS, NT>;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_w4_mu);
    const auto key = std::make_pair(reinterpret_cast<const void *>(kern), dev);
    if (!g_w4_attr.count(key)) {
      if (const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024))
        return e;
      g_w4_attr.insert(key);
    }
  }
  const size_t dyn = w4_smem(K, B);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GV_THREADS, dyn) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int rg = 8 / KS, sets = ((N + 15) / 16 + rg - 1) / rg;
  const int resident = per_sm * device_sm_count();  // one wave: the grid strides over the sets
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sets < resident ? sets : resident);
  cfg.blockDim = dim3(GV_THREADS);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, Wp, S, x, y, N, K, B, group, pdl ? trigger : 0);
}

template <int NT>
cudaError_t w4_ks(int ks, const uint8_t *Wp, const float *S, const bf16 *x, bf16 *y, int N, int K, int B, int group,
                  bool pdl, int trigger, cudaStream_t st) {
  switch (ks) {
    case 1: return w4_launch<1, NT>(Wp, S, x, y, N, K, B, group, pdl, trigger, st);
    case 2: return w4_launch<2, NT>(Wp, S, x, y, N, K, B, group, pdl, trigger, st);
    case 4: return w4_launch<4, NT>(Wp, S, x, y, N, K, B, group, pdl, trigger, st);
    default: return w4_launch<8, NT>(Wp, S, x, y, N, K, B, group, pdl, trigger, st);
  }
}

}  // namespace

// Slices per token of the INT4 GEMV: 3 for 1..4 tokens if its shared memory fits, else 0.
int gemv_w4_slices(int K, int B) {
  if (B < 1 || B > 4 || w4_smem(K, B) > 160 * 1024 || K > 8 * GV_THREADS * XS_CH / B) return 0;
  return 3;
}

cudaError_t launch_gemv_w4(const uint8_t *Wp, const float *S, const void *x, void *y, int N, int K, int group, int B,
                           bool pdl, int trigger, cudaStream_t st) {
  if (N <= 0 || B <= 0) return cudaSuccess;
  if (!gemv_w4_slices(K, B)) return cudaErrorInvalidValue;
  // K-slices per 16-row group: the fewest that give ~8 warps per SM, each slice a whole number of groups
  const long groups16 = (N + 15) / 16, target = 8L * device_sm_count();
  int ks = 1;
  while (ks < 8 && groups16 * ks < target && (K / (2 * ks)) % group == 0) ks *= 2;
  return B * 3 <= 8 ? w4_ks<1>(ks, Wp, S, (const bf16 *)x, (bf16 *)y, N, K, B, group, pdl, trigger, st)
                    : w4_ks<2>(ks, Wp, S, (const bf16 *)x, (bf16 *)y, N, K, B, group, pdl, trigger, st);
}

}  // namespace lfm2q
