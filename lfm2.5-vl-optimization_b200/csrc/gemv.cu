// Weight-only decode GEMV: y[b, n] = bf16( (sum_k W[n, k] * x[b, k]) * scale[n] ), W int8 (or bf16) [N, K]
// row-major, x / y bf16, fp32 accumulation, for 1..16 tokens per launch (more in chunks of 16).
//
// Reference: kernels/lfm2_decode.cu:576-661 (gemv_direct_kernel), :666-714 (gemv_dispatch / launch_gemv),
// binding kernels/lfm2_decode.cpp:73-85; fused epilogues kernels/lfm2_decode.cu:724-827 (gemv_epi_kernel).
//
// B200 design. The op is HBM-bound: every weight byte is read once, so the kernel must keep ~40 KB of loads in
// flight per SM and spend few ALU instructions per byte (at 85 % of 6.5 TB/s there are ~6 lane-instructions per
// weight). A warp owns a 16-row group of W and a K-slice; each lane streams two 16-byte chunks per 64-wide K step
// (rows g and g + 8 of the group), converts the int8 codes exactly to bf16 in registers (exponent-bias trick:
// byte + 128 placed in the mantissa of 2^23, one FADD removes the bias; the small integers are exact in bf16),
// and feeds warp-level bf16 MMAs (m16n8k16, fp32 accumulation) with the tokens on the N side. The MMA makes the
// cost per weight independent of the batch (8 tokens per MMA). The K order inside a 64-wide step is permuted
// identically for W and x (lane t, step s take physical k 16t+4s..16t+4s+3), which leaves the dot product
// unchanged. Small N is split over K-slices (KS warps per row group) whose fp32 partials meet in shared memory
// and are summed in a fixed order, so results are deterministic.
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <utility>

#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.h"

namespace lfm2q {
namespace {

// Plain GEMV. Block = RG row groups x KS K-slices (RG * KS == 8 warps); blocks walk the row-group sets in a grid
// stride (grid = min(sets, resident blocks)), so large N runs in one wave with balanced work.
template <typename WT, int NT, int KS>
__global__ void __launch_bounds__(GV_THREADS) gemv_kernel(const WT *__restrict__ W, const float *__restrict__ scale,
                                                          const bf16 *__restrict__ x, bf16 *__restrict__ y, int N, int K,
                                                          int B, int pdl) {
  constexpr int RG = 8 / KS;
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x GV_RING x 1 KB
  __shared__ float red[(KS > 1) ? RG * KS * 16 * 8 * NT : 1];
  if (pdl == 2) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = warp / KS, ks = warp % KS;
  const int kslice = K / KS;
  const int sets = ((N + 15) / 16 + RG - 1) / RG;
  for (int set = blockIdx.x; set < sets; set += gridDim.x) {
    const int r0 = (set * RG + rg) * 16;
    float acc[NT][4];
    warp_gemv<WT, NT>(W, x, N, K, B, r0, ks * kslice, (ks + 1) * kslice, acc, rings + warp * GV_RING * 1024,
                      pdl != 0 && set == blockIdx.x);
    // the block's weights are consumed: let the next kernel start streaming its own (pdl == 2: done at the start)
    if (pdl == 1 && set + (int)gridDim.x >= sets) pdl_trigger();
    if (KS == 1) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = r0 + frag_row(lane, e), b = frag_tok(lane, j, e);
          if (n < N && b < B) y[(size_t)b * N + n] = f2bf(scale ? acc[j][e] * scale[n] : acc[j][e]);
        }
      continue;
    }
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[((rg * KS + ks) * 16 + frag_row(lane, e)) * 8 * NT + frag_tok(lane, j, e)] = acc[j][e];
    __syncthreads();
    for (int i = threadIdx.x; i < RG * 16 * 8 * NT; i += GV_THREADS) {
      const int b = i % (8 * NT), rr = (i / (8 * NT)) % 16, g2 = i / (16 * 8 * NT);
      const int n = (set * RG + g2) * 16 + rr;
      if (n >= N || b >= B) continue;
      float v = 0.f;
#pragma unroll
      for (int s = 0; s < KS; ++s) v += red[((g2 * KS + s) * 16 + rr) * 8 * NT + b];
      y[(size_t)b * N + n] = f2bf(scale ? v * scale[n] : v);
    }
    __syncthreads();
  }
}

// A8 decode GEMV: y[b, n] = bf16(act(((float)(xq[b] . W[n]) * sx[b]) * sw[n] + bias[n])), the per-token W8A8
// epilogue of gemm_i8 on an exact int32 sum, for 1..16 tokens per launch. Block = RG row groups x KS K-slices;
// the K-slices' int32 partials are added in shared memory (exact, so the result does not depend on the split).
// FUSEQ: x is bf16 [B, K]; every block first quantizes it per token into shared memory (rows padded by 64 bytes so
// the fragment loads are bank-conflict-free), with the quant_rows arithmetic (same scale, same rounding), so one
// launch computes Int8Linear's per-token W8A8 result for a few tokens.
template <int NT, int KS, bool GELU, bool FUSEQ>
__global__ void __launch_bounds__(GV_THREADS) gemv_a8_kernel(const int8_t *__restrict__ W, const float *__restrict__ sw,
                                                             const int8_t *__restrict__ xq_g, const float *__restrict__ sx_g,
                                                             const bf16 *__restrict__ xbf, const bf16 *__restrict__ bias,
                                                             bf16 *__restrict__ y, int N, int K, int B, int pdl) {
  constexpr int RG = 8 / KS;
  extern __shared__ __align__(128) uint8_t rings[];
  __shared__ int red[(KS > 1) ? RG * KS * 16 * 8 * NT : 1];
  __shared__ float sx_s[16];
  if (pdl == 2) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int8_t *xq = xq_g;
  const float *sx = sx_g;
  int xstride = K;
  const int rg = warp / KS, ks = warp % KS;
  const int kslice = K / KS;
  const int sets = ((N + 15) / 16 + RG - 1) / RG;
  {
    // stream the first set's weights before anything waits on the previous kernel
    int dummy[NT][4];
    warp_gemv_a8<NT>(W, xq, xstride, N, K, B, (blockIdx.x * RG + rg) * 16, ks * kslice, (ks + 1) * kslice, dummy,
                     rings + warp * GV_RING * 1024, false, 1);
  }
  if (FUSEQ) {
    int8_t *xs = reinterpret_cast<int8_t *>(rings + 8 * GV_RING * 1024);
    xstride = K + 64;
    xq = xs;
    sx = sx_s;
    // weights first (the rings are filled inside warp_gemv_a8), so here only x: warp w quantizes tokens w, w + 8
    if (pdl) pdl_wait();
    for (int b = warp; b < B; b += 8) {
      const uint4 *xr = reinterpret_cast<const uint4 *>(xbf + (size_t)b * K);
      uint32_t m2 = 0;
      for (int c = lane; c < K / 8; c += 32) {
        const uint4 v = ld_cg16(xr + c);
        m2 = __vmaxu2(m2, __vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu));
        m2 = __vmaxu2(m2, __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
      }
      const float sc = __fdiv_rn(fmaxf(warp_max(fmaxf(bf_lo(m2), bf_hi(m2))), 1e-8f), 127.f);
      const float rinv = __frcp_rn(sc);
      if (lane == 0) sx_s[b] = sc;
      for (int c = lane; c < K / 8; c += 32) {
        const uint4 v = ld_cg16(xr + c);
        const uint32_t o0 = pack_sums4(q8r2(make_float2(bf_lo(v.x), bf_hi(v.x)), sc, rinv),
                                       q8r2(make_float2(bf_lo(v.y), bf_hi(v.y)), sc, rinv));
        const uint32_t o1 = pack_sums4(q8r2(make_float2(bf_lo(v.z), bf_hi(v.z)), sc, rinv),
                                       q8r2(make_float2(bf_lo(v.w), bf_hi(v.w)), sc, rinv));
        *reinterpret_cast<uint2 *>(xs + (size_t)b * xstride + c * 8) = make_uint2(o0, o1);
      }
    }
    __syncthreads();
  }
  for (int set = blockIdx.x; set < sets; set += gridDim.x) {
    const int r0 = (set * RG + rg) * 16;
    int acc[NT][4];
    warp_gemv_a8<NT>(W, xq, xstride, N, K, B, r0, ks * kslice, (ks + 1) * kslice, acc,
                     rings + warp * GV_RING * 1024, !FUSEQ && pdl != 0 && set == blockIdx.x,
                     set == blockIdx.x ? 2 : 0);
    if (pdl == 1 && set + (int)gridDim.x >= sets) pdl_trigger();
    if (KS == 1) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = r0 + frag_row(lane, e), b = frag_tok(lane, j, e);
          if (n < N && b < B)
            y[(size_t)b * N + n] =
                f2bf(epi_token<GELU>(acc[j][e], FUSEQ ? sx[b] : __ldcg(sx + b), sw[n], bias ? bf2f(bias[n]) : 0.f));
        }
      continue;
    }
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[((rg * KS + ks) * 16 + frag_row(lane, e)) * 8 * NT + frag_tok(lane, j, e)] = acc[j][e];
    __syncthreads();
    for (int i = threadIdx.x; i < RG * 16 * 8 * NT; i += GV_THREADS) {
      const int b = i % (8 * NT), rr = (i / (8 * NT)) % 16, g2 = i / (16 * 8 * NT);
      const int n = (set * RG + g2) * 16 + rr;
      if (n >= N || b >= B) continue;
      int v = 0;
#pragma unroll
      for (int s2 = 0; s2 < KS; ++s2) v += red[((g2 * KS + s2) * 16 + rr) * 8 * NT + b];
      y[(size_t)b * N + n] = f2bf(epi_token<GELU>(v, FUSEQ ? sx[b] : __ldcg(sx + b), sw[n], bias ? bf2f(bias[n]) : 0.f));
    }
    __syncthreads();
  }
}

// Weight-only GEMV on the int8 tensor path ("x-sliced"), for 1..4 tokens. Each token's bf16 activations are written
// exactly as NSL = 3 byte fixed point, q = x * 2^-E with E from the token's absmax so that |q| < 2^22, and q is split
// into 3 balanced signed bytes, q = sum_s q_s 256^s. The bytes of token b are the MMA columns 3 b + s (NT groups of 8
// columns: 1 up to 2 tokens, 2 up to 4), so the int8 weights feed m16n8k32 s8 MMAs unconverted (the A8 inner loop)
// and every partial sum A_s = sum_k W[n, k] q_s[k] is an exact int32. y[b, n] = bf16( ((sum_s 256^s A_s) * scale[n])
// * 2^E ), combined in fp32. Every bf16 element within 2^14 of the token's absmax is represented exactly (8
// significant bits above 2^E) and smaller ones to within 2^(E-1) <= 2^-22 of the absmax, so the result is the exact
// dot product rounded, at least as accurate as the reference's fp32 accumulation (kernels/lfm2_decode.cu:576-661)
// also with outlier channels. Every block slices x into shared memory after its first weights are in flight (rows of
// K + 64 bytes, bank-conflict-free fragment loads).
constexpr int XS_NSL = 3;
template <int KS, int NT, int RING>
__global__ void __launch_bounds__(GV_THREADS) gemv_xs_kernel(const int8_t *__restrict__ W, const float *__restrict__ scale,
                                                             const bf16 *__restrict__ x, bf16 *__restrict__ y, int N,
                                                             int K, int B, int pdl) {
  constexpr int RG = 8 / KS, NSL = XS_NSL;
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x RING x 1 KB, then the sliced tokens
  __shared__ int red[RG * KS * 16 * 8 * NT];
  __shared__ int e_s[4];
  __shared__ float red_max[4][8];
  if (pdl == 2) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = warp / KS, ks = warp % KS;
  const int kslice = K / KS;
  const int sets = ((N + 15) / 16 + RG - 1) / RG;
  const int xstride = K + 64;
  int8_t *xs = reinterpret_cast<int8_t *>(rings + 8 * RING * 1024);
  {
    // stream the first set's weights before anything waits on the previous kernel
    int dummy[NT][4];
    warp_gemv_a8<NT, RING>(W, xs, xstride, N, K, B * NSL, (blockIdx.x * RG + rg) * 16, ks * kslice, (ks + 1) * kslice,
                           dummy, rings + warp * RING * 1024, false, 1);
  }
  if (pdl) pdl_wait();
  slice_tokens<NSL>(x, K, B, xs, xstride, e_s, red_max);
  __syncthreads();
  for (int set = blockIdx.x; set < sets; set += gridDim.x) {
    const int r0 = (set * RG + rg) * 16;
    int acc[NT][4];
    warp_gemv_a8<NT, RING>(W, xs, xstride, N, K, B * NSL, r0, ks * kslice, (ks + 1) * kslice, acc,
                           rings + warp * RING * 1024, false, set == blockIdx.x ? 2 : 0);
    if (pdl == 1 && set + (int)gridDim.x >= sets) pdl_trigger();
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[((rg * KS + ks) * 16 + frag_row(lane, e)) * 8 * NT + frag_tok(lane, j, e)] = acc[j][e];
    __syncthreads();
    for (int i = threadIdx.x; i < RG * 16 * B; i += GV_THREADS) {
      const int b = i % B, rr = (i / B) % 16, g2 = i / (16 * B);
      const int n = (set * RG + g2) * 16 + rr;
      if (n >= N) continue;
      float f = 0.f;
#pragma unroll
      for (int sl = NSL - 1; sl >= 0; --sl) {
        int a = 0;
#pragma unroll
        for (int s2 = 0; s2 < KS; ++s2) a += red[((g2 * KS + s2) * 16 + rr) * 8 * NT + b * NSL + sl];
        f = __fmaf_rn(f, 256.f, (float)a);
      }
      y[(size_t)b * N + n] = f2bf(ldexpf(__fmul_rn(f, scale[n]), e_s[b]));
    }
    __syncthreads();
  }
}

// x-sliced GEMV with deep weight prefetch, for decode chains. Same arithmetic as gemv_xs_kernel (the tokens sliced
// into exact fixed-point bytes, exact int32 partials, the same fp32 combination), so the values are identical; the
// schedule differs. Grid = at most one block per SM. Each warp's steps over all of its sets (row group x K-slice)
// run through ONE ring of R 1 KB slots that continues across set boundaries, and the first R steps (up to 96 KB
// per block) are requested before the dependency wait. With pdl == 2 the dependent launch is triggered at the
// start; the block's shared memory stays below half an SM's, so the next GEMV's blocks are resident beside this one
// and fill their own rings while this one waits, slices and computes. The weight stream of consecutive GEMVs thus
// overlaps, instead of restarting from an empty pipe after every dependency (what bounds a chain of small GEMVs).
template <int KS, int NT, int R>
__global__ void __launch_bounds__(GV_THREADS, 2) gemv_deep_kernel(const int8_t *__restrict__ W,
                                                                   const float *__restrict__ scale,
                                                                   const bf16 *__restrict__ x, bf16 *__restrict__ y,
                                                                   int N, int K, int B, int pdl) {
  constexpr int RG = 8 / KS, NSL = XS_NSL;
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x R x 1 KB, then the sliced tokens
  __shared__ int red[RG * KS * 16 * 8 * NT];
  __shared__ int e_s[4];
  __shared__ float red_max[4][8];
  if (pdl == 2) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rg = warp / KS, ks = warp % KS;
  const int kslice = K / KS, nst = kslice / 64;
  const int sets = ((N + 15) / 16 + RG - 1) / RG;
  const int my_sets = (int)blockIdx.x < sets ? (sets - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_sets * nst;  // this warp's 64-wide K steps, over all of its sets
  const int xstride = K + 64;
  int8_t *xs = reinterpret_cast<int8_t *>(rings + 8 * R * 1024);
  const uint32_t slot0 = (uint32_t)__cvta_generic_to_shared(rings + warp * R * 1024) + g * 64 + t * 16;

  // issue cursor: the next step to request is step ist of set iset; rows g and g + 8 of its row group
  int iset = blockIdx.x, ist = 0;
  const int8_t *p0 = W, *p1 = W;
  auto rows_of = [&](int set) {
    const int r0 = (set * RG + rg) * 16;
    p0 = W + (size_t)min(r0 + g, N - 1) * K + ks * kslice + t * 16;
    p1 = W + (size_t)min(r0 + g + 8, N - 1) * K + ks * kslice + t * 16;
  };
  if (iset < sets) rows_of(iset);
  auto issue = [&](int slot) {
    if (iset < sets) {
      const uint32_t d = slot0 + slot * 1024;
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d), "l"(p0 + ist * 64) : "memory");
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d + 512), "l"(p1 + ist * 64) : "memory");
      if (++ist == nst) {
        ist = 0;
        iset += gridDim.x;
        if (iset < sets) rows_of(iset);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto lds = [&](int slot, uint4 &w0, uint4 &w1) {
    const uint32_t d = slot0 + slot * 1024;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w0.x), "=r"(w0.y), "=r"(w0.z), "=r"(w0.w) : "r"(d)
                 : "memory");
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w1.x), "=r"(w1.y), "=r"(w1.z), "=r"(w1.w)
                 : "r"(d + 512)
                 : "memory");
  };
  // MMA column c = g + 8 j holds token c / NSL, slice c % NSL (columns past B * NSL are zero)
  const int8_t *xrow = xs + ks * kslice + t * 16;
  auto ldx = [&](int st, uint4 (&xw)[NT]) {
#pragma unroll
    for (int j = 0; j < NT; ++j)
      xw[j] = g + 8 * j < B * NSL ? *reinterpret_cast<const uint4 *>(xrow + (size_t)(g + 8 * j) * xstride + st * 64)
                                  : make_uint4(0u, 0u, 0u, 0u);
  };

#pragma unroll
  for (int s = 0; s < R; ++s) issue(s);  // weights are immutable: requested before the dependency wait
  // the weight-row scales the epilogue items i = tid, tid + 256 of a set need, loaded a set ahead (the first set's
  // before the dependency wait), so no global load sits on the epilogue's critical path
  float sc[2] = {0.f, 0.f};
  auto scales_of = [&](int set) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = threadIdx.x + k * GV_THREADS;
      const int n = (set * RG + i / (16 * B)) * 16 + (i / B) % 16;
      if (set < sets && i < RG * 16 * B && n < N) sc[k] = __ldg(scale + n);
    }
  };
  scales_of(blockIdx.x);
  if (pdl) pdl_wait();
  slice_tokens<NSL>(x, K, B, xs, xstride, e_s, red_max);
  __syncthreads();

  uint4 wc0, wc1, xc[NT], wn0, wn1, xn[NT];
  asm volatile("cp.async.wait_group %0;" ::"n"(R - 1) : "memory");
  if (total > 0) {
    lds(0, wc0, wc1);
    ldx(0, xc);
  }
  int acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0;
  int slot = 0, st = 0, set = blockIdx.x;
  for (int c = 0; c < total; ++c) {
    const int nslot = slot + 1 == R ? 0 : slot + 1;
    const int nstp = st + 1 == nst ? 0 : st + 1;
    if (c + 1 < total) {
      asm volatile("cp.async.wait_group %0;" ::"n"(R - 2) : "memory");
      lds(nslot, wn0, wn1);
      ldx(nstp, xn);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint32_t a[4] = {(&wc0.x)[2 * s], (&wc1.x)[2 * s], (&wc0.x)[2 * s + 1], (&wc1.x)[2 * s + 1]};
#pragma unroll
      for (int j = 0; j < NT; ++j) mma_s8_16832(acc[j], a, (&xc[j].x)[2 * s], (&xc[j].x)[2 * s + 1]);
    }
    issue(slot);  // step c's slot (its data is in registers) takes step c + R
    slot = nslot;
    wc0 = wn0;
    wc1 = wn1;
#pragma unroll
    for (int j = 0; j < NT; ++j) xc[j] = xn[j];
    st = nstp;
    if (st == 0) {  // the set is complete: K-slices meet in shared memory, then the epilogue of gemv_xs_kernel
      if (pdl == 1 && set + (int)gridDim.x >= sets) pdl_trigger();
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          red[((rg * KS + ks) * 16 + frag_row(lane, e)) * 8 * NT + frag_tok(lane, j, e)] = acc[j][e];
          acc[j][e] = 0;
        }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + k * GV_THREADS;
        if (i >= RG * 16 * B) break;
        const int b = i % B, rr = (i / B) % 16, g2 = i / (16 * B);
        const int n = (set * RG + g2) * 16 + rr;
        if (n >= N) continue;
        float f = 0.f;
#pragma unroll
        for (int sl = NSL - 1; sl >= 0; --sl) {
          int a = 0;
#pragma unroll
          for (int s2 = 0; s2 < KS; ++s2) a += red[((g2 * KS + s2) * 16 + rr) * 8 * NT + b * NSL + sl];
          f = __fmaf_rn(f, 256.f, (float)a);
        }
        y[(size_t)b * N + n] = f2bf(ldexpf(__fmul_rn(f, sc[k]), e_s[b]));
      }
      __syncthreads();
      set += gridDim.x;
      scales_of(set);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Elementwise epilogue of the fused decode GEMVs on the NR bf16 GEMV values of output index n0 + threadIdx.x
// (threads 0..15; kernels/lfm2_decode.cu:770-805).
template <int NR, int EPI>
__device__ __forceinline__ void epi_tail(const float (&part)[NR][16], bf16 *__restrict__ y, int S, int n0,
                                         bf16 *__restrict__ state, const bf16 *__restrict__ cw,
                                         const bf16 *__restrict__ cbias) {
  if (threadIdx.x >= 16) return;
  const int m = n0 + threadIdx.x;
  if (m >= S) return;
  if (EPI == 0) {
    const float g = part[0][threadIdx.x], u = part[1][threadIdx.x];
    y[m] = f2bf(rbf(g / (1.f + __expf(-g))) * u);
  } else {
    const float bx = rbf(part[0][threadIdx.x] * part[NR - 1][threadIdx.x]);
    bf16 *st = state + (size_t)m * 3;
    const float s1 = bf2f(st[1]), s2 = bf2f(st[2]);
    st[0] = st[1];
    st[1] = st[2];
    st[2] = f2bf(bx);
    // conv = w0 * s1 + w1 * s2 + w2 * bx (+ bias), evaluated left to right with explicit fp32 roundings
    float acc2 = __fmul_rn(bf2f(cw[m * 3 + 0]), s1);
    acc2 = __fadd_rn(acc2, __fmul_rn(bf2f(cw[m * 3 + 1]), s2));
    acc2 = __fadd_rn(acc2, __fmul_rn(bf2f(cw[m * 3 + 2]), bx));
    if (cbias) acc2 = __fadd_rn(acc2, bf2f(cbias[m]));
    y[m] = f2bf(part[1][threadIdx.x] * rbf(acc2));
  }
}

// Batch-1 GEMV over NR stacked [S, K] blocks of W followed by an elementwise epilogue on the NR values of one
// output index (kernels/lfm2_decode.cu:718-805):
//   EPI 0, NR 2 (w1 | w3):         y[n] = bf16( bf16(silu(g)) * u ),  g, u = the bf16 the plain GEMV would store
//   EPI 1, NR 3 (in_proj B|C|x):   bx = bf16(B * x); conv state shift; y = bf16(C * bf16(w . window + bias))
// Block = NR parts x 8/NR... laid out as 2 row groups x 4 K-slices (NR=2) or 2 row groups x ... see host dispatch:
// the block covers 16 output indices; warp w handles part w / KSE and K-slice w % KSE.
template <typename WT, int NR, int EPI>
__global__ void __launch_bounds__(GV_THREADS) gemv_epi_kernel(const WT *__restrict__ W, const float *__restrict__ scale,
                                                              const bf16 *__restrict__ x, bf16 *__restrict__ y, int S,
                                                              int K, bf16 *__restrict__ state,
                                                              const bf16 *__restrict__ cw,
                                                              const bf16 *__restrict__ cbias, int pdl) {
  constexpr int KSE = (NR == 2) ? 4 : 2;  // K-slices per part (NR * KSE <= 8 warps)
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x GV_RING x 1 KB
  __shared__ float red[NR][KSE][16];
  __shared__ float part[NR][16];
  if (pdl) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = warp / KSE, ks = warp % KSE;
  const int n0 = blockIdx.x * 16;
  if (p < NR) {
    const int kslice = K / KSE;
    float acc[1][4];
    // rows of part p: p * S + n0 .. ; clamp inside the part so the loads stay in W
    const WT *Wp = W + (size_t)p * S * K;
    warp_gemv<WT, 1>(Wp, x, S, K, 1, n0, ks * kslice, (ks + 1) * kslice, acc, rings + warp * GV_RING * 1024, pdl != 0);
    // token 0 lives in lanes with t == 0, element e & 1 == 0
    if ((lane & 3) == 0) {
      red[p][ks][frag_row(lane, 0)] = acc[0][0];
      red[p][ks][frag_row(lane, 2)] = acc[0][2];
    }
  } else if (pdl) {
    pdl_wait();
  }
  __syncthreads();
  if (threadIdx.x < NR * 16) {
    const int pp = threadIdx.x / 16, r = threadIdx.x % 16, n = n0 + r;
    float v = 0.f;
#pragma unroll
    for (int s = 0; s < KSE; ++s) v += red[pp][s][r];
    part[pp][r] = (n < S) ? rbf(scale ? v * scale[pp * S + n] : v) : 0.f;
  }
  __syncthreads();
  epi_tail<NR, EPI>(part, y, S, n0, state, cw, cbias);
}

// gemv_epi on the x-sliced int8 path (see gemv_xs_kernel): the token is sliced into 3 exact fixed-point bytes in
// shared memory, each warp's int32 slice sums are exact, so the NR bf16 values equal the plain GEMV's outputs
// whatever the K-slicing. Same block layout and epilogue as gemv_epi_kernel.
template <int NR, int EPI, int RING>
__global__ void __launch_bounds__(GV_THREADS) gemv_epi_xs_kernel(const int8_t *__restrict__ W,
                                                                 const float *__restrict__ scale,
                                                                 const bf16 *__restrict__ x, bf16 *__restrict__ y,
                                                                 int S, int K, bf16 *__restrict__ state,
                                                                 const bf16 *__restrict__ cw,
                                                                 const bf16 *__restrict__ cbias, int pdl) {
  constexpr int KSE = (NR == 2) ? 4 : 2;
  constexpr int NSL = 3;
  extern __shared__ __align__(128) uint8_t rings[];  // 8 warps x RING x 1 KB, then the sliced token
  __shared__ int red[NR][KSE][16][NSL];
  __shared__ float part[NR][16];
  __shared__ int e_s[4];
  __shared__ float red_max[4][8];
  if (pdl) pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = warp / KSE, ks = warp % KSE;
  const int n0 = blockIdx.x * 16;
  const int kslice = K / KSE;
  const int xstride = K + 64;
  int8_t *xs = reinterpret_cast<int8_t *>(rings + 8 * RING * 1024);
  const int8_t *Wp = W + (size_t)(p < NR ? p : 0) * S * K;
  uint8_t *ring = rings + warp * RING * 1024;
  if (p < NR) {
    int dummy[1][4];
    warp_gemv_a8<1, RING>(Wp, xs, xstride, S, K, NSL, n0, ks * kslice, (ks + 1) * kslice, dummy, ring, false, 1);
  }
  if (pdl) pdl_wait();
  slice_tokens<NSL>(x, K, 1, xs, xstride, e_s, red_max);
  __syncthreads();
  if (p < NR) {
    int acc[1][4];
    warp_gemv_a8<1, RING>(Wp, xs, xstride, S, K, NSL, n0, ks * kslice, (ks + 1) * kslice, acc, ring, false, 2);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = frag_tok(lane, 0, e);
      if (col < NSL) red[p][ks][frag_row(lane, e)][col] = acc[0][e];
    }
  }
  __syncthreads();
  if (threadIdx.x < NR * 16) {
    const int pp = threadIdx.x / 16, r = threadIdx.x % 16, n = n0 + r;
    float f = 0.f;
#pragma unroll
    for (int sl = NSL - 1; sl >= 0; --sl) {
      int a = 0;
#pragma unroll
      for (int s2 = 0; s2 < KSE; ++s2) a += red[pp][s2][r][sl];
      f = __fmaf_rn(f, 256.f, (float)a);
    }
    part[pp][r] = (n < S) ? rbf(ldexpf(__fmul_rn(f, scale[pp * S + n]), e_s[0])) : 0.f;
  }
  __syncthreads();
  epi_tail<NR, EPI>(part, y, S, n0, state, cw, cbias);
}

constexpr int GV_DYN_SMEM = 8 * GV_RING * 1024;
constexpr int XS_RING = 6;  // ring depth of the x-sliced kernels (K steps of 1 KB per warp)
constexpr int EPI_RING = 5;  // ... of the SwiGLU epilogue GEMV
constexpr int CONV_RING = 10;  // ... of the short-conv epilogue GEMV
constexpr int GV_X_SMEM_MAX = 64 * 1024;  // fused-quantization A8 GEMV: B * (K + 64) bytes of int8 tokens
std::atomic<bool> g_early_trigger{false};
// 0 (default): deep-prefetch x-sliced kernel for 1-2 tokens, ring x-sliced kernel for 3-4 tokens from 8 M weights,
// else the bf16-MMA path; 1: always the bf16-MMA path; 2: the deep kernel wherever the slices fit; 4: the ring
// x-sliced kernel from 8 M weights (the deep kernel's predecessor, for comparisons)
std::atomic<int> g_gemv_impl{0};
std::atomic<bool> g_deep_late{false};  // deep kernel: trigger the dependent launch after the last set, not at start

// (kernel, device) pairs whose dynamic shared memory limit has been raised
std::mutex g_attr_mu;
std::set<std::pair<const void *, int>> g_attr_done;

// Raise the kernel's dynamic shared memory limit (rings + token buffer) once per device.
template <typename KernelT>
cudaError_t ensure_smem_attr(KernelT kernel) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_attr_mu);
  const auto key = std::make_pair(reinterpret_cast<const void *>(kernel), dev);
  if (!g_attr_done.count(key)) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_DYN_SMEM + GV_X_SMEM_MAX);
    if (e != cudaSuccess) return e;
    g_attr_done.insert(key);
  }
  return cudaSuccess;
}

// Blocks of `kernel` with `dyn_smem` bytes of dynamic shared memory that fit on the device at once (cached).
std::mutex g_occ_mu;
std::map<std::tuple<const void *, size_t, int>, int> g_occ;
template <typename KernelT>
int resident_blocks(KernelT kernel, size_t dyn_smem) {
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<const void *>(kernel), dyn_smem, dev);
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    const auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  int per_sm = 0;
  if (ensure_smem_attr(kernel) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, GV_THREADS, dyn_smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int n = per_sm * device_sm_count();
  std::lock_guard<std::mutex> lk(g_occ_mu);
  g_occ[key] = n;
  return n;
}

// Launch with `dyn_smem` bytes of dynamic shared memory (per-warp rings, then any token buffer) and, when asked,
// Programmatic Dependent Launch.
template <typename KernelT, typename... Args>
cudaError_t launch_dyn(KernelT kernel, dim3 grid, dim3 block, bool pdl, cudaStream_t st, size_t dyn_smem, Args... args) {
  if (const cudaError_t e = ensure_smem_attr(kernel)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = dyn_smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Launch with the default rings (GV_RING steps per warp) plus `extra_smem` bytes.
template <typename KernelT, typename... Args>
cudaError_t launch_ex(KernelT kernel, dim3 grid, dim3 block, bool pdl, cudaStream_t st, size_t extra_smem,
                      Args... args) {
  return launch_dyn(kernel, grid, block, pdl, st, GV_DYN_SMEM + extra_smem, args...);
}

template <typename WT, int NT>
cudaError_t gemv_ks(const WT *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int B, int ks, bool pdl,
                    cudaStream_t st) {
  const int groups = (N + 15) / 16, rg = 8 / ks;
  const int sets = (groups + rg - 1) / rg;
  const int resident = 4 * device_sm_count();  // 48 KB of rings per block: 4 blocks per SM
  const dim3 grid(sets < resident ? sets : resident);
  const int p = pdl ? (g_early_trigger ? 2 : 1) : 0;
  switch (ks) {
    case 1: return launch_ex(gemv_kernel<WT, NT, 1>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, N, K, B, p);
    case 2: return launch_ex(gemv_kernel<WT, NT, 2>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, N, K, B, p);
    case 4: return launch_ex(gemv_kernel<WT, NT, 4>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, N, K, B, p);
    default: return launch_ex(gemv_kernel<WT, NT, 8>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, N, K, B, p);
  }
}

// K-slices: the fewest that give ~8 warps per SM, keeping each slice a whole number of 64-wide steps
int pick_ks(int N, int K, int kstep, int rows_override) {
  if (rows_override == 1 || rows_override == 2 || rows_override == 4 || rows_override == 8) return rows_override;
  const long groups = (N + 15) / 16;
  const long target = 8L * device_sm_count();
  int ks = 1;
  while (ks < 8 && groups * ks < target && (K / (2 * ks)) % kstep == 0 && K / (2 * ks) >= kstep) ks *= 2;
  return ks;
}

template <typename WT>
cudaError_t gemv_dispatch(const WT *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int rows, int B,
                          bool pdl, cudaStream_t st) {
  const int ks = pick_ks(N, K, WFmt<WT>::KSTEP, rows);
  for (int b0 = 0; b0 < B; b0 += 16) {
    const int bs = min(16, B - b0);
    const bf16 *xb = x + (size_t)b0 * K;
    bf16 *yb = y + (size_t)b0 * N;
    const cudaError_t e = bs > 8 ? gemv_ks<WT, 2>(W, scale, xb, yb, N, K, bs, ks, pdl, st)
                                 : gemv_ks<WT, 1>(W, scale, xb, yb, N, K, bs, ks, pdl, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <typename WT>
cudaError_t gemv_epi_dispatch(int epi, const WT *W, const float *scale, const bf16 *x, bf16 *y, int S, int K,
                              bf16 *state, const bf16 *cw, const bf16 *cbias, bool pdl, cudaStream_t st) {
  const dim3 grid((S + 15) / 16);
  const int p = pdl ? 1 : 0;
  if (sizeof(WT) == 1 && g_gemv_impl != 1 && 3 * (size_t)(K + 64) <= (size_t)GV_X_SMEM_MAX && K % 256 == 0 &&
      K <= xs_max_k(1)) {
    const int8_t *Wi = reinterpret_cast<const int8_t *>(W);
    // SwiGLU (w1|w3): 5-deep rings, so four blocks fit per SM (smem) and the 512 blocks of an 8192-wide layer run
    // in one wave (6-deep: three blocks per SM, two waves)
    if (epi == 0)
      return launch_dyn(gemv_epi_xs_kernel<2, 0, EPI_RING>, grid, GV_THREADS, pdl, st,
                        (size_t)8 * EPI_RING * 1024 + 3 * (size_t)(K + 64), Wi, scale, x, y, S, K, state, cw, cbias, p);
    // short conv (in_proj, 16 outputs x 3 parts per block): ~one block per SM at the model's 2048 channels, so a
    // deeper ring keeps more of each block's weights in flight (where it fits the kernel's shared-memory limit)
    const size_t dconv = (size_t)8 * CONV_RING * 1024 + 3 * (size_t)(K + 64);
    if (dconv <= (size_t)(GV_DYN_SMEM + GV_X_SMEM_MAX))
      return launch_dyn(gemv_epi_xs_kernel<3, 1, CONV_RING>, grid, GV_THREADS, pdl, st, dconv, Wi, scale, x, y, S, K,
                        state, cw, cbias, p);
    return launch_dyn(gemv_epi_xs_kernel<3, 1, XS_RING>, grid, GV_THREADS, pdl, st,
                      (size_t)8 * XS_RING * 1024 + 3 * (size_t)(K + 64), Wi, scale, x, y, S, K, state, cw, cbias, p);
  }
  if (epi == 0)
    return launch_ex(gemv_epi_kernel<WT, 2, 0>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, S, K, state, cw, cbias, p);
  return launch_ex(gemv_epi_kernel<WT, 3, 1>, grid, GV_THREADS, pdl, st, 0, W, scale, x, y, S, K, state, cw, cbias, p);
}

}  // namespace

template <int NT, bool GELU, bool FUSEQ>
cudaError_t gemv_a8_ks(const int8_t *W, const float *sw, const int8_t *xq, const float *sx, const bf16 *xbf,
                       const bf16 *bias, bf16 *y, int N, int K, int B, int ks, bool pdl, cudaStream_t st) {
  const int groups = (N + 15) / 16, rg = 8 / ks;
  const int sets = (groups + rg - 1) / rg;
  // resident blocks per SM: 4 (48 KB of weight rings each); 32 and 64 tokens: 2 and 1 (registers: 128 / ~170 per thread)
  const int resident = (NT >= 8 ? 1 : (NT >= 4 ? 2 : 4)) * device_sm_count();
  const dim3 grid(sets < resident ? sets : resident);
  const int p = pdl ? (g_early_trigger ? 2 : 1) : 0;
  const size_t extra = FUSEQ ? (size_t)B * (K + 64) : 0;
  switch (ks) {
    case 1: return launch_ex(gemv_a8_kernel<NT, 1, GELU, FUSEQ>, grid, GV_THREADS, pdl, st, extra, W, sw, xq, sx, xbf, bias, y, N, K, B, p);
    case 2: return launch_ex(gemv_a8_kernel<NT, 2, GELU, FUSEQ>, grid, GV_THREADS, pdl, st, extra, W, sw, xq, sx, xbf, bias, y, N, K, B, p);
    case 4: return launch_ex(gemv_a8_kernel<NT, 4, GELU, FUSEQ>, grid, GV_THREADS, pdl, st, extra, W, sw, xq, sx, xbf, bias, y, N, K, B, p);
    default: return launch_ex(gemv_a8_kernel<NT, 8, GELU, FUSEQ>, grid, GV_THREADS, pdl, st, extra, W, sw, xq, sx, xbf, bias, y, N, K, B, p);
  }
}

template <int KS, int NT>
cudaError_t gemv_xs_launch(const int8_t *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int B, bool pdl,
                           cudaStream_t st) {
  auto kern = gemv_xs_kernel<KS, NT, XS_RING>;
  const int groups = (N + 15) / 16, rg = 8 / KS;
  const int sets = (groups + rg - 1) / rg;
  const size_t dyn = (size_t)8 * XS_RING * 1024 + (size_t)B * XS_NSL * (K + 64);
  const int resident = resident_blocks(kern, dyn);  // one wave: the grid strides over the sets
  const dim3 grid(sets < resident ? sets : resident);
  const int p = pdl ? (g_early_trigger ? 2 : 1) : 0;
  return launch_dyn(kern, grid, GV_THREADS, pdl, st, dyn, W, scale, x, y, N, K, B, p);
}

template <int NT>
cudaError_t gemv_xs_nt(const int8_t *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int B, int ks, bool pdl,
                       cudaStream_t st) {
  switch (ks) {
    case 1: return gemv_xs_launch<1, NT>(W, scale, x, y, N, K, B, pdl, st);
    case 2: return gemv_xs_launch<2, NT>(W, scale, x, y, N, K, B, pdl, st);
    case 4: return gemv_xs_launch<4, NT>(W, scale, x, y, N, K, B, pdl, st);
    default: return gemv_xs_launch<8, NT>(W, scale, x, y, N, K, B, pdl, st);
  }
}

// the ring x-sliced kernel for B <= 4 tokens: one MMA column group (8 columns) up to 2 tokens, two up to 4
cudaError_t gemv_xs_ks(const int8_t *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int B, int ks, bool pdl,
                       cudaStream_t st) {
  return B * XS_NSL <= 8 ? gemv_xs_nt<1>(W, scale, x, y, N, K, B, ks, pdl, st)
                         : gemv_xs_nt<2>(W, scale, x, y, N, K, B, ks, pdl, st);
}

// Deep-prefetch x-sliced GEMV (gemv_deep_kernel). Shared memory per block at most GV_DEEP_SMEM, so that two
// blocks (this GEMV's and the next one's) fit on an SM.
constexpr size_t GV_DEEP_SMEM = 104 * 1024;

template <int NT, int R>
cudaError_t gemv_deep_r(int ks, dim3 grid, size_t dyn, const int8_t *W, const float *scale, const bf16 *x, bf16 *y,
                        int N, int K, int B, bool pdl, int p, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_dyn(gemv_deep_kernel<1, NT, R>, grid, GV_THREADS, pdl, st, dyn, W, scale, x, y, N, K, B, p);
    case 2: return launch_dyn(gemv_deep_kernel<2, NT, R>, grid, GV_THREADS, pdl, st, dyn, W, scale, x, y, N, K, B, p);
    case 4: return launch_dyn(gemv_deep_kernel<4, NT, R>, grid, GV_THREADS, pdl, st, dyn, W, scale, x, y, N, K, B, p);
    default: return launch_dyn(gemv_deep_kernel<8, NT, R>, grid, GV_THREADS, pdl, st, dyn, W, scale, x, y, N, K, B, p);
  }
}

// K-slices for the deep kernel. Cost of a choice = sets per block x (steps per set + ~3 steps of per-set epilogue:
// block barriers and the reduction of the K-slices); a large GEMV (>= 16 M weights) also needs a block on every SM,
// because one SM streams only ~40-50 GB/s (measured: 16384 x 2048 on 128 blocks, 8.5 us; on 148, 6.9 us).
int deep_ks(int N, int K, int sms) {
  const long groups = (N + 15) / 16;
  const bool big = (long)N * K >= 16L * 1024 * 1024;
  int best = 0;
  long best_cost = 0;
  for (int pass = 0; pass < 2 && !best; ++pass)
    for (int ks = 1; ks <= 8; ks *= 2) {
      if ((K / 64) % ks) continue;
      const long sets = (groups * ks + 7) / 8;
      if (pass == 0 && big && sets < sms) continue;
      const long cost = (sets + sms - 1) / sms * (K / 64 / ks + 3);
      if (!best || cost < best_cost) {
        best_cost = cost;
        best = ks;
      }
    }
  return best ? best : 1;
}

// Ring depth that fits beside the token slices (0: none does)
int deep_ring(int K, int B) {
  const size_t xsb = (size_t)B * XS_NSL * (K + 64);
  for (int r : {12, 10, 8, 6})
    if ((size_t)r * 8 * 1024 + xsb <= GV_DEEP_SMEM) return r;
  return 0;
}

cudaError_t gemv_deep(const int8_t *W, const float *scale, const bf16 *x, bf16 *y, int N, int K, int B, bool pdl,
                      cudaStream_t st) {
  const int sms = device_sm_count();
  const int ks = deep_ks(N, K, sms), R = deep_ring(K, B);
  const long sets = ((long)(N + 15) / 16 * ks + 7) / 8;
  const dim3 grid((unsigned)(sets < sms ? sets : sms));
  const size_t dyn = (size_t)R * 8 * 1024 + (size_t)B * XS_NSL * (K + 64);
  const int p = pdl ? (g_deep_late ? 1 : 2) : 0;
  if (B * XS_NSL <= 8) {
    switch (R) {
      case 12: return gemv_deep_r<1, 12>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
      case 10: return gemv_deep_r<1, 10>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
      case 8: return gemv_deep_r<1, 8>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
      default: return gemv_deep_r<1, 6>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
    }
  }
  switch (R) {
    case 12: return gemv_deep_r<2, 12>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
    case 10: return gemv_deep_r<2, 10>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
    case 8: return gemv_deep_r<2, 8>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
    default: return gemv_deep_r<2, 6>(ks, grid, dyn, W, scale, x, y, N, K, B, pdl, p, st);
  }
}

// Slices per token for the x-sliced path: 3 for 1..4 tokens whose slices fit the shared-memory budget, else 0.
int gemv_xs_slices(int K, int B) {
  if (B < 1 || B > 4 || (size_t)B * XS_NSL * (K + 64) > (size_t)GV_X_SMEM_MAX || K % 64 != 0 || K > xs_max_k(B))
    return 0;
  return XS_NSL;
}

void gemv_set_early_trigger(bool early) { g_early_trigger = early; }
int gemv_trigger_mode() { return g_early_trigger ? 2 : 1; }
void gemv_set_impl(int impl) {
  g_gemv_impl = impl == 3 ? 2 : impl;
  g_deep_late = impl == 3;  // 3: the deep kernel everywhere, dependent launch triggered after the last set
}

cudaError_t launch_gemv(const void *W, bool int8, const float *scale, const void *x, void *y, int N, int K, int rows,
                        int B, bool pdl, cudaStream_t st) {
  if (N <= 0 || B <= 0) return cudaSuccess;
  const int impl = g_gemv_impl;
  if (int8 && impl != 1 && impl != 4 && (B <= 2 || impl == 2) && gemv_xs_slices(K, B) && deep_ring(K, B))
    return gemv_deep((const int8_t *)W, scale, (const bf16 *)x, (bf16 *)y, N, K, B, pdl, st);
  // the ring kernel's token prologue (absmax, slicing, two block barriers) is repaid by its faster weight stream
  // from ~8 M weights up; below that the bf16 path is quicker (measured on B200)
  if (int8 && impl != 1 && (long)N * K >= 8L * 1024 * 1024 && gemv_xs_slices(K, B))
    return gemv_xs_ks((const int8_t *)W, scale, (const bf16 *)x, (bf16 *)y, N, K, B, pick_ks(N, K, 64, rows), pdl, st);
  if (int8)
    return gemv_dispatch<int8_t>((const int8_t *)W, scale, (const bf16 *)x, (bf16 *)y, N, K, rows, B, pdl, st);
  return gemv_dispatch<bf16>((const bf16 *)W, scale, (const bf16 *)x, (bf16 *)y, N, K, rows, B, pdl, st);
}

// One GEMV of a chain: the x-sliced int8 path wherever its token buffer fits (the chain's contract: every layer gives
// the sliced path's exact-product values), else the bf16 path.
cudaError_t launch_gemv_sliced(const int8_t *W, const float *scale, const void *x, void *y, int N, int K, int B,
                               bool pdl, cudaStream_t st) {
  if (N <= 0 || B <= 0) return cudaSuccess;
  if (gemv_xs_slices(K, B)) {
    const int impl = g_gemv_impl;
    if (impl != 4 && (B <= 2 || impl == 2) && deep_ring(K, B))
      return gemv_deep(W, scale, (const bf16 *)x, (bf16 *)y, N, K, B, pdl, st);
    return gemv_xs_ks(W, scale, (const bf16 *)x, (bf16 *)y, N, K, B, pick_ks(N, K, 64, 0), pdl, st);
  }
  return gemv_dispatch<int8_t>(W, scale, (const bf16 *)x, (bf16 *)y, N, K, 0, B, pdl, st);
}

cudaError_t launch_gemv_epi(int epi, const void *W, bool int8, const float *scale, const void *x, void *y, int S, int K,
                            void *state, const void *cw, const void *cbias, bool pdl, cudaStream_t st) {
  if (S <= 0) return cudaSuccess;
  if (int8)
    return gemv_epi_dispatch<int8_t>(epi, (const int8_t *)W, scale, (const bf16 *)x, (bf16 *)y, S, K, (bf16 *)state,
                                     (const bf16 *)cw, (const bf16 *)cbias, pdl, st);
  return gemv_epi_dispatch<bf16>(epi, (const bf16 *)W, scale, (const bf16 *)x, (bf16 *)y, S, K, (bf16 *)state,
                                 (const bf16 *)cw, (const bf16 *)cbias, pdl, st);
}

cudaError_t launch_gemv_a8(const int8_t *W, const float *sw, const int8_t *xq, const float *sx, const void *bias, void *y,
                           int N, int K, int B, bool gelu, bool pdl, cudaStream_t st) {
  if (N <= 0 || B <= 0) return cudaSuccess;
  const int ks = pick_ks(N, K, 64, 0);
  // up to 64 tokens per pass over W (8 token groups of 8 per MMA row block); more tokens take more passes
  for (int b0 = 0; b0 < B; b0 += A8_MAX_TOKENS) {
    const int bs = min(A8_MAX_TOKENS, B - b0);
    const int8_t *xb = xq + (size_t)b0 * K;
    const float *sb = sx + b0;
    bf16 *yb = (bf16 *)y + (size_t)b0 * N;
    const bf16 *bi = (const bf16 *)bias;
    cudaError_t e;
    if (bs > 32)
      e = gelu ? gemv_a8_ks<8, true, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<8, false, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st);
    else if (bs > 16)
      e = gelu ? gemv_a8_ks<4, true, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<4, false, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st);
    else if (bs > 8)
      e = gelu ? gemv_a8_ks<2, true, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<2, false, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st);
    else
      e = gelu ? gemv_a8_ks<1, true, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<1, false, false>(W, sw, xb, sb, nullptr, bi, yb, N, K, bs, ks, pdl, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int gemv_a8_fused_max_tokens(int K) {
  const int b = GV_X_SMEM_MAX / (K + 64);
  return b < 16 ? b : 16;
}

cudaError_t launch_linear_a8(const void *x, const int8_t *W, const float *sw, const void *bias, void *y, int N, int K,
                             int B, bool gelu, bool pdl, cudaStream_t st) {
  if (N <= 0 || B <= 0) return cudaSuccess;
  const int ks = pick_ks(N, K, 64, 0);
  const int chunk = gemv_a8_fused_max_tokens(K);
  for (int b0 = 0; b0 < B; b0 += chunk) {
    const int bs = min(chunk, B - b0);
    const bf16 *xb = (const bf16 *)x + (size_t)b0 * K;
    bf16 *yb = (bf16 *)y + (size_t)b0 * N;
    const bf16 *bi = (const bf16 *)bias;
    cudaError_t e;
    if (bs > 8)
      e = gelu ? gemv_a8_ks<2, true, true>(W, sw, nullptr, nullptr, xb, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<2, false, true>(W, sw, nullptr, nullptr, xb, bi, yb, N, K, bs, ks, pdl, st);
    else
      e = gelu ? gemv_a8_ks<1, true, true>(W, sw, nullptr, nullptr, xb, bi, yb, N, K, bs, ks, pdl, st)
               : gemv_a8_ks<1, false, true>(W, sw, nullptr, nullptr, xb, bi, yb, N, K, bs, ks, pdl, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace lfm2q
