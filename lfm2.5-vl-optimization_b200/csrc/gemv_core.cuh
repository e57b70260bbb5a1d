// Warp-level building blocks of the decode GEMVs (gemv.cu, gemv_chain.cu): the per-warp cp.async weight ring, the
// bf16-MMA and int8-MMA inner loops, MMA fragment coordinates, and the exact fixed-point slicing of bf16 tokens.
// sm_100a only (mma.sync for the skinny, HBM-bound products; see gemv.cu for the design).
#pragma once

#include "common.cuh"

namespace lfm2q {
namespace {

constexpr int GV_THREADS = 256;  // 8 warps
constexpr int GV_RING = 6;       // K steps (1 KB each) a warp keeps in flight

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename WT>
struct WFmt;
// int8: one 16-byte chunk = 16 codes = 4 MMA k-steps of one row; a 64-wide K step is one chunk per lane-row
template <>
struct WFmt<int8_t> {
  static constexpr int KSTEP = 64;  // K covered per lane chunk pair
  static constexpr int STEPS = 4;   // MMA k16 steps per chunk
  __device__ static void frag(const uint4 &r0, const uint4 &r1, int s, uint32_t (&a)[4]) {
    const uint32_t w0 = (&r0.x)[s], w1 = (&r1.x)[s];
    i8x4_to_bf16x2x2(w0, a[0], a[2]);  // row g: k slots 2t,2t+1 | 2t+8,2t+9
    i8x4_to_bf16x2x2(w1, a[1], a[3]);  // row g + 8
  }
};
// bf16: one 16-byte chunk = 8 weights = 2 MMA k-steps of one row
template <>
struct WFmt<bf16> {
  static constexpr int KSTEP = 32;
  static constexpr int STEPS = 2;
  __device__ static void frag(const uint4 &r0, const uint4 &r1, int s, uint32_t (&a)[4]) {
    a[0] = (&r0.x)[2 * s];
    a[2] = (&r0.x)[2 * s + 1];
    a[1] = (&r1.x)[2 * s];
    a[3] = (&r1.x)[2 * s + 1];
  }
};

// x fragment words for lane (g, t) at K position k0 of token `tok`: the lane's chunk of x covers the same
// physical k as its weight chunk: int8 -> 16 bf16 (two 16-byte loads), bf16 -> 8 bf16 (one load)
template <typename WT>
__device__ __forceinline__ void load_x(const bf16 *__restrict__ x, int K, int tok, int B, int kphys, uint32_t (&xw)[8]) {
  constexpr int NW = WFmt<WT>::KSTEP / 8;  // 32-bit words per lane chunk: 8 (int8) or 4 (bf16)
  if (tok < B) {
    const uint4 *p = reinterpret_cast<const uint4 *>(x + (size_t)tok * K + kphys);
    const uint4 v0 = ld_cg16(p);
    xw[0] = v0.x; xw[1] = v0.y; xw[2] = v0.z; xw[3] = v0.w;
    if (NW == 8) {
      const uint4 v1 = ld_cg16(p + 1);
      xw[4] = v1.x; xw[5] = v1.y; xw[6] = v1.z; xw[7] = v1.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) xw[i] = 0u;
  }
}

// Core: one warp accumulates rows [r0, r0 + 16) x K-slice [kb, ke) for tokens 0..8*NT-1 into acc[NT][4].
// Weights travel global -> shared memory with cp.async (16 bytes per lane per row and step), GV_RING steps ahead, in
// a ring private to the warp (ring: GV_RING x 1 KB; each lane writes and later reads only its own 16-byte slots,
// at row * 64 + t * 16, which is bank-conflict-free), so no registers are tied up by loads in flight and a warp
// keeps ~5 KB of weights outstanding. A slot is refilled only after its data has been read and used.
template <typename WT, int NT>
__device__ __forceinline__ void warp_gemv(const WT *__restrict__ W, const bf16 *__restrict__ x, int N, int K, int B,
                                          int r0, int kb, int ke, float (&acc)[NT][4], uint8_t *ring, bool pdl) {
  constexpr int KSTEP = WFmt<WT>::KSTEP, STEPS = WFmt<WT>::STEPS;
  constexpr int CH = 16 / sizeof(WT);  // elements per 16-byte chunk
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const WT *row0 = W + (size_t)min(r0 + g, N - 1) * K + kb + t * CH;
  const WT *row1 = W + (size_t)min(r0 + g + 8, N - 1) * K + kb + t * CH;
  const uint32_t slot0 = (uint32_t)__cvta_generic_to_shared(ring) + g * 64 + t * 16;
  const int nsteps = (ke - kb) / KSTEP;

  auto issue = [&](int st) {
    if (st < nsteps) {
      const uint32_t d = slot0 + (st % GV_RING) * 1024;
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d), "l"(row0 + st * KSTEP) : "memory");
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d + 512), "l"(row1 + st * KSTEP)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto lds = [&](int st, uint4 &w0, uint4 &w1) {
    const uint32_t d = slot0 + (st % GV_RING) * 1024;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w0.x), "=r"(w0.y), "=r"(w0.z), "=r"(w0.w) : "r"(d)
                 : "memory");
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w1.x), "=r"(w1.y), "=r"(w1.z), "=r"(w1.w)
                 : "r"(d + 512)
                 : "memory");
  };

  // two independent accumulator chains (even / odd MMA k-steps), summed at the end
  float acc2[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = acc2[j][e] = 0.f;

#pragma unroll
  for (int st = 0; st < GV_RING; ++st) issue(st);  // weights are immutable: stream before the dependency wait
  if (pdl) pdl_wait();
  // software pipeline: the weights (shared memory) and x fragments (L1 / L2) of step st + 1 are loaded while
  // step st is converted and multiplied
  uint4 wc0, wc1, wn0, wn1;
  uint32_t xc[NT][8], xn[NT][8];
  asm volatile("cp.async.wait_group %0;" ::"n"(GV_RING - 1) : "memory");
  if (nsteps > 0) {
    lds(0, wc0, wc1);
#pragma unroll
    for (int j = 0; j < NT; ++j) load_x<WT>(x, K, g + 8 * j, B, kb + t * CH, xc[j]);
  }
  for (int st = 0; st < nsteps; ++st) {
    if (st + 1 < nsteps) {
      asm volatile("cp.async.wait_group %0;" ::"n"(GV_RING - 2) : "memory");
      lds(st + 1, wn0, wn1);
#pragma unroll
      for (int j = 0; j < NT; ++j) load_x<WT>(x, K, g + 8 * j, B, kb + (st + 1) * KSTEP + t * CH, xn[j]);
    }
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      uint32_t a[4];
      WFmt<WT>::frag(wc0, wc1, s, a);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        if (s & 1) mma_bf16_16816(acc2[j], a, xc[j][2 * s], xc[j][2 * s + 1]);
        else mma_bf16_16816(acc[j], a, xc[j][2 * s], xc[j][2 * s + 1]);
      }
    }
    issue(st + GV_RING);  // slot of step st: its data is already in registers
    wc0 = wn0;
    wc1 = wn1;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) xc[j][i] = xn[j][i];
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] += acc2[j][e];
}

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A8 core: int8 weights x int8 tokens (quantized per token) -> exact int32 sums, rows [r0, r0 + 16) x K-slice
// [kb, ke). Same cp.async ring and software pipeline as warp_gemv; no conversion at all: the 16 bytes a lane holds
// of rows g and g + 8 feed two m16n8k32 s8 MMAs directly. Lane (g, t), MMA s of a 64-byte step: logical k slots
// 4t..4t+3 / 16+4t..16+4t+3 take physical bytes 16t+8s..+3 / 16t+8s+4..+7, for W and x alike.
// phase 0: prefetch + compute; 1: only issue the first RING steps (weights, immutable); 2: compute after phase 1.
template <int NT, int RING = GV_RING>
__device__ __forceinline__ void warp_gemv_a8(const int8_t *__restrict__ W, const int8_t *xq, int xstride, int N, int K,
                                             int B, int r0, int kb, int ke, int (&acc)[NT][4], uint8_t *ring, bool pdl,
                                             int phase = 0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int8_t *row0 = W + (size_t)min(r0 + g, N - 1) * K + kb + t * 16;
  const int8_t *row1 = W + (size_t)min(r0 + g + 8, N - 1) * K + kb + t * 16;
  const uint32_t slot0 = (uint32_t)__cvta_generic_to_shared(ring) + g * 64 + t * 16;
  const int nsteps = (ke - kb) / 64;
  // step st goes to ring slot st mod RING; the loops below keep the slot of the current step incrementally
  auto issue = [&](int st, int slot) {
    if (st < nsteps) {
      const uint32_t d = slot0 + slot * 1024;
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d), "l"(row0 + st * 64) : "memory");
      asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(d + 512), "l"(row1 + st * 64) : "memory");
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
  // tokens in shared memory (sliced or quantized in this block) or in global memory (the previous kernel's output:
  // read through L2)
  const bool xg = !__isShared(xq);
  auto ldx = [&](int st, uint4 (&xw)[NT]) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int tok = g + 8 * j;
      const int8_t *p = xq + (size_t)tok * xstride + kb + st * 64 + t * 16;
      xw[j] = tok < B ? (xg ? ld_cg16(p) : *reinterpret_cast<const uint4 *>(p)) : make_uint4(0, 0, 0, 0);
    }
  };
  if (phase != 2) {
#pragma unroll
    for (int st = 0; st < RING; ++st) issue(st, st);
  }
  if (phase == 1) return;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0;
  if (pdl) pdl_wait();
  uint4 wc0, wc1, wn0, wn1, xc[NT], xn[NT];
  asm volatile("cp.async.wait_group %0;" ::"n"(RING - 1) : "memory");
  if (nsteps > 0) {
    lds(0, wc0, wc1);
    ldx(0, xc);
  }
  int slot = 0;  // ring slot of step st
  for (int st = 0; st < nsteps; ++st) {
    const int nslot = slot + 1 == RING ? 0 : slot + 1;
    if (st + 1 < nsteps) {
      asm volatile("cp.async.wait_group %0;" ::"n"(RING - 2) : "memory");
      lds(nslot, wn0, wn1);
      ldx(st + 1, xn);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint32_t a[4] = {(&wc0.x)[2 * s], (&wc1.x)[2 * s], (&wc0.x)[2 * s + 1], (&wc1.x)[2 * s + 1]};
#pragma unroll
      for (int j = 0; j < NT; ++j) mma_s8_16832(acc[j], a, (&xc[j].x)[2 * s], (&xc[j].x)[2 * s + 1]);
    }
    issue(st + RING, slot);  // step st's slot: its data is already in registers
    slot = nslot;
    wc0 = wn0;
    wc1 = wn1;
#pragma unroll
    for (int j = 0; j < NT; ++j) xc[j] = xn[j];
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Fragment accumulator element e of token group j -> (row in group, token)
__device__ __forceinline__ int frag_row(int lane, int e) { return (lane >> 2) + ((e & 2) ? 8 : 0); }
__device__ __forceinline__ int frag_tok(int lane, int j, int e) { return 8 * j + 2 * (lane & 3) + (e & 1); }

// Writes tokens 0..B-1 of x (bf16 [B, K]) as NSL-byte fixed point into shared memory, row b * NSL + s holding byte s
// of every element (q = sum_s q_s 256^s, balanced bytes), and the token's exponent E (x = q * 2^E) into e_s[b].
// All threads of the block take part (16-byte chunks c = tid, tid + 256, ..., held in registers across the absmax
// reduction, XS_CH chunks per thread and token at most: K <= 8 * 256 * XS_CH / B); the block is synchronised inside
// and the caller synchronises again before reading the slices.
constexpr int XS_CH = 8;
// EO: within every 8-element chunk the bytes are stored in the order of the elements 0, 2, 4, 6, 1, 3, 5, 7 (the
// order in which the INT4 GEMV unpacks a word of packed nibbles: low nibbles, then high nibbles).
// csum (optional, needs K % 128 == 0, B * NSL <= 16): the sums of the slice bytes of every 128 elements,
// csum[blk * 16 + b * NSL + s] for token b, slice s and block blk of 128 elements (16 chunks, held by 16 consecutive
// lanes).
// J: chunks per thread, a compile-time bound (J * 256 >= B * K / 8), so the register array and every loop are sized
// to the case at hand (a single-token K = 2048 call runs one chunk per thread without any idle iteration).
template <int NSL, bool EO, int J>
__device__ __forceinline__ void slice_tokens_j(const bf16 *__restrict__ x, int K, int B, int8_t *xs, int xstride,
                                               int *e_s, float (&red_max)[4][8], int *csum) {
  constexpr int QBITS = 8 * NSL - 2;  // |q| < 2^QBITS
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K8 = K / 8, total = B * K8;
  // token of chunk i (B <= 4), by comparisons
  auto tok = [K8](int i) { return (int)(i >= K8) + (int)(i >= 2 * K8) + (int)(i >= 3 * K8); };
  // this thread's chunks over all tokens: index i = tid + j * 256 -> token tok(i), chunk i - tok(i) * K8
  uint4 v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int i = threadIdx.x + j * GV_THREADS;
    v[j] = i < total ? ld_cg16(reinterpret_cast<const uint4 *>(x) + i) : make_uint4(0u, 0u, 0u, 0u);
  }
  {
    float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (j * GV_THREADS >= total) break;  // uniform; chunks past the end are zero and leave the maxima unchanged
      const int b = tok(threadIdx.x + j * GV_THREADS);
      const uint32_t m2 = __vmaxu2(__vmaxu2(v[j].x & 0x7FFF7FFFu, v[j].y & 0x7FFF7FFFu),
                                   __vmaxu2(v[j].z & 0x7FFF7FFFu, v[j].w & 0x7FFF7FFFu));
      const float mm = fmaxf(bf_lo(m2), bf_hi(m2));
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) m[bb] = bb == b ? fmaxf(m[bb], mm) : m[bb];
    }
#pragma unroll
    for (int bb = 0; bb < 4; ++bb)
      if (bb < B) {  // B is uniform: the whole warp takes part in each reduction it reaches
        const float w = warp_max(m[bb]);
        if (lane == 0) red_max[bb][warp] = w;
      }
  }
  __syncthreads();
  int E[4], f1b[4], f2b[4];
#pragma unroll
  for (int bb = 0; bb < 4; ++bb) {
    float amax = 0.f;
    if (bb < B) {
#pragma unroll
      for (int w = 0; w < 8; ++w) amax = fmaxf(amax, red_max[bb][w]);
    }
    // amax < 2^(ex + 1) with ex its binary exponent (bf16 subnormals: below the smallest normal, ex = -126 bounds
    // them); E = ex + 1 - QBITS. The scale 2^-E is applied as two exact power-of-two factors (it can exceed 2^127).
    const int ex = amax > 0.f ? max(((__float_as_int(amax) >> 23) & 255) - 127, -126) : 0;
    E[bb] = ex + 1 - QBITS;
    const int ne1 = min(max(-E[bb], -126), 127), ne2 = -E[bb] - ne1;
    f1b[bb] = (ne1 + 127) << 23;
    f2b[bb] = (ne2 + 127) << 23;
  }
  if (threadIdx.x < B)
    e_s[threadIdx.x] = threadIdx.x == 0 ? E[0] : (threadIdx.x == 1 ? E[1] : (threadIdx.x == 2 ? E[2] : E[3]));
#pragma unroll
  for (int j = 0; j < J; ++j) {
    if (j * GV_THREADS >= total) break;  // uniform
    const int i = threadIdx.x + j * GV_THREADS;
    if (i >= total) continue;  // whole 16-lane halves drop out together when total % 16 == 0
    const int b = tok(i), c = i - b * K8;
    int fb1 = f1b[0], fb2 = f2b[0];
#pragma unroll
    for (int bb = 1; bb < 4; ++bb)
      if (bb == b) {
        fb1 = f1b[bb];
        fb2 = f2b[bb];
      }
    const float f1 = __int_as_float(fb1), f2 = __int_as_float(fb2);
    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    // q = round(x 2^-E) (exact scaling, one rounding) is written in balanced bytes q = sum_s q_s 256^s. With
    // u = q + 128 (1 + 256 + ...), |q| <= 2^QBITS, every base-256 digit of u is q_s + 128 (no carries), so the slice
    // bytes are u's bytes with the top bit flipped. u comes from one add: y + 1.5 2^23 rounds y to an integer (round
    // to nearest even, as __float2int_rn) in the low mantissa bits, |y| <= 2^22.
    constexpr uint32_t BIAS = NSL == 3 ? 0x808080u : (NSL == 2 ? 0x8080u : 0x80u);
    constexpr uint32_t MAGIC = 0x4B400000u - BIAS;
    uint32_t u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xv = (e & 1) ? bf_hi(w[e >> 1]) : bf_lo(w[e >> 1]);
      u[e] = (uint32_t)__float_as_int(__fadd_rn(__fmul_rn(__fmul_rn(xv, f1), f2), 12582912.f)) - MAGIC;
    }
    uint32_t o[NSL][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // byte e of word h holds element 4h + e (EO: 2e + h) of the chunk
      const int e0 = EO ? h : 4 * h, de = EO ? 2 : 1;
#pragma unroll
      for (int sl = 0; sl < NSL; ++sl) {
        const uint32_t sel = sl | ((sl + 4) << 4);  // byte sl of each operand into bytes 0, 1
        const uint32_t lo = __byte_perm(u[e0], u[e0 + de], sel), hi = __byte_perm(u[e0 + 2 * de], u[e0 + 3 * de], sel);
        o[sl][h] = __byte_perm(lo, hi, 0x5410) ^ 0x80808080u;
      }
    }
#pragma unroll
    for (int sl = 0; sl < NSL; ++sl)
      *reinterpret_cast<uint2 *>(xs + (size_t)(b * NSL + sl) * xstride + c * 8) = make_uint2(o[sl][0], o[sl][1]);
    if (csum) {
      const unsigned half = 0xFFFFu << (lane & 16);
#pragma unroll
      for (int sl = 0; sl < NSL; ++sl) {
        int sum = __dp4a((int)o[sl][0], 0x01010101, __dp4a((int)o[sl][1], 0x01010101, 0));
#pragma unroll
        for (int o2 = 8; o2 > 0; o2 >>= 1) sum += __shfl_xor_sync(half, sum, o2);
        if ((lane & 15) == 0) csum[(c >> 4) * 16 + b * NSL + sl] = sum;
      }
    }
  }
}

template <int NSL, bool EO = false>
__device__ __forceinline__ void slice_tokens(const bf16 *__restrict__ x, int K, int B, int8_t *xs, int xstride, int *e_s,
                                             float (&red_max)[4][8], int *csum = nullptr) {
  const int total = B * (K / 8);
  if (total <= GV_THREADS) slice_tokens_j<NSL, EO, 1>(x, K, B, xs, xstride, e_s, red_max, csum);
  else if (total <= 2 * GV_THREADS) slice_tokens_j<NSL, EO, 2>(x, K, B, xs, xstride, e_s, red_max, csum);
  else if (total <= 4 * GV_THREADS) slice_tokens_j<NSL, EO, 4>(x, K, B, xs, xstride, e_s, red_max, csum);
  else slice_tokens_j<NSL, EO, XS_CH>(x, K, B, xs, xstride, e_s, red_max, csum);
}

// Largest K the sliced path handles for B tokens (chunks held in registers by the 256 threads of a block)
__host__ __device__ constexpr int xs_max_k(int B) { return 8 * GV_THREADS * XS_CH / (B > 0 ? B : 1); }

}  // namespace
}  // namespace lfm2q
