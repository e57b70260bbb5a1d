// Flash-decoding attention of one decode step over a bf16 KV cache (grouped-query attention, head dim 64, four
// query heads per KV head), split over positions, then a combine pass:
//   split s of (b, q head h): m_s = max_t score, l_s = sum_t e^(score - m_s), acc_s = sum_t e^(score - m_s) v_t over
//   the positions t of the split, score = (q * scale) . k_t; out[b, h] = bf16( sum_s acc_s e^(m_s - M) /
//   sum_s l_s e^(m_s - M) ), M = max_s m_s.
//
// Reference: decode_attention_split_kernel, attn_combine_kernel, launch_decode_attention_split
// (kernels/lfm2_decode.cu:284-426), binding decode_attention_split (kernels/lfm2_decode.cpp:64-71); its caller is the
// fused decode step (src/lfm2opt/runtime.py:258-264), which passes a caller-allocated fp32 workspace
// ws [B, NQ, S, 66] = (m, l, acc[64]) per (b, q head, split).
//
// B200 design. Grid (B * NKV, S); a block covers one KV head's positions [s chunk, (s + 1) chunk) of one sequence
// (chunk = ceil(max_len / S)): four consumer warps (the four query heads of the KV head) and one producer warp. The
// producer streams the split's K and V rows (128 bytes per position) into shared memory with cp.async.bulk copies in
// stages of 64 positions (8 KB of K and 8 KB of V), 3 or 6 deep, each stage completing on an mbarrier; the four
// warps read every staged row from shared memory (one DRAM read per row, no L1 dependence) and release the stage on
// a second mbarrier. Every wait is bounded (~1 s of SM clocks); a wait that gives up sets the device error word that
// lfm2q_check_device reports and the block stops.
// Per lane (position slot grp = lane / 8, dims 8 sub .. 8 sub + 7, sub = lane % 8) the arithmetic is the reference's
// operation for operation: the lane's partial dot product over its 8 dims, an xor-shuffle sum over the 8 slices, the
// online-softmax update per position in increasing order, the merge of the 4 slots by xor 8 then 16; the combine
// merges the splits in order. So the values equal the reference kernel's. What differs is the instruction stream:
// the 16 dot products of a stage are computed before its serial softmax updates, two positions (or two dims) per
// packed fp32x2 instruction, and bf16 is widened by moving bits (integer pipe) instead of by conversions (which issue
// at quarter rate and bounded the first version of this kernel).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace lfm2q {

__device__ int g_attn_err = 0;  // sticky: 1 = a stage wait gave up

namespace {

constexpr int AT_D = 64;                 // head dim
constexpr int AT_HEADS = 4;              // query heads per KV head (consumer warps)
constexpr int AT_THREADS = 32 * (AT_HEADS + 1);
constexpr int AT_ROWS = 64;              // positions per stage
constexpr int AT_MAX_STAGES = 6;
constexpr int AT_ROW_BYTES = AT_D * 2;   // one position of K (or V)
constexpr int AT_STAGE_BYTES = AT_ROWS * AT_ROW_BYTES;
constexpr int AT_MAX_SMEM = 2 * AT_MAX_STAGES * AT_STAGE_BYTES;  // 96 KB, dynamic
constexpr long long AT_WAIT_LIMIT = 1ll << 31;

__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bar_init(uint32_t b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait; false = gave up (or another role did): the caller stops
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t parity, volatile int *stop) {
  if (bar_try(b, parity)) return true;
  const long long t0 = clock64();
  while (!bar_try(b, parity)) {
    if (*stop) return false;
    if (clock64() - t0 > AT_WAIT_LIMIT) {
      *stop = 1;
      atomicCAS(&g_attn_err, 0, 1);
      return false;
    }
  }
  return true;
}
// bytes of global memory (16-byte aligned, a multiple of 16) into shared memory, completing on mbarrier b
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(b)
               : "memory");
}

// Two fp32 values in one 64-bit register, for the packed fp32 instructions of sm_100 (fma / mul / add .rn.f32x2):
// each half of a packed op is the IEEE operation of its scalar form, so packing changes no value.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 up2(f32x2 v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// One staged block of up to AT_ROWS positions for one warp: lane (grp, sub) takes positions grp, grp + 4, ... of the
// stage. The 16 dot products come first (independent: two positions per packed instruction, the loads and shuffles
// of all 16 overlapping), then the online-softmax updates run in position order. Each value is the reference
// kernel's (kernels/lfm2_decode.cu:329-365) with its operations spelled out as compiled: per pair of dims
// t = fma(q0, k0, q1 * k1), dot = dot + t; acc = fma(p, v, acc * corr); l = fma(l, corr, p) (each checked bit for bit
// against the reference kernel's output: the acc update fuses the second product). bf16 -> fp32 is exact
// (the 16 bits moved up). Groups of four positions past `rows` are skipped by the whole warp, as the reference's loop
// bound does; a lane's dot of a position past `rows` (within a pair still in range) is computed from stale shared
// memory inside the stage buffer and never used.
template <bool FULL>
__device__ __forceinline__ void attend_stage(const uint4 *Ks, const uint4 *Vs, int rows, const f32x2 (&q0)[4],
                                             const f32x2 (&q1)[4], int grp, int sub, float &m, float &l,
                                             f32x2 (&acc)[4]) {
  constexpr int IT = AT_ROWS / 4;
  float dot[IT];
#pragma unroll
  for (int i = 0; i < IT; i += 2) {  // positions 4i + grp and 4(i + 1) + grp
    if (!FULL && 4 * i >= rows) break;
    const uint4 ka = Ks[(4 * i + grp) * (AT_D / 8) + sub], kb = Ks[(4 * i + 4 + grp) * (AT_D / 8) + sub];
    const uint32_t wa[4] = {ka.x, ka.y, ka.z, ka.w}, wb[4] = {kb.x, kb.y, kb.z, kb.w};
    f32x2 d = pk2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const f32x2 t = fma2(q0[j], pk2(bf_lo(wa[j]), bf_lo(wb[j])), mul2(q1[j], pk2(bf_hi(wa[j]), bf_hi(wb[j]))));
      d = add2(d, t);
    }
    float2 dd = up2(d);
    dd.x += __shfl_xor_sync(0xffffffffu, dd.x, 4);
    dd.y += __shfl_xor_sync(0xffffffffu, dd.y, 4);
    dd.x += __shfl_xor_sync(0xffffffffu, dd.x, 2);
    dd.y += __shfl_xor_sync(0xffffffffu, dd.y, 2);
    dd.x += __shfl_xor_sync(0xffffffffu, dd.x, 1);
    dd.y += __shfl_xor_sync(0xffffffffu, dd.y, 1);
    dot[i] = dd.x;
    dot[i + 1] = dd.y;
  }
#pragma unroll
  for (int i = 0; i < IT; ++i) {
    const int t = 4 * i + grp;
    if (FULL || t < rows) {
      const uint4 vraw = Vs[t * (AT_D / 8) + sub];
      const uint32_t wv[4] = {vraw.x, vraw.y, vraw.z, vraw.w};
      const float mn = fmaxf(m, dot[i]), corr = __expf(m - mn), p = __expf(dot[i] - mn);
      l = __fmaf_rn(l, corr, p);
      const f32x2 c2 = pk2(corr, corr), p2 = pk2(p, p);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fma2(p2, pk2(bf_lo(wv[j]), bf_hi(wv[j])), mul2(acc[j], c2));
      m = mn;
    }
  }
}

// One block per (b * NKV + kv head, split): writes ws[((b * NQ + h) * S + s) * 66 + {0: m, 1: l, 2..65: acc}] for
// the block's four query heads h (acc only where the split holds positions). `stages` (1..AT_MAX_STAGES) is the ring
// depth; the dynamic shared memory holds 2 * stages * AT_STAGE_BYTES.
__global__ void __launch_bounds__(AT_THREADS) attn_split_kernel(const bf16 *__restrict__ q, const bf16 *__restrict__ kc,
                                                                const bf16 *__restrict__ vc,
                                                                const int64_t *__restrict__ pos_p, float *__restrict__ ws,
                                                                int NQ, int NKV, int max_len, int S, float scale,
                                                                int stages, int pdl) {
  extern __shared__ __align__(128) uint8_t at_smem[];  // [stage][K rows], then [stage][V rows]
  __shared__ __align__(8) uint64_t full[AT_MAX_STAGES], empty[AT_MAX_STAGES];
  __shared__ int stop;
  uint8_t(*stage_k)[AT_STAGE_BYTES] = reinterpret_cast<uint8_t(*)[AT_STAGE_BYTES]>(at_smem);
  uint8_t(*stage_v)[AT_STAGE_BYTES] = reinterpret_cast<uint8_t(*)[AT_STAGE_BYTES]>(at_smem + stages * AT_STAGE_BYTES);
  if (pdl) {
    pdl_trigger();
    pdl_wait();  // q, the newest cache row and pos come from the previous kernels
  }
  const int bk = blockIdx.x, s = blockIdx.y;
  const int b = bk / NKV, kvh = bk % NKV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long pv = __ldcg(reinterpret_cast<const long long *>(pos_p));
  const int len = pv + 1 < (long long)max_len ? (int)pv + 1 : max_len;  // positions past the cache are not read
  const int chunk = (max_len + S - 1) / S;
  const int t0 = s * chunk, t1 = min(len, t0 + chunk);
  if (t0 >= t1) {  // empty split: nothing to merge from it
    if (warp < AT_HEADS && lane == 0) {
      float *out = ws + (((size_t)b * NQ + kvh * AT_HEADS + warp) * S + s) * (AT_D + 2);
      out[0] = -INFINITY;
      out[1] = 0.f;
    }
    return;
  }
  const int nst = (t1 - t0 + AT_ROWS - 1) / AT_ROWS;  // stages of this split
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      bar_init(saddr(&full[i]), 1);
      bar_init(saddr(&empty[i]), AT_HEADS);
    }
    stop = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const size_t base = ((size_t)b * NKV + kvh) * max_len * AT_D;  // this KV head's cache rows

  if (warp == AT_HEADS) {
    // ---------------------------------------------------------------- producer: K and V rows of each stage
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int slot = i % stages;
        if (i >= stages && !bar_wait(saddr(&empty[slot]), (uint32_t)((i / stages - 1) & 1), &stop)) break;
        const int r0 = t0 + i * AT_ROWS;
        const int rows = min(AT_ROWS, t1 - r0);
        const uint32_t bytes = (uint32_t)(rows * AT_ROW_BYTES);
        bar_expect_tx(saddr(&full[slot]), 2 * bytes);
        bulk_g2s(saddr(stage_k[slot]), kc + base + (size_t)r0 * AT_D, bytes, saddr(&full[slot]));
        bulk_g2s(saddr(stage_v[slot]), vc + base + (size_t)r0 * AT_D, bytes, saddr(&full[slot]));
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumers: warp = query head of this KV head
  const int h = kvh * AT_HEADS + warp;
  const int grp = lane >> 3, sub = lane & 7;  // position slot in a group of four, 8-dim slice
  f32x2 q0[4], q1[4];  // (q * scale) of dims 8 sub + 2j and 8 sub + 2j + 1, each twice
  {
    const uint4 raw = ld_cg16(reinterpret_cast<const uint4 *>(q + ((size_t)b * NQ + h) * AT_D) + sub);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = bf_lo(w[j]) * scale, c = bf_hi(w[j]) * scale;
      q0[j] = pk2(a, a);
      q1[j] = pk2(c, c);
    }
  }
  float m = -INFINITY, l = 0.f;
  f32x2 accp[4] = {0ull, 0ull, 0ull, 0ull};  // (acc[2j], acc[2j + 1]); all-zero bits = (+0, +0)
  bool ok = true;
  for (int i = 0; i < nst && ok; ++i) {
    const int slot = i % stages;
    // every lane observes the stage's completion itself (the bulk copies' bytes are then visible to it)
    const bool fine = bar_wait(saddr(&full[slot]), (uint32_t)((i / stages) & 1), &stop);
    if (!__all_sync(0xffffffffu, fine)) {
      ok = false;
      break;
    }
    const int rows = min(AT_ROWS, t1 - (t0 + i * AT_ROWS));
    const uint4 *Ks = reinterpret_cast<const uint4 *>(stage_k[slot]);
    const uint4 *Vs = reinterpret_cast<const uint4 *>(stage_v[slot]);
    if (rows == AT_ROWS)
      attend_stage<true>(Ks, Vs, AT_ROWS, q0, q1, grp, sub, m, l, accp);
    else
      attend_stage<false>(Ks, Vs, rows, q0, q1, grp, sub, m, l, accp);
    __syncwarp();
    if (lane == 0) bar_arrive(saddr(&empty[slot]));  // this warp is done with the stage
  }
  float acc[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = up2(accp[j]);
    acc[2 * j] = a.x;
    acc[2 * j + 1] = a.y;
  }
  // merge the four position slots (same sub = same dims): xor 8, then 16
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, m2);
    const float c1 = (m == -INFINITY) ? 0.f : __expf(m - mn), c2 = (m2 == -INFINITY) ? 0.f : __expf(m2 - mn);
    l = l * c1 + l2 * c2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a2 = __shfl_xor_sync(0xffffffffu, acc[j], o);
      acc[j] = acc[j] * c1 + a2 * c2;
    }
    m = mn;
  }
  if (grp == 0) {
    float *out = ws + (((size_t)b * NQ + h) * S + s) * (AT_D + 2);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[2 + sub * 8 + j] = ok ? acc[j] : 0.f;
    if (sub == 0) {
      out[0] = ok ? m : -INFINITY;
      out[1] = ok ? l : 0.f;
    }
  }
}

// One block of 64 threads per (b, q head): the merge of the S partials, in split order, as the reference's combine
// (kernels/lfm2_decode.cu:389-416). M = max_s m_s is exact in any order (a max rounds nothing); the sums run in split
// order from partials staged in shared memory (all the loads of a chunk in flight at once instead of one dependent L2
// round trip per split). Up to AT_CMB_SPLITS splits everything is staged at once and M is read from shared memory:
// one round trip in all; beyond, M is a block reduction over the m values first, then chunk by chunk.
constexpr int AT_CMB_SPLITS = 64;
__global__ void __launch_bounds__(AT_D) attn_combine_kernel(const float *__restrict__ ws, bf16 *__restrict__ out, int S,
                                                            int pdl) {
  __shared__ float part[AT_CMB_SPLITS * (AT_D + 2)];
  __shared__ float wmax[AT_D / 32];
  if (pdl) {
    pdl_trigger();
    pdl_wait();
  }
  const int bh = blockIdx.x, d = threadIdx.x;
  const float *w = ws + (size_t)bh * S * (AT_D + 2);
  float M = -INFINITY, L = 0.f, o = 0.f;
  if (S <= AT_CMB_SPLITS) {
    // every partial in one round trip, M from shared memory (a max is exact in any order), then the sums
    for (int i = d; i < S * (AT_D + 2); i += AT_D) part[i] = __ldcg(w + i);
    __syncthreads();
    for (int s = 0; s < S; ++s) M = fmaxf(M, part[s * (AT_D + 2)]);
    for (int s = 0; s < S; ++s) {
      const float ls = part[s * (AT_D + 2) + 1];
      if (ls == 0.f) continue;
      const float c = __expf(part[s * (AT_D + 2)] - M);
      L += ls * c;
      o += part[s * (AT_D + 2) + 2 + d] * c;
    }
    out[(size_t)bh * AT_D + d] = f2bf(o / L);
    return;
  }
  for (int s = d; s < S; s += AT_D) M = fmaxf(M, __ldcg(w + (size_t)s * (AT_D + 2)));
  M = warp_max(M);
  if ((d & 31) == 0) wmax[d >> 5] = M;
  __syncthreads();
  M = fmaxf(wmax[0], wmax[1]);
  for (int c0 = 0; c0 < S; c0 += AT_CMB_SPLITS) {
    const int n = min(AT_CMB_SPLITS, S - c0);
    const float *wc = w + (size_t)c0 * (AT_D + 2);
    for (int i = d; i < n * (AT_D + 2); i += AT_D) part[i] = __ldcg(wc + i);
    __syncthreads();
    for (int s = 0; s < n; ++s) {
      const float ls = part[s * (AT_D + 2) + 1];
      if (ls == 0.f) continue;
      const float c = __expf(part[s * (AT_D + 2)] - M);
      L += ls * c;
      o += part[s * (AT_D + 2) + 2 + d] * c;
    }
    __syncthreads();
  }
  out[(size_t)bh * AT_D + d] = f2bf(o / L);
}

}  // namespace

cudaError_t launch_decode_attention_split(const void *q, const void *kc, const void *vc, const int64_t *pos, void *out,
                                          float *ws, int B, int NQ, int NKV, int max_len, int S, float scale, bool pdl,
                                          cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  static std::atomic<int> attr_set[64];  // the shared-memory opt-in, once per device
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    if (const cudaError_t e =
            cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_MAX_SMEM))
      return e;
    attr_set[dev].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cfg.stream = st;
  cfg.gridDim = dim3(B * NKV, S);
  cfg.blockDim = dim3(AT_THREADS);
  // Ring depth: 6 stages (96 KB, two blocks per SM) while the grid fits twice on the SMs, so that each SM keeps
  // 192 KB of rows in flight; 3 (48 KB, four blocks per SM) for larger grids; never more than a split's stages.
  const long long blocks = (long long)B * NKV * S;
  const int chunk = (max_len + S - 1) / S;
  const int stages = std::max(1, std::min(blocks <= 2LL * device_sm_count() ? 6 : 3, (chunk + AT_ROWS - 1) / AT_ROWS));
  cfg.dynamicSmemBytes = 2 * stages * AT_STAGE_BYTES;
  const int p = pdl ? 1 : 0;
  if (const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_split_kernel, (const bf16 *)q, (const bf16 *)kc,
                                               (const bf16 *)vc, pos, ws, NQ, NKV, max_len, S, scale, stages, p))
    return e;
  cfg.gridDim = dim3(B * NQ);
  cfg.blockDim = dim3(AT_D);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, attn_combine_kernel, (const float *)ws, (bf16 *)out, S, p);
}

// ---------------------------------------------------------------- allocation-free variant
// The per-split partials of lfm2q_decode_attention_split_noalloc: a fixed 8 MiB array in the library's own device
// image, present on every GPU that loads the library until the process exits. Host code may not pass the symbol
// itself to a kernel (on the host it names a host-side shadow, not device memory): its device address is looked up
// once per device, with that device current, and cached.
static __device__ __align__(256) float g_attn_static_ws[ATTN_STATIC_WS_FLOATS];

static cudaError_t attn_static_ws(float **ws) {
  static std::mutex mu;
  static float *addr[64] = {};
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {  // first call on this device: an error is returned and not cached, so a later call retries
    void *p = nullptr;
    if (const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_ws)) return e;
    addr[dev] = static_cast<float *>(p);
  }
  *ws = addr[dev];
  return cudaSuccess;
}

cudaError_t launch_decode_attention_split_static(const void *q, const void *kc, const void *vc, const int64_t *pos,
                                                 void *out, int B, int NQ, int NKV, int max_len, int S, float scale,
                                                 bool pdl, cudaStream_t st) {
  if ((long long)B * NQ * S * (AT_D + 2) > ATTN_STATIC_WS_FLOATS) return cudaErrorInvalidValue;
  float *ws = nullptr;
  if (const cudaError_t e = attn_static_ws(&ws)) return e;
  return launch_decode_attention_split(q, kc, vc, pos, out, ws, B, NQ, NKV, max_len, S, scale, pdl, st);
}

int attn_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace lfm2q
