// W8A8 GEMM on the B200 tensor cores: Y[M, N] = epilogue( Xq[M, K] . Wq[N, K]^T ), int8 x int8 -> exact int32.
//
// Reference: kernels/int8_gemm.cu:125-297 (gemm_i8_kernel, mma.sync m16n8k32 + cp.async), epilogue store_tile
// :93-115, grouped fold :202-230, QOUT requantization :234-285, launchers :741-763; bindings
// kernels/int8_gemm.cpp:39-69. The SiLU-gate epilogue has no counterpart in the reference GEMM: it fuses the
// reference's gemm_i8 (bf16 out) -> silu_mul (kernels/lfm2_decode.cu:954-963) composition.
//
// Epilogues (fp32, no FMA contraction where the reference has none):
//   EPI_TOKEN   y = bf16( act( ((float)acc * sx[m]) * sw[n] + b[n] ) ),          act = id | GELU(tanh)
//   EPI_GROUP   f = fold_g fma((float)acc_g, sxT[g][m], f) over 64-wide K groups; y = bf16(act(f * sw[n] + b[n]))
//   EPI_GROUP_Q as EPI_GROUP, then the bf16-rounded row segment of every 64 output columns is requantized:
//               yq int8 [M, N], ysT[n / 64][m] = max(|.|, 1e-8) / 127
//   EPI_SILU    weight rows [0, I) = gate, [I, 2I) = up; g, u = bf16 of the per-token epilogue;
//               y[m, n] = bf16( bf16(silu(g)) * u ),  silu(g) = g / (1 + __expf(-g)) (IEEE quotient),  y is [M, I]
//
// B200 structure (one persistent CTA per SM, 320 threads (grouped fold 576), warp-specialised):
//   warp 0      TMA producer: 128 x 128-byte A tile and BN x 128-byte B tile per stage, 128-byte swizzle,
//               OOB rows / K columns zero-filled by the copy engine (M, N and K tails need no code)
//   warp 1      allocates TMEM and issues tcgen05.mma.kind::i8 (K = 32 per instruction) from one thread;
//               tcgen05.commit releases a smem stage when its MMAs retire and hands a finished accumulator over
//   warps 2-9   epilogue, two warps per TMEM lane quarter (one per half of the tile's columns; the grouped fold:
//               warps 2-17, four per quarter, a quarter of the columns each): tcgen05.ld (32 lanes x 32 columns
//               per load) -> fp32 math -> 32 x 32 bf16 blocks written to a per-warp shared buffer and stored by TMA
//               (QOUT: int8 rows stored directly); each thread owns one output row, so per-row scales and the QOUT
//               row-group maxima stay in registers
//   W8A16       (EPI_W8, tcgen05.mma.kind::f16, 448 threads): the int8 weight rows arrive by TMA into a staging
//               area and eight converter warps write them as bf16 into the swizzled B stage; four epilogue warps
//               take all of the tile's columns
//   TMEM        2 accumulators of BN columns (TOKEN / SILU) or 4 of 128 (GROUP: one per 64-wide K group, so the
//               int32 partial sums of group g are folded while the MMAs of groups g+1.. run)
//   CTA pairs   (CG = 2, per-token and SiLU epilogues at large M x N): a cluster of two CTAs computes a 256-row tile
//               with tcgen05 cta_group::2 — each CTA stages its 128 A rows and half of the tile's B rows, the
//               leader issues M = 256 MMAs into both CTAs' TMEM.
// Every mbarrier wait is bounded (~1 s of SM clocks). On expiry the kernel records an error code in a device word,
// tells the other roles to stop through shared memory, frees its TMEM and returns; the host reads the code.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace lfm2q {

__device__ int g_gemm_err = 0;  // sticky: 1 = a pipeline wait timed out

namespace {

constexpr int TM = 128;        // output rows per tile (UMMA M, one TMEM lane per row)
constexpr int TK = 128;        // K bytes per pipeline stage: one 128-byte swizzle row
constexpr int NTHREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (2 per TMEM lane quarter)
constexpr int EPI_WARPS = 8;
// epilogue warps: W8 4 (warps 6-13 convert the weights); the grouped fold 16 (4 per TMEM lane quarter, 32 columns
// each: its per-group read-out and fold is the kernel's bottleneck, and 16 warps keep more of it in flight); else 8
__host__ __device__ constexpr int epi_warps(int epi) {
  return epi == EPI_W8 ? 4 : (epi == EPI_GROUP ? 2 * EPI_WARPS : EPI_WARPS);
}
// threads per CTA: producer + MMA warps, the epilogue warps, W8 also 8 converter warps
__host__ __device__ constexpr int cta_threads(int epi) { return 64 + 32 * epi_warps(epi) + (epi == EPI_W8 ? 256 : 0); }
constexpr long long WAIT_LIMIT = 1ll << 31;
constexpr uint32_t ACC_BIAS = 0x4B400000u;  // bit pattern of 1.5 * 2^23

struct GemmArgs {
  const float *sa;    // sx [M] (per token) or sxT [K/64][M] (grouped)
  const float *sb;    // sw [N] per weight row
  const bf16 *bias;   // [N] or null
  bf16 *Y;            // [M, Nout] bf16
  int8_t *Yq;         // QOUT: [M, Nout] int8
  float *YsT;         // QOUT: [Nout/64][M]
  int M, N, K;        // N = weight rows (SILU: 2 * Nout)
  int Nout;           // output columns
  int tiles_m, tiles_n;
  int m_fast;         // tile raster: 1 = consecutive tiles walk M (A stays in L2), 0 = walk N
  int pdl;            // launched as a programmatic dependent: weights may load before the previous grid completes
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// CL: acquire at cluster scope, for a barrier that threads of the other CTA of a pair arrive on
template <bool CL = false>
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if (CL)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity. Returns false when this or another role gave up.
template <bool CL = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *abort_flag, long long limit = WAIT_LIMIT) {
  if (mbar_try_wait<CL>(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait<CL>(bar, parity)) {
    if (*(volatile int *)abort_flag) return false;
    if (clock64() - t0 > limit) {
      atomicExch(abort_flag, 1);
      atomicCAS(&g_gemm_err, 0, 1);
      return false;
    }
  }
  return true;
}

// TMA tensor store of a shared-memory box to (x, y) of map's tensor (x >= 0, y >= 0), in this thread's bulk group
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n\t"
      "cp.async.bulk.commit_group;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(src)
      : "memory");
}
// this thread's bulk stores have read their shared-memory sources / have completed
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
// CTA-pair form: the destination is this CTA's shared memory, the mbarrier may be the pair leader's (a
// shared::cluster address), so both CTAs' bytes complete one transaction count. No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on a barrier of either CTA of the pair (release at CTA scope: what it orders is this thread's completed
// TMEM reads, made visible to the MMA by the tcgen05 fences around the barrier; a cluster-scope release would also
// wait for every global store this thread has in flight)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// K-major operand in the 128-byte swizzle layout the TMA writes: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address (16-byte units)
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                    // descriptor version (tcgen05)
  d |= (uint64_t)2 << 61;                    // 128-byte swizzle
  return d;
}
// Instruction descriptor: s8 x s8 -> s32, both operands K-major, M = 128 (one CTA) or 256 (CTA pair)
__host__ __device__ constexpr uint32_t idesc_i8(int n, int m) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both operands K-major
__host__ __device__ constexpr uint32_t idesc_bf16(int n, int m) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
template <int CG>
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  if constexpr (CG == 2)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// CTA pair: M = 256 MMA from the leader; A rows 0-127 / B rows [0, N/2) come from the leader's shared memory, A rows
// 128-255 / B rows [N/2, N) from the same offsets in the peer's, and D lands in both CTAs' TMEM (128 lanes each)
__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the mbarrier at this offset in both CTAs of the pair once the leader's MMAs so far have retired
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// Wait for this thread's TMEM loads with the destination registers tied to the wait, so no use of them can be
// scheduled before it.
__device__ __forceinline__ void tmem_wait_tie(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
        "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
        "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void st_shared16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tile_coord(int tile, const GemmArgs &a, int &mt, int &nt) {
  if (a.m_fast) {
    mt = tile % a.tiles_m;
    nt = tile / a.tiles_m;
  } else {
    nt = tile % a.tiles_n;
    mt = tile / a.tiles_n;
  }
}

// one elected lane waits, the warp follows its verdict (keeps the .sync.aligned TMEM loads convergent)
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int *abort_flag) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane == 0) ok = mbar_wait(bar, parity, abort_flag);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  return ok;
}

template <int BN, int STAGES, int W_BYTES_ = 0, int NOUT = EPI_WARPS>
struct Smem {
  static constexpr int A_BYTES = TM * TK;
  static constexpr int B_BYTES = BN * TK;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_BYTES;
  // W8: the stage's int8 weight rows as loaded by TMA (rows of 64 bytes), the converter warps' source
  static constexpr int W_BYTES = W_BYTES_;
  static constexpr int W_OFF = B_OFF + STAGES * B_BYTES;
  static constexpr int BAR_OFF = W_OFF + STAGES * W_BYTES;
  static constexpr int NBARS = 3 * STAGES + 8;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  // epilogue: per-warp staging of its columns' weight scales and bias (2 x 128 fp32 per warp)
  static constexpr int PAR_OFF = ((MISC_OFF + 16 + 1023) / 1024) * 1024;
  static constexpr int PAR_FLOATS = 256;
  // epilogue: per-warp 32 x 32 bf16 output block (64-byte rows, 64-byte TMA swizzle), the source of its TMA store
  static constexpr int OUT_OFF = PAR_OFF + EPI_WARPS * PAR_FLOATS * 4;
  static constexpr int OUT_BLOCK = 32 * 64;
  static constexpr int BYTES = OUT_OFF + NOUT * OUT_BLOCK;  // one output block per epilogue warp
  static constexpr int ALLOC = BYTES + 1024;  // room to align the base to 1024
  static_assert(ALLOC <= 232448, "shared memory per block");
};
// the layout of one instantiation: per CTA, A 128 rows and B BN / CG rows per stage (W8: plus the int8 weight rows)
template <int BN, int STAGES, int EPI, int CG>
using SmemOf = Smem<BN / CG, STAGES, EPI == EPI_W8 ? (BN / CG) * 64 : 0,
                    (epi_warps(EPI) > EPI_WARPS ? epi_warps(EPI) : EPI_WARPS)>;

// ------------------------------------------------------------------ the kernel
// CG = 1: one CTA per 128 x BN tile. CG = 2: a cluster of two CTAs (a CTA pair) per 256 x BN tile; CTA r loads A
// rows 128r.. and B rows [r BN/2, (r+1) BN/2) of the tile (SILU: r = 0 the gate rows, r = 1 the up rows), the leader
// (r = 0) issues the M = 256 MMAs, and each CTA's epilogue drains its own 128 TMEM lanes. Per SM this halves the B
// bytes staged in shared memory and cuts the L2 -> SM bytes per MMA by a third against one CTA on a 128 x 256 tile.
template <int BN, int STAGES, int NACC, int EPI, bool GELU, int CG>
__global__ void __launch_bounds__(cta_threads(EPI), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmY,
                   const GemmArgs args) {
  using L = SmemOf<BN, STAGES, EPI, CG>;
  constexpr bool GROUPED = (EPI == EPI_GROUP || EPI == EPI_GROUP_Q);
  static_assert(NACC * BN <= 512, "accumulators exceed TMEM");
  constexpr int TMEM_COLS = NACC * BN <= 256 ? 256 : 512;  // allocations are powers of two
  static_assert(!GROUPED || BN == 128, "grouped tiles are 128 columns wide");
  static_assert(CG == 1 || (CG == 2 && !GROUPED && BN % 32 == 0), "CTA pairs run the per-token epilogues");
  static_assert(EPI != EPI_SILU || BN == 256, "the SiLU tile holds 128 gate and 128 up rows");
  constexpr bool W8 = (EPI == EPI_W8);
  constexpr int EW = epi_warps(EPI);  // epilogue warps 2 .. 2 + EW - 1 (W8: warps 6-13 convert the weights)
  constexpr int PARTS = EW / 4;       // column parts per TMEM lane quarter
  constexpr int KPS = W8 ? TK / 2 : TK;   // K elements per stage (128 bytes of a row: int8 or bf16)
  static_assert(!W8 || (BN / CG) % 64 == 0, "eight converter warps stage B in 8-row groups");
  constexpr int TMU = TM * CG;  // output rows per tile
  constexpr uint32_t IDESC = W8 ? idesc_bf16(BN, TMU) : idesc_i8(BN, TMU);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::MISC_OFF);
  int *abort_flag = reinterpret_cast<int *>(smem + L::MISC_OFF + 4);
  auto bar_full = [&](int s) { return smem_addr(bars + s); };
  auto bar_empty = [&](int s) { return smem_addr(bars + STAGES + s); };
  auto bar_tfull = [&](int a) { return smem_addr(bars + 2 * STAGES + a); };
  auto bar_tempty = [&](int a) { return smem_addr(bars + 2 * STAGES + 4 + a); };
  auto bar_wfull = [&](int s) { return smem_addr(bars + 2 * STAGES + 8 + s); };  // W8: the stage's int8 weights

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = args.M, K = args.K;
  const int KB = (K + KPS - 1) / KPS;    // pipeline stages per tile
  const int G = K / 64;                  // grouped: 64-wide K groups (K % 64 == 0)
  const int tiles = args.tiles_m * args.tiles_n;
  // work unit = one CTA (CG = 1) or one CTA pair (CG = 2, consecutive blockIdx.x form a cluster)
  const int unit = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  // shared::cluster address of a barrier in the pair leader (its own address when CG = 1)
  auto lead = [&](uint32_t bar) { return CG == 2 ? mapa_shared(bar, 0) : bar; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // leader: its producer's arrive (expect_tx for both CTAs' TMA bytes), plus W8: one per converter warp of each CTA
      mbar_init(bar_full(s), W8 ? 1 + 8 * CG : 1);
      mbar_init(bar_empty(s), 1);  // every CTA: one commit from the (leader's) MMA thread
      mbar_init(bar_wfull(s), 1);  // W8, every CTA: its producer's expect_tx for its own weight rows
    }
    for (int a = 0; a < 4; ++a) {
      mbar_init(bar_tfull(a), 1);
      mbar_init(bar_tempty(a), EW * CG);  // one arrival per epilogue warp of every CTA of the unit
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (CG == 2) {  // the same warp of both CTAs allocates the pair's TMEM, same columns in both
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrive or transaction
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      constexpr uint32_t STAGE_TX = CG * (L::A_BYTES + (W8 ? 0 : L::B_BYTES));  // bytes the leader expects per stage
      auto load_b = [&](int st, int nt, int kb) {
        const uint32_t sb = sbase + L::B_OFF + st * L::B_BYTES;
        if constexpr (W8) {  // this CTA's int8 weight rows x 64 K, for its converter warps
          mbar_expect_tx(bar_wfull(st), L::W_BYTES);
          tma_load_2d(sbase + L::W_OFF + st * L::W_BYTES, &tmB, bar_wfull(st), kb * KPS, nt * BN + (int)rank * (BN / CG));
        } else if constexpr (CG == 2) {
          const int brow = (EPI == EPI_SILU) ? (rank ? args.Nout : 0) + nt * (BN / 2) : nt * BN + (int)rank * (BN / 2);
          tma_load_2d_pair(sb, &tmB, lead(bar_full(st)), kb * TK, brow);
        } else if (EPI == EPI_SILU) {
          tma_load_2d(sb, &tmB, bar_full(st), kb * TK, nt * (BN / 2));
          tma_load_2d(sb + (BN / 2) * TK, &tmB, bar_full(st), kb * TK, args.Nout + nt * (BN / 2));
        } else {
          tma_load_2d(sb, &tmB, bar_full(st), kb * TK, nt * BN);
        }
      };
      auto load_a = [&](int st, int mt, int kb) {
        const uint32_t sa = sbase + L::A_OFF + st * L::A_BYTES;
        if constexpr (CG == 2)
          tma_load_2d_pair(sa, &tmA, lead(bar_full(st)), kb * KPS, mt * TMU + (int)rank * TM);
        else
          tma_load_2d(sa, &tmA, bar_full(st), kb * KPS, mt * TM);
      };
      // Programmatic dependent launch: the weights of the first pipeline pass do not depend on the previous kernel,
      // so they load before griddepcontrol.wait; the activations (its output) after it.
      int pre = 0;
      if (args.pdl) {
        const int my_tiles = unit < tiles ? (tiles - 1 - unit) / units + 1 : 0;
        pre = my_tiles * KB < STAGES ? my_tiles * KB : STAGES;
        for (int j = 0; j < pre; ++j) {
          int mt, nt;
          tile_coord(unit + (j / KB) * units, args, mt, nt);
          if (rank == 0) mbar_expect_tx(bar_full(j), STAGE_TX);
          load_b(j, nt, j % KB);
        }
        pdl_wait();
      }
      int j = 0;
      for (int tile = unit; tile < tiles; tile += units) {
        int mt, nt;
        tile_coord(tile, args, mt, nt);
        for (int kb = 0; kb < KB; ++kb, ++j) {
          if (j < pre) {
            load_a(stage, mt, kb);  // fresh stage, B already on its way, expect_tx posted
          } else {
            if (!mbar_wait(bar_empty(stage), phase ^ 1, abort_flag)) goto producer_done;
            if (rank == 0) mbar_expect_tx(bar_full(stage), STAGE_TX);
            load_a(stage, mt, kb);
            load_b(stage, nt, kb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (args.pdl) pdl_trigger();  // every load is issued: the next kernel may start its own prologue
      // CTA pair: wait until every stage has been released once more, so no commit from the leader is still on its
      // way to this CTA's barriers when it exits
      if constexpr (CG == 2) {
        for (int i = 0; i < STAGES; ++i) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1, abort_flag)) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (the leader's, for a CTA pair)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      for (int tile = unit; tile < tiles; tile += units) {
        if (!GROUPED) {
          if (!mbar_wait<CG == 2>(bar_tempty(acc), aphase ^ 1, abort_flag)) goto mma_done;
          tc_fence_after();
          const uint32_t d = tmem_base + acc * BN;
          for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(bar_full(stage), phase, abort_flag)) goto mma_done;
            tc_fence_after();
            const uint64_t ad = sw128_desc(sbase + L::A_OFF + stage * L::A_BYTES);
            const uint64_t bd = sw128_desc(sbase + L::B_OFF + stage * L::B_BYTES);
#pragma unroll
            for (int k = 0; k < TK / 32; ++k) {  // +32 bytes of K per MMA = +2 in the 16-byte address field
              if constexpr (W8)
                umma_bf16<CG>(d, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
              else if constexpr (CG == 2)
                umma_i8_pair(d, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
              else
                umma_i8(d, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
            }
            if constexpr (CG == 2)
              umma_commit_pair(bar_empty(stage));
            else
              umma_commit(bar_empty(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if constexpr (CG == 2)
            umma_commit_pair(bar_tfull(acc));
          else
            umma_commit(bar_tfull(acc));
          if (++acc == NACC) {
            acc = 0;
            aphase ^= 1;
          }
        } else {
          for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(bar_full(stage), phase, abort_flag)) goto mma_done;
            tc_fence_after();
            const uint64_t ad = sw128_desc(sbase + L::A_OFF + stage * L::A_BYTES);
            const uint64_t bd = sw128_desc(sbase + L::B_OFF + stage * L::B_BYTES);
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
              if (2 * kb + gi >= G) break;
              if (!mbar_wait(bar_tempty(acc), aphase ^ 1, abort_flag)) goto mma_done;
              tc_fence_after();
              const uint32_t d = tmem_base + acc * BN;
              umma_i8(d, ad + 4 * gi, bd + 4 * gi, IDESC, 0u);
              umma_i8(d, ad + 4 * gi + 2, bd + 4 * gi + 2, IDESC, 1u);
              umma_commit(bar_tfull(acc));
              if (++acc == NACC) {
                acc = 0;
                aphase ^= 1;
              }
            }
            umma_commit(bar_empty(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
    mma_done:;
    }
  } else if (warp < 2 + EW) {
    // ---------------------------------------------------------------- epilogue warps 2..9 (W8: 2..5)
    // Warp w reads TMEM lane quarter w % 4 (tile rows 32q..32q+31) and owns one half of the tile's output columns
    // (W8: all of them).
    constexpr int PARW = EPI_WARPS * L::PAR_FLOATS / EW;  // parameter floats per warp: weight scales, then bias
    constexpr int PF = PARW / 64;                         // parameters per lane
    const int ew = warp - 2;          // epilogue warp 0..EW-1
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int half = ew >> 2;         // which part of the columns (PARTS per lane quarter)
    const int row = q * 32 + lane;    // tile row == TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    float *par_sw = reinterpret_cast<float *>(smem + L::PAR_OFF) + ew * PARW;  // [PARW / 2] weight scales
    float *par_b = par_sw + PARW / 2;                                           // [PARW / 2] bias
    const uint32_t out_buf = sbase + L::OUT_OFF + ew * L::OUT_BLOCK;
    int acc = 0;
    uint32_t aphase = 0;

    // Per-column epilogue parameters of this warp's columns: lane l holds entries l, l + 32, l + 64, l + 96 of the
    // next tile in registers (loaded one tile ahead, so their latency hides behind a whole tile of work) and writes
    // them to the warp's shared memory when that tile starts. Entry i: output column c0 + i; with `silu`, entries
    // CW.. hold the up rows (weight rows Nout + column).
    float pf_sw[PF], pf_b[PF], pf_sx = 0.f;
    auto prefetch = [&](int tile_i) {
      if (tile_i >= tiles) return;
      int pmt, pnt;
      tile_coord(tile_i, args, pmt, pnt);
      const int pm = pmt * TMU + (int)rank * TM + row;
      pf_sx = (pm < M && !GROUPED && !W8) ? __ldcg(args.sa + pm) : 0.f;  // the previous kernel wrote sa
      const int width = (EPI == EPI_SILU) ? BN / 4 : BN / PARTS;
      const int c0 = (EPI == EPI_SILU) ? pnt * (BN / 2) + half * width : pnt * BN + half * width;
      const int count = (EPI == EPI_SILU) ? 2 * width : width;
#pragma unroll
      for (int k = 0; k < PF; ++k) {
        const int i = lane + 32 * k;
        const int oc = c0 + ((EPI == EPI_SILU) ? (i % width) : i);
        const int col = (EPI == EPI_SILU && i >= width) ? args.Nout + oc : oc;
        const bool ok = i < count && oc < args.Nout;
        pf_sw[k] = ok ? __ldg(args.sb + col) : 0.f;
        pf_b[k] = (ok && args.bias) ? bf2f(args.bias[col]) : 0.f;
      }
    };
    auto stage_params = [&]() {
      __syncwarp();
#pragma unroll
      for (int k = 0; k < PF; ++k) {
        par_sw[lane + 32 * k] = pf_sw[k];
        par_b[lane + 32 * k] = pf_b[k];
      }
      __syncwarp();
    };
    // Store a 32-row x 32-column bf16 block (this lane's row: 16 packed words, 64 bytes) at (column x, row y0):
    // the lanes write their rows into the warp's shared buffer in the TMA 64-byte-swizzle layout (16-byte unit j of
    // row r at unit j ^ ((r >> 1) & 3): conflict-free), and one lane hands the block to a TMA tensor store, which
    // clips rows >= M and columns >= Nout. Against a transpose through shared memory and coalesced st.global, the
    // block crosses the shared-memory port twice instead of three times (measured: 1-10 % faster GEMMs, most at
    // short K). The buffer is rewritten only after the previous store has read it.
    auto store_chunk = [&](const uint32_t *o, int x, int y0) {
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
      const uint32_t sw = (uint32_t)((lane >> 1) & 3);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        st_shared16(out_buf + lane * 64 + ((j ^ sw) << 4), o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      fence_proxy_async_smem();  // the generic-proxy writes, before the TMA engine reads them
      __syncwarp();
      if (lane == 0 && x < args.Nout && y0 < M) tma_store_2d(&tmY, out_buf, x, y0);
    };
    auto release_acc = [&]() {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_cluster(lead(bar_tempty(acc)));
        else
          mbar_arrive(bar_tempty(acc));
      }
      if (++acc == NACC) {
        acc = 0;
        aphase ^= 1;
      }
    };

    if (args.pdl) pdl_wait();  // the per-token scales come from the previous kernel
    prefetch(unit);

    // Grouped: the activation scale of (this lane's row, K group) is loaded three groups ahead of its fold, into a
    // three-register queue that runs on into the next tile (a scale loaded one group ahead left every group waiting
    // out a DRAM round trip). sl_*: the next (tile, group) to load and that tile's row for this lane.
    auto tile_row = [&](int t) {
      int tm_, tn_;
      tile_coord(t, args, tm_, tn_);
      return tm_ * TMU + (int)rank * TM + row;
    };
    int sl_tile = unit, sl_g = 0, sl_m = unit < tiles ? tile_row(unit) : M;
    auto scale_next = [&]() {
      float v = 0.f;
      if (sl_tile < tiles) {
        if (sl_m < M) v = __ldcg(args.sa + (size_t)sl_g * M + sl_m);
        if (++sl_g == G) {
          sl_g = 0;
          sl_tile += units;
          sl_m = sl_tile < tiles ? tile_row(sl_tile) : M;
        }
      }
      return v;
    };
    float sq0 = 0.f, sq1 = 0.f, sq2 = 0.f;
    if constexpr (GROUPED) {
      sq0 = scale_next();
      sq1 = scale_next();
      sq2 = scale_next();
    }
    for (int tile = unit; tile < tiles; tile += units) {
      int mt, nt;
      tile_coord(tile, args, mt, nt);
      const int r0 = mt * TMU + (int)rank * TM;  // first row of this CTA's part of the tile
      const int m = r0 + row;
      const bool mrow = m < M;
      const int yrow = r0 + q * 32;  // first output row of this warp's blocks
      const float sxm = pf_sx;
      stage_params();
      prefetch(tile + units);
      if (EPI == EPI_TOKEN) {
        constexpr int CW = BN / 2, NCH = CW / 32;  // this warp's columns
        const int c0 = nt * BN + half * CW;
        if (!warp_wait(bar_tfull(acc), aphase, abort_flag)) break;
        tc_fence_after();
        const uint32_t tb = tmem_base + lane_addr + acc * BN + half * CW;
        uint32_t r[2][32];
        tmem_ld32(tb, r[0]);
        tmem_wait_tie(r[0]);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int cur = c & 1, nxt = cur ^ 1;
          if (c + 1 < NCH) tmem_ld32(tb + (c + 1) * 32, r[nxt]);
          else release_acc();  // every column of this warp is in registers
          uint32_t o[16];
          const float4 *ps = reinterpret_cast<const float4 *>(par_sw + c * 32);  // broadcast 16-byte reads
          const float4 *pb = reinterpret_cast<const float4 *>(par_b + c * 32);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 s4 = ps[j4], b4 = pb[j4];
            o[2 * j4] = epi_token2<GELU>(r[cur][4 * j4], r[cur][4 * j4 + 1], sxm, s4.x, s4.y, b4.x, b4.y);
            o[2 * j4 + 1] = epi_token2<GELU>(r[cur][4 * j4 + 2], r[cur][4 * j4 + 3], sxm, s4.z, s4.w, b4.z, b4.w);
          }
          store_chunk(o, c0 + c * 32, yrow);
          if (c + 1 < NCH) tmem_wait_tie(r[nxt]);
        }
      } else if (EPI == EPI_W8) {
        // fp32 accumulators: y = bf16(act(acc * sw[n] + b[n])), the reference's W8A16 epilogue order
        constexpr int NCH = BN / 32;  // the warp's 32 rows x all BN columns
        const int c0 = nt * BN;
        if (!warp_wait(bar_tfull(acc), aphase, abort_flag)) break;
        tc_fence_after();
        const uint32_t tb = tmem_base + lane_addr + acc * BN;
        uint32_t r[2][32];
        tmem_ld32(tb, r[0]);
        tmem_wait_tie(r[0]);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int cur = c & 1, nxt = cur ^ 1;
          if (c + 1 < NCH) tmem_ld32(tb + (c + 1) * 32, r[nxt]);
          else release_acc();
          uint32_t o[16];
          const float4 *ps = reinterpret_cast<const float4 *>(par_sw + c * 32);
          const float4 *pb = reinterpret_cast<const float4 *>(par_b + c * 32);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 s4 = ps[j4], b4 = pb[j4];
            const float sv[4] = {s4.x, s4.y, s4.z, s4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              y[e] = __fadd_rn(__fmul_rn(__uint_as_float(r[cur][4 * j4 + e]), sv[e]), bv[e]);
              if (GELU) y[e] = gelu_tanh(y[e]);
            }
            o[2 * j4] = pack_bf16x2(y[0], y[1]);
            o[2 * j4 + 1] = pack_bf16x2(y[2], y[3]);
          }
          store_chunk(o, c0 + c * 32, yrow);
          if (c + 1 < NCH) tmem_wait_tie(r[nxt]);
        }
      } else if (EPI == EPI_SILU) {
        constexpr int CW = BN / 4;  // 64 output columns per warp: gate TMEM columns [CW*half..), up [BN/2 + ..)
        const int c0 = nt * (BN / 2) + half * CW;
        if (!warp_wait(bar_tfull(acc), aphase, abort_flag)) break;
        tc_fence_after();
        const uint32_t tb = tmem_base + lane_addr + acc * BN + half * CW;
        // one 32-column chunk at a time (gate and up): 64 registers of TMEM data live, not 128; the accumulator is
        // released once the last chunk is in registers
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld32(tb + c * 32, rg);
          tmem_ld32(tb + BN / 2 + c * 32, ru);
          tmem_wait_tie(rg);
          tmem_wait_tie(ru);
          if (c == 1) release_acc();
          uint32_t o[16];
          const float4 *pgs = reinterpret_cast<const float4 *>(par_sw + c * 32);  // broadcast 16-byte reads
          const float4 *pgb = reinterpret_cast<const float4 *>(par_b + c * 32);
          const float4 *pus = reinterpret_cast<const float4 *>(par_sw + CW + c * 32);
          const float4 *pub = reinterpret_cast<const float4 *>(par_b + CW + c * 32);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 gs = pgs[j4], gb = pgb[j4], us = pus[j4], ub = pub[j4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int j = 4 * j4 + 2 * h;
              const float2 g = epi_pair(rg[j], rg[j + 1], sxm, h ? gs.z : gs.x, h ? gs.w : gs.y,
                                        h ? gb.z : gb.x, h ? gb.w : gb.y);
              const float2 u = epi_pair(ru[j], ru[j + 1], sxm, h ? us.z : us.x, h ? us.w : us.y,
                                        h ? ub.z : ub.x, h ? ub.w : ub.y);
              const float g0 = rbf(g.x), g1 = rbf(g.y);
              // IEEE quotient, as the reference's silu_mul: __fdividef flushes to 0 once the divisor passes 2^126
              // (g < -87.3), where the reference's value is still a normal float
              const float2 sg = make_float2(rbf(__fdiv_rn(g0, 1.f + __expf(-g0))), rbf(__fdiv_rn(g1, 1.f + __expf(-g1))));
              const float2 y = fmul2(sg, make_float2(rbf(u.x), rbf(u.y)));
              o[j / 2] = pack_bf16x2(y.x, y.y);
            }
          }
          store_chunk(o, c0 + c * 32, yrow);
        }
      } else {
        // grouped: fold every 64-wide K group into fp32 running sums held in registers (CW = 64 columns per warp; QOUT's
        // row-group scale needs a warp's 64 columns)
        constexpr int CW = BN / PARTS, NLD = CW / 32;
        const int c0 = nt * BN + half * CW;
        float f[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) f[j] = 0.f;
        bool ok = true;
        // f = fmaf((float)acc, s, f) per element, two at a time: the partial sums (|acc| < 2^22) become exact floats
        // through the 1.5 * 2^23 mantissa trick (integer add, packed subtract), then one packed fused multiply-add:
        // 2 instructions per element instead of 3, the same roundings
        const float2 big2 = make_float2(12582912.f, 12582912.f);
        auto fold = [&](const uint32_t(&r)[32], float s, int l) {
          const float2 s2 = make_float2(s, s);
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            const float2 a = fsub2(make_float2(__int_as_float((int)r[jj] + (int)ACC_BIAS),
                                               __int_as_float((int)r[jj + 1] + (int)ACC_BIAS)), big2);
            const float2 q = ffma2(a, s2, make_float2(f[32 * l + jj], f[32 * l + jj + 1]));
            f[32 * l + jj] = q.x;
            f[32 * l + jj + 1] = q.y;
          }
        };
        if constexpr (NLD == 1) {
          // 32 columns per warp: two K groups per handshake. Waiting for the later group's commit covers the earlier
          // group's MMAs too (a commit tracks every MMA issued before it); both accumulators are read, released and
          // folded in group order. The accumulator barriers of skipped waits are at most one phase ahead (the MMA
          // refills an accumulator only after its release), so the parity bookkeeping holds.
          for (int g = 0; g < G; g += 2) {
            const bool two = g + 1 < G;
            const float sa = sq0, sb = sq1;
            if (two) {
              sq0 = sq2;
              sq1 = scale_next();
              sq2 = scale_next();
            } else {
              sq0 = sq1;
              sq1 = sq2;
              sq2 = scale_next();
            }
            const int acc_b = acc + 1 == NACC ? 0 : acc + 1;
            const uint32_t ph_b = acc + 1 == NACC ? (aphase ^ 1u) : aphase;
            if (!warp_wait(bar_tfull(two ? acc_b : acc), two ? ph_b : aphase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            {
              uint32_t r[32];  // one accumulator's columns at a time (registers)
              tmem_ld32(tmem_base + lane_addr + acc * BN + half * CW, r);
              tmem_wait_tie(r);
              release_acc();
              fold(r, sa, 0);
            }
            if (two) {
              uint32_t r[32];
              tmem_ld32(tmem_base + lane_addr + acc * BN + half * CW, r);  // release_acc advanced acc to acc_b
              tmem_wait_tie(r);
              release_acc();
              fold(r, sb, 0);
            }
          }
        } else {  // 64 columns per warp (eight warps): the same pairing, one accumulator's registers at a time
          // (gemm_i8_q at 65536 x 2048 x 2048: 519 -> 543 TOPS with the pairing)
          auto drain = [&](float s) {  // read, release and fold the accumulator `acc` (advanced by release_acc)
            const uint32_t tb = tmem_base + lane_addr + acc * BN + half * CW;
            uint32_t r[NLD][32];
#pragma unroll
            for (int l = 0; l < NLD; ++l) tmem_ld32(tb + 32 * l, r[l]);
#pragma unroll
            for (int l = 0; l < NLD; ++l) tmem_wait_tie(r[l]);
            release_acc();
#pragma unroll
            for (int l = 0; l < NLD; ++l) fold(r[l], s, l);
          };
          for (int g = 0; g < G; g += 2) {
            const bool two = g + 1 < G;
            const float sa = sq0, sb = sq1;
            if (two) {
              sq0 = sq2;
              sq1 = scale_next();
              sq2 = scale_next();
            } else {
              sq0 = sq1;
              sq1 = sq2;
              sq2 = scale_next();
            }
            const int acc_b = acc + 1 == NACC ? 0 : acc + 1;
            const uint32_t ph_b = acc + 1 == NACC ? (aphase ^ 1u) : aphase;
            if (!warp_wait(bar_tfull(two ? acc_b : acc), two ? ph_b : aphase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            drain(sa);
            if (two) drain(sb);
          }
        }
        if (!ok) break;
        if (EPI == EPI_GROUP) {
#pragma unroll
          for (int c = 0; c < CW; c += 32) {
            uint32_t o[16];
            const float4 *ps = reinterpret_cast<const float4 *>(par_sw + c);  // broadcast 16-byte reads
            const float4 *pb = reinterpret_cast<const float4 *>(par_b + c);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 s4 = ps[j4], b4 = pb[j4];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int j = c + 4 * j4 + 2 * h;
                float2 y = make_float2(__fadd_rn(__fmul_rn(f[j], h ? s4.z : s4.x), h ? b4.z : b4.x),
                                       __fadd_rn(__fmul_rn(f[j + 1], h ? s4.w : s4.y), h ? b4.w : b4.y));
                if (GELU) {
                  y.x = gelu_tanh(y.x);
                  y.y = gelu_tanh(y.y);
                }
                o[2 * j4 + h] = pack_bf16x2(y.x, y.y);
              }
            }
            store_chunk(o, c0 + c, yrow);
          }
        } else if (mrow) {
          // QOUT: bf16-round the outputs, then one scale per (row, 64 columns): this warp's 64 columns are one
          // group (N % 128 == 0, whole tiles)
          float amax = 0.f;
#pragma unroll
          for (int j = 0; j < CW; ++j) {
            float y = __fadd_rn(__fmul_rn(f[j], par_sw[j]), par_b[j]);
            if (GELU) y = gelu_tanh(y);
            y = rbf(y);
            f[j] = y;
            amax = fmaxf(amax, fabsf(y));
          }
          const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
          const float rinv = __frcp_rn(sc);
          args.YsT[(size_t)(c0 >> 6) * M + m] = sc;
#pragma unroll
          for (int j16 = 0; j16 < CW; j16 += 16) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = pack_i8x4(q8r(f[j16 + 4 * i + 0], sc, rinv), q8r(f[j16 + 4 * i + 1], sc, rinv),
                               q8r(f[j16 + 4 * i + 2], sc, rinv), q8r(f[j16 + 4 * i + 3], sc, rinv));
            *reinterpret_cast<uint4 *>(args.Yq + (size_t)m * args.Nout + c0 + j16) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all0();  // this warp's output stores are complete before the CTA ends
  } else if constexpr (W8) {
    // ---------------------------------------------------------------- W8 weight converters, warps 6..13
    // Each stage, this CTA's BN / CG weight rows x 64 K of int8 (brought into shared memory by the producer's TMA,
    // STAGES stages ahead, zero-filled past N and K) become bf16 in the B stage: converter warp cw owns the 8-row
    // groups cw, cw + 8, ...; in a group, 4 lanes share a row (16 contiguous weights each, one conflict-free 16-byte
    // shared load), convert exactly (exponent-bias trick) and write the two 16-byte units of their 32 bf16 bytes at
    // the 128-byte-swizzled positions the MMA descriptor expects (unit u of row r at u ^ (r & 7)). Then: proxy fence
    // (the tensor core reads through the async proxy), and one arrival per warp on the pair leader's full barrier.
    constexpr int NCW = 8;                  // converter warps
    constexpr int BROWS = BN / CG;          // weight rows this CTA stages per tile
    constexpr int ITER = BROWS / (8 * NCW);  // 8-row groups per converter warp and stage
    static_assert(BROWS % (8 * NCW) == 0, "converter rows");
    const int cw = warp - 2 - EW;           // converter warp 0..NCW-1
    const int lr = lane >> 2, lc = lane & 3;
    const int my_tiles = unit < tiles ? (tiles - 1 - unit) / units + 1 : 0;
    const int total = my_tiles * KB;  // stages this CTA runs
    int stage = 0;
    uint32_t phase = 0;
    for (int j = 0; j < total; ++j) {
      if (!warp_wait(bar_empty(stage), phase ^ 1, abort_flag)) break;  // the MMA has read this B stage
      if (!warp_wait(bar_wfull(stage), phase, abort_flag)) break;      // the stage's int8 rows have landed
      mbar_try_wait<false>(bar_wfull(stage), phase);  // every lane observes the completed phase (acquire)
      const uint32_t sw8 = sbase + L::W_OFF + stage * L::W_BYTES;
      const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
#pragma unroll
      for (int it = 0; it < ITER; ++it) {
        const int rr = (it * NCW + cw) * 8 + lr;
        const uint4 v = ld_shared16(sw8 + rr * 64 + lc * 16);
        uint32_t o[8];
        i8x4_to_bf16x2x2(v.x, o[0], o[1]);
        i8x4_to_bf16x2x2(v.y, o[2], o[3]);
        i8x4_to_bf16x2x2(v.z, o[4], o[5]);
        i8x4_to_bf16x2x2(v.w, o[6], o[7]);
        const uint32_t rowa = sb + rr * 128;
        st_shared16(rowa + (((2 * lc) ^ (rr & 7)) << 4), o[0], o[1], o[2], o[3]);
        st_shared16(rowa + (((2 * lc + 1) ^ (rr & 7)) << 4), o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_cluster(lead(bar_full(stage)));
        else
          mbar_arrive(bar_full(stage));
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  if constexpr (CG == 2)
    cluster_sync_all();  // the peer's last remote arrivals have landed and its epilogue has left TMEM
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                   : "memory");
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D int8 matrix [rows, inner] row-major, box = 128 bytes x box_rows, 128-byte swizzle, OOB reads as zero
bool make_map(CUtensorMap *map, const void *ptr, int inner, int rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner};
  cuuint32_t box[2] = {(cuuint32_t)TK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D bf16 matrix [rows, inner] row-major, box = 64 elements (128 bytes) x box_rows, 128-byte swizzle, OOB reads zero
bool make_map_bf16(CUtensorMap *map, const void *ptr, int inner, int rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {(cuuint32_t)(TK / 2), (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// bf16 output [rows, cols] row-major, box = 32 x 32 (64-byte rows), 64-byte swizzle: the epilogue's store blocks
bool make_map_out(CUtensorMap *map, const void *ptr, int cols, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D int8 matrix [rows, inner] row-major, box = 64 bytes x box_rows, unswizzled (rows 64 bytes apart), OOB reads zero
bool make_map_w8(CUtensorMap *map, const void *ptr, int inner, int rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

std::atomic<int> g_tile_override{0};
// Per-token GEMMs with few rows: the A8 GEMV (one pass over W, int8 mma.sync, tokens on the MMA's N side) against
// the tcgen05 tiles, split-K or not (graph-timed on B200, weights beyond L2): the GEMV wins up to 16 rows, and up to
// 32 rows when the weights are small (<= 8 M: 2048 x 2048 at M = 32, 3.9 us against 4.9 us split-K); from 8 M
// weights split-K is faster (2048 x 8192 at M = 17..32: 7.9 us against 9.7-10.6 us).
bool a8_rows(int M, int N, int K) {
  if (K % 64 != 0) return false;
  if (M <= 16) return true;
  return M <= 32 && (long)N * K <= 8L * 1024 * 1024;
}
std::atomic<bool> g_gemm_pdl{true};  // GEMMs launch as programmatic dependents (lfm2q_set_pdl)

template <int BN, int STAGES, int NACC, int EPI, bool GELU, int CG>
cudaError_t run_tc(const void *A, const int8_t *B, GemmArgs a, cudaStream_t st) {
  using L = SmemOf<BN, STAGES, EPI, CG>;
  auto kern = gemm_tc_kernel<BN, STAGES, NACC, EPI, GELU, CG>;
  static std::once_flag once[64];
  static int max_units[64];  // co-resident work units (CTAs, or CTA pairs) per device
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (CG > 1) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = CG;
    attr[nattr].val.clusterDim.y = 1;
    attr[nattr].val.clusterDim.z = 1;
    ++nattr;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(cta_threads(EPI));
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
    int n = device_sm_count() / CG;
    if (attr_err == cudaSuccess && CG > 1) {
      cudaLaunchConfig_t q = cfg;
      q.gridDim = dim3(CG * n);
      int c = 0;
      if (cudaOccupancyMaxActiveClusters(&c, kern, &q) == cudaSuccess && c > 0) n = c < n ? c : n;
      cudaGetLastError();
    }
    max_units[dev & 63] = n;
  });
  if (attr_err != cudaSuccess) return attr_err;
  CUtensorMap ta, tb, ty;
  memset(&ty, 0, sizeof(ty));
  if (EPI != EPI_GROUP_Q && !make_map_out(&ty, a.Y, a.Nout, a.M)) return cudaErrorInvalidValue;
  if (EPI == EPI_W8) {  // bf16 activations; the int8 weights in 64-byte rows for the converter warps
    if (!make_map_bf16(&ta, A, a.K, a.M, TM) || !make_map_w8(&tb, B, a.K, a.N, BN / CG)) return cudaErrorInvalidValue;
  } else {
    const int box_b = (EPI == EPI_SILU) ? BN / 2 : BN / CG;
    if (!make_map(&ta, A, a.K, a.M, TM) || !make_map(&tb, B, a.K, a.N, box_b)) return cudaErrorInvalidValue;
  }
  const int tiles = a.tiles_m * a.tiles_n;
  const int units = tiles < max_units[dev & 63] ? tiles : max_units[dev & 63];
  cfg.gridDim = dim3(CG * units);
  a.pdl = g_gemm_pdl.load() ? 1 : 0;
  if (a.pdl) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = ++nattr;
  }
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, ty, a);
}

GemmArgs base_args(const float *sa, const float *sb, const void *bias, int M, int N, int K, int nout, int tile_n,
                   int tile_m = TM) {
  GemmArgs a = {};
  a.sa = sa;
  a.sb = sb;
  a.bias = (const bf16 *)bias;
  a.M = M;
  a.N = N;
  a.K = K;
  a.Nout = nout;
  a.tiles_m = (M + tile_m - 1) / tile_m;
  a.tiles_n = (nout + tile_n - 1) / tile_n;
  a.m_fast = M <= nout ? 1 : 0;  // walk the dimension whose operand is smaller, so it stays in L2
  return a;
}


// ------------------------------------------------------------------ split-K tiles for few rows
// Per-token W8A8 GEMMs with few rows (decode batches of 17-256 tokens) have too few 128 x 128 output tiles to put
// every SM on the weight stream, and each tile's time is its K loop of load round trips. Split-K: a cluster of S CTAs
// per tile, CTA r multiplying K blocks [r kbs, (r + 1) kbs) into its own TMEM. The S exact int32 partial tiles meet in
// distributed shared memory: each CTA writes its partial into its shared memory, the cluster synchronises, and CTA r
// adds the S partials of output columns [r 128/S, (r + 1) 128/S) (integers: exact in any order) and runs the
// per-token epilogue (epi_token, the same arithmetic as the one-CTA tile) on them. The result is bit-identical to
// the one-CTA tile. Roles: warp 0 TMA, warp 1 TMEM allocation and MMAs, warps 2-5 the epilogue (TMEM lane quarter
// warp % 4). No cluster multicast: every CTA loads its own A and B stages.
constexpr int SK_BN = 128;
constexpr int SK_THREADS = 192;
constexpr int SK_STAGES = 3;  // with <= 100 KB of shared memory a CTA of the next launch fits beside this one
// The partial tile in shared memory, laid out by the CTA that reduces each part: region p (the output columns
// [p W, (p + 1) W), W = 128 / S) holds 128 rows of W int32 plus a 16-byte pad per row (conflict-free row writes), so
// a peer reads its region as contiguous 16-byte chunks.
__host__ __device__ constexpr int sk_rstride(int S) { return SK_BN / S + 4; }
struct SkSmem {
  static constexpr int A_BYTES = TM * TK;
  static constexpr int B_BYTES = SK_BN * TK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 1024-byte multiple: every operand tile stays aligned
  static constexpr int PART_BYTES = 8 * TM * sk_rstride(8) * 4;  // the largest (S = 8); reuses the stages
  static constexpr int DATA_BYTES =
      SK_STAGES * STAGE_BYTES > PART_BYTES ? SK_STAGES * STAGE_BYTES : PART_BYTES;
  static constexpr int BAR_OFF = DATA_BYTES;
  static constexpr int NBARS = 2 * SK_STAGES + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  // this CTA's columns: weight scales [128], then bias [128]; the tile's per-token scales [128] (fp32, 16-byte reads)
  static constexpr int PAR_OFF = (MISC_OFF + 16 + 127) / 128 * 128;
  static constexpr int ALLOC = PAR_OFF + 3 * SK_BN * 4 + 1024;  // room to align the base to 1024
  static_assert(PAR_OFF % 16 == 0 && (sk_rstride(2) * 4) % 16 == 0 && (sk_rstride(8) * 4) % 16 == 0,
                "16-byte shared-memory vectors");
  static_assert(ALLOC <= 100 * 1024, "two CTAs per SM");
};

// a peer CTA's shared memory (the address from mapa, which itself follows the cluster barrier in program order); no
// memory clobber, so a run of these loads issues back to back
__device__ __forceinline__ uint4 ld_shared_cluster16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// S: CTAs per cluster (2, 4 or 8), kbs: K blocks (128 bytes of K) per CTA
template <bool GELU, int S>
__global__ void __launch_bounds__(SK_THREADS, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args, int kbs) {
  using L = SkSmem;
  constexpr uint32_t IDESC = idesc_i8(SK_BN, TM);
  constexpr uint32_t STAGE_TX = L::A_BYTES + L::B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::MISC_OFF);
  int *abort_flag = reinterpret_cast<int *>(smem + L::MISC_OFF + 4);
  auto bar_full = [&](int s) { return smem_addr(bars + s); };
  auto bar_empty = [&](int s) { return smem_addr(bars + SK_STAGES + s); };
  const uint32_t bar_tfull = smem_addr(bars + 2 * SK_STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = args.M, K = args.K;
  const uint32_t part = cluster_ctarank();  // this CTA's K part, and its share of the output columns
  int mt, nt;
  tile_coord((int)blockIdx.x / S, args, mt, nt);
  const int KB = (K + TK - 1) / TK;
  const int kb0 = (int)part * kbs;
  const int nkb = kb0 < KB ? (KB - kb0 < kbs ? KB - kb0 : kbs) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SK_STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    mbar_init(bar_tfull, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(SK_BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the epilogue's per-column parameters of this CTA's columns (immutable: loaded before any dependency wait, read
  // after the cluster barrier below)
  constexpr int W = SK_BN / S;
  const int c0 = (int)part * W;
  float *par_sw = reinterpret_cast<float *>(smem + L::PAR_OFF), *par_b = par_sw + SK_BN;
  float *par_sx = par_b + SK_BN;
  if (warp >= 2) {
    const int t = threadIdx.x - 64, n = nt * SK_BN + c0 + t;
    if (t < W) {
      par_sw[t] = n < args.Nout ? __ldg(args.sb + n) : 0.f;
      par_b[t] = (n < args.Nout && args.bias) ? bf2f(args.bias[n]) : 0.f;
    }
    // the per-token scales come from the previous kernel: waited for and loaded while the MMAs run
    if (args.pdl) pdl_wait();
    par_sx[t] = mt * TM + t < M ? __ldcg(args.sa + mt * TM + t) : 0.f;
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      auto sa = [&](int st) { return sbase + (uint32_t)(st * L::STAGE_BYTES); };
      auto sb = [&](int st) { return sbase + (uint32_t)(st * L::STAGE_BYTES + L::A_BYTES); };
      // programmatic dependent launch: the first stages' weights before the dependency wait, activations after it
      const int pre = args.pdl ? (nkb < SK_STAGES ? nkb : SK_STAGES) : 0;
      for (int j = 0; j < pre; ++j) {
        mbar_expect_tx(bar_full(j), STAGE_TX);
        tma_load_2d(sb(j), &tmB, bar_full(j), (kb0 + j) * TK, nt * SK_BN);
      }
      if (args.pdl) pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < nkb; ++i) {
        const int kx = (kb0 + i) * TK;
        if (i < pre) {
          tma_load_2d(sa(stage), &tmA, bar_full(stage), kx, mt * TM);  // B on its way, expect_tx posted
        } else {
          if (!mbar_wait(bar_empty(stage), phase ^ 1, abort_flag)) break;
          mbar_expect_tx(bar_full(stage), STAGE_TX);
          tma_load_2d(sa(stage), &tmA, bar_full(stage), kx, mt * TM);
          tma_load_2d(sb(stage), &tmB, bar_full(stage), kx, nt * SK_BN);
        }
        if (++stage == SK_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (args.pdl) pdl_trigger();  // every load is issued: the next kernel may start its own prologue
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(bar_full(stage), phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(sbase + (uint32_t)(stage * L::STAGE_BYTES));
        const uint64_t bd = sw128_desc(sbase + (uint32_t)(stage * L::STAGE_BYTES + L::A_BYTES));
#pragma unroll
        for (int k = 0; k < TK / 32; ++k) umma_i8(tmem_base, ad + 2 * k, bd + 2 * k, IDESC, (i | k) != 0);
        umma_commit(bar_empty(stage));
        if (++stage == SK_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      // the accumulator is complete once the MMAs retire; with nothing multiplied (or a wait given up) the epilogue
      // is released at once and writes zeros
      if (ok && nkb > 0)
        umma_commit(bar_tfull);
      else
        mbar_arrive(bar_tfull);
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps 2-5: the partial tile
    const int q = warp & 3, row = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    bool ok = warp_wait(bar_tfull, 0, abort_flag);
    int gave_up = lane == 0 ? *(volatile int *)abort_flag : 0;  // warp-uniform: the TMEM loads are .sync.aligned
    gave_up = __shfl_sync(0xffffffffu, gave_up, 0);
    ok = ok && nkb > 0 && !gave_up;
    tc_fence_after();
    constexpr int RS = sk_rstride(S);
#pragma unroll 1
    for (int c = 0; c < SK_BN / 32; ++c) {
      uint32_t r[32];
      if (ok) {
        tmem_ld32(tmem_base + lane_addr + c * 32, r);
        tmem_wait_tie(r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = c * 32 + 4 * j, p = col / W;  // region of the CTA that reduces this column
        st_shared16(sbase + (uint32_t)(((p * TM + row) * RS + col - p * W) * 4), r[4 * j], r[4 * j + 1], r[4 * j + 2],
                    r[4 * j + 3]);
      }
    }
    tc_fence_before();
  }
  __syncwarp();
  cluster_sync_all();  // every partial tile of the cluster is in its CTA's shared memory

  if (warp >= 2) {
    // ---------------------------------------------------------------- this CTA's columns: sum of S partials, epilogue
    // items = (row, 4-column chunk) of this CTA's region, consecutive threads on consecutive chunks of a row: every
    // warp-wide peer read is a few contiguous 128-byte runs
    constexpr int RS = sk_rstride(S), CPR = W / 4;  // chunks per row
    const int t = threadIdx.x - 64;
    const uint32_t region = sbase + (uint32_t)(part * TM * RS * 4);
    const int rows = M - mt * TM < TM ? M - mt * TM : TM;
    uint32_t peer[S];
#pragma unroll
    for (int p = 0; p < S; ++p) peer[p] = mapa_shared(region, (uint32_t)p);
#pragma unroll 2
    for (int i = t; i < rows * CPR; i += 128) {
      const int r = i / CPR, ch = i - r * CPR;
      const uint32_t off = (uint32_t)((r * RS + 4 * ch) * 4);
      uint4 v[S];
#pragma unroll
      for (int p = 0; p < S; ++p) v[p] = ld_shared_cluster16(peer[p] + off);
      int acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int p = 0; p < S; ++p) {
        acc[0] += (int)v[p].x;
        acc[1] += (int)v[p].y;
        acc[2] += (int)v[p].z;
        acc[3] += (int)v[p].w;
      }
      const int n = nt * SK_BN + c0 + 4 * ch;
      if (n >= args.Nout) continue;
      const float sxm = par_sx[r];
      const float4 s4 = *reinterpret_cast<const float4 *>(par_sw + 4 * ch);
      const float4 b4 = *reinterpret_cast<const float4 *>(par_b + 4 * ch);
      const float y0 = epi_token<GELU>(acc[0], sxm, s4.x, b4.x), y1 = epi_token<GELU>(acc[1], sxm, s4.y, b4.y);
      const float y2 = epi_token<GELU>(acc[2], sxm, s4.z, b4.z), y3 = epi_token<GELU>(acc[3], sxm, s4.w, b4.w);
      bf16 *yrow = args.Y + (size_t)(mt * TM + r) * args.Nout;
      if (n + 3 < args.Nout && (args.Nout & 3) == 0) {
        *reinterpret_cast<uint2 *>(yrow + n) = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
      } else {
        const float yv[4] = {y0, y1, y2, y3};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < args.Nout) yrow[n + e] = f2bf(yv[e]);
      }
    }
  }
  __syncwarp();
  // no CTA leaves while a peer may still read its partial tile. Relaxed: only execution is ordered here (every read
  // of a peer's partial has returned its value before this thread arrives); a release would also hold every thread
  // until its global stores of the output are acknowledged (measured: 4-6 us per launch)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(SK_BN) : "memory");
  }
}

// Clusters of S split-K CTAs that fit on the device at once (occupancy query, cached per device and S): a cluster's
// CTAs must share a GPC, and with one CTA per SM not every GPC holds two clusters of 8.
int sk_max_clusters(int S) {
  static std::once_flag once[64][4];
  static int n[64][4];
  int dev = 0;
  cudaGetDevice(&dev);
  const int si = S == 2 ? 1 : (S == 4 ? 2 : (S == 8 ? 3 : 0));
  std::call_once(once[dev & 63][si], [&] {
    int c = 0;
    const void *kern = S == 2 ? (const void *)gemm_sk_kernel<false, 2>
                              : (S == 4 ? (const void *)gemm_sk_kernel<false, 4> : (const void *)gemm_sk_kernel<false, 8>);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SkSmem::ALLOC) == cudaSuccess) {
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = S;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(S * 16);
      q.blockDim = dim3(SK_THREADS);
      q.dynamicSmemBytes = SkSmem::ALLOC;
      q.attrs = attr;
      q.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&c, kern, &q) != cudaSuccess) c = 0;
    }
    cudaGetLastError();
    n[dev & 63][si] = c;
  });
  return n[dev & 63][si];
}

// Split-K launch: grid = tiles x S CTAs, clusters of S consecutive CTAs along x (one tile each)
template <bool GELU, int S>
cudaError_t run_sk(const int8_t *A, const int8_t *B, GemmArgs a, cudaStream_t st) {
  auto kern = gemm_sk_kernel<GELU, S>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SkSmem::ALLOC);
  });
  if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
  CUtensorMap ta, tb;
  if (!make_map(&ta, A, a.K, a.M, TM) || !make_map(&tb, B, a.K, a.N, SK_BN)) return cudaErrorInvalidValue;
  const int KB = (a.K + TK - 1) / TK;
  const int kbs = (KB + S - 1) / S;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  attr[nattr].id = cudaLaunchAttributeClusterDimension;
  attr[nattr].val.clusterDim.x = S;
  attr[nattr].val.clusterDim.y = 1;
  attr[nattr].val.clusterDim.z = 1;
  ++nattr;
  a.pdl = g_gemm_pdl.load() ? 1 : 0;
  if (a.pdl) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.tiles_m * a.tiles_n * S);
  cfg.blockDim = dim3(SK_THREADS);
  cfg.dynamicSmemBytes = SkSmem::ALLOC;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, a, kbs);
}
template <bool GELU>
cudaError_t run_sk_s(const int8_t *A, const int8_t *B, GemmArgs a, int S, cudaStream_t st) {
  if (S == 2) return run_sk<GELU, 2>(A, B, a, st);
  if (S == 4) return run_sk<GELU, 4>(A, B, a, st);
  return run_sk<GELU, 8>(A, B, a, st);
}

}  // namespace

namespace {
// Failure-detection self-test: the pipeline's bounded wait on an mbarrier that nothing ever arrives on, with a short
// limit. The wait gives up, records the error word and returns; the kernel ends normally and the context stays usable.
__global__ void wait_timeout_selftest(long long limit) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_addr(&bar), 0, &abort_flag, limit);
}
}  // namespace

cudaError_t launch_wait_timeout_selftest(int limit_log2, cudaStream_t st) {
  wait_timeout_selftest<<<1, 32, 0, st>>>(1ll << limit_log2);
  return cudaGetLastError();
}

int gemm_device_error(bool clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(int));
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(int));
  }
  return v;
}

void gemm_set_pdl(bool on) { g_gemm_pdl.store(on); }

void gemm_set_tile_override(int bn) {
  g_tile_override = (bn == 1 || bn == 2 || bn == 4 || bn == 8 || bn == 64 || bn == 128 || bn == 256 || bn == -192 ||
                     bn == -256)
                        ? bn
                        : 0;
}

// CTAs per tile for split-K: while the 128 x 128 tiles fill fewer than half the SMs, the largest power of two <= 8
// that keeps the grid within the SMs and gives every CTA at least two 128-byte K blocks (force: regardless of the
// tile count). 1 = no split.
// Measured (graph-timed, M = 17..256): a long K gains most (K = 8192, N = 2048: 21.3 -> 7.9-13 us, S = 8 or 4); at
// K = 2048 only very few tiles gain (N = 2048: 7.5 -> 4.9-6.6 us with S = 4), while 48-64 tiles break even or lose
// (the partial tiles' exchange costs more than the shorter K loop saves).
int sk_split(int M, int N, int K, bool force) {
  const int sms = device_sm_count();
  const long tiles = (long)((M + TM - 1) / TM) * ((N + SK_BN - 1) / SK_BN);
  const int KB = (K + TK - 1) / TK;
  if (!force && (2 * tiles > sms || (KB < 32 && tiles > 16))) return 1;
  int S = (!force && KB < 32) ? 4 : 8;
  // at most one CTA per SM in all, and clusters the device can hold at once (with 100 KB per CTA two clusters' CTAs
  // share an SM, so up to twice the one-per-SM count)
  while (S > 1 && (tiles * S > sms || KB / S < 2 || tiles > 2 * sk_max_clusters(S))) S /= 2;
  return S;
}

cudaError_t launch_gemm_i8(const int8_t *A, const float *sa, const int8_t *B, const float *sb, const void *bias, void *Y,
                           int M, int N, int K, bool gelu, bool grouped, cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (grouped) {
    GemmArgs a = base_args(sa, sb, bias, M, N, K, N, 128);
    a.Y = (bf16 *)Y;
    return gelu ? run_tc<128, 5, 4, EPI_GROUP, true, 1>(A, B, a, st) : run_tc<128, 5, 4, EPI_GROUP, false, 1>(A, B, a, st);
  }
  const int ov = g_tile_override.load() == 64 ? 0 : g_tile_override.load();  // 64: a W8A16-only choice
  if (!ov && a8_rows(M, N, K)) {
    // skinny: the A8 GEMV streams W once with int8 MMAs (same exact int32 sums and the same epilogue)
    return launch_gemv_a8(B, sb, A, sa, bias, Y, N, K, M, gelu, g_gemm_pdl.load(), st);
  }
  // few tiles: K split over a cluster of CTAs per 128 x 128 tile (1: forced wherever K has two blocks per CTA;
  // 2, 4, 8: that many CTAs per tile)
  if (!ov || ov == 1 || ov == 2 || ov == 4 || ov == 8) {
    const int S = ov > 1 ? ov : sk_split(M, N, K, ov == 1);
    if (S > 1) {
      GemmArgs a = base_args(sa, sb, bias, M, N, K, N, SK_BN);
      a.Y = (bf16 *)Y;
      return gelu ? run_sk_s<true>(A, B, a, S, st) : run_sk_s<false>(A, B, a, S, st);
    }
  }
  int bn = (ov == 1 || ov == 2 || ov == 4 || ov == 8) ? 0 : ov;
  if (!bn) {
    // 256 x 256 CTA-pair tiles when there are at least 1.5 per cluster (3-10% faster than one CTA per 128 x 256 tile
    // at 65536 rows, K = 1152 .. 8192); fewer pair tiles leave too much of the last wave idle, so one CTA per
    // 128 x 256 tile while those fill half the SMs (M = 1024: 5-10% faster than 128 x 128), else 128 x 128
    const int sms = device_sm_count();
    const long tiles256 = (long)((M + TM - 1) / TM) * ((N + 255) / 256);
    const long pair_tiles = (long)((M + 2 * TM - 1) / (2 * TM)) * ((N + 255) / 256);
    bn = 2 * pair_tiles >= 3 * (sms / 2) ? -256 : (2 * tiles256 >= sms ? 256 : 128);
  }
  GemmArgs a = base_args(sa, sb, bias, M, N, K, N, bn < 0 ? -bn : bn, bn < 0 ? 2 * TM : TM);
  a.Y = (bf16 *)Y;
  if (bn == -256)
    return gelu ? run_tc<256, 6, 2, EPI_TOKEN, true, 2>(A, B, a, st)
                : run_tc<256, 6, 2, EPI_TOKEN, false, 2>(A, B, a, st);
  if (bn == -192)
    return gelu ? run_tc<192, 6, 2, EPI_TOKEN, true, 2>(A, B, a, st)
                : run_tc<192, 6, 2, EPI_TOKEN, false, 2>(A, B, a, st);
  if (bn == 256)
    return gelu ? run_tc<256, 4, 2, EPI_TOKEN, true, 1>(A, B, a, st)
                : run_tc<256, 4, 2, EPI_TOKEN, false, 1>(A, B, a, st);
  return gelu ? run_tc<128, 6, 2, EPI_TOKEN, true, 1>(A, B, a, st) : run_tc<128, 6, 2, EPI_TOKEN, false, 1>(A, B, a, st);
}

cudaError_t launch_gemm_i8_q(const int8_t *A, const float *saT, const int8_t *B, const float *sb, const void *bias,
                             int8_t *Yq, float *YsT, int M, int N, int K, bool gelu, cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  GemmArgs a = base_args(saT, sb, bias, M, N, K, N, 128);
  a.Yq = Yq;
  a.YsT = YsT;
  return gelu ? run_tc<128, 6, 4, EPI_GROUP_Q, true, 1>(A, B, a, st)
              : run_tc<128, 6, 4, EPI_GROUP_Q, false, 1>(A, B, a, st);
}

cudaError_t launch_gemm_i8_silu(const int8_t *A, const float *sa, const int8_t *B, const float *sb, const void *bias,
                                void *Y, int M, int I, int K, cudaStream_t st) {
  if (M <= 0 || I <= 0) return cudaSuccess;
  // CTA pairs (256 rows x 128 output columns per tile) when one-CTA tiles would fill the GPU, unless a one-CTA tile
  // width is forced
  const long tiles1 = (long)((M + TM - 1) / TM) * ((I + 127) / 128);
  const int ov = g_tile_override.load();
  const bool pair = ov < 0 || (ov == 0 && tiles1 >= device_sm_count());
  GemmArgs a = base_args(sa, sb, bias, M, 2 * I, K, I, 128, pair ? 2 * TM : TM);
  a.Y = (bf16 *)Y;
  if (pair) return run_tc<256, 6, 2, EPI_SILU, false, 2>(A, B, a, st);
  return run_tc<256, 4, 2, EPI_SILU, false, 1>(A, B, a, st);
}

}  // namespace lfm2q

namespace lfm2q {
// W8A16: y = bf16(act(((bf16 x) . (int8 W -> bf16)^T) * sw + b)), fp32 accumulation in TMEM (tcgen05 kind::f16).
// Reference: gemm_w8_kernel / launch_gemm_w8 (kernels/int8_gemm.cu:306-388, :765-780), op gemm_w8
// (kernels/int8_gemm.cpp:72-79). CTA pairs on 256 x 256 tiles when one-CTA 128 x 256 tiles fill the GPU, one CTA per
// 128 x 128 tile while those fill it, else one CTA per 128 x 64 tile; a forced tile width (lfm2q_set_gemm_tile) picks
// the same way by sign (64: the narrow tile).
cudaError_t launch_gemm_w8(const void *x, const int8_t *w, const float *sw, const void *bias, void *y, int M, int N,
                           int K, bool gelu, cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  const int ov = g_tile_override.load();
  if (M <= 16 && bias == nullptr && !gelu && K % 64 == 0 && ov == 0) {
    // a few tokens, no bias / activation: y = bf16(acc * sw) is the weight-only decode GEMV, which streams W once
    return launch_gemv(w, true, sw, x, y, N, K, 0, M, false, st);
  }
  const int sms = device_sm_count();
  const long tiles_m = (M + TM - 1) / TM;
  const bool pair = ov < 0 || (ov == 0 && tiles_m * ((N + 255) / 256) >= sms);
  // Few 128-column tiles (decode batches, small M): 64-column tiles put twice as many SMs on the weight stream; each
  // CTA's MMA and conversion work per stage halves, which is what bounds a one-tile-per-CTA launch.
  const bool narrow = ov == 64 || (ov == 0 && !pair && tiles_m * ((N + 127) / 128) < sms);
  const int bn = pair ? 256 : (narrow ? 64 : 128);
  GemmArgs a = base_args(nullptr, sw, bias, M, N, K, N, bn, pair ? 2 * TM : TM);
  a.Y = (bf16 *)y;
  if (pair)
    return gelu ? run_tc<256, 5, 2, EPI_W8, true, 2>(x, w, a, st) : run_tc<256, 5, 2, EPI_W8, false, 2>(x, w, a, st);
  if (narrow)
    return gelu ? run_tc<64, 7, 4, EPI_W8, true, 1>(x, w, a, st) : run_tc<64, 7, 4, EPI_W8, false, 1>(x, w, a, st);
  return gelu ? run_tc<128, 5, 2, EPI_W8, true, 1>(x, w, a, st) : run_tc<128, 5, 2, EPI_W8, false, 1>(x, w, a, st);
}
}  // namespace lfm2q
