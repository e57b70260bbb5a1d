// Shared device helpers for the lfm2q kernels (sm_100a only).
//
// Every kernel in this library is written for B200 (compute capability 10.0a): 32-wide warps, 148 SMs,
// tcgen05 tensor cores with TMEM accumulators, TMA bulk-tensor copies, HBM3e. Nothing here has a path
// for another architecture; the host layer refuses to launch on anything but an sm_100 device.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lfm2q {

typedef __nv_bfloat16 bf16;

// ------------------------------------------------------------------ scalar conversions
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
// round an fp32 value to bf16 and back (the rounding point of every bf16 tensor op)
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// symmetric int8 code of v at scale sc: the IEEE quotient rounded half-to-even, clamped to +-127
__device__ __forceinline__ int q8(float v, float sc) {
  const int q = __float2int_rn(__fdiv_rn(v, sc));
  return max(-127, min(127, q));
}

// The same code without a division per element (rinv = 1 / sc, IEEE). For |v / sc| <= 127.5 the estimate
// t = v * rinv lies within 2.3e-5 of the IEEE quotient, so both round to the same integer unless t is within that
// distance of a half-integer; only then (a few elements in 10^4) is the quotient divided out exactly. Rounding to
// an integer is an add of 1.5 * 2^23 (ties to even), and the integer is read from the sum's bits.
__device__ __forceinline__ int q8r(float v, float sc, float rinv) {
  const float big = 12582912.f;
  const float t = __fmul_rn(v, rinv);
  float tb = __fadd_rn(t, big);
  if (fabsf(__fsub_rn(t, __fsub_rn(tb, big))) > 0.49996f) tb = __fadd_rn(rintf(__fdiv_rn(v, sc)), big);
  return max(-127, min(127, __float_as_int(tb) - 0x4B400000));
}

// ------------------------------------------------------------------ packed fp32 pairs (sm_100 f32x2 arithmetic)
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// d = a * b + c on each half, one rounding each (two fmaf)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Two int8 codes at once, as q8r, returned as the rounding sums 1.5 * 2^23 + code: the code is the low byte of
// the sum's bits. No clamp is needed: with sc = RN(max(amax, 1e-8) / 127) and |v| <= amax, |v / sc| <= 127 *
// (1 + 2^-23), so both the estimate and the IEEE quotient round to an integer of magnitude <= 127.
__device__ __forceinline__ float2 q8r2(float2 v, float sc, float rinv) {
  const float2 big = make_float2(12582912.f, 12582912.f);
  const float2 t = fmul2(v, make_float2(rinv, rinv));
  float2 tb = fadd2(t, big);
  const float2 d = fsub2(t, fsub2(tb, big));
  if (fmaxf(fabsf(d.x), fabsf(d.y)) > 0.49996f) {
    tb.x = __fadd_rn(rintf(__fdiv_rn(v.x, sc)), 12582912.f);
    tb.y = __fadd_rn(rintf(__fdiv_rn(v.y, sc)), 12582912.f);
  }
  return tb;
}
// 4 int8 codes (bytes of w) -> two bf16x2 words (lo: bytes 0,1; hi: bytes 2,3), exact: each byte + 128 goes into
// the mantissa of 2^23 (one byte permute), a packed fp32 subtraction of 2^23 + 128 leaves the code as an exact fp32,
// whose upper half is its bf16 encoding (|q| <= 127 has at most 7 significant bits).
__device__ __forceinline__ void i8x4_to_bf16x2x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const uint32_t u = w ^ 0x80808080u;  // q + 128 in 0..255
  const float2 bias = make_float2(8388736.f, 8388736.f);  // 2^23 + 128
  const float2 f01 = fsub2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)),
                                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651))), bias);
  const float2 f23 = fsub2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)),
                                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653))), bias);
  lo = __byte_perm(__float_as_uint(f01.x), __float_as_uint(f01.y), 0x7632);
  hi = __byte_perm(__float_as_uint(f23.x), __float_as_uint(f23.y), 0x7632);
}

// low bytes of four rounding sums (see q8r2) -> one word of int8 codes
__device__ __forceinline__ uint32_t pack_sums4(float2 a, float2 b) {
  return __byte_perm(__byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x0040),
                     __byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x0040), 0x5410);
}

// four int8 codes -> one word (byte 0 = a)
__device__ __forceinline__ uint32_t pack_i8x4(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// 16-byte load through L2 (ld.global.cg), for data the previous kernel in the stream wrote. A kernel launched with
// programmatic dependent launch starts before its predecessor has finished; after griddepcontrol.wait the
// predecessor's stores are in L2, but a line of the same address cached in this SM's L1 or read-only path could be
// stale, so activations and their scales are never read through those caches.
__device__ __forceinline__ uint4 ld_cg16(const void *p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// ------------------------------------------------------------------ warp reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ W8A8 epilogue (shared by every W8A8 kernel)
// F.gelu(v, approximate="tanh") = 0.5 v (1 + tanh(u)), u = sqrt(2/pi) (v + 0.044715 v^3), evaluated as the equal
// v / (1 + exp(-2u)): no cancellation near tanh = -1, one exponential and one reciprocal per element.
__device__ __forceinline__ float gelu_tanh(float v) {
  const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return __fdividef(v, 1.f + __expf(-2.f * u));
}
// y = act(((float)acc * sx[m]) * sw[n] + b[n]) in the reference's fp32 operation order (kernels/int8_gemm.cu:93-115,
// no contraction); (float)acc rounds the exact int32 to nearest even, as torch's .float() does.
template <bool GELU>
__device__ __forceinline__ float epi_token(int acc, float sxm, float sw, float b) {
  float y = __fmul_rn((float)acc, sxm);
  y = __fadd_rn(__fmul_rn(y, sw), b);
  if (GELU) y = gelu_tanh(y);
  return y;
}

// The first product of two adjacent columns is one packed f32x2 multiply; the scale-and-bias step stays scalar:
// ptxas may contract a packed mul.rn.f32x2 feeding an add into a fused multiply-add (observed on sm_100a), which
// would skip the reference's rounding of the product. Each value is rounded as in epi_token, bit for bit.
__device__ __forceinline__ float2 epi_pair(uint32_t acc0, uint32_t acc1, float sxm, float sw0, float sw1, float b0,
                                           float b1) {
  const float2 y = fmul2(make_float2((float)(int)acc0, (float)(int)acc1), make_float2(sxm, sxm));
  return make_float2(__fadd_rn(__fmul_rn(y.x, sw0), b0), __fadd_rn(__fmul_rn(y.y, sw1), b1));
}
// Two adjacent columns of epi_token, returned as two packed bf16.
template <bool GELU>
__device__ __forceinline__ uint32_t epi_token2(uint32_t acc0, uint32_t acc1, float sxm, float sw0, float sw1,
                                               float b0, float b1) {
  float2 y = epi_pair(acc0, acc1, sxm, sw0, sw1, b0, b1);
  if (GELU) {
    y.x = gelu_tanh(y.x);
    y.y = gelu_tanh(y.y);
  }
  return pack_bf16x2(y.x, y.y);
}

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while its predecessor drains.
// Before pdl_wait() it may only read immutable data (weights); pdl_wait() returns once the previous
// grid's writes are visible. Both are no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace lfm2q
