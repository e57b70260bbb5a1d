// C ABI of liblfm2q (include/lfm2q.h): host-side argument checks, device check, dispatch to the launchers.
//
// The checks restate the reference bindings' TORCH_CHECKs (kernels/int8_gemm.cpp:20-141,
// kernels/lfm2_decode.cpp:73-150) with the limits of this build, and run before anything touches the device,
// so a bad call returns LFM2Q_EINVAL (and a message) on any machine, with or without a GPU.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lfm2q.h"
#include "launch.h"

namespace lfm2q {

static thread_local std::string g_last_error;
static std::atomic<bool> g_pdl{true};

static int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device facts, filled once per device (std::call_once: concurrent first calls from several threads see the
// complete record).
struct DevInfo {
  int sms = 0;
  int supported = 0;
};
static DevInfo g_dev[64];
static std::once_flag g_dev_once[64];

static const DevInfo &dev_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    static const DevInfo none;
    return none;
  }
  std::call_once(g_dev_once[dev], [dev] {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_dev[dev].sms = sms;
    g_dev[dev].supported = (major == 10 && minor == 0) ? 1 : 0;
  });
  return g_dev[dev];
}

int device_sm_count() {
  const int s = dev_info().sms;
  return s > 0 ? s : 148;
}
bool device_is_sm100() { return dev_info().supported == 1; }

static int device_gate() {
  if (!device_is_sm100())
    return fail(LFM2Q_ENOTSUP, "lfm2q: the current CUDA device is not an sm_100 (B200) GPU, or no device is visible");
  return LFM2Q_OK;
}

static int launched(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return LFM2Q_OK;
  return fail(LFM2Q_ECUDA, std::string("lfm2q: ") + what + ": " + cudaGetErrorString(e));
}

#define REQUIRE(cond, msg) \
  do {                     \
    if (!(cond)) return fail(LFM2Q_EINVAL, std::string("lfm2q: ") + (msg)); \
  } while (0)

}  // namespace lfm2q

using namespace lfm2q;

extern "C" {

const char *lfm2q_last_error(void) { return g_last_error.c_str(); }

const char *lfm2q_version(void) { return "lfm2q 0.1.0 (sm_100a)"; }

int lfm2q_device_supported(void) { return device_is_sm100() ? 1 : 0; }

int lfm2q_check_device(int clear) {
  if (int e = device_gate()) return e;
  const int v = gemm_device_error(clear != 0);
  const int a = attn_device_error(clear != 0);
  if (v) return fail(LFM2Q_ETIMEOUT, "lfm2q: a GEMM pipeline wait timed out on the device");
  if (a) return fail(LFM2Q_ETIMEOUT, "lfm2q: a decode-attention stage wait timed out on the device");
  return LFM2Q_OK;
}

int lfm2q_selftest_wait_timeout(int limit_log2, void *stream) {
  REQUIRE(limit_log2 >= 10 && limit_log2 <= 31, "limit_log2 must be in [10, 31] (clock cycles = 2^limit_log2)");
  if (int e = device_gate()) return e;
  return launched(launch_wait_timeout_selftest(limit_log2, (cudaStream_t)stream), "selftest_wait_timeout");
}

void lfm2q_set_pdl(int on) {
  g_pdl.store(on != 0);
  gemm_set_pdl(on != 0);
}
void lfm2q_set_gemv_trigger(int early) { gemv_set_early_trigger(early != 0); }
void lfm2q_set_gemv_impl(int) {}
void lfm2q_set_gemv_path(int path) { gemv_set_impl(path >= 1 && path <= 4 ? path : 0); }
void lfm2q_set_gemm_tile(int bn) { gemm_set_tile_override(bn); }

// ------------------------------------------------------------------ quantizers
int lfm2q_quant_rows(const uint16_t *x, int8_t *q, float *s, int rows, int K, void *stream) {
  REQUIRE(rows >= 0 && K > 0, "rows must be >= 0 and K > 0");
  REQUIRE(K % 8 == 0 && K <= 16384, "K must be a multiple of 8, <= 16384");
  REQUIRE(rows == 0 || (x && q && s), "x, q and s must be non-null");
  REQUIRE(aligned16(x) && aligned16(q), "x and q must be 16-byte aligned");
  if (rows == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  // programmatic dependent launch at every size: the quantizer's launch overlaps the previous kernel's tail and the
  // GEMM after it starts its weight loads early (config-5 job at 8192 rows per GPU: 13.6 -> 13.2 ms per step; no
  // change at 65536 rows)
  return launched(launch_quant_rows(x, q, s, rows, K, g_pdl.load(), (cudaStream_t)stream), "quant_rows");
}

int lfm2q_quant_groups(const uint16_t *x, int8_t *q, float *sT, int rows, int K, void *stream) {
  REQUIRE(rows >= 0 && K > 0, "rows must be >= 0 and K > 0");
  REQUIRE(K % 64 == 0 && K <= 16384, "grouped shapes: K must be a multiple of 64, <= 16384");
  REQUIRE(rows == 0 || (x && q && sT), "x, q and s must be non-null");
  REQUIRE(aligned16(x) && aligned16(q), "x and q must be 16-byte aligned");
  if (rows == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_quant_groups(x, q, sT, rows, K, g_pdl.load(), (cudaStream_t)stream),
                  "quant_groups");
}

// ------------------------------------------------------------------ GEMMs
static int check_gemm_common(const void *w, const float *sw, const uint16_t *bias, const void *y, int M, int N,
                             int K) {
  REQUIRE(M >= 0 && N > 0 && K > 0, "need M >= 0, N > 0, K > 0");
  REQUIRE(K % 16 == 0 && N % 8 == 0, "need K % 16 == 0 and N % 8 == 0");
  REQUIRE(w && sw && y, "w, sw and y must be non-null");
  REQUIRE(aligned16(w) && aligned16(sw) && aligned16(y) && aligned16(bias), "w, sw, bias and y must be 16-byte aligned");
  return LFM2Q_OK;
}

int lfm2q_gemm_i8(const int8_t *xq, const float *sx, int grouped, const int8_t *w, const float *sw,
                  const uint16_t *bias, uint16_t *y, int M, int N, int K, int gelu, void *stream) {
  if (int e = check_gemm_common(w, sw, bias, y, M, N, K)) return e;
  REQUIRE(M == 0 || (xq && sx), "xq and sx must be non-null");
  REQUIRE(aligned16(xq), "xq must be 16-byte aligned");
  if (grouped) REQUIRE(K % 64 == 0, "sx shape: grouped scales need K % 64 == 0");
  if (M == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_gemm_i8(xq, sx, w, sw, bias, y, M, N, K, gelu != 0, grouped != 0, (cudaStream_t)stream),
                  "gemm_i8");
}

int lfm2q_gemm_i8_q(const int8_t *xq, const float *sxT, const int8_t *w, const float *sw, const uint16_t *bias,
                    int8_t *yq, float *ysT, int M, int N, int K, int gelu, void *stream) {
  REQUIRE(M >= 0 && N > 0 && K > 0, "need M >= 0, N > 0, K > 0");
  REQUIRE(K % 64 == 0, "sxT shape: K must be a multiple of 64");
  REQUIRE(N % 128 == 0, "w [N, K] with N % 128 == 0");
  REQUIRE(w && sw && yq && ysT && (M == 0 || (xq && sxT)), "pointers must be non-null");
  REQUIRE(aligned16(xq) && aligned16(w) && aligned16(sw) && aligned16(bias) && aligned16(yq),
          "xq, w, sw, bias and yq must be 16-byte aligned");
  if (M == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_gemm_i8_q(xq, sxT, w, sw, bias, yq, ysT, M, N, K, gelu != 0, (cudaStream_t)stream),
                  "gemm_i8_q");
}

int lfm2q_gemm_i8_silu(const int8_t *xq, const float *sx, const int8_t *w, const float *sw, const uint16_t *bias,
                       uint16_t *y, int M, int I, int K, void *stream) {
  REQUIRE(M >= 0 && I > 0 && K > 0, "need M >= 0, I > 0, K > 0");
  REQUIRE(K % 16 == 0 && I % 8 == 0, "need K % 16 == 0 and I % 8 == 0");
  REQUIRE(w && sw && y && (M == 0 || (xq && sx)), "pointers must be non-null");
  REQUIRE(aligned16(xq) && aligned16(w) && aligned16(sw) && aligned16(bias) && aligned16(y),
          "xq, w, sw, bias and y must be 16-byte aligned");
  REQUIRE(aligned16(sw + I) && aligned16(bias ? bias + I : nullptr), "I must keep the up-half scales 16-byte aligned");
  if (M == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_gemm_i8_silu(xq, sx, w, sw, bias, y, M, I, K, (cudaStream_t)stream), "gemm_i8_silu");
}

int lfm2q_gemm_w8(const uint16_t *x, const int8_t *w, const float *sw, const uint16_t *bias, uint16_t *y, int M,
                  int N, int K, int gelu, void *stream) {
  if (int e = check_gemm_common(w, sw, bias, y, M, N, K)) return e;
  REQUIRE(M == 0 || x, "x must be non-null");
  REQUIRE(aligned16(x), "x must be 16-byte aligned");
  if (M == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_gemm_w8(x, w, sw, bias, y, M, N, K, gelu != 0, (cudaStream_t)stream), "gemm_w8");
}

// ------------------------------------------------------------------ producers
int lfm2q_add_layernorm_q(uint16_t *h, const uint16_t *y, const uint16_t *w, const uint16_t *b, int8_t *q, float *s,
                          int rows, int D, float eps, int grouped, void *stream) {
  REQUIRE(rows >= 0 && D > 0, "rows must be >= 0 and D > 0");
  REQUIRE(D % 8 == 0 && D <= 16384, "D must be a multiple of 8, <= 16384");
  if (grouped) REQUIRE(D % 64 == 0, "s shape: grouped scales need D % 64 == 0");
  REQUIRE(h && w && b && q && s, "h, w, b, q and s must be non-null");
  REQUIRE(aligned16(h) && aligned16(y) && aligned16(w) && aligned16(b) && aligned16(q),
          "h, y, w, b and q must be 16-byte aligned");
  if (rows == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_add_layernorm_q(h, y, w, b, q, s, rows, D, eps, grouped != 0, (cudaStream_t)stream),
                  "add_layernorm_q");
}

int lfm2q_add_rmsnorm_q(uint16_t *h, const uint16_t *y, const uint16_t *w, int8_t *q, float *s, int rows, int H,
                        float eps, int grouped, void *stream) {
  REQUIRE(rows >= 0 && H > 0, "rows must be >= 0 and H > 0");
  REQUIRE(H % 8 == 0 && H <= 16384, "w shape: H must be a multiple of 8, <= 16384");
  if (grouped) REQUIRE(H % 64 == 0, "s shape: grouped scales need H % 64 == 0");
  REQUIRE(h && w && q && s, "h, w, q and s must be non-null");
  REQUIRE(aligned16(h) && aligned16(y), "h and y must be 16-byte aligned");
  if (rows == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_add_rmsnorm_q(h, y, w, q, s, rows, H, eps, grouped != 0, (cudaStream_t)stream),
                  "add_rmsnorm_q");
}

int lfm2q_silu_mul_q(const uint16_t *g, int8_t *q, float *s, int rows, int I, int grouped, void *stream) {
  REQUIRE(rows >= 0 && I > 0, "rows must be >= 0 and I > 0");
  REQUIRE(I % 8 == 0 && I <= 16384, "I shape: I must be a multiple of 8, <= 16384");
  if (grouped) REQUIRE(I % 64 == 0, "s shape: grouped scales need I % 64 == 0");
  REQUIRE(g && q && s, "g, q and s must be non-null");
  REQUIRE(aligned16(g), "g must be 16-byte aligned");
  if (rows == 0) return LFM2Q_OK;
  if (int e = device_gate()) return e;
  return launched(launch_silu_mul_q(g, q, s, rows, I, grouped != 0, (cudaStream_t)stream), "silu_mul_q");
}

// ------------------------------------------------------------------ GEMV
int lfm2q_gemv(const void *W, int w_is_int8, const float *scale, const uint16_t *x, uint16_t *y, int N, int K,
               int rows, int B, void *stream) {
  REQUIRE(N > 0 && K > 0 && B >= 1, "x [B, K], y [B, N]: need N > 0, K > 0, B >= 1");
  REQUIRE(K % (w_is_int8 ? 512 : 256) == 0, "K must be a multiple of 256 (bf16) / 512 (int8)");
  REQUIRE(W && x && y, "W, x and y must be non-null");
  REQUIRE(!w_is_int8 || scale, "int8 W needs fp32 scale");
  REQUIRE(aligned16(W) && aligned16(x), "W and x must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_gemv(W, w_is_int8 != 0, scale, x, y, N, K, rows, B, g_pdl.load(), (cudaStream_t)stream),
                  "gemv");
}

int lfm2q_gemv_a8(const int8_t *W, const float *sw, const int8_t *xq, const float *sx, const uint16_t *bias,
                  uint16_t *y, int N, int K, int B, int gelu, void *stream) {
  REQUIRE(N > 0 && K > 0 && B >= 1, "xq [B, K], y [B, N]: need N > 0, K > 0, B >= 1");
  REQUIRE(K % 64 == 0, "K must be a multiple of 64");
  REQUIRE(W && sw && xq && sx && y, "W, sw, xq, sx and y must be non-null");
  REQUIRE(aligned16(W) && aligned16(xq) && aligned16(y) && aligned16(bias), "W, xq, bias and y must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_gemv_a8(W, sw, xq, sx, bias, y, N, K, B, gelu != 0, g_pdl.load(), (cudaStream_t)stream),
                  "gemv_a8");
}

int lfm2q_linear_a8(const uint16_t *x, const int8_t *W, const float *sw, const uint16_t *bias, uint16_t *y, int N,
                    int K, int B, int gelu, void *stream) {
  REQUIRE(N > 0 && K > 0 && B >= 1, "x [B, K], y [B, N]: need N > 0, K > 0, B >= 1");
  REQUIRE(K % 64 == 0 && K <= 16384, "K must be a multiple of 64, <= 16384");
  REQUIRE(W && sw && x && y, "W, sw, x and y must be non-null");
  REQUIRE(aligned16(W) && aligned16(x) && aligned16(y) && aligned16(bias), "W, x, bias and y must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_linear_a8(x, W, sw, bias, y, N, K, B, gelu != 0, g_pdl.load(), (cudaStream_t)stream),
                  "linear_a8");
}

int lfm2q_gemv_chain(const lfm2q_gemv_layer *layers, int n_layers, int B, void *stream) {
  REQUIRE(n_layers >= 1 && n_layers <= LFM2Q_CHAIN_MAX_LAYERS, "n_layers must be in [1, 96]");
  REQUIRE(B >= 1 && B <= LFM2Q_CHAIN_MAX_TOKENS, "x [B, K]: the chained GEMV takes 1 <= B <= 4 tokens");
  REQUIRE(layers != nullptr, "layers must be non-null");
  std::vector<ChainLayer> L((size_t)n_layers);
  for (int l = 0; l < n_layers; ++l) {
    const lfm2q_gemv_layer &g = layers[l];
    const std::string at = "layer " + std::to_string(l) + ": ";
    REQUIRE(g.W && g.scale && g.x && g.y, at + "W, scale, x and y must be non-null");
    REQUIRE(aligned16(g.W) && aligned16(g.x), at + "W and x must be 16-byte aligned");
    REQUIRE(g.N > 0 && g.K >= 512 && g.K % 512 == 0, at + "need N > 0 and K a positive multiple of 512");
    const uintptr_t x0 = reinterpret_cast<uintptr_t>(g.x), x1 = x0 + (size_t)B * g.K * 2;
    const uintptr_t y0 = reinterpret_cast<uintptr_t>(g.y), y1 = y0 + (size_t)B * g.N * 2;
    REQUIRE(x1 <= y0 || y1 <= x0, at + "y must not overlap x");
    L[(size_t)l] = ChainLayer{g.W, g.scale, g.x, g.y, g.N, g.K};
  }
  if (int e = device_gate()) return e;
  return launched(launch_gemv_chain(L.data(), n_layers, B, g_pdl.load(), (cudaStream_t)stream), "gemv_chain");
}

int lfm2q_gemv_w4(const uint8_t *Wp, const float *S, const uint16_t *x, uint16_t *y, int N, int K, int group, int B,
                  void *stream) {
  REQUIRE(N > 0 && K > 0 && B >= 1 && B <= 4, "Wp [N, K/2], x [B, K]: need N > 0, K > 0, 1 <= B <= 4");
  REQUIRE(group > 0 && group % 128 == 0 && K % group == 0, "group size must be a multiple of 128 dividing K");
  REQUIRE(Wp && S && x && y, "Wp, S, x and y must be non-null");
  REQUIRE(aligned16(Wp) && aligned16(x), "Wp and x must be 16-byte aligned");
  REQUIRE(gemv_w4_slices(K, B) != 0, "K too large for this batch (B * K <= 16384 and the token slices in 160 KB)");
  if (int e = device_gate()) return e;
  return launched(launch_gemv_w4(Wp, S, x, y, N, K, group, B, g_pdl.load(), gemv_trigger_mode(), (cudaStream_t)stream),
                  "gemv_w4");
}

int lfm2q_gemv_epi(int epi, const void *W, int w_is_int8, const float *scale, const uint16_t *x, uint16_t *y, int S,
                   int K, uint16_t *state, const uint16_t *cw, const uint16_t *cbias, void *stream) {
  REQUIRE(epi == 0 || epi == 1, "epi 0 (swiglu) or 1 (shortconv)");
  REQUIRE(S > 0 && K > 0, "batch 1: x [1, K], y [1, S]");
  REQUIRE(K % (w_is_int8 ? 512 : 256) == 0, "K must be a multiple of 256 (bf16) / 512 (int8)");
  REQUIRE(W && x && y, "W, x and y must be non-null");
  REQUIRE(!w_is_int8 || scale, "int8 W needs fp32 scale");
  REQUIRE(epi == 0 || (state && cw), "shortconv epilogue needs state and conv weight");
  REQUIRE(aligned16(W) && aligned16(x), "W and x must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_gemv_epi(epi, W, w_is_int8 != 0, scale, x, y, S, K, state, cw, cbias, g_pdl.load(),
                                  (cudaStream_t)stream),
                  "gemv_epi");
}

// ------------------------------------------------------------------ decode step kernels
int lfm2q_add_rmsnorm(uint16_t *h, const uint16_t *y, const uint16_t *w, uint16_t *x, int rows, int H, float eps,
                      void *stream) {
  REQUIRE(rows >= 0 && H > 0 && H <= 8192, "h [rows, H]: need rows >= 0 and 0 < H <= 8192");
  if (rows == 0) return LFM2Q_OK;
  REQUIRE(h && w && x, "h, w and x must be non-null");
  if (int e = device_gate()) return e;
  return launched(launch_add_rmsnorm(h, y, w, x, rows, H, eps, g_pdl.load(), (cudaStream_t)stream), "add_rmsnorm");
}

int lfm2q_embed_rmsnorm(const int64_t *tok, const uint16_t *embed, const uint16_t *w, uint16_t *h, uint16_t *x,
                        int rows, int H, float eps, void *stream) {
  REQUIRE(rows >= 0 && H > 0 && H <= 8192, "embed [V, H], h / x [rows, H]: need rows >= 0 and 0 < H <= 8192");
  if (rows == 0) return LFM2Q_OK;
  REQUIRE(tok && embed && w && h && x, "tok, embed, w, h and x must be non-null");
  if (int e = device_gate()) return e;
  return launched(launch_embed_rmsnorm(tok, embed, w, h, x, rows, H, eps, g_pdl.load(), (cudaStream_t)stream),
                  "embed_rmsnorm");
}

int lfm2q_argmax_next(const uint16_t *logits, int64_t *tok, int64_t *pos, int B, int V, void *stream) {
  REQUIRE(B >= 0 && B <= 65535 && V > 0, "logits [B, V]: need 0 <= B <= 65535 and V > 0");
  if (B == 0) return LFM2Q_OK;
  REQUIRE(logits && tok, "logits and tok must be non-null");
  REQUIRE(aligned16(logits) && (V % 8 == 0 || B == 1),
          "logits must be 16-byte aligned, and V a multiple of 8 when B > 1 (every row 16-byte aligned)");
  if (int e = device_gate()) return e;
  return launched(launch_argmax_next(logits, tok, pos, B, V, g_pdl.load(), (cudaStream_t)stream), "argmax_next");
}

int lfm2q_shortconv_step(const uint16_t *bcx, uint16_t *state, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                         int B, int H, void *stream) {
  REQUIRE(B >= 0 && H > 0, "bcx [B, 3H], state [B, H, 3], w [H, 3], y [B, H]: need B >= 0, H > 0");
  REQUIRE(B <= 65535, "B <= 65535");
  if (B == 0) return LFM2Q_OK;
  REQUIRE(bcx && state && w && y, "bcx, state, w and y must be non-null");
  if (int e = device_gate()) return e;
  return launched(launch_shortconv_step(bcx, state, w, bias, y, B, H, g_pdl.load(), (cudaStream_t)stream),
                  "shortconv_step");
}

int lfm2q_qk_norm_rope_kv(const uint16_t *qkv, const uint16_t *qw, const uint16_t *kw, const float *inv_freq,
                          float scaling, const int64_t *pos, uint16_t *q_out, uint16_t *kc, uint16_t *vc, int B,
                          int NQ, int NKV, int max_len, float eps, void *stream) {
  REQUIRE(B >= 0 && NQ > 0 && NKV > 0 && max_len > 0, "qkv [B, (NQ + 2 NKV) * 64]: need B >= 0, NQ, NKV, max_len > 0");
  REQUIRE((long long)B * (NQ + 2 * NKV) <= 0x7fffffffLL, "B * (NQ + 2 NKV) too large");
  if (B == 0) return LFM2Q_OK;
  REQUIRE(qkv && qw && kw && inv_freq && pos && q_out && kc && vc, "every pointer must be non-null");
  REQUIRE(aligned16(qkv) && aligned16(vc), "qkv and vc must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_qk_norm_rope_kv(qkv, qw, kw, inv_freq, scaling, pos, q_out, kc, vc, B, NQ, NKV, max_len, eps,
                                         g_pdl.load(), (cudaStream_t)stream),
                  "qk_norm_rope_kv");
}

// ------------------------------------------------------------------ decode attention
int lfm2q_decode_attention_split(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, const int64_t *pos,
                                 uint16_t *out, float *ws, int B, int NQ, int NKV, int max_len, int S, float scale,
                                 void *stream) {
  REQUIRE(B >= 0 && NKV > 0 && max_len > 0, "q [B, NQ, 64], kc / vc [B, NKV, max_len, 64]: need B >= 0, NKV > 0, "
                                            "max_len > 0");
  REQUIRE(NQ == 4 * NKV, "head_dim 64 and 4 query heads per KV head only");
  REQUIRE(S >= 1 && S <= 65535, "ws [B, NQ, S, 66]: need 1 <= S <= 65535");
  REQUIRE((long long)B * NKV <= 0x7fffffffLL, "B * NKV too large");
  if (B == 0) return LFM2Q_OK;
  REQUIRE(q && kc && vc && pos && out && ws, "q, kc, vc, pos, out and ws must be non-null");
  REQUIRE(aligned16(q) && aligned16(kc) && aligned16(vc), "q, kc and vc must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_decode_attention_split(q, kc, vc, pos, out, ws, B, NQ, NKV, max_len, S, scale, g_pdl.load(),
                                                (cudaStream_t)stream),
                  "decode_attention_split");
}

// Allocation-free variant: the partials live in the library's static device workspace (ATTN_STATIC_WS_FLOATS).
int lfm2q_decode_attention_split_noalloc(const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                         const int64_t *pos, uint16_t *out, int B, int NQ, int NKV, int max_len, int S,
                                         float scale, void *stream) {
  static_assert(ATTN_STATIC_WS_FLOATS == LFM2Q_ATTN_NOALLOC_MAX_WS_FLOATS, "header and library disagree");
  REQUIRE(B >= 0 && NKV > 0 && max_len > 0, "q [B, NQ, 64], kc / vc [B, NKV, max_len, 64]: need B >= 0, NKV > 0, "
                                            "max_len > 0");
  REQUIRE(NQ == 4 * NKV, "head_dim 64 and 4 query heads per KV head only");
  REQUIRE(S >= 1 && S <= 65535, "need 1 <= S <= 65535");
  REQUIRE((long long)B * NQ * S * 66 <= ATTN_STATIC_WS_FLOATS,
          "B * NQ * S * 66 exceeds the static workspace of decode_attention_split_noalloc (" +
              std::to_string(ATTN_STATIC_WS_FLOATS) + " floats, 8 MiB): use lfm2q_decode_attention_split with a "
              "caller-allocated ws, or fewer splits");
  if (B == 0) return LFM2Q_OK;
  REQUIRE(q && kc && vc && pos && out, "q, kc, vc, pos and out must be non-null");
  REQUIRE(aligned16(q) && aligned16(kc) && aligned16(vc), "q, kc and vc must be 16-byte aligned");
  if (int e = device_gate()) return e;
  return launched(launch_decode_attention_split_static(q, kc, vc, pos, out, B, NQ, NKV, max_len, S, scale,
                                                       g_pdl.load(), (cudaStream_t)stream),
                  "decode_attention_split_noalloc");
}

}  // extern "C"
