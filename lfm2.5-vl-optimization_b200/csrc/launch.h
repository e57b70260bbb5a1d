// Internal launcher interface between the CUDA translation units and the C ABI (capi.cpp).
// Launchers assume validated arguments (capi.cpp checks shapes, alignment and the device) and only
// enqueue work on `st`; they return the launch status.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace lfm2q {

// quant.cu
// pdl: launch with programmatic stream serialization (small decode batches: overlaps the neighbouring launches)
cudaError_t launch_quant_rows(const void *x, int8_t *q, float *s, int rows, int K, bool pdl, cudaStream_t st);
cudaError_t launch_quant_groups(const void *x, int8_t *q, float *sT, int rows, int K, bool pdl, cudaStream_t st);

// producers.cu
cudaError_t launch_add_layernorm_q(void *h, const void *y, const void *w, const void *b, int8_t *q, float *s, int rows,
                                   int D, float eps, bool grouped, cudaStream_t st);
cudaError_t launch_add_rmsnorm_q(void *h, const void *y, const void *w, int8_t *q, float *s, int rows, int H, float eps,
                                 bool grouped, cudaStream_t st);
cudaError_t launch_silu_mul_q(const void *g, int8_t *q, float *s, int rows, int I, bool grouped, cudaStream_t st);

// gemv.cu
cudaError_t launch_gemv(const void *W, bool int8, const float *scale, const void *x, void *y, int N, int K, int rows,
                        int B, bool pdl, cudaStream_t st);
// tuning: let dependents launch at kernel start (default: after the K loop)
void gemv_set_early_trigger(bool early);
int gemv_trigger_mode();  // the PDL trigger argument of the GEMV kernels: 1 = after the K loop, 2 = at the start
void gemv_set_impl(int impl);
// per-token W8A8 linear for few tokens in one launch: quant_rows(x) fused into the A8 GEMV
cudaError_t launch_linear_a8(const void *x, const int8_t *W, const float *sw, const void *bias, void *y, int N, int K,
                             int B, bool gelu, bool pdl, cudaStream_t st);
// A8 decode GEMV: int8 tokens (per-token scales) x int8 W, exact int32, the per-token W8A8 epilogue (gemm_i8's);
// up to A8_MAX_TOKENS tokens per pass over W
constexpr int A8_MAX_TOKENS = 64;
cudaError_t launch_gemv_a8(const int8_t *W, const float *sw, const int8_t *xq, const float *sx, const void *bias, void *y,
                           int N, int K, int B, bool gelu, bool pdl, cudaStream_t st);
cudaError_t launch_gemv_epi(int epi, const void *W, bool int8, const float *scale, const void *x, void *y, int S, int K,
                            void *state, const void *cw, const void *cbias, bool pdl, cudaStream_t st);

// gemv_chain.cu: a list of weight-only int8 GEMVs, one PDL launch each
constexpr int CHAIN_MAX = 96;
constexpr int CHAIN_MAX_TOKENS = 4;
struct ChainLayer {
  const int8_t *W;      // int8 [N, K]
  const float *scale;   // fp32 [N]
  const uint16_t *x;    // bf16 [B, K]
  uint16_t *y;          // bf16 [B, N]
  int N, K;
};
cudaError_t launch_gemv_chain(const ChainLayer *layers, int n, int B, bool pdl, cudaStream_t st);
// gemv.cu: one weight-only int8 GEMV of a chain (the x-sliced path where it applies, else the bf16 path)
cudaError_t launch_gemv_sliced(const int8_t *W, const float *scale, const void *x, void *y, int N, int K, int B,
                               bool pdl, cudaStream_t st);

// gemv_w4.cu: INT4 weight-only GEMV (packed nibbles, one fp32 scale per group of `group` inputs, group % 128 == 0)
int gemv_w4_slices(int K, int B);  // 0: this K / B does not fit the kernel's shared memory
cudaError_t launch_gemv_w4(const uint8_t *Wp, const float *S, const void *x, void *y, int N, int K, int group, int B,
                           bool pdl, int trigger, cudaStream_t st);

// gemm_tc.cu: tcgen05 W8A8 GEMMs
enum GemmEpi { EPI_TOKEN = 0, EPI_GROUP = 1, EPI_GROUP_Q = 2, EPI_SILU = 3, EPI_W8 = 4 };
cudaError_t launch_gemm_i8(const int8_t *A, const float *sa, const int8_t *B, const float *sb, const void *bias, void *Y,
                           int M, int N, int K, bool gelu, bool grouped, cudaStream_t st);
cudaError_t launch_gemm_i8_q(const int8_t *A, const float *saT, const int8_t *B, const float *sb, const void *bias,
                             int8_t *Yq, float *YsT, int M, int N, int K, bool gelu, cudaStream_t st);
cudaError_t launch_gemm_i8_silu(const int8_t *A, const float *sa, const int8_t *B, const float *sb, const void *bias,
                                void *Y, int M, int I, int K, cudaStream_t st);
int gemm_device_error(bool clear);
cudaError_t launch_wait_timeout_selftest(int limit_log2, cudaStream_t st);  // sticky code written by a bounded wait that gave up (0 = none)
void gemm_set_tile_override(int bn);  // 0 = heuristic, 128 / 256 = force the per-token tile width (< 0: CTA pairs), 1 = split-K
void gemm_set_pdl(bool on);            // GEMMs launch as programmatic dependents

// gemm_tc.cu: tcgen05 W8A16 GEMM
cudaError_t launch_gemm_w8(const void *A, const int8_t *B, const float *sb, const void *bias, void *Y, int M, int N,
                           int K, bool gelu, cudaStream_t st);

// attention.cu: split-over-positions decode attention + combine
cudaError_t launch_decode_attention_split(const void *q, const void *kc, const void *vc, const int64_t *pos, void *out,
                                          float *ws, int B, int NQ, int NKV, int max_len, int S, float scale, bool pdl,
                                          cudaStream_t st);
int attn_device_error(bool clear);
// the same with the per-split partials in the library's static device workspace (capacity in floats below)
cudaError_t launch_decode_attention_split_static(const void *q, const void *kc, const void *vc, const int64_t *pos,
                                                 void *out, int B, int NQ, int NKV, int max_len, int S, float scale,
                                                 bool pdl, cudaStream_t st);
constexpr long long ATTN_STATIC_WS_FLOATS = 1ll << 21;

// decode.cu: the decode step's small kernels
cudaError_t launch_add_rmsnorm(void *h, const void *y, const void *w, void *x, int rows, int H, float eps, bool pdl,
                               cudaStream_t st);
cudaError_t launch_shortconv_step(const void *bcx, void *state, const void *w, const void *bias, void *y, int B, int H,
                                  bool pdl, cudaStream_t st);
cudaError_t launch_embed_rmsnorm(const int64_t *tok, const void *embed, const void *w, void *h, void *x, int rows,
                                 int H, float eps, bool pdl, cudaStream_t st);
cudaError_t launch_argmax_next(const void *logits, int64_t *tok, int64_t *pos, int B, int V, bool pdl,
                               cudaStream_t st);
cudaError_t launch_qk_norm_rope_kv(const void *qkv, const void *qw, const void *kw, const float *inv_freq,
                                   float scaling, const int64_t *pos, void *q_out, void *kc, void *vc, int B, int NQ,
                                   int NKV, int max_len, float eps, bool pdl, cudaStream_t st);

// device facts cached per device
int device_sm_count();
bool device_is_sm100();

}  // namespace lfm2q
