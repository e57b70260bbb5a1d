// TEST INFRASTRUCTURE ONLY (not part of the product library): a C-ABI shim over the reference's own CUDA launchers,
// compiled together with the reference's kernel sources (kernels/int8_gemm.cu, kernels/lfm2_decode.cu, built for
// sm_100a from where they lie) into oracle/_ref/librefk.so by oracle/Makefile. The GPU parity tests call the
// reference kernels through it on the same device buffers as lfm2q's, and time both.
//
// The prototypes below restate the reference launchers' signatures (kernels/int8_gemm.cu:741-742, :751-752,
// :765-766, :782, :787-788, :798-799, :810, :822; kernels/lfm2_decode.cu:36, :123, :157, :204-206, :418-419, :708,
// :818-819, :938, :965); they must match for the link to resolve.
#include <cuda_runtime.h>
#include <stdint.h>

void launch_gemm_i8(const void *A, const float *sa, const void *B, const float *sb, const void *bias, void *Y, int M,
                    int N, int K, bool gelu, bool grouped, cudaStream_t st);
void launch_gemm_w8(const void *A, const void *B, const float *sb, const void *bias, void *Y, int M, int N, int K,
                    bool gelu, cudaStream_t st);
void launch_gemm_i8_q(const void *A, const float *saT, const void *B, const float *sb, const void *bias, void *Yq,
                      float *YsT, int M, int N, int K, bool gelu, cudaStream_t st);
void launch_quant_rows(const void *x, void *q, float *s, int rows, int K, cudaStream_t st);
void launch_quant_groups(const void *x, void *q, float *sT, int rows, int K, cudaStream_t st);
void launch_add_layernorm_q(void *h, const void *y, const void *w, const void *b, void *q, float *s, int rows, int D,
                            float eps, bool grouped, cudaStream_t st);
void launch_add_rmsnorm_q(void *h, const void *y, const void *w, void *q, float *s, int rows, int H, float eps,
                          bool grouped, cudaStream_t st);
void launch_silu_mul_q(const void *g, void *q, float *s, int rows, int I, bool grouped, cudaStream_t st);
void launch_silu_mul(const void *g, void *y, int B, int I, cudaStream_t st);
void launch_gemv_epi(int epi, const void *W, bool int8, const float *scale, const void *x, void *y, int S, int K,
                     void *state, const void *cw, const void *cbias, cudaStream_t st);
void launch_gemv_w4(const void *Wp, const float *S, const void *x, void *y, int N, int K, int group, int rows,
                    cudaStream_t st);
void launch_gemv(const void *W, bool int8, const float *scale, const void *x, void *y, int N, int K, int rows, int B,
                 cudaStream_t st);
void launch_decode_attention_split(const void *q, const void *kc, const void *vc, const int64_t *pos, void *out,
                                   float *ws, int B, int NQ, int NKV, int max_len, int S, float scale, cudaStream_t st);
void launch_add_rmsnorm(void *h, const void *y, const void *w, void *x, int rows, int H, float eps, cudaStream_t st);
void launch_shortconv_step(const void *bcx, void *state, const void *w, const void *bias, void *y, int B, int H,
                           cudaStream_t st);
void launch_qk_norm_rope_kv(const void *qkv, const void *qw, const void *kw, const float *inv_freq, float scaling,
                            const int64_t *pos, void *q_out, void *kc, void *vc, int B, int NQ, int NKV, int max_len,
                            float eps, cudaStream_t st);
void set_pdl(bool on);

// Each wrapper launches on `stream` and returns the launch status (cudaError_t as int; 0 = success).
extern "C" {
int refk_gemm_i8(const void *xq, const float *sx, const void *w, const float *sw, const void *bias, void *y, int M,
                 int N, int K, int gelu, int grouped, void *stream) {
  launch_gemm_i8(xq, sx, w, sw, bias, y, M, N, K, gelu != 0, grouped != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_gemm_w8(const void *x, const void *w, const float *sw, const void *bias, void *y, int M, int N, int K,
                 int gelu, void *stream) {
  launch_gemm_w8(x, w, sw, bias, y, M, N, K, gelu != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_quant_rows(const void *x, void *q, float *s, int rows, int K, void *stream) {
  launch_quant_rows(x, q, s, rows, K, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_gemv(const void *w, int w_is_int8, const float *scale, const void *x, void *y, int N, int K, int B,
              void *stream) {
  launch_gemv(w, w_is_int8 != 0, scale, x, y, N, K, 0, B, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_gemm_i8_q(const void *xq, const float *sxT, const void *w, const float *sw, const void *bias, void *yq,
                   float *ysT, int M, int N, int K, int gelu, void *stream) {
  launch_gemm_i8_q(xq, sxT, w, sw, bias, yq, ysT, M, N, K, gelu != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_quant_groups(const void *x, void *q, float *sT, int rows, int K, void *stream) {
  launch_quant_groups(x, q, sT, rows, K, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_add_layernorm_q(void *h, const void *y, const void *w, const void *b, void *q, float *s, int rows, int D,
                         float eps, int grouped, void *stream) {
  launch_add_layernorm_q(h, y, w, b, q, s, rows, D, eps, grouped != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_add_rmsnorm_q(void *h, const void *y, const void *w, void *q, float *s, int rows, int H, float eps,
                       int grouped, void *stream) {
  launch_add_rmsnorm_q(h, y, w, q, s, rows, H, eps, grouped != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_silu_mul_q(const void *g, void *q, float *s, int rows, int I, int grouped, void *stream) {
  launch_silu_mul_q(g, q, s, rows, I, grouped != 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_silu_mul(const void *g, void *y, int B, int I, void *stream) {
  launch_silu_mul(g, y, B, I, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_gemv_epi(int epi, const void *W, int w_is_int8, const float *scale, const void *x, void *y, int S, int K,
                  void *state, const void *cw, const void *cbias, void *stream) {
  launch_gemv_epi(epi, W, w_is_int8 != 0, scale, x, y, S, K, state, cw, cbias, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_gemv_w4(const void *Wp, const float *S, const void *x, void *y, int N, int K, int group, void *stream) {
  launch_gemv_w4(Wp, S, x, y, N, K, group, 0, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_decode_attention_split(const void *q, const void *kc, const void *vc, const int64_t *pos, void *out, float *ws,
                                int B, int NQ, int NKV, int max_len, int S, float scale, void *stream) {
  launch_decode_attention_split(q, kc, vc, pos, out, ws, B, NQ, NKV, max_len, S, scale, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_add_rmsnorm(void *h, const void *y, const void *w, void *x, int rows, int H, float eps, void *stream) {
  launch_add_rmsnorm(h, y, w, x, rows, H, eps, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_shortconv_step(const void *bcx, void *state, const void *w, const void *bias, void *y, int B, int H,
                        void *stream) {
  launch_shortconv_step(bcx, state, w, bias, y, B, H, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
int refk_qk_norm_rope_kv(const void *qkv, const void *qw, const void *kw, const float *inv_freq, float scaling,
                         const int64_t *pos, void *q_out, void *kc, void *vc, int B, int NQ, int NKV, int max_len,
                         float eps, void *stream) {
  launch_qk_norm_rope_kv(qkv, qw, kw, inv_freq, scaling, pos, q_out, kc, vc, B, NQ, NKV, max_len, eps,
                         (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
void refk_set_pdl(int on) { set_pdl(on != 0); }
}
