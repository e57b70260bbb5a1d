/*
 * lfm2q — B200-native (sm_100a) INT8 matrix-multiply hot path of LFM2.5-VL-Optimization, C ABI.
 *
 * Plain pointers and sizes only: device pointers for all tensors, a cudaStream_t passed as `void *`
 * (NULL = the legacy default stream). Every entry point validates its arguments on the host, enqueues
 * the work on `stream` without synchronising, and returns an lfm2q_status; lfm2q_last_error() gives the
 * message of the last failure on the calling thread. Callers allocate every output. No entry point
 * allocates device memory.
 *
 * Element types: "bf16" tensors are uint16_t bit patterns of bfloat16; int8 tensors are int8_t; scales fp32.
 * Layouts are row-major and dense. Every pointer must be 16-byte aligned.
 *
 * Each declaration names the reference interface it replaces (path:line in the reference project).
 */
#ifndef LFM2Q_H
#define LFM2Q_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LFM2Q_OK = 0,
  LFM2Q_EINVAL = -22,   /* bad shape, size, alignment or null pointer; nothing was launched */
  LFM2Q_ENOTSUP = -95,  /* no sm_100 device current, or the driver lacks the tensor-map entry point */
  LFM2Q_ECUDA = -5,     /* the CUDA runtime reported an error while launching */
  LFM2Q_ETIMEOUT = -62  /* a kernel's bounded pipeline wait gave up (see lfm2q_check_device) */
} lfm2q_status;

/* Message of the last non-OK status returned on this thread ("" if none). */
const char *lfm2q_last_error(void);

/* Library version string. */
const char *lfm2q_version(void);

/* 1 if the current device is an sm_100 part this library can launch on, else 0. */
int lfm2q_device_supported(void);

/* Reads (and with clear != 0 resets) the sticky device error words that the tcgen05 GEMMs and the decode attention
 * set when one of their bounded pipeline waits gives up (no other kernel of this library waits on anything).
 * Returns LFM2Q_OK or LFM2Q_ETIMEOUT. Synchronous (copies two ints from the device). Poll it after a batch of work
 * whose outputs matter. */
int lfm2q_check_device(int clear);

/* ------------------------------------------------------------------ activation quantizers
 * Replaces launch_quant_rows / launch_quant_groups (kernels/int8_gemm.cu:822-825, :782-785) behind the
 * quant_rows binding (kernels/int8_gemm.cpp:83-96).
 * x bf16 [rows, K] -> q int8 [rows, K], s fp32 [rows] = max(|x_row|, 1e-8) / 127, q = clamp(rint(x / s), +-127).
 * Needs K % 8 == 0 and K <= 16384 (the reference needs K % 128 == 0 and K <= 2048). */
int lfm2q_quant_rows(const uint16_t *x, int8_t *q, float *s, int rows, int K, void *stream);
/* Grouped: sT fp32 [K/64, rows], one scale per row and 64-wide group. Needs K % 64 == 0, K <= 16384. */
int lfm2q_quant_groups(const uint16_t *x, int8_t *q, float *sT, int rows, int K, void *stream);

/* ------------------------------------------------------------------ W8A8 GEMM (tcgen05)
 * Replaces launch_gemm_i8 (kernels/int8_gemm.cu:741-748) behind gemm_i8 (kernels/int8_gemm.cpp:39-50).
 * y bf16 [M, N] = bf16(act(((float)(xq . w^T)[m, n] * sx[m]) * sw[n] + bias[n])), act = GELU(tanh) if gelu.
 * xq int8 [M, K], w int8 [N, K], sw fp32 [N], bias bf16 [N] or NULL.
 * grouped == 0: sx fp32 [M] (one scale per token).
 * grouped != 0: sx fp32 [K/64, M]; the int32 sum of every 64-wide K group is folded into fp32 with its scale.
 * Needs K % 16 == 0, N % 8 == 0 (grouped: K % 64 == 0). */
int lfm2q_gemm_i8(const int8_t *xq, const float *sx, int grouped, const int8_t *w, const float *sw,
                  const uint16_t *bias, uint16_t *y, int M, int N, int K, int gelu, void *stream);

/* Replaces launch_gemm_i8_q (kernels/int8_gemm.cu:751-763) behind gemm_i8_q (kernels/int8_gemm.cpp:53-69).
 * Grouped W8A8 whose bf16-rounded output is requantized for the next W8A8 GEMM: yq int8 [M, N],
 * ysT fp32 [N/64, M]. sxT fp32 [K/64, M]. Needs K % 64 == 0, N % 128 == 0. */
int lfm2q_gemm_i8_q(const int8_t *xq, const float *sxT, const int8_t *w, const float *sw, const uint16_t *bias,
                    int8_t *yq, float *ysT, int M, int N, int K, int gelu, void *stream);

/* New fused epilogue with no single-kernel counterpart in the reference: it replaces the composition
 * gemm_i8 (kernels/int8_gemm.cpp:39-50, bf16 out) -> silu_mul (kernels/lfm2_decode.cu:954-969).
 * w = [w1 | w3] int8 [2I, K] with sw fp32 [2I], bias bf16 [2I] or NULL, per-token sx fp32 [M];
 * y bf16 [M, I] = bf16(bf16(silu(g)) * u), g and u the bf16 per-token epilogue outputs of rows n and I + n.
 * Needs K % 16 == 0, I % 8 == 0. */
int lfm2q_gemm_i8_silu(const int8_t *xq, const float *sx, const int8_t *w, const float *sw, const uint16_t *bias,
                       uint16_t *y, int M, int I, int K, void *stream);

/* Replaces launch_gemm_w8 (kernels/int8_gemm.cu:765-780) behind gemm_w8 (kernels/int8_gemm.cpp:72-79).
 * W8A16: y bf16 [M, N] = bf16(act((x . w^T) * sw[n] + bias[n])), x bf16 [M, K], w int8 [N, K].
 * Needs K % 16 == 0, N % 8 == 0. */
int lfm2q_gemm_w8(const uint16_t *x, const int8_t *w, const float *sw, const uint16_t *bias, uint16_t *y, int M,
                  int N, int K, int gelu, void *stream);

/* ------------------------------------------------------------------ fused producers
 * Replace launch_add_layernorm_q / launch_add_rmsnorm_q / launch_silu_mul_q (kernels/int8_gemm.cu:787-820) behind
 * the bindings of the same names (kernels/int8_gemm.cpp:107-141). grouped != 0 selects s [K/64, rows].
 * h is updated in place (h += y) when y is non-NULL. */
int lfm2q_add_layernorm_q(uint16_t *h, const uint16_t *y, const uint16_t *w, const uint16_t *b, int8_t *q, float *s,
                          int rows, int D, float eps, int grouped, void *stream);
int lfm2q_add_rmsnorm_q(uint16_t *h, const uint16_t *y, const uint16_t *w, int8_t *q, float *s, int rows, int H,
                        float eps, int grouped, void *stream);
/* g bf16 [rows, 2I] -> q int8 [rows, I] + scales of bf16(bf16(silu(g[:, :I])) * g[:, I:]). */
int lfm2q_silu_mul_q(const uint16_t *g, int8_t *q, float *s, int rows, int I, int grouped, void *stream);

/* ------------------------------------------------------------------ decode GEMV
 * Replaces launch_gemv (kernels/lfm2_decode.cu:708-714) behind gemv (kernels/lfm2_decode.cpp:73-85).
 * y bf16 [B, N] = bf16((x . W^T) * scale[n]), fp32 accumulation. w_is_int8 != 0: W int8 [N, K] with scale fp32
 * [N] (required); else W bf16 [N, K] and scale optional (NULL = 1). x bf16 [B, K]. Needs K % 512 == 0 (int8) or
 * K % 256 == 0 (bf16). Int8 weights with 1-4 tokens run the x-sliced tensor-core path (the tokens as exact fixed-point
 * bytes, exact int32 partial sums; see lfm2q_set_gemv_path), else bf16 MMAs on the exactly converted weights.
 * `rows` (the reference's kernel-choice argument): 0 = automatic; 1, 2, 4 or 8 forces that many K-slices per 16-row
 * group on the ring and bf16 paths (the deep-prefetch kernel sizes its own). Results agree to fp32 summation order. */
int lfm2q_gemv(const void *W, int w_is_int8, const float *scale, const uint16_t *x, uint16_t *y, int N, int K,
               int rows, int B, void *stream);

/* A8 decode GEMV, bit-exact at int32: the W8A8 path of gemm_i8 for few tokens (no single counterpart in the
 * reference, whose decode GEMV is weight-only; the result equals gemm_i8 (kernels/int8_gemm.cpp:39-50) on the same
 * int8 inputs, and lfm2q_gemm_i8 itself routes per-token calls here at M <= 16, at M <= 64 when K >= 4096, and at
 * M <= 32 when N * K <= 8 M).
 * y bf16 [B, N] = bf16(act(((float)(xq . W^T)[b, n] * sx[b]) * sw[n] + bias[n])), xq int8 [B, K] quantized per token
 * (lfm2q_quant_rows), sx fp32 [B], W int8 [N, K], sw fp32 [N], bias bf16 [N] or NULL, act = GELU(tanh) if gelu.
 * Needs K % 64 == 0, B >= 1 (any B: up to 64 tokens per pass over W). */
int lfm2q_gemv_a8(const int8_t *W, const float *sw, const int8_t *xq, const float *sx, const uint16_t *bias,
                  uint16_t *y, int N, int K, int B, int gelu, void *stream);

/* Per-token W8A8 linear for a few tokens in one launch: the composition quant_rows (kernels/int8_gemm.cpp:83-96)
 * -> gemm_i8 (kernels/int8_gemm.cpp:39-50) that the reference's Int8Linear.__call__ (src/lfm2opt/int8.py:84-88)
 * performs for group 0, with the quantization fused into the A8 GEMV. x bf16 [B, K] -> y bf16 [B, N]; identical to
 * lfm2q_quant_rows + lfm2q_gemm_i8 on the same inputs. Needs K % 64 == 0 (any B: chunks of up to 16 tokens). */
int lfm2q_linear_a8(const uint16_t *x, const int8_t *W, const float *sw, const uint16_t *bias, uint16_t *y, int N,
                    int K, int B, int gelu, void *stream);

/* Replaces launch_gemv_w4 (kernels/lfm2_decode.cu:938-945) behind gemv_w4 (kernels/lfm2_decode.cpp:87-98).
 * INT4 weight-only GEMV: Wp uint8 [N, K/2], byte j of a row holding inputs 2j (low nibble) and 2j + 1 (high nibble),
 * each stored as q + 8, q in [-8, 7]; S fp32 [N, K / group], one scale per row and group of `group` inputs
 * (lfm2opt.quant.quantize_int4). y bf16 [B, N] = bf16(sum_g S[n, g] * (x . q)_g). x bf16 [B, K], 1 <= B <= 4 (the
 * reference: batch 1). Needs group % 128 == 0 (the reference: % 32; its models use 128), K % group == 0,
 * B * K <= 16384. */
int lfm2q_gemv_w4(const uint8_t *Wp, const float *S, const uint16_t *x, uint16_t *y, int N, int K, int group, int B,
                  void *stream);

/* ------------------------------------------------------------------ chained decode GEMV
 * No single counterpart in the reference: it replaces a run of gemv launches (kernels/lfm2_decode.cu:708-714 behind
 * gemv, kernels/lfm2_decode.cpp:73-85) that the reference's decode step issues back to back inside its captured
 * graph (src/lfm2opt/runtime.py:223-244, :247-294). The layers run in list order, each after the previous one has
 * completed (so a layer may read an earlier layer's y as its x); each is lfm2q_gemv with int8 weights, y = bf16((x .
 * W^T) * scale), computed on the int8 tensor path with the tokens sliced into exact fixed-point bytes where the
 * slices fit in shared memory (B * 3 * (K + 64) <= 65536 and B * K <= 16384; else the bf16 path). For B <= 2 each
 * layer is the deep-prefetch kernel: its blocks start while the previous layer runs and have their weights in flight
 * before the dependency wait. One kernel launch per layer, capturable in a CUDA graph; nothing is allocated. */
typedef struct {
  const int8_t *W;    /* int8 [N, K], 16-byte aligned */
  const float *scale; /* fp32 [N] */
  const uint16_t *x;  /* bf16 [B, K], 16-byte aligned; may be an earlier layer's y */
  uint16_t *y;        /* bf16 [B, N]; must not overlap this layer's x */
  int N;
  int K;              /* a multiple of 512 */
} lfm2q_gemv_layer;

#define LFM2Q_CHAIN_MAX_LAYERS 96
#define LFM2Q_CHAIN_MAX_TOKENS 4

/* Runs layers[0 .. n_layers) (a host array, read during the call) for B tokens, 1 <= B <= 4, 1 <= n_layers <= 96,
 * on `stream`. */
int lfm2q_gemv_chain(const lfm2q_gemv_layer *layers, int n_layers, int B, void *stream);

/* Replaces launch_gemv_epi (kernels/lfm2_decode.cu:818-827) behind gemv_epi (kernels/lfm2_decode.cpp:130-150).
 * Batch 1. epi 0: W = w1|w3 [2S, K] -> y [S] = bf16(bf16(silu(g)) * u).
 *          epi 1: W = in_proj [3S, K] (B|C|x) -> short-conv step, state bf16 [S, 3] updated in place,
 *                 cw bf16 [S, 3], cbias bf16 [S] or NULL. */
int lfm2q_gemv_epi(int epi, const void *W, int w_is_int8, const float *scale, const uint16_t *x, uint16_t *y, int S,
                   int K, uint16_t *state, const uint16_t *cw, const uint16_t *cbias, void *stream);

/* ------------------------------------------------------------------ decode step kernels
 * Replace launch_add_rmsnorm / launch_shortconv_step / launch_qk_norm_rope_kv (kernels/lfm2_decode.cu:123-130,
 * :157-161, :204-212) behind add_rmsnorm / shortconv_step / qk_norm_rope_kv (kernels/lfm2_decode.cpp:32-55). Outputs
 * bit-identical to the reference kernels. All bf16 except inv_freq (fp32 [32]) and pos (int64 [1] on the device).
 *
 * add_rmsnorm: h [rows, H] (updated in place to bf16(h + y) when y is non-NULL), w [H], x [rows, H] =
 * bf16(w * bf16(h * rsqrt(mean(h^2) + eps))). Needs H <= 8192. */
int lfm2q_add_rmsnorm(uint16_t *h, const uint16_t *y, const uint16_t *w, uint16_t *x, int rows, int H, float eps,
                      void *stream);
/* shortconv_step: bcx [B, 3H] = (B | C | x), state [B, H, 3] (shifted in place), w [H, 3], bias [H] or NULL,
 * y [B, H] = bf16(C * bf16(w . (s1, s2, bf16(B x)) + bias)). */
int lfm2q_shortconv_step(const uint16_t *bcx, uint16_t *state, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                         int B, int H, void *stream);
/* No counterpart in the reference: the embedding lookup (F.embedding) and the first add_rmsnorm (no residual) of its
 * decode step (src/lfm2opt/runtime.py:249-251) in one launch. h [rows, H] = embed[tok[r]] (bf16 [V, H], bits
 * unchanged), x = rmsnorm(h) * w as lfm2q_add_rmsnorm with y NULL. tok: int64 [rows] on the device, each in [0, V)
 * (not checked: the values are on the device). H <= 8192. */
int lfm2q_embed_rmsnorm(const int64_t *tok, const uint16_t *embed, const uint16_t *w, uint16_t *h, uint16_t *x,
                        int rows, int H, float eps, void *stream);
/* No counterpart in the reference: the end of its decode step (src/lfm2opt/runtime.py:286-294: torch.argmax over the
 * logits, the token copied into the next input, the position advanced) in one launch. tok[b] = the first index of
 * the largest value of logits row b (bf16 [B, V]; NaN counts as the largest, as torch.argmax), then pos[0] += 1 if pos
 * is not NULL. logits 16-byte aligned; V a multiple of 8 when B > 1. */
int lfm2q_argmax_next(const uint16_t *logits, int64_t *tok, int64_t *pos, int B, int V, void *stream);
/* qk_norm_rope_kv: qkv [B, (NQ + 2 NKV) * 64] (q | k | v heads, head dim 64), qw / kw [64] per-head RMSNorm weights,
 * rope cos / sin = bf16(cos / sin(pos * inv_freq[d % 32]) * scaling); q_out [B, NQ, 64]; k and v written to
 * kc / vc [B, NKV, max_len, 64] at position pos (the caller keeps pos < max_len). */
int lfm2q_qk_norm_rope_kv(const uint16_t *qkv, const uint16_t *qw, const uint16_t *kw, const float *inv_freq,
                          float scaling, const int64_t *pos, uint16_t *q_out, uint16_t *kc, uint16_t *vc, int B,
                          int NQ, int NKV, int max_len, float eps, void *stream);

/* ------------------------------------------------------------------ decode attention
 * Replaces launch_decode_attention_split (kernels/lfm2_decode.cu:418-426) behind decode_attention_split
 * (kernels/lfm2_decode.cpp:64-71). One decode step of grouped-query attention over a bf16 KV cache, head dim 64, four
 * query heads per KV head (NQ == 4 * NKV): q bf16 [B, NQ, 64] (unscaled: score = (q * scale) . k),
 * kc / vc bf16 [B, NKV, max_len, 64], pos int64 [1] on the device (positions 0 .. pos are attended, for every
 * sequence; positions at or past max_len are not read), out bf16 [B, NQ, 64]. The positions are cut into S splits of
 * ceil(max_len / S); ws fp32 [B, NQ, S, 66] receives (m, l, acc[64]) of every split and is then merged into out
 * (no value of ws needs to be set before the call). Per-position arithmetic in the reference kernel's order. */
int lfm2q_decode_attention_split(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, const int64_t *pos,
                                 uint16_t *out, float *ws, int B, int NQ, int NKV, int max_len, int S, float scale,
                                 void *stream);

/* No counterpart in the reference. lfm2q_decode_attention_split without the ws argument, for callers that cannot
 * allocate device memory: a C or FFI host that only receives device pointers for q, kc, vc, pos and out from another
 * runtime and holds no allocator, or a decode loop where a cudaMalloc / cudaFree would synchronize the device and
 * stall the other streams. The per-split partials go to a workspace inside the library itself: a static device array
 * of LFM2Q_ATTN_NOALLOC_MAX_WS_FLOATS floats (8 MiB), which every GPU that loads the library holds until the process
 * exits. Needs B * NQ * S * 66 <= LFM2Q_ATTN_NOALLOC_MAX_WS_FLOATS (else LFM2Q_EINVAL, nothing launched); otherwise
 * the same arguments, checks and results as lfm2q_decode_attention_split. Nothing in the workspace needs to start at
 * zero (every split writes its partials before the combine reads them), but all calls on one device share it: two
 * calls whose kernels overlap on the GPU (other streams, other host threads) race and corrupt each other's results,
 * so serialise them. The first call on each device finds the workspace's device address (cudaGetSymbolAddress, with
 * that device current) and sets the kernel's shared-memory limit; make that first call before any stream capture.
 * Allocates nothing. */
#define LFM2Q_ATTN_NOALLOC_MAX_WS_FLOATS (1 << 21)
int lfm2q_decode_attention_split_noalloc(const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                         const int64_t *pos, uint16_t *out, int B, int NQ, int NKV, int max_len, int S,
                                         float scale, void *stream);

/* Replace set_pdl / set_gemv_impl (kernels/lfm2_decode.cpp:165-166). set_pdl toggles Programmatic Dependent
 * Launch for the GEMV kernels (default on). set_gemv_impl is accepted for compatibility; this build has one
 * GEMV implementation. */
void lfm2q_set_pdl(int on);
void lfm2q_set_gemv_impl(int impl);

/* Path of the int8 weight-only GEMV (lfm2q_gemv, lfm2q_gemv_chain and lfm2q_gemv_epi with w_is_int8). The int8
 * tensor path slices the tokens into exact fixed-point bytes (B <= 4, B * 3 * (K + 64) <= 64 KB, K <= 16384 / B);
 * two kernels implement it with identical values: the deep-prefetch kernel (one block per SM, weights requested
 * before the dependency wait while the previous GEMV still runs) and the ring kernel.
 *   0 (default): deep kernel for B <= 2; ring kernel for B = 3, 4 from N * K >= 8 M; else the bf16 path
 *   1: always the bf16 path (weights converted exactly to bf16, bf16 MMAs)
 *   2: deep kernel wherever the slices fit    3: as 2, next launch triggered after the last row group
 *   4: ring kernel from N * K >= 8 M (the earlier default)
 * No counterpart in the reference (its set_gemv_impl chooses how x is loaded, kernels/lfm2_decode.cu:662-675).
 * Tuning and testing only; a process-wide setting. */
void lfm2q_set_gemv_path(int path);

/* GEMV kernels launched with Programmatic Dependent Launch let the next kernel launch after their K loop
 * (early == 0, default) or at their start (early != 0). Tuning only; results are unchanged. */
void lfm2q_set_gemv_trigger(int early);

/* Failure-detection self-test (no counterpart in the reference): launches one block that runs the GEMM pipeline's
 * bounded mbarrier wait on a barrier nothing arrives on, with a limit of 2^limit_log2 clock cycles (10..31). The wait
 * gives up, sets the device error word and the kernel ends normally; lfm2q_check_device then reports LFM2Q_ETIMEOUT
 * (and clears it with clear != 0). The context stays usable. Asynchronous on `stream`. */
int lfm2q_selftest_wait_timeout(int limit_log2, void *stream);

/* Forces the per-token GEMM tile: 128 or 256 = one CTA per 128-row tile of that many columns; -192 or -256 = a CTA
 * pair (cluster of two, tcgen05 cta_group::2) per 256-row tile of that many columns; 0 = automatic. The SiLU GEMM
 * follows the sign (one CTA or a pair, 128 output columns per tile); 64 = one CTA per 128 x 64 tile (W8A16 only, its
 * small-M choice; the int8 GEMMs treat it as automatic); 1 = the per-token W8A8 GEMM splits K over a cluster of
 * CTAs per 128 x 128 tile wherever K has two 128-byte blocks per CTA (automatic: when the tiles fill fewer than half
 * the SMs). Tuning and testing only. */
void lfm2q_set_gemm_tile(int bn);

#ifdef __cplusplus
}
#endif

#endif /* LFM2Q_H */
