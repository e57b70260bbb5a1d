"""The two extension objects the reference loads (src/lfm2opt/kernels.py:16-68 of the reference), backed by the
prebuilt sm_100a library liblfm2q.so instead of a JIT build.

    int8_ext()  ops of the reference's lfm2_int8_gemm extension (kernels/int8_gemm.cpp:143-151):
                gemm_i8, gemm_i8_q, gemm_w8, quant_rows, add_layernorm_q, add_rmsnorm_q, silu_mul_q,
                plus gemm_i8_silu (W8A8 GEMM with the SiLU(w1) * w3 gate fused into its epilogue)
    ext()       the GEMV part of the reference's lfm2_decode extension (kernels/lfm2_decode.cpp:152-168):
                gemv, gemv_epi, gemv_w4, set_pdl, set_gemv_impl, plus gemv_a8 (int8 tokens x int8 weights, exact int32)

Argument names, meaning, in-place outputs and the RuntimeError messages of the shape checks follow the reference
bindings (kernels/int8_gemm.cpp:20-141, kernels/lfm2_decode.cpp:30-150). Every op enqueues on PyTorch's current
stream of the tensors' device and returns None. The decode extension's non-GEMV kernels (attention, RoPE, conv,
norms) are not part of this library; reaching for them raises AttributeError.
"""

import ctypes
import os

import torch

from . import _capi

_I8, _BF, _F32 = torch.int8, torch.bfloat16, torch.float32


def _check(t, dtype, name):
    if not (t.is_cuda and t.dtype == dtype and t.is_contiguous()):
        raise RuntimeError(f"{name} must be contiguous CUDA {_DT_NAME[dtype]}")


_DT_NAME = {_I8: "at::kChar", _BF: "at::kBFloat16", _F32: "at::kFloat"}


def _req(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


class _DeviceOf:
    """Make t's device current for the duration of a call (ops launch on the current device)."""

    __slots__ = ("idx", "prev")

    def __init__(self, t):
        self.idx = t.device.index

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev != self.idx:
            torch.cuda.set_device(self.prev)


class Int8GemmExt:
    """Ops of the reference's lfm2_int8_gemm extension."""

    @staticmethod
    def _common(w, sw, bias, y, M, K):
        _check(w, _I8, "w")
        _check(sw, _F32, "sw")
        _check(y, _BF, "y")
        _req(w.dim() == 2 and w.size(1) == K, "w must be [N, K]")
        N = w.size(0)
        _req(K % 16 == 0 and N % 8 == 0, "need K % 16 == 0 and N % 8 == 0")
        _req(sw.numel() == N and y.numel() == M * N, "sw / y shape")
        if bias is not None:
            _check(bias, _BF, "(*bias)")
            _req(bias.numel() == N, "bias shape")
        return N

    def gemm_i8(self, xq, sx, w, sw, bias, y, gelu):
        """W8A8: y[M, N] = (xq[M, K] . w[N, K]^T) * sx[m] * sw[n] (+ bias) (GELU), bf16 out. sx [M]: one scale per
        row; sx [K/64, M]: one scale per row and group of 64 input channels."""
        _check(xq, _I8, "xq")
        _check(sx, _F32, "sx")
        K = xq.size(-1)
        M = xq.numel() // K
        grouped = sx.dim() == 2
        _req((K % 64 == 0 and sx.size(0) == K // 64 and sx.size(1) == M) if grouped else sx.numel() == M, "sx shape")
        N = self._common(w, sw, bias, y, M, K)
        with _DeviceOf(xq):
            _capi.call("lfm2q_gemm_i8", xq.data_ptr(), sx.data_ptr(), int(grouped), w.data_ptr(), sw.data_ptr(),
                       _ptr(bias), y.data_ptr(), M, N, K, int(bool(gelu)), _stream(xq))

    def gemm_i8_q(self, xq, sxT, w, sw, bias, yq, ysT, gelu):
        """Grouped W8A8 with an INT8 output for the next W8A8 GEMM: (yq [M, N], ysT [N/64, M])."""
        for t, n, d in ((xq, "xq", _I8), (sxT, "sxT", _F32), (w, "w", _I8), (sw, "sw", _F32), (yq, "yq", _I8),
                        (ysT, "ysT", _F32)):
            _check(t, d, n)
        K = xq.size(-1)
        M, N = xq.numel() // K, w.size(0)
        _req(sxT.dim() == 2 and K % 64 == 0 and sxT.size(0) == K // 64 and sxT.size(1) == M, "sxT shape")
        _req(w.dim() == 2 and w.size(1) == K and N % 128 == 0 and sw.numel() == N, "w [N, K] with N % 128 == 0")
        _req(yq.numel() == M * N and ysT.dim() == 2 and ysT.size(0) == N // 64 and ysT.size(1) == M, "yq / ysT shape")
        if bias is not None:
            _check(bias, _BF, "(*bias)")
            _req(bias.numel() == N, "bias shape")
        with _DeviceOf(xq):
            _capi.call("lfm2q_gemm_i8_q", xq.data_ptr(), sxT.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias),
                       yq.data_ptr(), ysT.data_ptr(), M, N, K, int(bool(gelu)), _stream(xq))

    def gemm_i8_silu(self, xq, sx, w, sw, bias, y):
        """W8A8 over w = [w1 | w3] [2I, K] with the SwiGLU gate in the epilogue: y [M, I] = bf16(bf16(silu(g)) * u),
        g / u = the bf16 per-token outputs of rows n / I + n (gemm_i8 followed by silu_mul, in one kernel)."""
        _check(xq, _I8, "xq")
        _check(sx, _F32, "sx")
        K = xq.size(-1)
        M = xq.numel() // K
        _req(sx.dim() == 1 and sx.numel() == M, "sx shape: the SiLU-gate epilogue takes per-token scales [M]")
        _check(w, _I8, "w")
        _check(sw, _F32, "sw")
        _check(y, _BF, "y")
        _req(w.dim() == 2 and w.size(1) == K and w.size(0) % 2 == 0, "w must be [2I, K]")
        I = w.size(0) // 2
        _req(K % 16 == 0 and I % 8 == 0, "need K % 16 == 0 and I % 8 == 0")
        _req(sw.numel() == 2 * I and y.numel() == M * I, "sw / y shape")
        if bias is not None:
            _check(bias, _BF, "(*bias)")
            _req(bias.numel() == 2 * I, "bias shape")
        with _DeviceOf(xq):
            _capi.call("lfm2q_gemm_i8_silu", xq.data_ptr(), sx.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias),
                       y.data_ptr(), M, I, K, _stream(xq))

    def linear_a8(self, x, w, sw, bias, y, gelu):
        """Per-token W8A8 for a few tokens in one launch: quant_rows(x) fused into the A8 GEMV, bit-identical to
        quant_rows followed by gemm_i8 (no counterpart op in the reference)."""
        _check(x, _BF, "x")
        K = x.size(-1)
        M = x.numel() // K
        N = self._common(w, sw, bias, y, M, K)
        _req(K % 64 == 0 and K <= 16384, "K must be a multiple of 64, <= 16384")
        with _DeviceOf(x):
            _capi.call("lfm2q_linear_a8", x.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias), y.data_ptr(), N, K, M,
                       int(bool(gelu)), _stream(x))

    def gemm_w8(self, x, w, sw, bias, y, gelu):
        """W8A16: y[M, N] = (x[M, K] . w[N, K]^T) * sw[n] (+ bias) (GELU), bf16 in / out."""
        _check(x, _BF, "x")
        K = x.size(-1)
        M = x.numel() // K
        N = self._common(w, sw, bias, y, M, K)
        with _DeviceOf(x):
            _capi.call("lfm2q_gemm_w8", x.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias), y.data_ptr(), M, N, K,
                       int(bool(gelu)), _stream(x))

    def quant_rows(self, x, q, s):
        """Per-row (token) symmetric quantization: s = max(|x|) / 127, q = round(x / s); with s of shape [K/64, rows]:
        one scale per row and group of 64 channels (transposed, as gemm_i8 reads it)."""
        _check(x, _BF, "x")
        _check(q, _I8, "q")
        _check(s, _F32, "s")
        K = x.size(-1)
        rows = x.numel() // K
        if s.dim() == 2:
            _req(K % 64 == 0 and K <= 16384 and s.size(0) == K // 64 and s.size(1) == rows and q.numel() == x.numel(),
                 "grouped shapes")
            with _DeviceOf(x):
                _capi.call("lfm2q_quant_groups", x.data_ptr(), q.data_ptr(), s.data_ptr(), rows, K, _stream(x))
            return
        _req(K % 8 == 0 and K <= 16384, "K must be a multiple of 8, <= 16384")
        _req(q.numel() == x.numel() and s.numel() == rows, "q / s shape")
        with _DeviceOf(x):
            _capi.call("lfm2q_quant_rows", x.data_ptr(), q.data_ptr(), s.data_ptr(), rows, K, _stream(x))

    @staticmethod
    def _check_qs(q, s, rows, K):
        _check(q, _I8, "q")
        _check(s, _F32, "s")
        grouped = s.dim() == 2
        _req(q.numel() == rows * K, "q shape")
        _req((K % 64 == 0 and s.size(0) == K // 64 and s.size(1) == rows) if grouped else s.numel() == rows,
             "s shape")
        return grouped

    def add_layernorm_q(self, h, y, w, b, q, s, eps):
        """Vision: h += y (optional, in place); (q, s) = quant(LayerNorm(h) * w + b)."""
        _check(h, _BF, "h")
        _check(w, _BF, "w")
        _check(b, _BF, "b")
        if y is not None:
            _check(y, _BF, "(*y)")
            _req(y.numel() == h.numel(), "y shape")
        D = h.size(-1)
        rows = h.numel() // D
        _req(D % 8 == 0 and D <= 16384 and w.numel() == D and b.numel() == D, "D must be a multiple of 8, <= 16384")
        grouped = self._check_qs(q, s, rows, D)
        with _DeviceOf(h):
            _capi.call("lfm2q_add_layernorm_q", h.data_ptr(), _ptr(y), w.data_ptr(), b.data_ptr(), q.data_ptr(),
                       s.data_ptr(), rows, D, float(eps), int(grouped), _stream(h))

    def add_rmsnorm_q(self, h, y, w, q, s, eps):
        """LM prefill: h += y (optional, in place); (q, s) = quant(w * rmsnorm(h))."""
        _check(h, _BF, "h")
        _check(w, _BF, "w")
        if y is not None:
            _check(y, _BF, "(*y)")
            _req(y.numel() == h.numel(), "y shape")
        H = h.size(-1)
        rows = h.numel() // H
        _req(w.numel() == H and H % 8 == 0 and H <= 16384, "w shape")
        grouped = self._check_qs(q, s, rows, H)
        with _DeviceOf(h):
            _capi.call("lfm2q_add_rmsnorm_q", h.data_ptr(), _ptr(y), w.data_ptr(), q.data_ptr(), s.data_ptr(), rows,
                       H, float(eps), int(grouped), _stream(h))

    def silu_mul_q(self, g, q, s):
        """LM prefill: g [rows, 2I] = w1 | w3 outputs -> (q, s) = quant(silu(g1) * g3)."""
        _check(g, _BF, "g")
        I = g.size(-1) // 2
        rows = g.numel() // (2 * I)
        _req(I % 8 == 0 and I <= 16384, "I shape")
        grouped = self._check_qs(q, s, rows, I)
        with _DeviceOf(g):
            _capi.call("lfm2q_silu_mul_q", g.data_ptr(), q.data_ptr(), s.data_ptr(), rows, I, int(grouped),
                       _stream(g))


class DecodeGemvExt:
    """The GEMV ops of the reference's lfm2_decode extension."""

    def gemv(self, W, scale, x, y, rows=0):
        """y [B, N] = x [B, K] @ W^T, W [N, K] BF16 or INT8 (then scale [N] fp32 is required); B >= 1."""
        if not (x.is_cuda and x.dtype == _BF and x.is_contiguous()):
            raise RuntimeError("x must be contiguous CUDA bf16")
        if not (y.is_cuda and y.dtype == _BF and y.is_contiguous()):
            raise RuntimeError("y must be contiguous CUDA bf16")
        _req(W.is_cuda and W.is_contiguous() and W.dim() == 2, "W must be a contiguous CUDA matrix")
        int8 = W.dtype == _I8
        _req(int8 or W.dtype == _BF, "W must be bf16 or int8")
        _req(not int8 or (scale is not None and scale.dtype == _F32), "int8 W needs fp32 scale")
        N, K = W.shape
        B = x.numel() // K
        _req(x.numel() == B * K and y.numel() == B * N and B >= 1, "x [B, K], y [B, N]")
        _req(K % (32 * (16 if int8 else 8)) == 0, "K must be a multiple of 256 (bf16) / 512 (int8)")
        if scale is not None:
            _req(scale.is_cuda and scale.is_contiguous() and scale.numel() == N, "scale must be contiguous CUDA [N]")
        with _DeviceOf(x):
            _capi.call("lfm2q_gemv", W.data_ptr(), int(int8), _ptr(scale), x.data_ptr(), y.data_ptr(), N, K,
                       int(rows), B, _stream(x))

    def gemv_epi(self, epi, W, scale, x, y, state=None, cw=None, cbias=None):
        """Batch-1 GEMV + fused epilogue. epi 0: W = w1|w3 [2S, K] -> y [1, S] = silu(w1 x) * (w3 x);
        epi 1: W = in_proj [3S, K] -> y [1, S] = shortconv_step(in_proj x), conv state updated in place."""
        for t, n in ((x, "x"), (y, "y")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        _req(W.is_cuda and W.is_contiguous() and W.dim() == 2, "W must be a contiguous CUDA matrix")
        int8 = W.dtype == _I8
        _req(int8 or W.dtype == _BF, "W must be bf16 or int8")
        _req(not int8 or (scale is not None and scale.dtype == _F32), "int8 W needs fp32 scale")
        _req(epi in (0, 1), "epi 0 (swiglu) or 1 (shortconv)")
        NR = 2 if epi == 0 else 3
        K = W.size(1)
        S = W.size(0) // NR
        _req(W.size(0) == NR * S and x.numel() == K and y.numel() == S, "batch 1: x [1, K], y [1, S]")
        _req(K % (32 * (16 if int8 else 8)) == 0, "K must be a multiple of 256 (bf16) / 512 (int8)")
        if epi == 1:
            _req(state is not None and cw is not None, "shortconv epilogue needs state and conv weight")
            for t, n in ((state, "(*state)"), (cw, "(*cw)")):
                if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                    raise RuntimeError(f"{n} must be contiguous CUDA bf16")
            _req(state.numel() == S * 3 and cw.numel() == S * 3, "state [1, S, 3], cw [S, 3]")
            if cbias is not None and not (cbias.is_cuda and cbias.dtype == _BF and cbias.is_contiguous()):
                raise RuntimeError("(*cbias) must be contiguous CUDA bf16")
        with _DeviceOf(x):
            _capi.call("lfm2q_gemv_epi", int(epi), W.data_ptr(), int(int8), _ptr(scale), x.data_ptr(), y.data_ptr(),
                       S, K, _ptr(state) if epi == 1 else None, _ptr(cw) if epi == 1 else None,
                       _ptr(cbias) if epi == 1 else None, _stream(x))

    def gemv_a8(self, W, sw, xq, sx, y, bias=None, gelu=False):
        """A8 decode GEMV (no counterpart in the reference): y [B, N] = bf16(act((xq . W^T) * sx[b] * sw[n] + bias)),
        xq int8 [B, K] with per-token scales sx [B] (from quant_rows), exact int32 sums: equal to gemm_i8 on the same
        operands."""
        _check(W, _I8, "W")
        _check(sw, _F32, "sw")
        _check(xq, _I8, "xq")
        _check(sx, _F32, "sx")
        _check(y, _BF, "y")
        N, K = W.shape
        B = xq.numel() // K
        _req(W.dim() == 2 and xq.numel() == B * K and B >= 1 and y.numel() == B * N, "xq [B, K], y [B, N]")
        _req(sx.numel() == B and sw.numel() == N, "sx [B], sw [N]")
        _req(K % 64 == 0, "K must be a multiple of 64")
        if bias is not None:
            _check(bias, _BF, "(*bias)")
            _req(bias.numel() == N, "bias shape")
        with _DeviceOf(xq):
            _capi.call("lfm2q_gemv_a8", W.data_ptr(), sw.data_ptr(), xq.data_ptr(), sx.data_ptr(), _ptr(bias),
                       y.data_ptr(), N, K, B, int(bool(gelu)), _stream(xq))

    def gemv_w4(self, Wp, S, x, y, rows=0):
        """INT4 weight-only GEMV: y [1, N] = x [1, K] . dequant(Wp)^T, Wp uint8 [N, K/2] (two codes + 8 per byte, low
        nibble first), S fp32 [N, K / group] (lfm2opt.quant.quantize_int4). rows: accepted for compatibility."""
        _req(Wp.is_cuda and Wp.is_contiguous() and Wp.dtype == torch.uint8 and Wp.dim() == 2,
             "Wp: contiguous uint8 [N, K/2]")
        _req(S.is_cuda and S.is_contiguous() and S.dtype == _F32, "S: contiguous fp32 [N, K/128]")
        _check(x, _BF, "x")
        _check(y, _BF, "y")
        N, K = Wp.size(0), Wp.size(1) * 2
        _req(S.size(0) == N and K % S.size(1) == 0, "S must be [N, K / group]")
        group = K // S.size(1)
        _req(group % 32 == 0, "group size must be a multiple of 32")
        _req(x.numel() == K and y.numel() == N, "batch 1 only")
        with _DeviceOf(x):
            _capi.call("lfm2q_gemv_w4", Wp.data_ptr(), S.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, group, 1,
                       _stream(x))

    def add_rmsnorm(self, h, y, w, x, eps):
        """h += y (if y is not None); x = w * rmsnorm(h), bf16, rows of H (the reference's add_rmsnorm binding,
        kernels/lfm2_decode.cpp:32-37)."""
        for t, n in ((h, "h"), (w, "w"), (x, "x")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        if y is not None and not (y.is_cuda and y.dtype == _BF and y.is_contiguous()):
            raise RuntimeError("(*y) must be contiguous CUDA bf16")
        H = h.size(-1)
        rows = h.numel() // H
        _req(w.numel() == H and x.numel() == h.numel() and (y is None or y.numel() == h.numel()), "shapes")
        with _DeviceOf(h):
            _capi.call("lfm2q_add_rmsnorm", h.data_ptr(), _ptr(y), w.data_ptr(), x.data_ptr(), rows, H, float(eps),
                       _stream(h))

    def embed_rmsnorm(self, tok, embed, w, h, x, eps):
        """h = embed[tok] (bits unchanged), x = w * rmsnorm(h): F.embedding + add_rmsnorm(h, None, w, x, eps) in one
        launch (no counterpart in the reference). tok int64 [rows] on the device, embed bf16 [V, H]."""
        for t, n in ((embed, "embed"), (w, "w"), (h, "h"), (x, "x")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        _req(tok.is_cuda and tok.dtype == torch.int64 and tok.is_contiguous(), "tok: contiguous CUDA int64")
        H = embed.size(1)
        rows = tok.numel()
        _req(h.numel() == rows * H and x.numel() == rows * H and w.numel() == H, "h, x [rows, H], w [H]")
        with _DeviceOf(h):
            _capi.call("lfm2q_embed_rmsnorm", tok.data_ptr(), embed.data_ptr(), w.data_ptr(), h.data_ptr(),
                       x.data_ptr(), rows, H, float(eps), _stream(h))

    def argmax_next(self, logits, tok, pos=None):
        """tok[b] = argmax(logits[b]) (first index of the maximum, NaN largest, as torch.argmax), then pos += 1:
        the end of a decode step in one launch (no counterpart in the reference)."""
        if not (logits.is_cuda and logits.dtype == _BF and logits.is_contiguous()):
            raise RuntimeError("logits must be contiguous CUDA bf16")
        _req(tok.is_cuda and tok.dtype == torch.int64 and tok.is_contiguous(), "tok: contiguous CUDA int64")
        _req(pos is None or (pos.is_cuda and pos.dtype == torch.int64), "pos: CUDA int64 [1]")
        B = tok.numel()
        V = logits.numel() // max(B, 1)
        _req(logits.numel() == B * V, "logits [B, V]")
        with _DeviceOf(logits):
            _capi.call("lfm2q_argmax_next", logits.data_ptr(), tok.data_ptr(), _ptr(pos), B, V, _stream(logits))

    def shortconv_step(self, bcx, state, w, bias, y):
        """One short-convolution decode step (the reference's shortconv_step binding,
        kernels/lfm2_decode.cpp:39-45): bcx [B, 3H], state [B, H, 3] updated in place, w [H, 3], bias [H] or None,
        y [B, H]."""
        for t, n in ((bcx, "bcx"), (state, "state"), (w, "w"), (y, "y")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        _req(state.size(-1) == 3, "conv state length must be 3")
        B, H = bcx.size(0), bcx.size(-1) // 3
        _req(state.numel() == B * H * 3 and w.numel() == H * 3 and y.numel() == B * H, "shapes")
        if bias is not None:
            _req(bias.is_cuda and bias.dtype == _BF and bias.is_contiguous() and bias.numel() == H, "bias [H] bf16")
        with _DeviceOf(bcx):
            _capi.call("lfm2q_shortconv_step", bcx.data_ptr(), state.data_ptr(), w.data_ptr(), _ptr(bias),
                       y.data_ptr(), B, H, _stream(bcx))

    def qk_norm_rope_kv(self, qkv, qw, kw, inv_freq, scaling, pos, q_out, kc, vc, eps):
        """Per-head RMSNorm of q and k, RoPE, k and v into the cache at pos (the reference's qk_norm_rope_kv
        binding, kernels/lfm2_decode.cpp:47-55): qkv [B, (NQ + 2 NKV) * 64], q_out [B, NQ, 64], kc / vc
        [B, NKV, max_len, 64]."""
        for t, n in ((qkv, "qkv"), (qw, "qw"), (kw, "kw"), (q_out, "q_out"), (kc, "kc"), (vc, "vc")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        _req(inv_freq.dtype == _F32 and pos.dtype == torch.int64, "inv_freq fp32, pos int64")
        _req(kc.size(3) == 64, "head_dim 64 only")
        B, NQ, NKV, max_len = qkv.size(0), q_out.size(1), kc.size(1), kc.size(2)
        _req(qkv.numel() == B * (NQ + 2 * NKV) * 64 and vc.shape == kc.shape and inv_freq.numel() >= 32, "shapes")
        with _DeviceOf(qkv):
            _capi.call("lfm2q_qk_norm_rope_kv", qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), inv_freq.data_ptr(),
                       float(scaling), pos.data_ptr(), q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, NQ, NKV,
                       max_len, float(eps), _stream(qkv))

    def decode_attention_split(self, q, kc, vc, pos, out, ws, scale):
        """One decode step of attention over the KV cache, split over positions (the reference's
        decode_attention_split binding, kernels/lfm2_decode.cpp:64-71): q bf16 [B, NQ, 64], kc / vc bf16
        [B, NKV, max_len, 64] with NQ == 4 * NKV, pos int64 [1] (positions 0 .. pos attended), out bf16 [B, NQ, 64],
        ws fp32 [B, NQ, S, 66] the per-split partials (S = ws.size(2))."""
        for t, n in ((q, "q"), (kc, "kc"), (vc, "vc"), (out, "out")):
            if not (t.is_cuda and t.dtype == _BF and t.is_contiguous()):
                raise RuntimeError(f"{n} must be contiguous CUDA bf16")
        _req(kc.dim() == 4 and kc.size(3) == 64 and q.dim() == 3 and q.size(1) == 4 * kc.size(1),
             "head_dim 64 and 4 query heads per KV head only")
        B, NQ = q.size(0), q.size(1)
        NKV, max_len = kc.size(1), kc.size(2)
        _req(q.size(2) == 64 and kc.size(0) == B and vc.shape == kc.shape and out.shape == q.shape,
             "q [B, NQ, 64], kc / vc [B, NKV, max_len, 64], out [B, NQ, 64]")
        _req(ws.is_cuda and ws.dtype == _F32 and ws.is_contiguous() and ws.dim() == 4 and ws.size(3) == 66
             and ws.size(0) == B and ws.size(1) == NQ, "ws: fp32 [B, NQ, S, 66]")
        _req(pos.is_cuda and pos.dtype == torch.int64 and pos.numel() >= 1, "pos: CUDA int64 [1]")
        with _DeviceOf(q):
            _capi.call("lfm2q_decode_attention_split", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                       out.data_ptr(), ws.data_ptr(), B, NQ, NKV, max_len, ws.size(2), float(scale), _stream(q))

    def set_pdl(self, on):
        """Enable/disable Programmatic Dependent Launch for the GEMV kernels (default on)."""
        _capi.lib().lfm2q_set_pdl(int(bool(on)))

    def set_gemv_impl(self, impl):
        """Accepted for compatibility with the reference (0 = staged x, 1 = direct x); this build has one GEMV."""
        _capi.lib().lfm2q_set_gemv_impl(int(impl))


class GemvChain:
    """A fixed list of int8 weight-only decode GEMVs run in order (lfm2q_gemv_chain, include/lfm2q.h): the run of gemv
    calls a decode step makes back to back, with the weights of the layers ahead streamed into L2 meanwhile.

    layers: sequence of (W int8 [N, K], scale fp32 [N], x bf16 [B, K], y bf16 [B, N]) with one B (1..4) for all; a
    layer's x may be an earlier layer's y. The tensors are referenced, not copied: calling the chain reads the current
    contents of every x and writes every y, on the current stream (capturable in a CUDA graph)."""

    def __init__(self, layers):
        layers = list(layers)
        _req(1 <= len(layers) <= 96, "a chain holds 1 to 96 layers")
        B = layers[0][2].shape[0]
        _req(1 <= B <= 4, "x [B, K]: the chained GEMV takes 1 <= B <= 4 tokens")
        arr = (_capi.GemvLayer * len(layers))()
        for i, (W, scale, x, y) in enumerate(layers):
            _check(W, _I8, "W")
            _check(scale, _F32, "scale")
            _check(x, _BF, "x")
            _check(y, _BF, "y")
            _req(W.dim() == 2, "W must be [N, K]")
            N, K = W.shape
            _req(K % 512 == 0, f"layer {i}: K must be a multiple of 512")
            _req(x.dim() == 2 and x.shape == (B, K), f"layer {i}: x must be [B, K] with the chain's B")
            _req(y.numel() == B * N and scale.numel() == N, f"layer {i}: y / scale shape")
            _req(W.device == x.device == y.device == scale.device == layers[0][0].device, "one device for all")
            arr[i] = _capi.GemvLayer(W.data_ptr(), scale.data_ptr(), x.data_ptr(), y.data_ptr(), N, K)
        self.B, self.n, self.arr = B, len(layers), arr
        self.device = layers[0][0].device
        self._keep = layers  # the launches read these pointers

    def __call__(self):
        with _DeviceOf(self._keep[0][0]):
            _capi.call("lfm2q_gemv_chain", ctypes.cast(self.arr, ctypes.c_void_p), self.n, self.B,
                       torch.cuda.current_stream(self.device).cuda_stream)


def check_device(clear=False):
    """Raise RuntimeError if a bounded pipeline wait inside a tcgen05 GEMM or the decode attention gave up since the
    last clear (the outputs of
    that work are then invalid). Synchronises with the current device. clear: reset the word."""
    st = _capi.lib().lfm2q_check_device(int(bool(clear)))
    if st != _capi.OK:
        raise RuntimeError(_capi.lib().lfm2q_last_error().decode() or f"lfm2q_check_device: status {st}")


_INT8 = None
_DEC = None


def int8_ext():
    """INT8 tensor-core GEMMs for prefill and the vision encoder (replaces the reference's JIT-built extension)."""
    global _INT8
    if _INT8 is None:
        _capi.lib()  # fail here, loudly, if the library is missing
        _INT8 = Int8GemmExt()
    return _INT8


def ext():
    """Decode GEMV kernels. Programmatic Dependent Launch is on unless LFM2_PDL=0, as in the reference."""
    global _DEC
    if _DEC is None:
        _capi.lib()
        _DEC = DecodeGemvExt()
        _DEC.set_pdl(os.environ.get("LFM2_PDL", "1") != "0")
        _capi.lib().lfm2q_set_gemv_trigger(int(os.environ.get("LFM2_GEMV_TRIGGER", "late") == "early"))
    return _DEC
