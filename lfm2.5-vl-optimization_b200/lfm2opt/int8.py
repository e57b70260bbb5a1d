"""INT8 linear layers for prefill and the vision encoder, on the B200 kernels of liblfm2q.

Drop-in for the reference module src/lfm2opt/int8.py (Int8Linear :54-91, quantize_rows :45-51, qbuf :39-42,
act_group :27-36, a16_kinds :22-24): same names, arguments, environment variables and return values.

  a8  (W8A8):  activations quantized on the fly (quantize_rows) with one scale per token (LFM2_INT8_GROUP=0) or per
               token and group of 64 input channels (LFM2_INT8_GROUP=64, the default), int8 x int8 tcgen05 GEMM with
               the scales, bias and GELU in the epilogue (per-token calls of <= 16 tokens, and of up to 64 with
               long K, run the A8 GEMV inside gemm_i8: same exact int32 sums, same epilogue).
  a16 (W8A16): bf16 activations, int8 weights (LFM2_INT8_A16 lists the layer kinds).

Additions over the reference (all optional, defaults keep the reference's behaviour):
  Int8Linear(..., group=None)            explicit activation granularity (None = act_group(kind, K)); the
                                         per-token quantizer here handles K up to 16384, so wide inputs may run
                                         per token when asked for explicitly.
  Int8Linear.__call__(x, silu_gate=True) weight = [w1 | w3] (2I rows): returns bf16(bf16(silu(x w1^T)) * (x w3^T)),
                                         [..., I], from one GEMM whose epilogue applies the gate.
"""

import os

import torch

from .kernels import int8_ext
from .quant import quantize_int8


def a16_kinds():
    """The set of layer kinds named in LFM2_INT8_A16 (comma-separated): those layers take bf16 activations and int8
    weights (W8A16); every other kind runs W8A8."""
    return set(filter(None, os.environ.get("LFM2_INT8_A16", "").split(",")))


def act_group(kind=None, K=0):
    """How finely a W8A8 layer's activations are scaled: 0 = one scale per token, 64 = one per token and 64-channel
    slice of the input. LFM2_INT8_GROUP (0 or 64, default 64) chooses it; LFM2_INT8_GROUP_KINDS, a comma-separated
    list of kinds, restricts the 64-wide scales to those kinds. Layers with K > 2048 always get 64-wide scales,
    which is the reference's rule (its per-token quantizer stops at K = 2048)."""
    g = int(os.environ.get("LFM2_INT8_GROUP", "64"))
    if g not in (0, 64):
        raise ValueError("LFM2_INT8_GROUP must be 0 or 64: the kernel folds one scale per 64-wide K group")
    kinds = set(filter(None, os.environ.get("LFM2_INT8_GROUP_KINDS", "").split(",")))
    if K > 2048:
        return 64
    return g if (not kinds or kind in kinds) else 0


def qbuf(rows, K, group, device):
    """Uninitialised output buffers for a kernel that writes a W8A8 layer's quantized input itself: int8 [rows, K]
    codes and fp32 scales, [rows] for group 0 or [K / 64, rows] for group 64."""
    return (torch.empty(rows, K, device=device, dtype=torch.int8),
            torch.empty((K // 64, rows) if group else (rows,), device=device, dtype=torch.float32))


def quantize_rows(x2, group=0):
    """Quantize bf16 activations x2 [M, K] to int8 on the GPU. Returns (codes int8 [M, K], fp32 scales): with
    group 0 one scale per row, [M] (row absmax / 127); with group 64 one per row and 64 columns, laid out [K / 64, M]."""
    M, K = x2.shape
    q = torch.empty(x2.shape, device=x2.device, dtype=torch.int8)
    s = torch.empty((K // 64, M) if group else (M,), device=x2.device, dtype=torch.float32)
    int8_ext().quant_rows(x2, q, s)
    return q, s


class Int8Linear:
    def __init__(self, weight=None, bias=None, a8=True, q=None, scale=None, pad_n=0, pad_k=0, kind=None, group=None):
        """Build the layer either from a bf16 weight [N, K], which is quantized per output row here, or from an
        already quantized pair (q int8 [N, K], scale fp32 [N]). pad_n adds zero weight rows (and zero bias) at the
        end, pad_k zero input columns, before quantizing; the grouped activation scales need K % 128 == 0, so a
        4304-wide layer is padded to 4352 (pad_n=48 on the layer that produces it, pad_k=48 on the one that reads
        it). kind names the layer for LFM2_INT8_A16 / LFM2_INT8_GROUP_KINDS; group overrides act_group."""
        if q is None:
            weight = torch.nn.functional.pad(weight, (0, pad_k, 0, pad_n))
            if bias is not None and pad_n:
                bias = torch.nn.functional.pad(bias, (0, pad_n))
            q, scale = quantize_int8(weight)
        self.q, self.s, self.bias, self.a8 = q, scale, bias, a8
        self.N, self.K = q.shape
        if group is not None and group not in (0, 64):
            raise ValueError("group must be 0 (per token) or 64")
        self.group = (act_group(kind, self.K) if group is None else group) if a8 else 0
        self.ext = int8_ext()

    def __call__(self, x, gelu=False, quant_out=False, silu_gate=False):
        """Apply the layer. x is bf16 [..., K] or, when a producer kernel already quantized it, the pair
        (int8 [..., K], scales) that kernel wrote. Returns bf16 [..., N] with GELU applied when gelu is set.
        quant_out: return the result already quantized for the next W8A8 layer, (int8 [M, N], scales [N/64, M]),
        from this GEMM's epilogue (grouped W8A8 only, N % 128 == 0).
        silu_gate: the weight rows are [w1 | w3]; returns bf16(bf16(silu(g)) * u) [..., N/2] from one GEMM (per-token
        W8A8 only: a layer built with a8=False or with 64-wide activation scales raises ValueError)."""
        if quant_out:
            xq, sx = x if isinstance(x, tuple) else quantize_rows(x.reshape(-1, self.K).contiguous(), 64)
            M = xq.numel() // self.K
            yq, ys = qbuf(M, self.N, 64, xq.device)
            self.ext.gemm_i8_q(xq, sx, self.q, self.s, self.bias, yq, ys, gelu)
            return yq, ys
        if silu_gate:
            if gelu:
                raise ValueError("silu_gate and gelu are exclusive epilogues")
            if not self.a8 or self.group != 0:
                raise ValueError("silu_gate runs the per-token W8A8 epilogue: build the layer with a8=True and "
                                 "group=0 (it has " + ("a8=False" if not self.a8 else f"group={self.group}") + ")")
            if isinstance(x, tuple):
                xq, sx = x
                lead = xq.shape[:-1]
            else:
                lead = x.shape[:-1]
                xq, sx = quantize_rows(x.reshape(-1, self.K).contiguous(), 0)
            y = torch.empty(xq.numel() // self.K, self.N // 2, device=xq.device, dtype=torch.bfloat16)
            self.ext.gemm_i8_silu(xq, sx, self.q, self.s, self.bias, y)
            return y.view(*lead, self.N // 2)
        if isinstance(x, tuple):
            xq, sx = x
            y = torch.empty(xq.numel() // self.K, self.N, device=xq.device, dtype=torch.bfloat16)
            self.ext.gemm_i8(xq, sx, self.q, self.s, self.bias, y, gelu)
            return y.view(*xq.shape[:-1], self.N)
        x2 = x.reshape(-1, self.K)
        y = torch.empty(x2.shape[0], self.N, device=x.device, dtype=torch.bfloat16)
        if self.a8:
            xq, sx = quantize_rows(x2.contiguous(), self.group)
            self.ext.gemm_i8(xq, sx, self.q, self.s, self.bias, y, gelu)
        else:
            self.ext.gemm_w8(x2.contiguous(), self.q, self.s, self.bias, y, gelu)
        return y.view(*x.shape[:-1], self.N)
