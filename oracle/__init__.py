"""TEST INFRASTRUCTURE ONLY — CPU oracle for the lfm2q INT8 matrix-multiply hot path.

A CPU restatement of the reference's algorithm (jainilbavishi24/LFM2.5-VL-Optimization): the PyTorch reference
expressions its tests check the CUDA kernels against (tests/test_int8_gemm.py, tests/test_kernels.py) and the
semantics of its kernels (kernels/int8_gemm.cu, kernels/lfm2_decode.cu), every function citing the file:line it
follows. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference`) may import
it, and only as the checker or the timed CPU baseline. The product (liblfm2q.so and the lfm2opt package) never
imports, links or calls anything here.

Parity is pinned: tests/golden/ holds vectors produced by the reference's own Python code, run on CPU in the build
container (tests/golden/make_golden.py); tests/test_oracle.py checks this oracle against them bit for bit.
"""

from .quant import quantize_int8_ref, quantize_int4_ref, quant_rows_ref, quant_groups_ref  # noqa: F401
from .gemm import (gemm_i8_ref, gemm_i8_grouped_ref, gemm_i8_grouped_f64, gemm_i8_q_ref, gemm_i8_silu_ref,  # noqa: F401
                   gemm_w8_f64, int_mm_exact, bf16_ulps, silu_chain_close, gelu_close)
from .gemv import gemv_ref, gemv_f64, gemv_epi_ref, gemv_w4_ref, gemv_w4_f64, dequantize_int4_ref  # noqa: F401
from .attention import decode_attention_f64, decode_attention_sdpa, split_partials_f64  # noqa: F401
from .decode import add_rmsnorm_ref, shortconv_step_ref, qk_norm_rope_kv_ref  # noqa: F401
