"""lfm2opt — the INT8 matrix-multiply hot path of LFM2.5-VL-Optimization, rebuilt for B200 (sm_100a).

Drop-in for the reference package's hot-path modules: `lfm2opt.int8` (Int8Linear, quantize_rows, qbuf, act_group,
a16_kinds), `lfm2opt.quant` (quantize_int8) and `lfm2opt.kernels` (int8_ext, ext), backed by the prebuilt C-ABI
library liblfm2q.so. `lfm2opt.parallel` adds row sharding of large-M GEMMs and the N-split lm_head with an NCCL
all-gather.
"""

__version__ = "0.1.0"
