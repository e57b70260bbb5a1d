"""The device quantizers' fast int8 rounding (lfm2.5-vl-optimization_b200/csrc/common.cuh, q8r), emulated in
IEEE fp32 with numpy: it must return rint(v / sc) of the IEEE quotient (ties to even), clamped to +-127, for every
v with |v| <= amax, sc = max(amax, 1e-8) / 127 — the reference quantizer (kernels/int8_gemm.cu:419-430)."""

import numpy as np

F = np.float32
BIG = F(12582912.0)  # 1.5 * 2^23
MARGIN = F(0.5) - F(4e-5)


def q8r(v, sc):
    rinv = (F(1) / sc).astype(F)
    t = (v * rinv).astype(F)
    tb = (t + BIG).astype(F)
    k = (tb - BIG).astype(F)
    near = np.abs((t - k).astype(F)) > MARGIN
    exact = np.rint((v / sc).astype(F)).astype(F)
    tb = np.where(near, (exact + BIG).astype(F), tb)
    qi = tb.view(np.int32) - np.int32(0x4B400000)
    return np.clip(qi, -127, 127), near


def ref(v, sc):
    return np.clip(np.rint((v / sc).astype(F)), -127, 127).astype(np.int32)


def test_random_rows():
    rng = np.random.default_rng(0)
    for _ in range(20):
        amax = F(10.0 ** rng.uniform(-9, 4))
        v = (rng.uniform(-1, 1, 200_000) * amax).astype(F)
        v[0] = amax
        v[1] = -amax
        sc = (np.maximum(np.abs(v).max(), F(1e-8)) / F(127)).astype(F)
        q, near = q8r(v, sc)
        assert np.array_equal(q, ref(v, sc))
        assert near.mean() < 1e-3


def test_adversarial_half_integers():
    # values whose exact quotient sits on or next to k + 0.5 (the rounding boundary), over many scales
    rng = np.random.default_rng(1)
    for _ in range(200):
        amax = F(10.0 ** rng.uniform(-6, 3))
        sc = (amax / F(127)).astype(F)
        k = rng.integers(-127, 127, 4000).astype(F) + F(0.5)
        v = (k * sc).astype(F)
        ulp = np.spacing(np.abs(v)).astype(F)
        for d in (-3, -2, -1, 0, 1, 2, 3):
            vv = (v + F(d) * ulp).astype(F)
            vv = np.clip(vv, -amax, amax).astype(F)
            q, _ = q8r(vv, sc)
            assert np.array_equal(q, ref(vv, sc))


def test_bf16_inputs_exhaustive_scales():
    # every bf16 value in [-amax, amax] for a spread of row maxima (activations are bf16)
    allbits = np.arange(0, 1 << 16, dtype=np.uint32)
    vals = (allbits << 16).view(np.float32)
    vals = vals[np.isfinite(vals)]
    rng = np.random.default_rng(2)
    for amax in list((10.0 ** rng.uniform(-8, 4, 40)).astype(F)) + [F(1e-8), F(37.0), F(127.0)]:
        v = vals[np.abs(vals) <= amax]
        sc = (np.maximum(amax, F(1e-8)) / F(127)).astype(F)
        q, _ = q8r(v, sc)
        assert np.array_equal(q, ref(v, sc)), amax
