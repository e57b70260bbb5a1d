"""Generate the golden vectors in tests/golden/ from the reference's own Python code, run on CPU in the build
container (the reference tree is not present on the GPU box; the vectors travel as committed .npz files).

What is executed from the reference (jainilbavishi24/LFM2.5-VL-Optimization, checked out read-only):
  * src/lfm2opt/quant.py            quantize_int4, dequantize_int4 (imported as a module)
  * src/lfm2opt/quant.py            quantize_int8 (imported as a module)
  * tests/test_int8_gemm.py         ref_quant, ref_quant_groups, bf16_ulps, test_quant_rows, test_quant_groups,
                                    test_i8, test_i8_grouped (function definitions taken from the file's AST)
  * tests/test_kernels.py           test_gemv (function definition from the AST; its shape list is swapped for
                                    small shapes so the CPU run stays quick); rms, test_add_rmsnorm, test_shortconv,
                                    test_qk_rope_kv, test_attention and the module's model constants (H, NQ, NKV, D,
                                    EPS), test_attention at a small cache (B = 1, 512 slots, position 300)
The test functions are executed with dev = "cpu" and with stand-ins for the CUDA extension calls; a `check`
stand-in captures the reference tensors the test computes (its locals), which become the golden outputs.

    python tests/golden/make_golden.py [--reference /path/to/reference]
"""

import argparse
import os
import ast
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def load_functions(path: Path, names, replace_lists=None):
    """Compile the named top-level functions of `path` (optionally with the first list literal of a function
    replaced) into a code object per function."""
    tree = ast.parse(path.read_text())
    out = {}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            if replace_lists and node.name in replace_lists:
                new = ast.parse(replace_lists[node.name], mode="eval").body

                class Swap(ast.NodeTransformer):
                    done = False

                    def visit_List(self, n):
                        if not Swap.done:
                            Swap.done = True
                            return ast.copy_location(new, n)
                        return n

                node = Swap().visit(node)
                ast.fix_missing_locations(node)
            out[node.name] = ast.Module(body=[node], type_ignores=[])
    missing = set(names) - set(out)
    if missing:
        raise RuntimeError(f"functions {missing} not found in {path}")
    return out


def load_assign(path: Path, name):
    """The top-level assignment statement of `path` that binds `name` (e.g. a tuple of model constants)."""
    tree = ast.parse(path.read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign):
            for t in node.targets:
                names = [e.id for e in t.elts] if isinstance(t, ast.Tuple) else [getattr(t, "id", None)]
                if name in names:
                    return ast.Module(body=[node], type_ignores=[])
    raise RuntimeError(f"no assignment of {name} in {path}")


def run_in(ns, mod):
    exec(compile(mod, "<reference>", "exec"), ns)


class Capture:
    """Stand-in for the reference's `check`/`report`: keeps the caller's local tensors."""

    def __init__(self):
        self.cases = []

    def __call__(self, *args, **kwargs):
        frame = sys._getframe(1)
        case = {k: v.clone() if isinstance(v, torch.Tensor) else v for k, v in frame.f_locals.items()}
        case["_args"] = tuple(v.clone() if isinstance(v, torch.Tensor) else v for v in args)
        self.cases.append(case)


class Stub:
    """Stand-in for a CUDA extension object: every op is a no-op (the reference values come from the test's own
    torch expressions, not from the kernel)."""

    def __getattr__(self, name):
        return lambda *a, **k: None


def t2np(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().copy()
    return t.numpy().copy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LFM2_REFERENCE"),
                    help="the reference project's source tree (or set LFM2_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("name the reference's source tree with --reference or LFM2_REFERENCE")
    ref = Path(a.reference)
    sys.path.insert(0, str(ref / "src"))
    import lfm2opt.quant as rq  # the reference's own module

    # ---------------------------------------------------------------- weight quantizer (imported)
    out = {}
    g = torch.Generator().manual_seed(0)
    for i, (N, K) in enumerate([(8, 64), (64, 128), (33, 2048), (16, 1152)]):
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        if i == 2:
            w[3] = 0  # an all-zero row: scale clamps to 1e-12
            w[5, 7] = 0.5  # an outlier
        q, s = rq.quantize_int8(w)
        out[f"w{i}"], out[f"q{i}"], out[f"s{i}"] = t2np(w), t2np(q), t2np(s)
    np.savez_compressed(HERE / "quantize_int8.npz", **out)

    # ---------------------------------------------------------------- INT4 weight quantizer (imported)
    out4 = {}
    g = torch.Generator().manual_seed(4)
    cases4 = [(8, 256, 128, False), (33, 1024, 128, True), (16, 2048, 256, False), (5, 512, 128, True)]
    for i, (N, K, group, clip) in enumerate(cases4):
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        if i == 1:
            w[2, :128] = 0  # an all-zero group: its scale clamps to 1e-12 / 7
            w[4, 9] = 0.4  # an outlier in one group
        p4, s4 = rq.quantize_int4(w, group, clip_search=clip)
        out4[f"w{i}"], out4[f"p{i}"], out4[f"s{i}"] = t2np(w), t2np(p4), t2np(s4)
        out4[f"d{i}"] = t2np(rq.dequantize_int4(p4, s4))
        out4[f"meta{i}"] = np.array([N, K, group, int(clip)])
    np.savez_compressed(HERE / "quantize_int4.npz", **out4)

    # ---------------------------------------------------------------- activation quantizers + W8A8 (test functions)
    tests = load_functions(ref / "tests/test_int8_gemm.py",
                           ["ref_quant", "ref_quant_groups", "bf16_ulps", "test_quant_rows", "test_quant_groups",
                            "test_i8", "test_i8_grouped"])
    cap = Capture()
    ns = {"torch": torch, "F": F, "dev": "cpu", "bf": torch.bfloat16, "E": Stub(), "check": cap,
          "quantize_int8": rq.quantize_int8}
    for name, mod in tests.items():
        run_in(ns, mod)
    ns["quantize_rows"] = lambda x, group=0: ns["ref_quant_groups"](x) if group else ns["ref_quant"](x)

    torch.manual_seed(0)
    qr = {}
    for i, (M, K) in enumerate([(1, 2048), (37, 1152), (5, 128)]):
        ns["test_quant_rows"](M, K)
        c = cap.cases[-1]
        qr[f"x{i}"], qr[f"q{i}"], qr[f"s{i}"] = t2np(c["x"]), t2np(c["rq"]), t2np(c["rs"])
    for i, (M, K) in enumerate([(1, 2048), (37, 1152), (3, 256)]):
        ns["test_quant_groups"](M, K)
        c = cap.cases[-1]
        qr[f"gx{i}"], qr[f"gq{i}"], qr[f"gs{i}"] = t2np(c["x"]), t2np(c["rq"]), t2np(c["rs"])
    np.savez_compressed(HERE / "quant_rows.npz", **qr)

    torch.manual_seed(1)
    gm = {}
    cases = [(17, 256, 64, False, False), (9, 1152, 128, True, False), (33, 512, 96, True, True),
             (1, 2048, 64, False, False)]
    for i, (M, K, N, bias, gelu) in enumerate(cases):
        ns["test_i8"](M, K, N, bias, gelu)
        c = cap.cases[-1]
        gm[f"xq{i}"], gm[f"sx{i}"], gm[f"wq{i}"], gm[f"sw{i}"] = (t2np(c["xq"]), t2np(c["sx"]), t2np(c["wq"]),
                                                                 t2np(c["sw"]))
        gm[f"b{i}"] = t2np(c["b"]) if c["b"] is not None else np.zeros(0, np.int16)
        gm[f"y{i}"] = t2np(c["r"])
        gm[f"meta{i}"] = np.array([M, K, N, int(bias), int(gelu)])
    np.savez_compressed(HERE / "gemm_i8.npz", **gm)

    torch.manual_seed(2)
    gg = {}
    cases = [(17, 256, 64, False, False), (9, 1152, 128, True, False), (5, 512, 64, True, True)]
    for i, (M, K, N, bias, gelu) in enumerate(cases):
        ns["test_i8_grouped"](M, K, N, bias, gelu)
        c = cap.cases[-1]
        gg[f"xq{i}"], gg[f"sx{i}"], gg[f"wq{i}"], gg[f"sw{i}"] = (t2np(c["xq"]), t2np(c["sxT"]), t2np(c["wq"]),
                                                                 t2np(c["sw"]))
        gg[f"b{i}"] = t2np(c["b"]) if c["b"] is not None else np.zeros(0, np.int16)
        gg[f"r{i}"] = t2np(c["r"])  # the fp64 reference the test compares against
        gg[f"meta{i}"] = np.array([M, K, N, int(bias), int(gelu)])
    np.savez_compressed(HERE / "gemm_i8_grouped.npz", **gg)

    # ---------------------------------------------------------------- decode GEMV (test_kernels.test_gemv)
    tk = load_functions(ref / "tests/test_kernels.py", ["test_gemv"],
                        replace_lists={"test_gemv": "[(64, 512), (40, 1024)]"})
    cap2 = Capture()
    ns2 = {"torch": torch, "F": F, "dev": "cpu", "bf": torch.bfloat16, "K": Stub(), "report": cap2}
    run_in(ns2, tk["test_gemv"])
    torch.manual_seed(3)
    ns2["test_gemv"]()
    gv, g4 = {}, {}
    n = n4 = 0
    for c in cap2.cases:
        name, _, ref_y = c["_args"]
        if "int4" in name:  # the reference's expression: F.linear(x.float(), dequantize_int4(Wp, S4)).to(bf16)
            g4[f"name{n4}"] = np.array(name)
            g4[f"p{n4}"], g4[f"s{n4}"], g4[f"x{n4}"], g4[f"y{n4}"] = (t2np(c["Wp"]), t2np(c["S4"]), t2np(c["x"]),
                                                                      t2np(ref_y))
            n4 += 1
            continue
        batched = "B=" in name
        xin = c["xb"] if batched else c["x"]
        if "int8" in name:
            W, sc = c["Wq"], c["scale"]
        else:
            W, sc = c["W"], None
        gv[f"name{n}"] = np.array(name)
        gv[f"W{n}"], gv[f"x{n}"], gv[f"y{n}"] = t2np(W), t2np(xin), t2np(ref_y)
        gv[f"s{n}"] = t2np(sc) if sc is not None else np.zeros(0, np.float32)
        n += 1
    np.savez_compressed(HERE / "gemv.npz", **gv)
    np.savez_compressed(HERE / "gemv_w4.npz", **g4)

    # ---------------------------------------------------------------- decode-step kernels and attention
    kpath = ref / "tests/test_kernels.py"
    tk3 = load_functions(kpath, ["rms", "test_add_rmsnorm", "test_shortconv", "test_qk_rope_kv", "test_attention"])
    cap3 = Capture()
    ns3 = {"torch": torch, "F": F, "dev": "cpu", "bf": torch.bfloat16, "K": Stub(), "report": cap3}
    run_in(ns3, load_assign(kpath, "EPS"))  # H, I, NQ, NKV, D, EPS as the reference's test defines them
    for name in ("rms", "test_add_rmsnorm", "test_shortconv", "test_qk_rope_kv", "test_attention"):
        run_in(ns3, tk3[name])
    dk = {}
    torch.manual_seed(5)
    ns3["test_add_rmsnorm"]()
    c_res, c_norm, c_noadd = cap3.cases[-3:]
    dk["norm_h"], dk["norm_y"], dk["norm_w"] = t2np(c_res["h"]), t2np(c_res["y"]), t2np(c_res["w"])
    dk["norm_ref_h"], dk["norm_ref_x"] = t2np(c_res["ref_h"]), t2np(c_norm["ref_x"])
    dk["norm_ref_x_noadd"] = t2np(c_noadd["_args"][2])
    torch.manual_seed(6)
    ns3["test_shortconv"]()
    c_out, c_state = cap3.cases[-2:]
    dk["conv_bcx"], dk["conv_state"], dk["conv_w"] = t2np(c_out["bcx"]), t2np(c_out["state"]), t2np(c_out["w"])
    dk["conv_ref_y"], dk["conv_ref_state"] = t2np(c_out["ref"]), t2np(c_state["st"])
    torch.manual_seed(7)
    ns3["test_qk_rope_kv"]()
    c_q, c_k, c_v = cap3.cases[-4:-1]
    dk["qk_qkv"], dk["qk_qw"], dk["qk_kw"] = t2np(c_q["qkv"]), t2np(c_q["qw"]), t2np(c_q["kw"])
    dk["qk_inv_freq"], dk["qk_meta"] = t2np(c_q["inv_freq"]), np.array([c_q["B"], c_q["max_len"], c_q["pos"]])
    dk["qk_ref_q"], dk["qk_ref_k"], dk["qk_ref_v"] = (t2np(c_q["_args"][2]), t2np(c_k["_args"][2]),
                                                      t2np(c_v["_args"][2]))
    np.savez_compressed(HERE / "decode_kernels.npz", **dk)
    at = {}
    torch.manual_seed(8)
    ns3["test_attention"](B=1, max_len=512, pos=300)
    c_full, c_one = cap3.cases[-5], cap3.cases[-2]
    at["q"], at["kc"], at["vc"] = t2np(c_full["q"]), t2np(c_full["kc"]), t2np(c_full["vc"])
    at["scale"], at["meta"] = np.array(c_full["scale"], np.float64), np.array([1, 512, 300])
    at["ref"], at["ref_len1"] = t2np(c_full["ref"]), t2np(c_one["_args"][2])
    np.savez_compressed(HERE / "attention.npz", **at)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
