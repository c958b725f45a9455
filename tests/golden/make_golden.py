"""Generate the golden parity vectors in this directory from the reference's own code.

Run on a host that has the reference checkout (it is NOT needed at test time):

    python tests/golden/make_golden.py /path/to/ArtHIP

The script imports the reference suite's float64 NumPy references
(``tests/correctness/harness/reference.py``: ``ramp``/``logical_input``, ``conv3x3``,
``depth_to_space_dcr``) straight from the reference checkout and evaluates, for each
case the reference's ``test_engine.py`` checks, the value that suite asserts the engine
output against. Weights and biases are the fixture generator's
(``tests/correctness/harness/modelgen.py:124-129``: ``RandomState(seed).uniform(-0.5,
0.5)`` kernels, ``linspace`` biases, fp16-rounded), reproduced by
``arthip_b200.modelgen`` so the test side builds byte-identical ONNX fixtures.

Each case is stored as ``<case>.npz`` with the fixture name, the logical NCHW input,
and the reference's expected output (float32).
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from arthip_b200 import modelgen  # noqa: E402

# The reference's geometry sweep (test_engine.py:18-31) minus the two large bands,
# which are covered by size-independent properties in the GPU suite instead.
GEOMETRY = [(8, 8), (8, 17), (8, 24), (8, 25), (17, 16), (17, 17), (33, 17), (16, 33), (33, 33), (64, 64)]


def _load_reference(ref_root: Path):
    path = ref_root / "tests" / "correctness" / "harness" / "reference.py"
    spec = importlib.util.spec_from_file_location("arthip_reference_py", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(argv):
    if not argv:
        print("usage: python tests/golden/make_golden.py <reference project root>")
        return 2
    ref_root = Path(argv[0])
    ref = _load_reference(ref_root)
    cases = {}

    def conv_case(case, fx_name, h, w):
        fx = modelgen.FIXTURES[fx_name]()
        x = ref.logical_input(fx.input_channels, h, w, in_fp32=False)
        bias = None if fx.bias is None else fx.bias.astype(np.float64)
        y = ref.conv3x3(x, fx.weights.astype(np.float64), bias)
        cases[case] = dict(fixture=fx_name, x=x, expected=y)
        return y

    for h, w in GEOMETRY:
        conv_case(f"direct_c1m8_{h}x{w}", "conv_c1m8", h, w)
        conv_case(f"winograd_c4m4_{h}x{w}", "conv_c4m4", h, w)
    for name in ("conv_c4m8", "conv_c4m64"):
        conv_case(f"{name}_16x16", name, 16, 16)
    # Tensor-core-width convs with the fused epilogues (ReLU / SiLU), two column strips.
    y = conv_case("wide_c64m64_relu_24x200", "wide_c64m64_relu", 24, 200)
    cases["wide_c64m64_relu_24x200"]["expected"] = np.maximum(y, 0.0)
    y = conv_case("wide_c64m64_silu_20x136", "wide_c64m64_silu", 20, 136)
    cases["wide_c64m64_silu_20x136"]["expected"] = y / (1.0 + np.exp(-y))
    conv_case("wide_c96m96_18x70", "wide_c96m96", 18, 70)
    conv_case("wide_c48m80_9x130", "wide_c48m80", 9, 130)

    # Identity conv (test_engine.py:109-119): output equals the fp16 input exactly.
    fx = modelgen.FIXTURES["identity_raw"]()
    x = ref.logical_input(1, 17, 8, in_fp32=False)
    cases["identity_17x8"] = dict(fixture="identity_raw", x=x, expected=x.copy())

    # DepthToSpace block sizes and DCR channel order (test_engine.py:146-179).
    for name in ("dts_b1", "dts_b2", "dts_b3", "dts_multi_b2", "dts_multi_b2_f16", "dts_multi_b3"):
        fx = modelgen.FIXTURES[name]()
        x = ref.logical_input(1, 16, 16, in_fp32=False)
        conv = ref.conv3x3(x, fx.weights.astype(np.float64), fx.bias.astype(np.float64))
        cases[f"{name}_16x16"] = dict(fixture=name, x=x, expected=ref.depth_to_space_dcr(conv, fx.blocksize))

    # Fusion declined for shared intermediates (test_engine.py:187-215).
    fx = modelgen.FIXTURES["silu_shared"]()
    x = ref.logical_input(4, 16, 16, in_fp32=False)
    raw = ref.conv3x3(x, fx.weights.astype(np.float64), fx.bias.astype(np.float64))
    cases["silu_shared_16x16"] = dict(fixture="silu_shared", x=x, expected=raw + raw / (1.0 + np.exp(-raw)))
    fx = modelgen.FIXTURES["add_shared_conv_out"]()
    a = ref.conv3x3(x, fx.weights.astype(np.float64), fx.bias.astype(np.float64))
    bb = ref.conv3x3(a, fx.weights.astype(np.float64), fx.bias.astype(np.float64))
    cases["add_shared_conv_out_16x16"] = dict(fixture="add_shared_conv_out", x=x, expected=bb * (a + bb))
    # Clip without bounds is a no-op (test_engine.py:229-238).
    fx = modelgen.FIXTURES["clip_no_bounds"]()
    cases["clip_no_bounds_16x16"] = dict(
        fixture="clip_no_bounds", x=x,
        expected=ref.conv3x3(x, fx.weights.astype(np.float64), fx.bias.astype(np.float64)))

    manifest = {}
    for case, d in cases.items():
        np.savez_compressed(HERE / f"{case}.npz", x=d["x"].astype(np.float32),
                            expected=d["expected"].astype(np.float32))
        manifest[case] = {"fixture": d["fixture"], "shape": list(d["expected"].shape)}
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(cases)} golden cases to {HERE}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
