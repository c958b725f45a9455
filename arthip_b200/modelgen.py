"""ONNX model generators: the BASELINE conv-chain configs and the engine test fixtures.

Two families, both written with :mod:`arthip_b200.onnx_proto` (no ``onnx`` package):

* **Conv-chain configs** (``conv_chain``): ArtCNN-style ReLU upscalers
  ``head conv -> N x [conv+ReLU, conv, add block input] -> add head output
  -> tail conv -> DepthToSpace(2, DCR)``. BASELINE config 0 is C4F32 (4 blocks,
  32 ch), config 2 R8F64, config 3 R16F96, config 4 R8F64 at 2160p. Weights are
  He-normal (std sqrt(2/(9*C_in))), the second conv of each block scaled by 0.1,
  biases N(0, 0.01) (0.01 is the standard deviation); all stored fp16.
  Seeds: weights from ``numpy.random.default_rng(seed + 1000)``, the input frame
  from ``numpy.random.default_rng(seed)`` (``synthetic_frame``).
* **Engine fixtures** (``FIXTURES``): the same small single-property models the
  reference suite generates (``tests/correctness/harness/modelgen.py:124-525``):
  weights ``RandomState(seed).uniform(-0.5, 0.5)`` and linspace biases.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable

import numpy as np

from . import onnx_proto as op

OPSET = 17


# ---------------------------------------------------------------------------
# Conv-chain
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class ChainSpec:
    name: str
    blocks: int
    features: int
    in_ch: int = 1
    out_ch: int = 1
    scale: int = 2


CONFIGS = {
    "C4F32": ChainSpec("C4F32", 4, 32),
    "R8F64": ChainSpec("R8F64", 8, 64),
    "R16F96": ChainSpec("R16F96", 16, 96),
}


@dataclass
class ChainModel:
    model: op.Model
    convs: list  # [(weight fp16 OIHW, bias fp16)] in graph order
    spec: ChainSpec


def _he(rng, m, c, scale=1.0):
    std = np.sqrt(2.0 / (9.0 * c)) * scale
    return (rng.standard_normal((m, c, 3, 3)) * std).astype(np.float16)


def conv_chain(spec: ChainSpec, seed: int) -> ChainModel:
    rng = np.random.default_rng(seed + 1000)
    f, b = spec.features, spec.blocks
    r = spec.scale
    nodes, inits, convs = [], [], []

    def conv(x, m, c, out, scale=1.0):
        w = _he(rng, m, c, scale)
        bias = (rng.standard_normal(m) * 0.01).astype(np.float16)
        wn, bn = f"{out}_w", f"{out}_b"
        inits.append(op.tensor_from_array(wn, w))
        inits.append(op.tensor_from_array(bn, bias))
        nodes.append(op.make_node("Conv", [x, wn, bn], [out], kernel_shape=[3, 3],
                                  pads=[1, 1, 1, 1], strides=[1, 1], dilations=[1, 1], group=1))
        convs.append((w, bias))
        return out

    h = conv("input", f, spec.in_ch, "head")
    x = h
    for i in range(b):
        a = conv(x, f, f, f"b{i}_a")
        nodes.append(op.make_node("Relu", [a], [f"b{i}_r"]))
        c2 = conv(f"b{i}_r", f, f, f"b{i}_b", scale=0.1)
        nodes.append(op.make_node("Add", [c2, x], [f"b{i}_s"]))
        x = f"b{i}_s"
    nodes.append(op.make_node("Add", [x, h], ["skip"]))
    t = conv("skip", spec.out_ch * r * r, f, "tail")
    nodes.append(op.make_node("DepthToSpace", [t], ["output"], blocksize=r, mode="DCR"))
    g = op.Graph(nodes=nodes,
                 inputs=[op.value_info("input", op.FLOAT16, [1, spec.in_ch, "H", "W"])],
                 outputs=[op.value_info("output", op.FLOAT16, [1, spec.out_ch, "2*H", "2*W"])],
                 initializers=inits, name=spec.name)
    return ChainModel(op.Model(graph=g, opset=OPSET), convs, spec)


def artcnn_silu(blocks: int = 8, features: int = 64, in_ch: int = 1, out_ch: int = 1, scale: int = 2,
                fp32_io: bool = False, seed: int = 0) -> ChainModel:
    """The topology of the shipped ArtCNN models (random weights of the same shapes):
    ``head conv -> N x [conv+SiLU, conv+SiLU, conv, add block input] -> conv -> add head
    output -> tail conv -> DepthToSpace(scale, DCR) (scale > 1) -> Clip(0, 1)``, with SiLU
    as Sigmoid + Mul, ``auto_pad = SAME_UPPER`` convs and Clip bounds as initializers.
    ``fp32_io`` wraps the fp16 graph in boundary Casts (fp32 input and output), as the
    fp32 chroma / dehalo models look after fp16 conversion with kept IO types."""
    rng = np.random.default_rng(seed + 2000)
    nodes, inits, convs = [], [], []
    f = features

    def conv(x, m, c, out, wscale=1.0):
        w = _he(rng, m, c, wscale)
        bias = (rng.standard_normal(m) * 0.01).astype(np.float16)
        inits.append(op.tensor_from_array(f"{out}_w", w))
        inits.append(op.tensor_from_array(f"{out}_b", bias))
        nodes.append(op.make_node("Conv", [x, f"{out}_w", f"{out}_b"], [out], kernel_shape=[3, 3],
                                  auto_pad="SAME_UPPER", strides=[1, 1], dilations=[1, 1], group=1))
        convs.append((w, bias))
        return out

    def silu(x, out):
        nodes.append(op.make_node("Sigmoid", [x], [f"{out}_sig"]))
        nodes.append(op.make_node("Mul", [x, f"{out}_sig"], [out]))
        return out

    src = "input"
    if fp32_io:
        nodes.append(op.make_node("Cast", ["input"], ["input_h"], to=op.FLOAT16))
        src = "input_h"
    h = conv(src, f, in_ch, "head")
    x = h
    for i in range(blocks):
        a = silu(conv(x, f, f, f"b{i}_a"), f"b{i}_as")
        b = silu(conv(a, f, f, f"b{i}_b"), f"b{i}_bs")
        c = conv(b, f, f, f"b{i}_c", wscale=0.1)
        nodes.append(op.make_node("Add", [c, x], [f"b{i}_s"]))
        x = f"b{i}_s"
    body = conv(x, f, f, "body")
    nodes.append(op.make_node("Add", [body, h], ["skip"]))
    t = conv("skip", out_ch * scale * scale, f, "tail")
    if scale > 1:
        nodes.append(op.make_node("DepthToSpace", [t], ["dts"], blocksize=scale, mode="DCR"))
        t = "dts"
    inits.append(op.tensor_from_array("clip_lo", np.array(0.0, dtype=np.float16)))
    inits.append(op.tensor_from_array("clip_hi", np.array(1.0, dtype=np.float16)))
    out = "clipped" if fp32_io else "output"
    nodes.append(op.make_node("Clip", [t, "clip_lo", "clip_hi"], [out]))
    if fp32_io:
        nodes.append(op.make_node("Cast", [out], ["output"], to=op.FLOAT))
    io = op.FLOAT if fp32_io else op.FLOAT16
    g = op.Graph(nodes=nodes,
                 inputs=[op.value_info("input", io, [1, in_ch, "H", "W"])],
                 outputs=[op.value_info("output", io, [1, out_ch, "H2", "W2"])],
                 initializers=inits, name=f"artcnn_silu_b{blocks}f{f}")
    spec = ChainSpec(f"SiLU-B{blocks}F{f}", blocks, f, in_ch, out_ch, scale)
    return ChainModel(op.Model(graph=g, opset=19), convs, spec)


def synthetic_frame(seed: int, c: int, h: int, w: int) -> np.ndarray:
    """Seeded U[0,1) frame, NCHW float16."""
    rng = np.random.default_rng(seed)
    return rng.random((1, c, h, w), dtype=np.float32).astype(np.float16)


def conv_chain_flops(spec: ChainSpec, h: int, w: int) -> tuple[float, float]:
    """Algorithmic direct-conv FLOPs and fused-design HBM bytes for one frame.

    FLOPs = sum over convs of 2*9*C_in*C_out*H*W. Bytes: each conv reads its input
    (+ residual and skip operands) and writes its output once (fp16), plus the weights.
    """
    f, p = spec.features, h * w
    fl = 0.0
    by = 0.0
    layers = [(spec.in_ch, f, 0)]
    for i in range(spec.blocks):
        layers.append((f, f, 0))
        layers.append((f, f, 1 if i < spec.blocks - 1 else 2))
    layers.append((f, spec.out_ch * spec.scale ** 2, 0))
    for c, m, adds in layers:
        fl += 2.0 * 9 * c * m * p
        by += 2.0 * p * (c + m + adds * m) + 2.0 * (9 * c * m + m)
    return fl, by


# ---------------------------------------------------------------------------
# Engine fixtures (mirror of the reference suite's tiny models)
# ---------------------------------------------------------------------------

@dataclass
class Fixture:
    name: str
    model: op.Model
    input_channels: int
    output_channels: int
    weights: np.ndarray | None = None
    bias: np.ndarray | None = None
    blocksize: int = 1
    fp32_io: bool = False
    extra: dict = field(default_factory=dict)


def kern(seed: int, m: int, c: int, k: int = 3) -> np.ndarray:
    return np.random.RandomState(seed).uniform(-0.5, 0.5, (m, c, k, k)).astype(np.float32)


def linspace(m: int, lo: float = -0.1, hi: float = 0.1) -> np.ndarray:
    return np.linspace(lo, hi, m).astype(np.float32)


def _vi(name, shape, dt=op.FLOAT16):
    return op.value_info(name, dt, shape)


def _model(nodes, in_name, in_shape, in_t, out_name, out_shape, out_t, inits):
    g = op.Graph(nodes=nodes, inputs=[_vi(in_name, in_shape, in_t)],
                 outputs=[_vi(out_name, out_shape, out_t)], initializers=inits, name="fixture")
    return op.Model(graph=g, opset=OPSET)


def _conv_node(x, w, b, out, *, kernel=3, pads=(1, 1, 1, 1)):
    ins = [x, w] + ([b] if b else [])
    return op.make_node("Conv", ins, [out], kernel_shape=[kernel, kernel], pads=list(pads),
                        strides=[1, 1], dilations=[1, 1], group=1)


def _half(name, a, **kw):
    return op.tensor_from_array(name, np.asarray(a, dtype=np.float16), **kw)


def _float(name, a):
    return op.tensor_from_array(name, np.asarray(a, dtype=np.float32))


FIXTURES: dict[str, Callable[[], Fixture]] = {}


def fixture(name):
    def deco(fn):
        FIXTURES[name] = fn
        return fn
    return deco


def _single_conv(name, *, m, c, seed, bias="full", kernel=3, pads=(1, 1, 1, 1), external=False):
    w = kern(seed, m, c, kernel)
    inits = [_half("w", w, external=external)]
    bias_name, b16 = None, None
    if bias != "none":
        blen = m if bias == "full" else int(bias)
        b = linspace(blen)
        inits.append(_half("b", b))
        bias_name = "b"
        if blen == m:
            b16 = b.astype(np.float16)
    node = _conv_node("x", "w", bias_name, "y", kernel=kernel, pads=pads)
    model = _model([node], "x", [1, c, "h", "w"], op.FLOAT16, "y", [1, m, "h", "w"], op.FLOAT16, inits)
    return Fixture(name, model, c, m, w.astype(np.float16), b16)


for _n, _m, _c, _s in [("conv_c4m4", 4, 4, 11), ("conv_c4m8", 8, 4, 12), ("conv_c4m64", 64, 4, 13),
                       ("conv_c1m8", 8, 1, 21)]:
    FIXTURES[_n] = (lambda n=_n, m=_m, c=_c, s=_s: _single_conv(n, m=m, c=c, seed=s))


@fixture("conv_m128")
def _conv_m128():
    return _single_conv("conv_m128", m=128, c=4, seed=51, bias="none")


@fixture("conv_m512")
def _conv_m512():
    """Beyond the engine's 256-output-channel limit."""
    return _single_conv("conv_m512", m=512, c=4, seed=52, bias="none")


@fixture("conv_1x1")
def _conv_1x1():
    return _single_conv("conv_1x1", m=4, c=4, seed=31, bias="none", kernel=1)


@fixture("conv_short_bias")
def _conv_short_bias():
    return _single_conv("conv_short_bias", m=4, c=4, seed=41, bias=2)


@fixture("conv_external")
def _conv_external():
    return _single_conv("conv_external", m=4, c=4, seed=95, bias="none", external=True)


@fixture("conv_pads_asym")
def _conv_pads_asym():
    return _single_conv("conv_pads_asym", m=4, c=4, seed=33, bias="none", pads=(1, 0, 1, 0))


def _identity(name, typed):
    ident = np.zeros((1, 1, 3, 3), dtype=np.float32)
    ident[0, 0, 1, 1] = 1.0
    init = _half("w", ident, typed_half=typed)
    model = _model([_conv_node("x", "w", None, "y")], "x", [1, 1, "h", "w"], op.FLOAT16,
                   "y", [1, 1, "h", "w"], op.FLOAT16, [init])
    return Fixture(name, model, 1, 1, ident.astype(np.float16))


FIXTURES["identity_raw"] = lambda: _identity("identity_raw", False)
FIXTURES["identity_typed_half"] = lambda: _identity("identity_typed_half", True)


@fixture("add_const")
def _add_const():
    w = kern(61, 4, 4)
    k = np.full((1, 1, 1, 1), 0.25, dtype=np.float32)
    nodes = [_conv_node("x", "w", None, "raw"), op.make_node("Add", ["raw", "k"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _float("k", k)])
    return Fixture("add_const", model, 4, 4, w.astype(np.float16))


@fixture("add_broadcast")
def _add_broadcast():
    w, w2 = kern(71, 4, 4), kern(72, 1, 4)
    nodes = [_conv_node("x", "w", None, "a"), _conv_node("x", "w2", None, "b"),
             op.make_node("Add", ["a", "b"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("w2", w2)])
    return Fixture("add_broadcast", model, 4, 4, w.astype(np.float16))


def _dts(name, blocksize):
    m = blocksize * blocksize
    w = kern(80 + blocksize, m, 1)
    b = linspace(m, -0.05, 0.05)
    nodes = [_conv_node("x", "w", "b", "raw"),
             op.make_node("DepthToSpace", ["raw"], ["sq"], blocksize=blocksize, mode="DCR"),
             op.make_node("Cast", ["sq"], ["y"], to=op.FLOAT)]
    model = _model(nodes, "x", [1, 1, "h", "w"], op.FLOAT16, "y", [1, 1, "h", "w"], op.FLOAT,
                   [_half("w", w), _half("b", b)])
    return Fixture(name, model, 1, 1, w.astype(np.float16), b.astype(np.float16), blocksize, True)


for _b in (1, 2, 3):
    FIXTURES[f"dts_b{_b}"] = (lambda b=_b: _dts(f"dts_b{b}", b))


def _dts_multi(name, *, blocksize, cout, fp32_out):
    m = cout * blocksize * blocksize
    w = kern(90 + blocksize * 10 + cout, m, 1)
    b = linspace(m, -0.05, 0.05)
    nodes = [_conv_node("x", "w", "b", "raw"),
             op.make_node("DepthToSpace", ["raw"], ["sq"], blocksize=blocksize, mode="DCR")]
    if fp32_out:
        nodes.append(op.make_node("Cast", ["sq"], ["y"], to=op.FLOAT))
        out_name, out_t = "y", op.FLOAT
    else:
        out_name, out_t = "sq", op.FLOAT16
    model = _model(nodes, "x", [1, 1, "h", "w"], op.FLOAT16, out_name, [1, cout, "h", "w"], out_t,
                   [_half("w", w), _half("b", b)])
    return Fixture(name, model, 1, cout, w.astype(np.float16), b.astype(np.float16), blocksize, fp32_out)


FIXTURES["dts_multi_b2"] = lambda: _dts_multi("dts_multi_b2", blocksize=2, cout=2, fp32_out=True)
FIXTURES["dts_multi_b2_f16"] = lambda: _dts_multi("dts_multi_b2_f16", blocksize=2, cout=2, fp32_out=False)
FIXTURES["dts_multi_b3"] = lambda: _dts_multi("dts_multi_b3", blocksize=3, cout=2, fp32_out=True)


@fixture("dts_crd")
def _dts_crd():
    """CRD mode: the engine supports DCR only and must refuse it."""
    w = kern(99, 4, 1)
    nodes = [_conv_node("x", "w", None, "raw"),
             op.make_node("DepthToSpace", ["raw"], ["y"], blocksize=2, mode="CRD")]
    model = _model(nodes, "x", [1, 1, "h", "w"], op.FLOAT16, "y", [1, 1, "h", "w"], op.FLOAT16,
                   [_half("w", w)])
    return Fixture("dts_crd", model, 1, 1, w.astype(np.float16))


@fixture("silu_shared")
def _silu_shared():
    w, b = kern(63, 4, 4), linspace(4)
    nodes = [_conv_node("x", "w", "b", "raw"), op.make_node("Sigmoid", ["raw"], ["sig"]),
             op.make_node("Mul", ["raw", "sig"], ["z"]), op.make_node("Add", ["raw", "z"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    return Fixture("silu_shared", model, 4, 4, w.astype(np.float16), b.astype(np.float16))


@fixture("relu_shared")
def _relu_shared():
    """raw = conv(x); y = raw + relu(raw): the Relu must not be fused into the conv."""
    w, b = kern(65, 4, 4), linspace(4)
    nodes = [_conv_node("x", "w", "b", "raw"), op.make_node("Relu", ["raw"], ["r"]),
             op.make_node("Add", ["raw", "r"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    return Fixture("relu_shared", model, 4, 4, w.astype(np.float16), b.astype(np.float16))


@fixture("add_shared_conv_out")
def _add_shared_conv_out():
    w = (kern(64, 4, 4) * 0.2).astype(np.float32)
    b = linspace(4)
    nodes = [_conv_node("x", "w", "b", "a"), _conv_node("a", "w", "b", "bb"),
             op.make_node("Add", ["a", "bb"], ["s"]), op.make_node("Mul", ["bb", "s"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    return Fixture("add_shared_conv_out", model, 4, 4, w.astype(np.float16), b.astype(np.float16))


@fixture("clip_no_bounds")
def _clip_no_bounds():
    w = kern(34, 4, 4)
    b = np.full((4,), 2.0, dtype=np.float32)
    nodes = [_conv_node("x", "w", "b", "raw"), op.make_node("Clip", ["raw"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    return Fixture("clip_no_bounds", model, 4, 4, w.astype(np.float16), b.astype(np.float16))


@fixture("clip_dynamic_bound")
def _clip_dynamic_bound():
    w = kern(35, 4, 4)
    nodes = [_conv_node("x", "w", None, "raw"), op.make_node("Clip", ["raw", "raw"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w", w)])
    return Fixture("clip_dynamic_bound", model, 4, 4, w.astype(np.float16))


@fixture("ep_two_inputs")
def _ep_two_inputs():
    g = op.Graph(nodes=[op.make_node("Add", ["x1", "x2"], ["y"])],
                 inputs=[_vi("x1", [1, 4, "h", "w"]), _vi("x2", [1, 4, "h", "w"])],
                 outputs=[_vi("y", [1, 4, "h", "w"])], initializers=[], name="fixture")
    return Fixture("ep_two_inputs", op.Model(graph=g, opset=OPSET), 4, 4)


@fixture("ep_two_convs_one_input")
def _ep_two_convs_one_input():
    w1, w2 = kern(81, 4, 4), kern(82, 4, 4)
    b1, b2 = linspace(4), linspace(4, -0.2, 0.2)
    nodes = [_conv_node("x", "w1", "b1", "ca"), _conv_node("x", "w2", "b2", "cb"),
             op.make_node("Add", ["ca", "cb"], ["y"])]
    model = _model(nodes, "x", [1, 4, "h", "w"], op.FLOAT16, "y", [1, 4, "h", "w"], op.FLOAT16,
                   [_half("w1", w1), _half("b1", b1), _half("w2", w2), _half("b2", b2)])
    return Fixture("ep_two_convs_one_input", model, 4, 4, w1.astype(np.float16), b1.astype(np.float16),
                   extra={"w2": w2.astype(np.float16), "b2": b2.astype(np.float16)})


@fixture("identity_fp32io")
def _identity_fp32io():
    ident = np.zeros((1, 1, 3, 3), dtype=np.float32)
    ident[0, 0, 1, 1] = 1.0
    nodes = [op.make_node("Cast", ["x"], ["xh"], to=op.FLOAT16), _conv_node("xh", "w", None, "raw"),
             op.make_node("Cast", ["raw"], ["y"], to=op.FLOAT)]
    model = _model(nodes, "x", [1, 1, "h", "w"], op.FLOAT, "y", [1, 1, "h", "w"], op.FLOAT,
                   [_half("w", ident)])
    return Fixture("identity_fp32io", model, 1, 1, ident.astype(np.float16), fp32_io=True)


@fixture("ep_conv_fp32io")
def _ep_conv_fp32io():
    w, b = kern(5, 1, 1), linspace(1)
    nodes = [op.make_node("Cast", ["x"], ["xh"], to=op.FLOAT16), _conv_node("xh", "w", "b", "raw"),
             op.make_node("Cast", ["raw"], ["y"], to=op.FLOAT)]
    model = _model(nodes, "x", [1, 1, "h", "w"], op.FLOAT, "y", [1, 1, "h", "w"], op.FLOAT,
                   [_half("w", w), _half("b", b)])
    return Fixture("ep_conv_fp32io", model, 1, 1, w.astype(np.float16), b.astype(np.float16), fp32_io=True)


def _single_conv_wide(name, *, m, c, seed, act=None):
    """A tensor-core-width conv (C and M multiples of 16) with an optional epilogue."""
    w = (kern(seed, m, c) * (1.0 / np.sqrt(c))).astype(np.float32)
    b = linspace(m)
    nodes = [_conv_node("x", "w", "b", "raw" if act else "y")]
    if act == "relu":
        nodes.append(op.make_node("Relu", ["raw"], ["y"]))
    elif act == "silu":
        nodes += [op.make_node("Sigmoid", ["raw"], ["sg"]), op.make_node("Mul", ["raw", "sg"], ["y"])]
    model = _model(nodes, "x", [1, c, "h", "w"], op.FLOAT16, "y", [1, m, "h", "w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    return Fixture(name, model, c, m, w.astype(np.float16), b.astype(np.float16))


for _c, _m in [(16, 16), (32, 32), (64, 64), (64, 32), (32, 64), (96, 96), (48, 80), (128, 128), (64, 256)]:
    FIXTURES[f"wide_c{_c}m{_m}"] = (lambda c=_c, m=_m: _single_conv_wide(f"wide_c{c}m{m}", m=m, c=c,
                                                                          seed=200 + c + m))
FIXTURES["wide_c64m64_relu"] = lambda: _single_conv_wide("wide_c64m64_relu", m=64, c=64, seed=300, act="relu")
FIXTURES["wide_c64m64_silu"] = lambda: _single_conv_wide("wide_c64m64_silu", m=64, c=64, seed=301, act="silu")


def write_fixture(name: str, out_dir: Path) -> tuple[Fixture, Path]:
    fx = FIXTURES[name]()
    out_dir.mkdir(parents=True, exist_ok=True)
    path = out_dir / f"{name}.onnx"
    op.save_model(fx.model, path)
    return fx, path
