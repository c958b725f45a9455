"""CPU restatement of ONNX Runtime's execution of an fp16 conv-chain graph (test oracle).

Test infrastructure only (see the package docstring). Each node follows the ONNX
operator definition; the reference file each piece follows is cited inline.
"""

from __future__ import annotations

import math

import numpy as np

from arthip_b200 import onnx_proto as op

try:  # torch is only used for the fast fp32 path on large frames
    import torch
    import torch.nn.functional as F
except Exception:  # pragma: no cover - torch is present in this image
    torch = None

RAMP_MODULUS = 251
RAMP_MULT = 37
RAMP_ADD = 11


def ramp(numel: int) -> np.ndarray:
    """Deterministic dense [0,1) ramp ``((i*37+11) mod 251)/251`` used by the reference
    suite's inputs (``tests/correctness/harness/reference.py:16-31``)."""
    i = np.arange(numel, dtype=np.int64)
    return (((i * RAMP_MULT) + RAMP_ADD) % RAMP_MODULUS).astype(np.float32) / np.float32(RAMP_MODULUS)


def logical_ramp_input(c: int, h: int, w: int, in_fp32: bool = False) -> np.ndarray:
    """The ramp as a logical NCHW float64 tensor, fp16-rounded for fp16-input models
    (``reference.py:44-54``)."""
    flat = ramp(c * h * w).reshape(1, c, h, w)
    if in_fp32:
        return flat.astype(np.float64)
    return flat.astype(np.float16).astype(np.float64)


# ---------------------------------------------------------------------------
# Node kernels
# ---------------------------------------------------------------------------

def conv3x3_nchw(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None = None,
                 pads=(1, 1, 1, 1)) -> np.ndarray:
    """Float64 direct convolution, stride 1, dilation 1, group 1.

    ``pads`` is ONNX order [top, left, bottom, right]. Computed as a sum of shifted
    views (one GEMM per tap) so it is independent of the torch path below and of the
    reference's loop form (``reference.py:67-81``)."""
    m, c, kh, kw = weight.shape
    n, cx, h, w = x.shape
    assert cx == c, f"channel mismatch {cx} vs {c}"
    top, left, bottom, right = pads
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (top, bottom), (left, right)))
    oh = h + top + bottom - kh + 1
    ow = w + left + right - kw + 1
    out = np.zeros((n, m, oh, ow), dtype=np.float64)
    wt = weight.astype(np.float64)
    for ky in range(kh):
        for kx in range(kw):
            view = xp[:, :, ky:ky + oh, kx:kx + ow]          # n, c, oh, ow
            out += np.einsum("mc,nchw->nmhw", wt[:, :, ky, kx], view, optimize=True)
    if bias is not None:
        out += bias.astype(np.float64).reshape(1, m, 1, 1)
    return out


def depth_to_space(x: np.ndarray, b: int, mode: str = "DCR") -> np.ndarray:
    """ONNX DepthToSpace. DCR: input channel (r*b + q)*Cout + c feeds output
    (c, h*b + r, w*b + q); CRD: c*b*b + r*b + q (``hip_kernels.h:521-551``,
    ``reference.py:84-93``)."""
    n, c, h, w = x.shape
    assert c % (b * b) == 0
    co = c // (b * b)
    if mode == "DCR":
        t = x.reshape(n, b, b, co, h, w).transpose(0, 3, 4, 1, 5, 2)
    else:
        t = x.reshape(n, co, b, b, h, w).transpose(0, 1, 4, 2, 5, 3)
    return t.reshape(n, co, h * b, w * b)


def psnr(got: np.ndarray, ref: np.ndarray, peak: float = 1.0) -> float:
    mse = float(np.mean((got.astype(np.float64) - ref.astype(np.float64)) ** 2))
    if mse == 0.0:
        return float("inf")
    return 10.0 * math.log10(peak * peak / mse)


# ---------------------------------------------------------------------------
# Graph executor
# ---------------------------------------------------------------------------

def _conv_pads(node: op.Node, kh: int, kw: int):
    pads = node.attr("pads")
    auto_pad = node.attr("auto_pad", "NOTSET")
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        # stride 1: total pad = k-1, the extra one goes to the end (UPPER) or begin (LOWER)
        th, tw = kh - 1, kw - 1
        if auto_pad == "SAME_UPPER":
            return (th // 2, tw // 2, th - th // 2, tw - tw // 2)
        return (th - th // 2, tw - tw // 2, th // 2, tw // 2)
    if pads:
        return tuple(int(p) for p in pads)
    return (0, 0, 0, 0)


class _Exec:
    def __init__(self, mode: str, use_torch: bool, device: str = "cpu", reverse_channels: bool = False):
        assert mode in ("fp16_nodes", "fp32_nodes", "float64")
        self.mode = mode
        self.use_torch = use_torch and torch is not None and mode != "float64"
        self.device = device
        # Same arithmetic, different fp32 summation order: measures how far two equally
        # valid fp16-per-node executions drift apart through a deep chain.
        self.reverse_channels = reverse_channels
        if self.use_torch and device != "cpu":
            # a reference must not silently drop to TF32 inside cuDNN
            torch.backends.cudnn.allow_tf32 = False
            torch.backends.cuda.matmul.allow_tf32 = False

    # values are float64 numpy arrays (float64 mode) or float32 torch tensors
    def node_out(self, v, dtype):
        if self.mode == "fp16_nodes" and dtype == op.FLOAT16:
            return self.round16(v)
        return v

    def round16(self, v):
        if self.use_torch:
            return v.to(torch.float16).to(torch.float32)
        return v.astype(np.float16).astype(v.dtype)

    def const(self, arr: np.ndarray):
        if self.use_torch:
            return torch.from_numpy(np.ascontiguousarray(arr.astype(np.float32))).to(self.device)
        return arr.astype(np.float64 if self.mode == "float64" else np.float32)

    def conv(self, x, w, b, pads):
        if self.use_torch:
            top, left, bottom, right = pads
            xp = F.pad(x, (left, right, top, bottom))
            if self.reverse_channels:
                return F.conv2d(xp.flip(1), w.flip(1), b)
            return F.conv2d(xp, w, b)
        if self.mode == "float64":
            return conv3x3_nchw(x, w, b, pads)
        return conv3x3_nchw(x, w, b, pads).astype(np.float32)

    def to_numpy(self, v):
        if self.use_torch:
            return v.cpu().numpy().astype(np.float64)
        return np.asarray(v, dtype=np.float64)


def run_model(model: op.Model, x_nchw: np.ndarray, *, mode: str = "fp16_nodes",
              use_torch: bool = True, convert_fp32_weights_to_fp16: bool = False,
              threads: int | None = None, device: str = "cpu", reverse_channels: bool = False) -> np.ndarray:
    """Execute ``model`` on one NCHW input and return the graph output as float64.

    ``convert_fp32_weights_to_fp16`` reproduces the fp16 conversion the engine applies
    to fp32 initializers (IEEE round-to-nearest-even, ``hip_engine.cc:1190-1232``), so
    an fp32-weight model can be compared with the fp16 engine on equal weights."""
    g = model.graph
    ex = _Exec(mode, use_torch, device, reverse_channels)
    if threads is not None and ex.use_torch:
        torch.set_num_threads(int(threads))
    inits = {t.name: t.to_numpy() for t in g.initializers}
    dtypes: dict[str, int] = {}
    env = {}
    gin = g.inputs[0]
    x = np.asarray(x_nchw, dtype=np.float64)
    if gin.elem_type == op.FLOAT16:
        x = x.astype(np.float16).astype(np.float64)
    env[gin.name] = ex.const(x) if ex.use_torch else (x if mode == "float64" else x.astype(np.float32))
    dtypes[gin.name] = gin.elem_type

    def weight(name):
        arr = inits[name]
        if convert_fp32_weights_to_fp16 and arr.dtype == np.float32:
            arr = arr.astype(np.float16)
        return arr

    def val(name):
        if name in env:
            return env[name]
        if name in inits:
            return ex.const(weight(name).astype(np.float64))
        raise KeyError(f"tensor '{name}' not computed")

    def dt(name):
        if name in dtypes:
            return dtypes[name]
        if name in inits:
            a = inits[name]
            return op.FLOAT16 if a.dtype == np.float16 else op.FLOAT
        return op.FLOAT

    for n in g.nodes:
        t = n.op_type
        if t == "Conv":
            w = weight(n.inputs[1])
            b = weight(n.inputs[2]) if len(n.inputs) > 2 and n.inputs[2] else None
            pads = _conv_pads(n, w.shape[2], w.shape[3])
            assert all(s == 1 for s in (n.attr("strides") or [1, 1]))
            assert all(d == 1 for d in (n.attr("dilations") or [1, 1]))
            assert (n.attr("group") or 1) == 1
            y = ex.conv(val(n.inputs[0]), ex.const(w.astype(np.float64)),
                        None if b is None else ex.const(b.astype(np.float64)), pads)
            odt = dt(n.inputs[0])
        elif t == "Relu":
            v = val(n.inputs[0])
            y = torch.clamp_min(v, 0.0) if ex.use_torch else np.maximum(v, 0.0)
            odt = dt(n.inputs[0])
        elif t == "Sigmoid":
            v = val(n.inputs[0])
            y = torch.sigmoid(v) if ex.use_torch else 1.0 / (1.0 + np.exp(-v))
            odt = dt(n.inputs[0])
        elif t in ("Add", "Mul"):
            a, b2 = val(n.inputs[0]), val(n.inputs[1])
            y = a + b2 if t == "Add" else a * b2
            odt = dt(n.inputs[0])
        elif t == "Clip":
            v = val(n.inputs[0])
            lo = n.attr("min", None)
            hi = n.attr("max", None)
            if len(n.inputs) > 1 and n.inputs[1]:
                lo = float(np.asarray(inits[n.inputs[1]], dtype=np.float64).reshape(-1)[0])
            if len(n.inputs) > 2 and n.inputs[2]:
                hi = float(np.asarray(inits[n.inputs[2]], dtype=np.float64).reshape(-1)[0])
            y = v
            if ex.use_torch:
                if lo is not None:
                    y = torch.clamp_min(y, lo)
                if hi is not None:
                    y = torch.clamp_max(y, hi)
            else:
                if lo is not None:
                    y = np.maximum(y, lo)
                if hi is not None:
                    y = np.minimum(y, hi)
            odt = dt(n.inputs[0])
        elif t == "DepthToSpace":
            b = int(n.attr("blocksize"))
            mode_ = n.attr("mode", "DCR")
            v = val(n.inputs[0])
            if ex.use_torch:
                y = torch.from_numpy(depth_to_space(v.cpu().numpy(), b, mode_).copy()).to(ex.device)
            else:
                y = depth_to_space(v, b, mode_)
            odt = dt(n.inputs[0])
        elif t == "Cast":
            v = val(n.inputs[0])
            to = int(n.attr("to"))
            y = ex.round16(v) if to == op.FLOAT16 else v
            odt = to
        else:
            raise NotImplementedError(f"oracle: op {t}")
        env[n.outputs[0]] = ex.node_out(y, odt)
        dtypes[n.outputs[0]] = odt

    out_name = g.outputs[0].name
    out = env[out_name]
    if g.outputs[0].elem_type == op.FLOAT16:
        out = ex.round16(out)
    return ex.to_numpy(out)


def conv_layer_nhwc(x_nhwc: np.ndarray, w_oihw: np.ndarray, bias: np.ndarray | None,
                    relu: bool, threads: int | None = None) -> np.ndarray:
    """One fp16 3x3 conv + bias (+ReLU) on an NHWC frame, fp32 compute, fp16-rounded
    output (the single-layer microbench). Returns float32 NHWC."""
    assert torch is not None
    if threads is not None:
        torch.set_num_threads(int(threads))
    x = torch.from_numpy(np.ascontiguousarray(x_nhwc.astype(np.float32))).permute(0, 3, 1, 2)
    w = torch.from_numpy(w_oihw.astype(np.float32))
    b = None if bias is None else torch.from_numpy(bias.astype(np.float32))
    y = F.conv2d(x, w, b, padding=1)
    y = y.to(torch.float16).to(torch.float32)
    if relu:
        y = torch.clamp_min(y, 0.0)
    return y.permute(0, 2, 3, 1).contiguous().numpy()
