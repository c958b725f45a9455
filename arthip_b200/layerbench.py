"""Single conv layer benchmark (the 64->64 + bias + ReLU microbench on a 1080x1920 NHWC frame
by default), through the ``ah_conv3x3_*`` C ABI.

    python -m arthip_b200.layerbench [--C 64 --M 64 --H 1080 --W 1920 --act 1 --adds 0]
                                     [--warmup 3 --iters 20] [--algo direct|winograd]

Prints one JSON line: mean launch time from CUDA events around `iters` back-to-back
launches on the current stream, the algorithmic direct-conv FLOPs (2*9*C*M*H*W) and bytes
(input + residual inputs + weights read once, output written once) per launch, and their
rates against the measured B200 peaks (MEASURED_PEAKS.json beside the repository root when
present, else the pool's earlier figures). At the default size every tensor (265 MB) is
larger than the 126 MB L2, so consecutive launches do not hit in L2.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _peaks():
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"])}, "measured"
        except Exception:
            pass
    return dict(_FALLBACK), "fallback"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--C", type=int, default=64)
    ap.add_argument("--M", type=int, default=64)
    ap.add_argument("--H", type=int, default=1080)
    ap.add_argument("--W", type=int, default=1920)
    ap.add_argument("--act", type=int, default=1, help="0 none, 1 ReLU, 2 SiLU")
    ap.add_argument("--adds", type=int, default=0, choices=[0, 1, 2])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--in-place", action="store_true",
                    help="write over the last residual operand (reduce-add stores); the "
                         "operand then accumulates across launches, which does not change the timing")
    ap.add_argument("--algo", default="direct", choices=["direct", "winograd", "pair"],
                    help="conv kernel: the direct implicit GEMM, Winograd F(2x2,3x3), or the direct conv on "
                         "two SMs per MMA (the last two 64 -> 64 only)")
    ap.add_argument("--model", choices=["C4F32", "R8F64", "R16F96"],
                    help="time whole frames of this BASELINE chain (luma, 2x) at --H x --W through the "
                         "engine's CUDA graph instead of one layer (a small-frame case for profilers)")
    args = ap.parse_args(argv)
    if args.model:
        return _model_frames(args)

    import torch

    from arthip_b200.engine import Conv3x3

    dev = torch.device("cuda:0")
    C, M, H, W = args.C, args.M, args.H, args.W
    g = torch.Generator(device="cpu").manual_seed(args.seed)
    x = torch.rand(1, H, W, C, generator=g).half().to(dev)
    adds = [torch.rand(1, H, W, M, generator=g).half().to(dev) for _ in range(args.adds)]
    out = torch.empty(1, H, W, M, dtype=torch.float16, device=dev)
    rng = np.random.default_rng(args.seed)
    w = (rng.standard_normal((M, C, 3, 3)) * (2.0 / (9 * C)) ** 0.5).astype(np.float16)
    b = (rng.standard_normal(M) * 0.01).astype(np.float16).astype(np.float32)
    conv = Conv3x3(w, b, act=args.act, algo=args.algo)
    s = torch.cuda.current_stream().cuda_stream
    ptrs = [a.data_ptr() for a in adds]
    if args.in_place:
        if not adds:
            ap.error("--in-place needs --adds 1 or 2")
        out = adds[-1]

    def launch():
        conv.run(x.data_ptr(), H, W, out.data_ptr(), *ptrs, stream=s)

    for _ in range(max(1, args.warmup)):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        launch()
    e1.record()
    torch.cuda.synchronize()
    status = conv.status()
    ms = e0.elapsed_time(e1) / args.iters
    flops = 2.0 * 9 * C * M * H * W
    nbytes = 2.0 * H * W * (C + M * (1 + args.adds)) + 2.0 * 9 * C * M + 4.0 * M
    peaks, src = _peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    gbs = nbytes / (ms * 1e-3) / 1e9
    roof_ms = max(flops / (peaks["bf16_tflops"] * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9)) * 1e3
    print(json.dumps({
        "layer": f"conv3x3 {C}->{M} act{args.act} adds{args.adds}{' in place' if args.in_place else ''} {H}x{W}", "kernel": conv.kind,
        "us_per_launch": ms * 1e3, "tflops": tflops, "gbs": gbs, "algorithmic_flops": flops,
        "algorithmic_bytes": nbytes, "roofline_us": roof_ms * 1e3, "roofline_frac": roof_ms / ms,
        "tflops_frac": tflops / peaks["bf16_tflops"], "peaks": src, "iters": args.iters, "status": status,
    }))
    conv.close()
    return 0 if status == 0 else 1


def _model_frames(args) -> int:
    import tempfile
    import time

    import torch

    from arthip_b200 import modelgen, onnx_proto as op
    from arthip_b200.engine import Engine

    H, W = args.H, args.W
    with tempfile.TemporaryDirectory() as td:
        cm = modelgen.conv_chain(modelgen.CONFIGS[args.model], seed=args.seed)
        path = Path(td) / f"{args.model}.onnx"
        op.save_model(cm.model, path)
        eng = Engine(path)
        eng.set_conv_algo(args.algo)
        in_ptr, _, in_bytes, _ = eng.prepare(1, H, W)
        dev = torch.device("cuda:0")
        frame = torch.from_numpy(modelgen.synthetic_frame(args.seed, 1, H, W).reshape(-1)).to(dev)
        torch.cuda.synchronize()

        class _B:  # the engine's input buffer as a torch view
            __cuda_array_interface__ = {"shape": (in_bytes // 2,), "typestr": "<f2", "data": (in_ptr, False),
                                        "version": 3}
        torch.as_tensor(_B(), device=dev).copy_(frame)
        torch.cuda.synchronize()
        for _ in range(max(1, args.warmup)):
            eng.enqueue()
        eng.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.iters):
            eng.enqueue()
        eng.synchronize()
        ms = (time.perf_counter() - t0) * 1e3 / args.iters
        print(json.dumps({"model": f"{args.model} {H}x{W}", "algo": args.algo, "ms_per_frame": ms, "fps": 1e3 / ms,
                          "iters": args.iters, "timing": "host wall clock around enqueued graph replays"}))
        eng.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
