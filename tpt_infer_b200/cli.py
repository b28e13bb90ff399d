"""Command line of the CUDA backend: ``python -m tpt_infer_b200 <command>``.

Mirrors the reference CLI (crates/tpt-infer-cli/src/main.rs:29-59, 129-183)
with the backend chosen by ``--backend`` (only ``cuda`` exists here: there is no
CPU fallback) instead of the hard-wired ``select_backend()`` (main.rs:164):

  inspect MODEL               node / initializer / input / output counts, the
                              operator histogram, the outputs, and whether every
                              operator lowers onto the CUDA plan
  run MODEL [--input F]       loads the ONNX model, lowers it, runs it on the GPU
                              and prints the output shape, its first values and
                              the argmax (main.rs:129-183 output format); F holds
                              raw little-endian f32 values of the runtime input,
                              else the reference's deterministic pseudo-random
                              input is used; --int8 lowers rank-2 MatMuls with
                              INT8 per-output-channel weights, calibrated on
                              that input
  bench CONFIG                one of the benchmark workloads on the GPU through
                              the public API (mlp, mlp-int8, resnet18, bert, w8a8,
                              w4), device-resident inputs, printed as one JSON line

Exit status 0 on success, 1 with ``error: ...`` on stderr otherwise (main.rs:45-58).
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from collections import Counter

import numpy as np


def _backend(name, device):
    if name != "cuda":
        raise RuntimeError(f"unsupported backend {name!r}: this build provides the CUDA backend only")
    from .backend import CudaBackend

    be = CudaBackend.new(device)
    if be is None:
        raise RuntimeError("no usable sm_100 CUDA device")
    return be


def _runtime_input(g):
    """find_runtime_input (main.rs:108-125)."""
    ins = g.inputs()
    if not ins:
        raise RuntimeError("model has no runtime input (every graph input is a weight initializer)")
    return g.nodes[ins[0]]


def _pseudo_random(n):
    """main.rs:151-155: ((i * 12.9898).sin() * 43758.547).fract(), in f32."""
    i = np.arange(n, dtype=np.float32)
    v = np.sin(i * np.float32(12.9898)).astype(np.float32) * np.float32(43758.547)
    return (v - np.trunc(v)).astype(np.float32)


def cmd_inspect(args):
    from . import lowering, onnx

    g = onnx.load(args.model)
    print(f"nodes:        {len(g.nodes)}")
    print(f"initializers: {len(g.initializers)}")
    print(f"inputs:       {sum(1 for n in g.nodes if n.op.kind == 'Input')}")
    print(f"outputs:      {len(g.outputs)}")
    print("\noperator histogram:")
    for op, c in sorted(Counter(n.op.name for n in g.nodes).items()):
        print(f"  {op:<16} {c}")
    print("\noutputs:")
    for o in g.outputs:
        n = g.nodes[o]
        print(f"  node {o} ({n.name or '<unnamed>'}): shape {list(n.dims)}")
    unsupported = sorted({n.op.name for n in g.nodes if n.op.kind not in lowering.SUPPORTED})
    print("\nCUDA lowering: " + ("supported - every operator in this graph lowers onto the device plan"
                                 if not unsupported else f"not supported - {', '.join(unsupported)}"))
    return 0


def cmd_run(args):
    from . import lowering, onnx

    g = onnx.load(args.model)
    node = _runtime_input(g)
    numel = int(np.prod(node.dims, dtype=np.int64))
    if args.input:
        raw = open(args.input, "rb").read()
        if len(raw) != numel * 4:
            raise RuntimeError(f"input file '{args.input}' is {len(raw)} bytes; expected {numel * 4} "
                               f"({numel} f32 elements for shape {list(node.dims)})")
        x = np.frombuffer(raw, "<f4").astype(np.float32)
    else:
        print(f"no --input given; using deterministic pseudo-random input of shape {list(node.dims)}")
        x = _pseudo_random(numel)
    feeds = [x] + [np.zeros(int(np.prod(g.nodes[i].dims, dtype=np.int64)), np.float32) for i in g.inputs()[1:]]
    be = _backend(args.backend, args.device)
    lg = lowering.lower(g, be, quantized="all" if args.int8 else None)
    try:
        if args.int8:
            lg.calibrate([feeds])
        out = lg.run(feeds)[0]
    finally:
        lg.close()
        be.close()
    flat = out.ravel()
    print(f"output shape: {list(out.shape)}")
    prev = ", ".join(f"{v:.6f}" for v in flat[:10])
    print(f"output[..{min(10, flat.size)}]: [{prev}{', ...' if flat.size > 10 else ''}]")
    print(f"argmax: {int(np.argmax(flat))}")
    return 0


def _time(fn, sync, reps):
    fn()
    sync()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    sync()
    return (time.perf_counter() - t0) / reps


def cmd_bench(args):
    """One workload through the public API, inputs resident on the device, timed
    on the host around args.steps runs after a warm-up (each run ends with a
    stream synchronisation)."""
    from . import graphs, synth

    be = _backend(args.backend, args.device)
    res = {"config": args.config, "steps": args.steps}
    try:
        if args.config in ("mlp", "mlp-int8"):
            B = args.batch or 64
            W = graphs.mlp_weights()
            if args.config == "mlp":
                p, x, y, _ = graphs.build_mlp_f32(be, B, W)
            else:
                p, x, y, _, _ = graphs.build_mlp_int8(be, B, W)
                p.calibrate(True)
                for i in range(4):
                    p.run({x: synth.uniform(B * 784, 1000 + i)}, [y])
                p.freeze()
            p.set_graph(True)
            p.run({x: synth.uniform(B * 784, 77)}, [y])
            t = _time(p.run_device, be.sync, args.steps)
            res.update(batch=B, us_per_forward=t * 1e6, inferences_per_s=B / t)
            p.close()
        elif args.config == "resnet18":
            B, IMG = args.batch or 256, 3 * 224 * 224
            p, x, y = graphs.build_resnet18(be, B, graphs.resnet18_weights(be))
            p.calibrate(True)
            p.run({x: synth.normal(B * IMG, 31)}, [y])
            p.freeze()
            p.set_graph(True)  # the forward as one recorded launch sequence
            p.run({x: synth.normal(B * IMG, 32)}, [y])
            t = _time(p.run_device, be.sync, args.steps)
            res.update(batch=B, ms_per_batch=t * 1e3, images_per_s=B / t)
            p.close()
        elif args.config == "bert":
            B, S, H = args.batch or 64, args.seq, 768
            p, x, y = graphs.build_bert(be, B, S, graphs.bert_weights(be, layers=args.layers))
            p.calibrate(True)
            p.run({x: synth.normal(B * S * H, 41)}, [y])
            p.freeze()
            p.set_graph(True)
            p.run({x: synth.normal(B * S * H, 42)}, [y])
            t = _time(p.run_device, be.sync, args.steps)
            res.update(batch=B, seq=S, layers=args.layers, ms_per_batch=t * 1e3, sequences_per_s=B / t)
            p.close()
        elif args.config in ("w8a8", "w4"):
            import torch

            M, K = args.m, 4096
            N = 4096 if args.config == "w8a8" else 11008
            dev = f"cuda:{args.device}"
            wt = synth.normal(N * K, 1000, 0.0, 0.02)
            bias = torch.from_numpy(synth.normal(N, 1002, 0.0, 0.01)).to(dev)
            y = torch.empty(M * N, dtype=torch.float32, device=dev)
            if args.config == "w8a8":
                wq, ws = be.quantize_i8_symmetric_per_channel(wt, N)
                w = be.upload_i8(wq, ws, N, K)
                aq, sa = be.quantize_i8_symmetric(synth.normal(M * K, 1001))
                a = torch.from_numpy(aq).to(dev)
                t = _time(lambda: be.w8a8_gemm_dev(a, M, sa, w, bias, 0, y), be.sync, args.steps)
                res.update(M=M, N=N, K=K, us=t * 1e6, TOPs=2.0 * M * N * K / t / 1e12)
            else:
                pk, s = be.quantize_i4_symmetric_per_channel(wt, N)
                w = be.upload_i4(pk, s, N, K)
                xx = torch.from_numpy(synth.normal(M * K, 1001)).to(dev)
                t = _time(lambda: be.w4_gemm_dev(xx, M, w, bias, 0, y), be.sync, args.steps)
                res.update(M=M, N=N, K=K, us=t * 1e6, TFLOPs=2.0 * M * N * K / t / 1e12)
            w.free()
        else:
            raise RuntimeError(f"unknown bench config {args.config!r}")
    finally:
        be.close()
    print(json.dumps(res))
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(prog="tpt-infer-cuda",
                                 description="Inspect, run and benchmark ONNX models on the B200 CUDA backend")
    ap.add_argument("--backend", default="cuda", help="compute backend (cuda)")
    ap.add_argument("--device", type=int, default=0)
    sub = ap.add_subparsers(dest="command", required=True)
    s = sub.add_parser("inspect")
    s.add_argument("model")
    s = sub.add_parser("run")
    s.add_argument("model")
    s.add_argument("--input")
    s.add_argument("--int8", action="store_true")
    s = sub.add_parser("bench")
    s.add_argument("config", choices=["mlp", "mlp-int8", "resnet18", "bert", "w8a8", "w4"])
    s.add_argument("--steps", type=int, default=20)
    s.add_argument("--batch", type=int, default=0)
    s.add_argument("--seq", type=int, default=128)
    s.add_argument("--layers", type=int, default=12)
    s.add_argument("--m", type=int, default=4096)
    args = ap.parse_args(argv)
    try:
        return {"inspect": cmd_inspect, "run": cmd_run, "bench": cmd_bench}[args.command](args)
    except Exception as e:  # main.rs:45-58: "error: ..." and a failing exit status
        print(f"error: {e}", file=sys.stderr)
        return 1
