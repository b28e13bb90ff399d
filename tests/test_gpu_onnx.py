"""ONNX-loaded graphs on the CUDA backend, and the command line.

Models are written by tpt_infer_b200.onnx.save (no ONNX package exists in this
image), loaded back by the loader, lowered onto a device plan and compared with
the oracle's walk of the same loaded graph: bit-exact for the f32 operators,
within 1e-5 (1 + |want|) after Softmax (CUDA expf). The command line's
``run`` prints the reference CLI's output format (main.rs:167-181) for the same
model and input.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import graph_exec

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bert_block(L, S=16, D=32):
    """A transformer block in the shape of the reference's bert_tiny_style
    fixture, with the real LayerNorm: q/k/v projections (MatMul + bias Add),
    scores Q K^T (Transpose + batched-free rank-2 MatMul), Softmax, context,
    residual Add, LayerNorm, ReLU FFN."""
    r = np.random.default_rng(11)
    g = L.ComputationGraph()
    x = g.add_input([S, D], "x")

    def lin(inp, name, n_in, n_out):
        m = g.add_node(L.Operator.matmul(), [inp, g.add_weight(name + "_w", [n_in, n_out],
                                                                r.normal(0, 0.2, n_in * n_out))], [S, n_out])
        return g.add_node(L.Operator.add(), [m, g.add_weight(name + "_b", [n_out], r.normal(0, 0.1, n_out))],
                          [S, n_out])

    q, k, v = lin(x, "q", D, D), lin(x, "k", D, D), lin(x, "v", D, D)
    kt = g.add_node(L.Operator.transpose([1, 0]), [k], [D, S])
    sc = g.add_node(L.Operator.matmul(), [q, kt], [S, S])
    sc = g.add_node(L.Operator.mul(), [sc, g.add_weight("scale", [1], [1.0 / np.sqrt(D)])], [S, S])
    p = g.add_node(L.Operator.softmax(-1), [sc], [S, S])
    ctx = g.add_node(L.Operator.matmul(), [p, v], [S, D])
    res = g.add_node(L.Operator.add(), [ctx, x], [S, D])
    ln = g.add_node(L.Operator.layer_norm(1e-5), [res, g.add_weight("g", [D], np.ones(D)),
                                                   g.add_weight("b", [D], np.zeros(D))], [S, D])
    h = g.add_node(L.Operator.relu(), [lin(ln, "f1", D, 2 * D)], [S, 2 * D])
    out = g.add_node(L.Operator.add(), [lin(h, "f2", 2 * D, D), ln], [S, D])
    g.mark_output(out)
    g.mark_output(p)
    return g


def test_onnx_mobilenet_style_runs_bit_exact(cuda, tmp_path):
    from tests.test_gpu_lowering import lcg, mobilenet_v2_style
    from tpt_infer_b200 import lowering as L
    from tpt_infer_b200 import onnx

    path = tmp_path / "mobilenet_style.onnx"
    onnx.save(mobilenet_v2_style(L), str(path))
    g = onnx.load(str(path))
    x = lcg(8 * 32 * 32, 7, 0.5)
    lg = L.lower(g, cuda)
    got = lg.run([x])[0]
    lg.close()
    want = graph_exec.execute_graph(g, [x])[0]
    assert np.array_equal(got, want)
    # the command line on the same model and input (raw little-endian f32)
    inp = tmp_path / "x.bin"
    inp.write_bytes(x.astype("<f4").tobytes())
    r = subprocess.run([sys.executable, "-m", "tpt_infer_b200", "--backend", "cuda", "run", str(path), "--input",
                        str(inp)], capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert "output shape: [1, 1000]" in lines
    assert f"argmax: {int(np.argmax(want))}" in lines
    first = [ln for ln in lines if ln.startswith("output[..10]: [")][0]
    vals = [float(v) for v in first[len("output[..10]: ["):].rstrip(", ...]").split(", ")]
    assert np.allclose(vals, want.ravel()[:10], atol=5e-7)


def test_onnx_transformer_block(cuda):
    from tpt_infer_b200 import lowering as L
    from tpt_infer_b200 import onnx

    g = onnx.load_from_bytes(onnx.save_bytes(_bert_block(L)))
    assert any(n.op.kind == "LayerNorm" for n in g.nodes)
    x = np.random.default_rng(12).normal(0, 1, 16 * 32).astype(np.float32)
    lg = L.lower(g, cuda)
    out, p = lg.run([x])
    lg.close()
    want_out, want_p = graph_exec.execute_graph(g, [x])
    assert np.all(np.abs(p - want_p) <= 1e-5 * (1 + np.abs(want_p)))
    assert np.max(np.abs(out - want_out)) <= 1e-4 * (1 + np.max(np.abs(want_out)))


def test_cli_errors_and_bench(tmp_path):
    r = subprocess.run([sys.executable, "-m", "tpt_infer_b200", "--backend", "cpu", "run", "missing.onnx"],
                       capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert r.returncode == 1 and r.stderr.startswith("error: ")
    r = subprocess.run([sys.executable, "-m", "tpt_infer_b200", "bench", "mlp", "--steps", "5"],
                       capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["config"] == "mlp" and res["inferences_per_s"] > 0
