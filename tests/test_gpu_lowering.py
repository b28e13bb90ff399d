"""Whole graphs lowered onto one device plan (tpt_infer_b200.lowering) against
the oracle's node-by-node execution of the same graph (oracle/graph_exec.py,
the reference runtime's dispatch of crates/tpt-infer-runtime/src/exec.rs).

The f32 operators are bit-exact (MatMul, Conv2d, broadcast Add/Sub/Mul/Div,
ReLU, pooling, BatchNorm, Concat, Transpose, Reshape/Flatten, batched MatMul,
ONNX Gemm); Sigmoid/GELU/Softmax use CUDA's expf/tanhf and are compared within
1e-5 (1 + |want|), as the Backend element-op tests are.
"""
import numpy as np
import pytest

from oracle import graph_exec
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def lcg(n, seed, scale):
    """tests.rs:20-30: LCG values (u * 2 - 1) * scale, u = (s >> 8) / 2^24, in f32."""
    s = seed
    out = np.empty(n, np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u = np.float32(s >> 8) / np.float32(1 << 24)
        out[i] = (u * np.float32(2.0) - np.float32(1.0)) * np.float32(scale)
    return out


def mobilenet_v2_style(L):
    """The structure of the reference's MobileNetV2-shaped fixture (tests.rs:104-200):
    3x3/2 stem, four inverted-residual-ish blocks (1x1 expand, ReLU, 3x3, ReLU, 1x1
    project, residual Add when shapes match), global average pool, Flatten, MatMul
    head to 1000 classes."""
    g = L.ComputationGraph()
    seed = [0]

    def nxt():
        seed[0] += 1
        return seed[0]

    def conv(x, name, wd, strides, pad, od):
        w = g.add_weight(name, wd, lcg(int(np.prod(wd)), nxt(), 0.05))
        return g.add_node(L.Operator.conv2d(strides, pad), [x, w], od)

    def block(x, xd, ce, co, stride, tag):
        n, ci, h, w = xd
        oh, ow = (h + 2 - 3) // stride + 1, (w + 2 - 3) // stride + 1
        t = conv(x, tag + "_e", [ce, ci, 1, 1], [1, 1], [0, 0], [n, ce, h, w])
        t = g.add_node(L.Operator.relu(), [t], [n, ce, h, w])
        t = conv(t, tag + "_s", [ce, ce, 3, 3], [stride, stride], [1, 1], [n, ce, oh, ow])
        t = g.add_node(L.Operator.relu(), [t], [n, ce, oh, ow])
        t = conv(t, tag + "_p", [co, ce, 1, 1], [1, 1], [0, 0], [n, co, oh, ow])
        if stride == 1 and ci == co:
            t = g.add_node(L.Operator.add(), [x, t], [n, co, oh, ow])
        return t, [n, co, oh, ow]

    x = g.add_input([1, 8, 32, 32], "data")
    cur = conv(x, "stem_w", [16, 8, 3, 3], [2, 2], [1, 1], [1, 16, 16, 16])
    cur = g.add_node(L.Operator.relu(), [cur], [1, 16, 16, 16])
    d = [1, 16, 16, 16]
    for ce, co, s, tag in ((32, 16, 2, "b1"), (32, 16, 1, "b2"), (48, 16, 2, "b3"), (48, 16, 1, "b4")):
        cur, d = block(cur, d, ce, co, s, tag)
    gap = g.add_node(L.Operator.average_pool2d(d[2:], [1, 1], [0, 0]), [cur], [d[0], d[1], 1, 1])
    flat = g.add_node(L.Operator.flatten(1), [gap], [d[0], d[1]])
    fc = g.add_weight("fc_w", [d[1], 1000], lcg(d[1] * 1000, nxt(), 0.1))
    head = g.add_node(L.Operator.matmul(), [flat, fc], [d[0], 1000])
    g.mark_output(head)
    return g


def test_mobilenet_style_graph_bit_exact(cuda):
    # mobilenet_v2_end_to_end (tests.rs:202-230): [1, 1000] logits, finite, and
    # the same bits on a second run; here also the same bits as the oracle
    from tpt_infer_b200 import lowering as L

    g = mobilenet_v2_style(L)
    assert len(g.nodes) > 30
    x = lcg(8 * 32 * 32, 7, 0.5)
    lg = L.lower(g, cuda)
    got = lg.run([x])[0]
    again = lg.run([x])[0]
    want = graph_exec.execute_graph(g, [x])[0]
    lg.close()
    assert got.shape == (1, 1000) and np.all(np.isfinite(got))
    assert np.array_equal(got, again)
    assert np.array_equal(got, want)
    assert int(np.argmax(got)) == int(np.argmax(want))


def test_dispatch_operator_coverage_graph(cuda):
    # dispatch_operator_coverage (tests.rs:232-292): the reference's expected
    # values, and the oracle's outputs
    from tpt_infer_b200 import lowering as L

    g = L.ComputationGraph()
    x = g.add_input([1, 1, 4, 4], "x")
    mp = g.add_node(L.Operator.max_pool2d([2, 2], [2, 2], [0, 0]), [x], [1, 1, 2, 2])
    cat = g.add_node(L.Operator.concat(1), [mp, mp], [1, 2, 2, 2])
    flat = g.add_node(L.Operator.flatten(1), [cat], [1, 8])
    tr = g.add_node(L.Operator.transpose([0, 1, 3, 2]), [mp], [1, 1, 2, 2])
    outs = [flat, tr]
    for k in ("sub", "mul", "div", "sigmoid", "gelu"):
        outs.append(g.add_node(getattr(L.Operator, k)(), [mp, mp] if k in ("sub", "mul", "div") else [mp],
                               [1, 1, 2, 2]))
    for o in outs:
        g.mark_output(o)
    xin = np.arange(16, dtype=np.float32)
    lg = L.lower(g, cuda)
    r = lg.run([xin])
    lg.close()
    want = graph_exec.execute_graph(g, [xin])
    assert len(r) == 7
    assert r[0].ravel().tolist() == [5, 7, 13, 15, 5, 7, 13, 15]
    assert r[1].ravel().tolist() == [5, 13, 7, 15]
    assert r[2].ravel().tolist() == [0, 0, 0, 0]
    for i in range(5):
        assert np.array_equal(r[i], want[i])
    for i in (5, 6):
        assert np.all(np.abs(r[i] - want[i]) <= 1e-5 * (1 + np.abs(want[i])))


def test_extended_operator_graph(cuda):
    # BatchNorm in both modes, padded average pooling, broadcast Sub/Div/Mul,
    # Concat on an inner axis, a rank-4 Transpose, a rank-4 MatMul with a
    # broadcast batch dim, Softmax, ONNX Gemm with transB and C, LayerNorm
    from tpt_infer_b200 import lowering as L

    r = np.random.default_rng(5)
    g = L.ComputationGraph()
    x = g.add_input([2, 3, 9, 7], "x")
    bn = g.add_node(L.Operator.batch_norm(1e-3),
                    [x] + [g.add_weight(f"bn{i}", [3], v) for i, v in
                           enumerate((r.normal(1, .2, 3), r.normal(0, .1, 3), r.normal(0, .5, 3), r.uniform(.5, 2, 3)))],
                    [2, 3, 9, 7])
    ap = g.add_node(L.Operator.average_pool2d([3, 3], [2, 2], [1, 1]), [bn], [2, 3, 5, 4])
    mx = g.add_node(L.Operator.max_pool2d([3, 2], [1, 2], [1, 0]), [bn], [2, 3, 9, 3])
    rowv = g.add_weight("rowv", [1, 3, 1, 4], r.normal(0, 1, 12))
    sub = g.add_node(L.Operator.sub(), [ap, rowv], [2, 3, 5, 4])
    div = g.add_node(L.Operator.div(), [sub, g.add_weight("d", [4], r.uniform(.5, 2, 4))], [2, 3, 5, 4])
    cat = g.add_node(L.Operator.concat(2), [div, sub], [2, 3, 10, 4])
    tr = g.add_node(L.Operator.transpose([0, 3, 1, 2]), [cat], [2, 4, 3, 10])
    bw = g.add_weight("bw", [1, 4, 10, 6], r.normal(0, .3, 240))
    bmm = g.add_node(L.Operator.matmul(), [tr, bw], [2, 4, 3, 6])
    sm = g.add_node(L.Operator.softmax(-1), [bmm], [2, 4, 3, 6])
    flat = g.add_node(L.Operator.reshape([24, 6]), [sm], [24, 6])
    gw = g.add_weight("gw", [5, 6], r.normal(0, 1, 30))
    gc = g.add_weight("gc", [5], r.normal(0, 1, 5))
    gm = g.add_node(L.Operator.gemm(alpha=0.5, beta=2.0, trans_b=True), [flat, gw, gc], [24, 5])
    ew = [g.add_weight(f"e{i}", [24, 5], v) for i, v in enumerate((r.normal(1, .1, 120), r.normal(0, .1, 120),
                                                                    r.normal(0, .1, 120), r.uniform(.5, 1, 120)))]
    bne = g.add_node(L.Operator.batch_norm(1e-5), [gm] + ew, [24, 5])
    mul = g.add_node(L.Operator.mul(), [bne, g.add_weight("m", [24, 1], r.normal(0, 1, 24))], [24, 5])
    outs = [ap, mx, cat, tr, bmm, sm, gm, bne, mul]
    for o in outs:
        g.mark_output(o)
    xin = r.normal(0, 1, 2 * 3 * 9 * 7).astype(np.float32)
    lg = L.lower(g, cuda)
    got = lg.run([xin])
    lg.close()
    want = graph_exec.execute_graph(g, [xin])
    for o, a, b in zip(outs, got, want):
        if o == sm:
            assert np.all(np.abs(a - b) <= 1e-5 * (1 + np.abs(b)))
        elif o in (gm, bne, mul):  # downstream of the softmax: compare against the device's softmax
            continue
        else:
            assert np.array_equal(a, b), g.nodes[o].op.kind
    # the tail from the device's own softmax output on: exact
    g2 = L.ComputationGraph()
    s_in = g2.add_input([24, 6], "s")
    gm2 = g2.add_node(L.Operator.gemm(alpha=0.5, beta=2.0, trans_b=True),
                      [s_in, g2.add_weight("gw", [5, 6], g.initializers["gw"].data),
                       g2.add_weight("gc", [5], g.initializers["gc"].data)], [24, 5])
    g2.initializers.update({k: v for k, v in g.initializers.items() if k.startswith("e") or k == "m"})
    ew2 = [g2.add_input([24, 5], f"e{i}") for i in range(4)]
    bne2 = g2.add_node(L.Operator.batch_norm(1e-5), [gm2] + ew2, [24, 5])
    mul2 = g2.add_node(L.Operator.mul(), [bne2, g2.add_input([24, 1], "m")], [24, 5])
    for o in (gm2, bne2, mul2):
        g2.mark_output(o)
    lg2 = L.lower(g2, cuda)
    got2 = lg2.run([got[5]])
    lg2.close()
    want2 = graph_exec.execute_graph(g2, [got[5]])
    for a, b in zip(got2 + [got[6], got[7], got[8]], want2 + want2):
        assert np.array_equal(a, b)


def test_layernorm_node(cuda):
    from tpt_infer_b200 import lowering as L

    r = np.random.default_rng(9)
    g = L.ComputationGraph()
    x = g.add_input([4, 37, 768], "x")
    ln = g.add_node(L.Operator.layer_norm(1e-5), [x, g.add_weight("g", [768], r.normal(1, .1, 768)),
                                                  g.add_weight("b", [768], r.normal(0, .1, 768))], [4, 37, 768])
    g.mark_output(ln)
    xin = r.normal(0, 2, 4 * 37 * 768).astype(np.float32)
    lg = L.lower(g, cuda)
    got = lg.run([xin])[0]
    lg.close()
    want = graph_exec.execute_graph(g, [xin])[0]
    assert np.max(np.abs(got - want)) <= 1e-5 * (1 + np.max(np.abs(want)))


def test_int8_weight_lowering_matches_oracle(cuda):
    # the MLP as a graph with INT8 weights: MatMul -> QUANTIZE + W8A8 GEMM with
    # per-output-channel weights quantized on the device, calibrated activation
    # scales; bit-exact against the oracle given the same scales and weights
    from tpt_infer_b200 import graphs, lowering as L, synth

    W = graphs.mlp_weights()
    g = L.ComputationGraph()
    x = g.add_input([64, 784], "x")
    h = g.add_node(L.Operator.matmul(), [x, g.add_weight("w1", [784, 512], W.w1)], [64, 512])
    h = g.add_node(L.Operator.add(), [h, g.add_weight("b1", [512], synth.normal(512, 3, 0, .1))], [64, 512])
    h = g.add_node(L.Operator.relu(), [h], [64, 512])
    z = g.add_node(L.Operator.matmul(), [h, g.add_weight("w2", [512, 16], synth.normal(512 * 16, 4, 0, .06))],
                   [64, 16])
    g.mark_output(z)
    lg = L.lower(g, cuda, quantized="all")
    cal = [[synth.uniform(64 * 784, 1000 + i)] for i in range(4)]
    lg.calibrate(cal)
    scales = lg.plan.scales()
    assert scales.size == 2
    xin = synth.uniform(64 * 784, 77)
    got = lg.run([xin])[0]
    lg.close()
    q = {}
    for name, n in (("w1", 512), ("w2", 16)):
        w = g.initializers[name].data.reshape(-1, n)
        q[name] = O.quantize_i8_symmetric_per_channel(np.ascontiguousarray(w.T), n)
    calib = []
    for b in cal:
        graph_exec.execute_graph(g, b, quantized=q, calib=calib)
    want_scales = [O.sym_scale(max(calib[i::2])) for i in range(2)]
    assert np.array_equal(scales, np.array(want_scales, np.float32))
    want = graph_exec.execute_graph(g, [xin], quantized=q, scales=scales)[0]
    assert np.array_equal(got, want)


def test_lowering_errors(cuda):
    from tpt_infer_b200 import lowering as L
    from tpt_infer_b200.backend import OpError

    g = L.ComputationGraph()
    x = g.add_input([2, 3], "x")
    g.mark_output(g.add_node(L.Operator.custom("NonMaxSuppression"), [x], [2, 3]))
    with pytest.raises(L.UnsupportedOp):
        L.lower(g, cuda)
    g = L.ComputationGraph()
    x = g.add_input([2, 3], "x")
    g.mark_output(g.add_node(L.Operator.softmax(0), [x], [2, 3]))
    with pytest.raises(L.UnsupportedOp):  # the HAL softmax normalizes the last axis only
        L.lower(g, cuda)
    g = L.ComputationGraph()
    a, b = g.add_input([3], "a"), g.add_input([4], "b")
    g.mark_output(g.add_node(L.Operator.add(), [a, b], [4]))
    with pytest.raises(OpError) as e:  # binary_incompatible_broadcast_errors (kernels.rs:616-622)
        L.lower(g, cuda)
    assert e.value.code == 2
    g = L.ComputationGraph()
    a, b = g.add_input([2, 3], "a"), g.add_input([4, 5], "b")
    g.mark_output(g.add_node(L.Operator.matmul(), [a, b], [2, 5]))
    with pytest.raises(OpError) as e:  # validate_matmul: k mismatch
        L.lower(g, cuda)
    assert e.value.code == 2
