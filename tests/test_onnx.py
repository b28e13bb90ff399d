"""ONNX loader and writer (tpt_infer_b200/onnx.py), on the CPU.

- The reference's own committed fixtures, when the reference tree is present:
  the structural assertions of crates/tpt-infer-onnx/tests/
  real_model_fixtures.rs:16-60 and :185-230, and an execution through the
  oracle's graph walk (finite outputs of the declared shape).
- Writer -> loader round trips of generated graphs reproduce the graph and its
  oracle outputs bit for bit.
- Malformed bytes raise OnnxError (load.rs decode / invalid-model errors).
"""
import os

import numpy as np
import pytest

from oracle import graph_exec

FIX = "/root/reference/crates/tpt-infer-onnx/tests/fixtures"


def _kinds(g, kind):
    return sum(1 for n in g.nodes if n.op.kind == kind)


@pytest.mark.skipif(not os.path.isdir(FIX), reason="reference fixtures not present")
def test_reference_mobilenet_fixture():
    from tpt_infer_b200 import onnx

    g = onnx.load(os.path.join(FIX, "mobilenet_v2_style.onnx"))
    assert len(g.nodes) >= 20
    assert len(g.initializers) == 12
    assert _kinds(g, "Input") == 1 + 12
    x = [n for n in g.nodes if n.name == "x"]
    assert x and x[0].dims == (1, 3, 16, 16)
    assert len(g.outputs) == 1 and g.nodes[g.outputs[0]].dims == (1, 10)
    for k in ("Conv2d", "BatchNorm", "Relu", "Add", "AveragePool2d", "MatMul"):
        assert _kinds(g, k) >= 1, k
    out = graph_exec.execute_graph(g, [np.linspace(-1, 1, 3 * 16 * 16, dtype=np.float32)])[0]
    assert out.shape == (1, 10) and np.all(np.isfinite(out))


@pytest.mark.skipif(not os.path.isdir(FIX), reason="reference fixtures not present")
def test_reference_bert_tiny_fixture():
    from tpt_infer_b200 import onnx

    g = onnx.load(os.path.join(FIX, "bert_tiny_style.onnx"))
    assert len(g.nodes) >= 15
    assert len(g.initializers) == 10
    x = [n for n in g.nodes if n.name == "x"]
    assert x and x[0].dims == (1, 8)
    assert len(g.outputs) == 1 and g.nodes[g.outputs[0]].dims == (1, 8)
    assert _kinds(g, "MatMul") >= 5 and _kinds(g, "Add") >= 4
    assert _kinds(g, "Softmax") == 1 and _kinds(g, "BatchNorm") == 1 and _kinds(g, "Relu") == 1
    out = graph_exec.execute_graph(g, [np.linspace(-1, 1, 8, dtype=np.float32)])[0]
    assert out.shape == (1, 8) and np.all(np.isfinite(out))


def _sample_graph(L):
    r = np.random.default_rng(3)
    g = L.ComputationGraph()
    x = g.add_input([2, 4, 8, 8], "img")
    c = g.add_node(L.Operator.conv2d([2, 2], [1, 1]), [x, g.add_weight("w", [6, 4, 3, 3], r.normal(0, .2, 216)),
                                                       g.add_weight("b", [1, 6, 1, 1], r.normal(0, .1, 6))],
                   [2, 6, 4, 4])
    bn = g.add_node(L.Operator.batch_norm(1e-4), [c] + [g.add_weight(f"p{i}", [6], v) for i, v in enumerate(
        (r.normal(1, .1, 6), r.normal(0, .1, 6), r.normal(0, .1, 6), r.uniform(.5, 1.5, 6)))], [2, 6, 4, 4])
    rl = g.add_node(L.Operator.relu(), [bn], [2, 6, 4, 4])
    mp = g.add_node(L.Operator.max_pool2d([2, 2], [2, 2], [0, 0]), [rl], [2, 6, 2, 2])
    tr = g.add_node(L.Operator.transpose([0, 2, 3, 1]), [mp], [2, 2, 2, 6])
    rs = g.add_node(L.Operator.reshape([2, 24]), [tr], [2, 24])
    gm = g.add_node(L.Operator.gemm(1.5, 0.5, False, True), [rs, g.add_weight("gw", [5, 24], r.normal(0, .2, 120)),
                                                             g.add_weight("gc", [5], r.normal(0, 1, 5))], [2, 5])
    ln = g.add_node(L.Operator.layer_norm(1e-5), [gm, g.add_weight("lg", [5], np.ones(5)),
                                                  g.add_weight("lb", [5], np.zeros(5))], [2, 5])
    sm = g.add_node(L.Operator.softmax(-1), [ln], [2, 5])
    g.mark_output(sm)
    g.mark_output(mp)
    return g


def test_writer_loader_round_trip():
    from tpt_infer_b200 import lowering as L
    from tpt_infer_b200 import onnx

    g = _sample_graph(L)
    g2 = onnx.load_from_bytes(onnx.save_bytes(g))
    assert [n.op.kind for n in g2.nodes if n.op.kind != "Input"] == \
        [n.op.kind for n in g.nodes if n.op.kind != "Input"]
    assert set(g2.initializers) >= set(g.initializers)
    for name, init in g.initializers.items():
        assert np.array_equal(g2.initializers[name].data, init.data)
    for a, b in zip([n for n in g.nodes if n.op.kind != "Input"], [n for n in g2.nodes if n.op.kind != "Input"]):
        assert a.dims == b.dims
        for k, v in a.op.attrs.items():
            assert b.op.attrs[k] == pytest.approx(v) if isinstance(v, float) else tuple(np.ravel(b.op.attrs[k])) == \
                tuple(np.ravel(v)), (a.op.kind, k)
    x = np.random.default_rng(4).normal(0, 1, 2 * 4 * 8 * 8).astype(np.float32)
    for u, v in zip(graph_exec.execute_graph(g, [x]), graph_exec.execute_graph(g2, [x])):
        assert np.array_equal(u, v)


def test_loader_rejects_malformed_bytes():
    from tpt_infer_b200 import onnx

    with pytest.raises(onnx.OnnxError):
        onnx.load_from_bytes(b"\x3a\xff\xff")  # truncated length-delimited graph field
    with pytest.raises(onnx.OnnxError):
        onnx.load_from_bytes(b"\x08\x08")  # a model with no graph
    with pytest.raises(onnx.OnnxError):  # opset beyond the supported version (load.rs:168-175)
        from tpt_infer_b200 import lowering as L

        good = onnx.save_bytes(_sample_graph(L))
        onnx.load_from_bytes(good[:-1] + bytes([99]))


def test_shape_inference_reference_cases():
    # crates/tpt-infer-onnx/src/shapes.rs:308-373: the shapes of MatMul, Conv,
    # Flatten and a dynamic batch, and kernels that do not fit their input
    from tpt_infer_b200 import onnx
    from tpt_infer_b200.lowering import Operator as Op

    assert onnx._infer(Op.matmul(), [[1, 784], [784, 10]]) == [1, 10]
    assert onnx._infer(Op.conv2d((1, 1), (1, 1)), [[1, 3, 224, 224], [8, 3, 3, 3]]) == [1, 8, 224, 224]
    assert onnx._infer(Op.flatten(1), [[1, 3, 32, 32]]) == [1, 3072]
    assert onnx._infer(Op.relu(), [[0, 128]]) == [0, 128]
    assert onnx._infer(Op.average_pool2d((0, 0), (1, 1), (0, 0)), [[2, 5, 7, 7]]) == [2, 5, 1, 1]
    with pytest.raises(onnx.OnnxError):
        onnx._infer(Op.conv2d((1, 1), (0, 0)), [[1, 3, 4, 4], [8, 3, 999, 999]])
    with pytest.raises(onnx.OnnxError):
        onnx._infer(Op.max_pool2d((999, 999), (1, 1), (0, 0)), [[1, 3, 4, 4]])


def test_loader_rejects_kernel_larger_than_input():
    # load.rs:1060-1105: a Conv whose 999 x 999 kernel exceeds its 4 x 4 input,
    # with no declared output shape (so shape inference runs), is an invalid model
    from tpt_infer_b200 import onnx as X

    conv = (X._ld(1, "x") + X._ld(1, "w") + X._ld(2, "y") + X._ld(3, "conv") + X._ld(4, "Conv") +
            X._attr_ints("strides", [1, 1]) + X._attr_ints("pads", [0, 0, 0, 0]) +
            X._attr_ints("kernel_shape", [999, 999]))
    body = (X._ld(1, conv) + X._ld(5, X._tensor_msg("w", [1, 1, 999, 999], np.zeros(999 * 999, np.float32))) +
            X._vi(11, "x", [1, 1, 4, 4]) + X._ld(12, X._ld(1, "y")))
    body = X._ld(2, "conv_bad") + body
    model = X._key(1, 0) + X._enc_varint(8) + X._ld(7, body) + X._ld(8, X._ld(1, "") + X._key(2, 0) + X._enc_varint(17))
    with pytest.raises(X.OnnxError, match="invalid model"):
        X.load_from_bytes(model)


def _model_bytes(X, nodes, inits, ins, outs):
    body = b"".join(X._ld(1, n) for n in nodes) + b"".join(X._ld(5, t) for t in inits)
    body += b"".join(X._vi(11, n, d) for n, d in ins) + b"".join(X._vi(12, n, d) for n, d in outs)
    body = X._ld(2, "g") + body
    return X._key(1, 0) + X._enc_varint(8) + X._ld(7, body) + X._ld(8, X._ld(1, "") + X._key(2, 0) + X._enc_varint(17))


def test_loader_limits_and_initializer_checks():
    # load.rs tests: oversized_model_bytes_rejected, oversized_graph_item_count_rejected,
    # negative_initializer_dim_rejected, mismatched_initializer_length_rejected
    from tpt_infer_b200 import onnx as X

    relu = X._ld(1, "x") + X._ld(2, "y") + X._ld(3, "relu0") + X._ld(4, "Relu")
    b = _model_bytes(X, [relu], [], [("x", [1, 4])], [("y", [1, 4])])
    assert [n.op.kind for n in X.load_from_bytes(b).nodes] == ["Input", "Relu"]
    with pytest.raises(X.OnnxError, match="invalid model"):
        X.load_from_bytes(b, max_bytes=len(b) - 1)
    with pytest.raises(X.OnnxError, match="invalid model"):
        X.load_from_bytes(b, max_graph_items=0)

    def tensor(name, dims, data):  # dims as int64 varints (two's complement for negatives)
        raw = np.ascontiguousarray(data, "<f4").tobytes()
        return (X._ld(1, b"".join(X._enc_varint(d & (2 ** 64 - 1)) for d in dims)) + X._key(2, 0) +
                X._enc_varint(1) + X._ld(8, name) + X._ld(9, raw))

    mm = X._ld(1, "x") + X._ld(1, "w") + X._ld(2, "y") + X._ld(3, "mm0") + X._ld(4, "MatMul")
    for dims, n in (([-4, 5], 20), ([4, 5], 3)):
        b2 = _model_bytes(X, [mm], [tensor("w", dims, np.zeros(n, np.float32))], [("x", [1, 4])], [("y", [1, 5])])
        with pytest.raises(X.OnnxError, match="invalid model"):
            X.load_from_bytes(b2)


def test_loader_same_padding_int64_reshape_and_dynamic_batch():
    # load.rs tests: conv_auto_pad_same_upper_resolves_symmetric_padding,
    # reshape_target_from_int64_initializer_input, dynamic_batch_zero
    from tpt_infer_b200 import onnx as X

    conv = (X._ld(1, "x") + X._ld(1, "conv_w") + X._ld(2, "c") + X._ld(3, "conv") + X._ld(4, "Conv") +
            X._attr_ints("strides", [1, 1]) + X._attr_ints("kernel_shape", [5, 5]) +
            X._ld(5, X._ld(1, "auto_pad") + X._ld(4, "SAME_UPPER") + X._key(20, 0) + X._enc_varint(3)))
    g = X.load_from_bytes(_model_bytes(X, [conv], [X._tensor_msg("conv_w", [8, 1, 5, 5], np.zeros(200, np.float32))],
                                       [("x", [1, 1, 28, 28])], [("c", [1, 8, 28, 28])]))
    c = [n for n in g.nodes if n.op.kind == "Conv2d"][0]
    assert tuple(c.op.attrs["padding"]) == (2, 2) and tuple(c.dims) == (1, 8, 28, 28)

    rs = X._ld(1, "x") + X._ld(1, "target_shape") + X._ld(2, "y") + X._ld(3, "reshape0") + X._ld(4, "Reshape")
    g = X.load_from_bytes(_model_bytes(X, [rs], [X._tensor_msg("target_shape", [2], np.array([1, 12], np.int64), 7)],
                                       [("x", [1, 3, 4])], [("y", [1, 12])]))
    r = [n for n in g.nodes if n.op.kind == "Reshape"][0]
    assert tuple(r.op.attrs["shape"]) == (1, 12) and "target_shape" in g.initializers

    def vi(f, name, dims):  # dim values as int64 varints, -1 included
        dm = b"".join(X._ld(1, X._key(1, 0) + X._enc_varint(d & (2 ** 64 - 1))) for d in dims)
        return X._ld(f, X._ld(1, name) + X._ld(2, X._ld(1, X._key(1, 0) + X._enc_varint(1) + X._ld(2, dm))))

    relu = X._ld(1, "x") + X._ld(2, "y") + X._ld(3, "r") + X._ld(4, "Relu")
    body = X._ld(2, "dyn") + X._ld(1, relu) + vi(11, "x", [-1, 4]) + vi(12, "y", [-1, 4])
    model = X._key(1, 0) + X._enc_varint(8) + X._ld(7, body) + X._ld(8, X._ld(1, "") + X._key(2, 0) + X._enc_varint(17))
    g = X.load_from_bytes(model)
    assert [tuple(n.dims) for n in g.nodes] == [(0, 4), (0, 4)]
