"""Model-level GPU parity: the device-resident plans against the oracle's
node-by-node replay of the same graphs (oracle/models.py).

MLP (f32): logits bit-exact (f32 MatMul is bit-identical to naive.rs), softmax
within 1e-5*(1+|want|). MLP (INT8 PTQ) and the ResNet-18-shaped CNN: the
calibrated activation scales and the logits are bit-exact -- every op on those
paths (quantize, W8A8 GEMM, bias/ReLU, max pool, residual add, sequential
global average pool, f32 MatMul) is exact. BERT-shaped encoder: LayerNorm,
the fused attention (softmax through exp_det) and the GELU epilogue follow a
fixed evaluation order that the oracle restates, so calibration and hidden
states are bit-exact too: at 2 layers with the calibration replayed, and at
the benchmarked 12 x 64 x 128 shape on sampled sequences with the device's
frozen scales.
"""
import numpy as np
import pytest

from oracle import models as OM
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _relerr(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want.astype(np.float64)), 1e-30))


def test_mlp_f32_plan(cuda):
    from tpt_infer_b200 import graphs, synth

    W = graphs.mlp_weights()
    p, x, y, z = graphs.build_mlp_f32(cuda, 64, W)
    xin = synth.uniform(64 * 784, 77)  # U[0,1)
    got_y, got_z = p.run({x: xin}, [y, z])
    h = O.matmul(xin, (64, 784), W.w1, (784, 512))
    h = np.where(O.add_bias_rows(h, 64, 512, W.b1) > 0, O.add_bias_rows(h, 64, 512, W.b1), 0).astype(np.float32)
    want_z = O.add_bias_rows(O.matmul(h, (64, 512), W.w2, (512, 10)), 64, 10, W.b2)
    assert np.array_equal(got_z, want_z)
    want_y = OM.mlp_f32(xin, W, 64)
    assert np.all(np.abs(got_y - want_y) <= 1e-5 * (1 + np.abs(want_y)))
    p.close()


def test_mlp_int8_plan_calibration_and_parity(cuda):
    from tpt_infer_b200 import graphs, synth

    W = graphs.mlp_weights()
    p, x, y, z, q = graphs.build_mlp_int8(cuda, 64, W)
    # the device-quantized weights equal the oracle's per-channel quantization
    q1o, s1o = O.quantize_i8_symmetric_per_channel(np.ascontiguousarray(W.w1.T), 512)
    assert np.array_equal(q[0], q1o) and np.array_equal(q[1], s1o)
    cal = [synth.uniform(64 * 784, 1000 + i) for i in range(4)]  # 256 seeded inputs
    p.calibrate(True)
    for xb in cal:
        p.run({x: xb}, [y])
    p.freeze()
    want_scales = OM.mlp_int8_calibrate(cal, W, 64, q)
    assert np.array_equal(p.scales(), np.array(want_scales, np.float32))
    xin = synth.uniform(64 * 784, 77)
    got_y, got_z = p.run({x: xin}, [y, z])
    q1, s1, q2, s2 = q
    a1, a2 = want_scales
    hq = O.quantize_i8_static(O.w8a8_gemm(O.quantize_i8_static(xin, a1), q1, 64, 512, 784, a1, s1, W.b1,
                                          O.ACT_RELU), a2)
    want_z = O.w8a8_gemm(hq, q2, 64, 10, 512, a2, s2, W.b2, O.ACT_NONE)
    assert np.array_equal(got_z, want_z)
    want_y = OM.mlp_int8(xin, W, 64, q, want_scales)
    assert np.all(np.abs(got_y - want_y) <= 1e-5 * (1 + np.abs(want_y)))
    # and the INT8 classifier agrees with the f32 one on most rows
    pf, xf, yf, _ = graphs.build_mlp_f32(cuda, 64, W)
    f32_y, = pf.run({xf: xin}, [yf])
    agree = np.mean(np.argmax(f32_y.reshape(64, 10), 1) == np.argmax(got_y.reshape(64, 10), 1))
    assert agree >= 0.9
    p.close()
    pf.close()


def test_resnet18_plan_bit_exact_batch2(cuda):
    from tpt_infer_b200 import graphs, synth

    spec = graphs.resnet18_weights(cuda)
    p, x, logits = graphs.build_resnet18(cuda, 2, spec)
    xcal = synth.normal(2 * 3 * 224 * 224, 31)
    p.calibrate(True)
    p.run({x: xcal}, [logits])
    p.freeze()
    cal = OM._Scales()
    OM.resnet18(xcal, spec, 2, calib=cal)
    assert np.array_equal(p.scales(), cal.frozen())
    xin = synth.normal(2 * 3 * 224 * 224, 32)
    got, = p.run({x: xin}, [logits])
    want = OM.resnet18(xin, spec, 2, scales=cal.frozen())
    assert np.array_equal(got, want), _relerr(got, want)
    p.close()


@pytest.mark.parametrize("B,S", [(2, 128), (3, 80)])
def test_bert_plan_two_layers(cuda, B, S):
    # calibration and hidden states bit-exact: LayerNorm, attention (softmax
    # through exp_det) and the GELU epilogue all have exact CPU restatements
    from tpt_infer_b200 import graphs, synth

    layers = graphs.bert_weights(cuda, layers=2)
    p, x, out = graphs.build_bert(cuda, B, S, layers)
    xcal = synth.normal(B * S * 768, 41)
    p.calibrate(True)
    p.run({x: xcal}, [out])
    p.freeze()
    cal = OM._Scales()
    OM.bert(xcal, layers, B, S, calib=cal)
    assert np.array_equal(p.scales(), cal.frozen())
    xin = synth.normal(B * S * 768, 42)
    got, = p.run({x: xin}, [out])
    want = OM.bert(xin, layers, B, S, scales=cal.frozen())
    assert np.array_equal(got, want), _relerr(got, want)
    p.close()


def test_bert_plan_benchmark_shape(cuda):
    # the benchmarked encoder: 12 layers, batch 64, seq 128, calibrated on one
    # batch; sampled sequences replayed by the oracle with the device's frozen
    # scales are bit-exact (sequences are independent given the scales)
    from tpt_infer_b200 import graphs, synth

    B, S, H, L = 64, 128, 768, 12
    layers = graphs.bert_weights(cuda, layers=L)
    p, x, out = graphs.build_bert(cuda, B, S, layers)
    p.calibrate(True)
    p.run({x: synth.normal(B * S * H, 41)}, [out])
    p.freeze()
    scales = p.scales()
    assert scales.size == 4 * L and np.all(scales > 0)
    xin = synth.normal(B * S * H, 42)
    got, = p.run({x: xin}, [out])
    p.close()
    got = got.reshape(B, S * H)
    pick = [0, 37, 63]
    want = OM.bert(np.concatenate([xin[b * S * H:(b + 1) * S * H] for b in pick]), layers, len(pick), S,
                   scales=scales).reshape(len(pick), S * H)
    for i, b in enumerate(pick):
        assert np.array_equal(got[b], want[i]), (b, _relerr(got[b], want[i]))


@pytest.mark.parametrize("rows,cols", [(300, 768), (37, 500)])
def test_plan_add_layernorm_fusion(cuda, rows, cols):
    # ADD_ACT -> LAYERNORM (-> QUANTIZE) runs as one residual layernorm when the
    # sum is not fetched: the LayerNorm output and its int8 copy are the same
    # bits as the separate ops give (the sum fetched), for the 768-wide and the
    # generic kernel
    from tpt_infer_b200 import graphs, synth

    a, r = synth.normal(rows * cols, 71), synth.normal(rows * cols, 72)
    g, b = synth.normal(cols, 73, 1.0, 0.1), synth.normal(cols, 74, 0.0, 0.1)
    p = graphs.Plan(cuda)
    ta, tr = p.tensor(graphs.F32, rows * cols), p.tensor(graphs.F32, rows * cols)
    ts, th = p.tensor(graphs.F32, rows * cols), p.tensor(graphs.F32, rows * cols)
    tq = p.tensor(graphs.I8, rows * cols)
    p.op(graphs.OP_ADD_ACT, ta, ts, in1=tr, dims=(rows * cols,))
    p.op(graphs.OP_LAYERNORM, ts, th, in1=p.const(g), in2=p.const(b), f0=1e-5, dims=(rows, cols))
    p.op(graphs.OP_QUANTIZE, th, tq, dims=(rows * cols,))
    p.finalize()
    p.calibrate(True)
    p.run({ta: a, tr: r}, [th])
    p.freeze()
    s_sep, h_sep, q_sep = p.run({ta: a, tr: r}, [ts, th, tq])  # the sum fetched: separate ops
    h_fused, q_fused = p.run({ta: a, tr: r}, [th, tq])         # fused
    assert np.array_equal(s_sep, (a + r).astype(np.float32))
    assert np.array_equal(h_fused, h_sep)
    n = rows * cols  # int8 outputs come back as raw bytes at the front of the buffer
    assert np.array_equal(np.frombuffer(q_fused.tobytes()[:n], np.int8), np.frombuffer(q_sep.tobytes()[:n], np.int8))
    assert np.array_equal(h_fused, O.layernorm((a + r).astype(np.float32), rows, cols, g, b, 1e-5))
    x = (a + r).astype(np.float64).reshape(rows, cols)
    ref = (x - x.mean(1, keepdims=True)) / np.sqrt(x.var(1, keepdims=True) + 1e-5) * g + b
    assert np.max(np.abs(h_fused.reshape(rows, cols) - ref)) < 1e-4
    p.close()


@pytest.mark.parametrize("B,S", [(2, 128), (1, 77), (3, 40), (1, 1), (16, 128), (64, 100)])
def test_attention_op(cuda, B, S):
    # the fused attention op alone against the oracle's MatMul / Softmax / MatMul
    from tpt_infer_b200 import graphs, synth

    qkv = synth.normal(B * S * 3 * 768, 45)
    pa = graphs.Plan(cuda)
    tq = pa.tensor(graphs.F32, qkv.size)
    to = pa.tensor(graphs.F32, B * S * 768)
    pa.op(graphs.OP_ATTENTION, tq, to, f0=0.125, dims=(B, S, 12, 64))
    pa.finalize()
    att = pa.run({tq: qkv}, [to])[0]
    pa.close()
    want = OM._attention(qkv, B, S, 12, 64, 0.125).ravel()
    assert np.array_equal(att, want)  # the defined evaluation order, bit for bit
    # and close to the plain MatMul / Softmax / MatMul composition
    ref = np.empty_like(want).reshape(B, S, 768)
    q3 = qkv.reshape(B, S, 3, 12, 64).astype(np.float64)
    for b in range(B):
        for h in range(12):
            sc = (q3[b, :, 0, h] * 0.125) @ q3[b, :, 1, h].T
            e = np.exp(sc - sc.max(1, keepdims=True))
            ref[b, :, h * 64:(h + 1) * 64] = (e / e.sum(1, keepdims=True)) @ q3[b, :, 2, h]
    assert np.max(np.abs(att - ref.ravel())) <= 1e-5 * (1 + np.max(np.abs(ref)))


@pytest.mark.parametrize("m", [96, 12])
def test_plan_fusion_rules(cuda, m):
    # LINEAR -> QUANTIZE runs as one requantizing launch only when the f32
    # tensor is not fetched; fetched or not, the int8 result is the same, and both
    # match the oracle's separate quantize (M = 12: the small-batch MMA kernel).
    import torch

    from tpt_infer_b200 import graphs, synth

    k, n = 512, 384
    x = synth.normal(m * k, 61)
    wq, ws = cuda.quantize_i8_symmetric_per_channel(synth.normal(n * k, 62, 0.0, 0.05), n)
    bias = synth.normal(n, 63, 0.0, 0.1)
    p = graphs.Plan(cuda)
    w = cuda.upload_i8(wq, ws, n, k)
    p.weights.append(w)
    tx, tq = p.tensor(graphs.F32, m * k), p.tensor(graphs.I8, m * k)
    ty, tyq = p.tensor(graphs.F32, m * n), p.tensor(graphs.I8, m * n)
    p.op(graphs.OP_QUANTIZE, tx, tq, dims=(m * k,))
    p.op(graphs.OP_LINEAR, tq, ty, in1=p.const(bias), w=w, act=graphs.ACT_RELU, dims=(m,))
    p.op(graphs.OP_QUANTIZE, ty, tyq, dims=(m * n,))
    p.finalize()
    p.calibrate(True)
    p.run({tx: x}, [ty])
    p.freeze()
    sx, sy = p.scales()

    class _Dev:  # a view of a plan tensor for torch
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|i1", "data": (ptr, False), "version": 3}

    def read_q():
        torch.cuda.synchronize()
        return torch.as_tensor(_Dev(p.ptr(tyq), m * n), device="cuda").cpu().numpy().copy()

    y_unfused = p.run({tx: x}, [ty])[0]  # the f32 tensor is fetched: separate QUANTIZE
    q_unfused = read_q()
    p.run({tx: x}, [])                   # not fetched: requantizing epilogue
    q_fused = read_q()
    assert np.array_equal(q_unfused, q_fused)
    xq = O.quantize_i8_static(x, sx)
    want_y = O.w8a8_gemm(xq, wq, m, n, k, sx, ws, bias, O.ACT_RELU)
    assert np.array_equal(y_unfused, want_y)
    assert np.array_equal(q_fused, O.quantize_i8_static(want_y, sy))
    p.close()


def test_resnet18_plan_bit_exact_batch256(cuda):
    # the benchmarked shape: batch 256 (TMA-im2col operands, several persistent
    # tile rounds per conv, every run-time fusion). The calibration over the whole
    # batch and the logits of all 256 images are bit-exact against the oracle's
    # replay of the same graph.
    from tpt_infer_b200 import graphs, synth

    B, IMG = 256, 3 * 224 * 224
    spec = graphs.resnet18_weights(cuda)
    p, x, logits = graphs.build_resnet18(cuda, B, spec)
    xcal = synth.normal(B * IMG, 31)
    p.calibrate(True)
    p.run({x: xcal}, [logits])
    p.freeze()
    cal = OM._Scales()
    OM.resnet18(xcal, spec, B, calib=cal)
    del xcal
    assert np.array_equal(p.scales(), cal.frozen())
    xin = synth.normal(B * IMG, 32)
    got, = p.run({x: xin}, [logits])
    p.close()
    for b0 in range(0, B, 64):
        want = OM.resnet18(xin[b0 * IMG:(b0 + 64) * IMG], spec, 64, scales=cal.frozen())
        g = got[b0 * 1000:(b0 + 64) * 1000]
        assert np.array_equal(g, want), (b0, _relerr(g, want))


def test_liveness_arena_same_results_smaller(cuda):
    # arena offsets by liveness (tpt_cuda_plan_reuse_arena): the same logits and
    # hidden states as the one-slot-per-tensor layout, in a fraction of the bytes
    from tpt_infer_b200 import graphs, synth

    spec = graphs.resnet18_weights(cuda)
    outs, sizes = [], []
    for reuse in (False, True):
        p, x, logits = graphs.build_resnet18(cuda, 4, spec, reuse=reuse)
        p.calibrate(True)
        p.run({x: synth.normal(4 * 3 * 224 * 224, 31)}, [logits])
        p.freeze()
        outs.append(p.run({x: synth.normal(4 * 3 * 224 * 224, 32)}, [logits])[0])
        sizes.append(p.arena_bytes())
        p.close()
    assert np.array_equal(outs[0], outs[1])
    assert sizes[1] * 3 <= sizes[0], sizes
    layers = graphs.bert_weights(cuda, layers=3)
    outs, sizes = [], []
    for reuse in (False, True):
        p, x, h = graphs.build_bert(cuda, 2, 64, layers, reuse=reuse)
        p.calibrate(True)
        p.run({x: synth.normal(2 * 64 * 768, 41)}, [h])
        p.freeze()
        p.set_graph(True)
        xin = synth.normal(2 * 64 * 768, 42)
        outs.append(p.run({x: xin}, [h])[0])
        outs.append(p.run({x: xin}, [h])[0])  # graph replay
        sizes.append(p.arena_bytes())
        p.close()
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    assert sizes[1] * 3 <= sizes[0], sizes


def test_liveness_arena_rejects_fetch_of_dropped_tensor(cuda):
    from tpt_infer_b200 import graphs
    from tpt_infer_b200.backend import OpError

    W = graphs.mlp_weights()
    p = graphs.Plan(cuda)
    x, h, y = p.tensor(graphs.F32, 2 * 784), p.tensor(graphs.F32, 2 * 512), p.tensor(graphs.F32, 2 * 10)
    p.op(graphs.OP_MATMUL, x, h, in1=p.const(W.w1), act=graphs.ACT_RELU, dims=(2, 784, 512))
    p.op(graphs.OP_MATMUL, h, y, in1=p.const(W.w2), dims=(2, 512, 10))
    p.reuse([x, y])
    p.finalize()
    xin = np.ones(2 * 784, np.float32)
    assert p.run({x: xin}, [y])[0].shape == (20,)
    with pytest.raises(OpError):
        p.run({x: xin}, [h])  # not kept: its bytes may hold a later tensor
    p.close()


def test_run_batches_equals_separate_runs(cuda):
    # tpt_cuda_plan_run_batches: consecutive batches with the next batch's H2D
    # overlapped (page-locked and pageable host buffers) give the outputs of
    # separate tpt_cuda_plan_run calls, also when called twice in a row
    import torch

    from tpt_infer_b200 import graphs, synth

    spec = graphs.resnet18_weights(cuda)
    p, x, logits = graphs.build_resnet18(cuda, 2, spec)
    p.calibrate(True)
    p.run({x: synth.normal(2 * 3 * 224 * 224, 31)}, [logits])
    p.freeze()
    xs = [synth.normal(2 * 3 * 224 * 224, 50 + s) for s in range(5)]
    want = [p.run({x: v}, [logits])[0] for v in xs]
    pinned = [torch.from_numpy(v).pin_memory().numpy() for v in xs]
    for src in (pinned, xs):
        for _ in range(2):
            got = p.run_batches([x], [[v] for v in src], [logits])
            for g, w in zip(got, want):
                assert np.array_equal(g[0], w)
    p.close()
