"""Pins the CPU oracle to tpt-infer's own known-answer tests.

Every case below replays a test from the reference repository (file:line
relative to its root) against the oracle's restatement, so the oracle that
checks the CUDA backend is itself checked against the reference's vectors.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O


# ---------------------------------------------------------------- naive.rs tests
def test_matmul_known_values():
    # crates/tpt-infer-ops/src/naive.rs:212-219
    out = O.matmul_naive([1, 2, 3, 4], (2, 2), [5, 6, 7, 8], (2, 2))
    assert out.tolist() == [19.0, 22.0, 43.0, 50.0]
    assert O.matmul([1, 2, 3, 4], (2, 2), [5, 6, 7, 8], (2, 2)).tolist() == [19.0, 22.0, 43.0, 50.0]


def test_matmul_shape_mismatch():
    # naive.rs:221-228
    with pytest.raises(O.OracleError) as e:
        O.matmul_naive(np.ones(6), (2, 3), np.ones(12), (4, 3), out_len=6)
    assert e.value.code == O.SHAPE_MISMATCH


def test_matmul_size_mismatch():
    # naive.rs:230-243: expected 6, actual 5
    with pytest.raises(O.OracleError) as e:
        O.matmul_naive(np.ones(5), (2, 3), np.ones(9), (3, 3), out_len=6)
    assert (e.value.code, e.value.expected, e.value.actual) == (O.SIZE_MISMATCH, 6, 5)


def test_conv2d_known_values():
    # naive.rs:245-260
    out = O.conv2d(np.arange(1, 10), (1, 1, 3, 3), [1, 0, 0, -1], (1, 1, 2, 2))
    assert out.tolist() == [-4.0, -4.0, -4.0, -4.0]


def test_conv2d_stride2_pad0_output_shape():
    # naive.rs:262-282
    out = O.conv2d(np.ones(64), (1, 1, 8, 8), np.ones(9), (1, 1, 3, 3), stride=(2, 2))
    assert out.size == 9 and np.all(out == 9.0)


def test_conv2d_channel_count_mismatch():
    # naive.rs:284-300
    with pytest.raises(O.OracleError) as e:
        O.conv2d(np.zeros(8), (1, 2, 2, 2), np.zeros(6), (1, 3, 2, 2), out_len=4)
    assert e.value.code == O.SHAPE_MISMATCH


def test_conv2d_zero_stride_rejected():
    # naive.rs:302-321
    with pytest.raises(O.OracleError) as e:
        O.conv2d(np.zeros(16), (1, 1, 4, 4), np.zeros(9), (1, 1, 3, 3), stride=(0, 1), out_len=16)
    assert e.value.code == O.INVALID


def test_relu_clips_negatives():
    # naive.rs:323-329
    assert O.relu([-1.0, 0.0, 1.0, 0.5]).tolist() == [0.0, 0.0, 1.0, 0.5]


def test_sigmoid_at_zero_is_half():
    # naive.rs:331-337
    assert abs(O.sigmoid([0.0])[0] - 0.5) < 1e-6


def test_gelu_at_zero_is_zero():
    # naive.rs:339-347
    out = O.gelu([0.0, -1.0, 1.0])
    assert out[0] == 0.0 and out[1] < 0.0 and out[2] > 0.0


def test_softmax_rows_sum_to_one():
    # naive.rs:349-359
    out = O.softmax([1.0, 2.0, 3.0, 1000.0, 1000.0, 1000.0], 3)
    assert abs(out[:3].sum() - 1.0) < 1e-5 and abs(out[3:].sum() - 1.0) < 1e-5
    assert 0.3 < out[3] < 0.34


def test_softmax_invalid_row_len():
    # naive.rs:361-367
    for rl in (0, 2):
        with pytest.raises(O.OracleError) as e:
            O.softmax([1.0, 2.0, 3.0], rl)
        assert e.value.code == O.INVALID


def test_elementwise_add_length_check():
    # naive.rs:369-380: expected 2, actual 1
    with pytest.raises(O.OracleError) as e:
        O.elementwise_add([1.0, 2.0], [1.0], out_len=2)
    assert (e.value.code, e.value.expected, e.value.actual) == (O.SIZE_MISMATCH, 2, 1)


# ---------------------------------------------------------------- dispatch.rs parity harness
def test_lcg_matches_reference_formula():
    # crates/tpt-infer-ops/src/dispatch.rs:274-282, recomputed in Python
    s, want = 1, []
    for _ in range(16):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        want.append(np.float32((s >> 8) / float(1 << 24)) * np.float32(2.0) - np.float32(1.0))
    assert np.array_equal(O.lcg_sym(16, 1), np.array(want, np.float32))


@pytest.mark.parametrize("m,k,n,sa,sb", [(3, 4, 5, 1, 2), (1, 784, 10, 3, 4), (13, 17, 19, 5, 6),
                                         (32, 64, 48, 7, 8)])
def test_avx_matmul_bit_identical_to_naive(m, k, n, sa, sb):
    # dispatch.rs:318-341 and :501-511: AVX2/AVX-512 backends agree with naive
    a, b = O.lcg_sym(m * k, sa), O.lcg_sym(k * n, sb)
    assert np.array_equal(O.matmul(a, (m, k), b, (k, n), threads=2), O.matmul_naive(a, (m, k), b, (k, n)))


# ---------------------------------------------------------------- quant.rs tests
def test_quantize_i8_symmetric_doc_example():
    # crates/tpt-infer-quantize/src/quant.rs:18-24
    q, s = O.quantize_i8_symmetric([-1.0, 0.0, 1.0])
    assert q.tolist() == [-127, 0, 127]
    assert abs(s - 1.0 / 127.0) < 1e-6


def test_i8_symmetric_roundtrip_unit_range():
    # quant.rs:210-219
    data = np.array([i / 50.0 for i in range(-50, 51)], np.float32)
    q, s = O.quantize_i8_symmetric(data)
    assert np.all(np.abs(q.astype(np.float32) * s - data) < 0.01)


def test_i8_asymmetric_roundtrip():
    # quant.rs:221-229
    data = np.array([0.0, 0.25, 0.5, 1.0, 2.0], np.float32)
    q, s, zp = O.quantize_i8_asymmetric(data)
    d = (q.astype(np.float32) - np.float32(zp)) * s
    assert np.all(np.abs(d - data) < 0.01)


def test_per_channel_not_worse_than_per_tensor():
    # quant.rs:231-259
    data = np.zeros(64, np.float32)
    data[:32] = np.arange(32, dtype=np.float32) / np.float32(31.0) * np.float32(10.0)
    data[32:] = (np.arange(32, 64, dtype=np.float32) - np.float32(32.0)) / np.float32(31.0) * np.float32(0.1)
    qt, st = O.quantize_i8_symmetric(data)
    qc, sc = O.quantize_i8_symmetric_per_channel(data, 2)
    assert sc.size == 2
    err_t = np.abs(qt.astype(np.float32) * st - data).sum()
    err_c = sum(abs(float(qc[i]) * float(sc[i // 32]) - float(data[i])) for i in range(64))
    assert err_c <= err_t + 1e-5


def test_i4_pack_unpack_roundtrip():
    # quant.rs:261-272 and the doc example quant.rs:116-122
    vals = np.arange(-8, 8, dtype=np.int8)
    p = O.pack_i4(vals)
    assert p.size == 8 and np.array_equal(O.unpack_i4(p, 16), vals)
    odd = np.array([1, -1, 7], np.int8)
    p = O.pack_i4(odd)
    assert p.size == 2 and np.array_equal(O.unpack_i4(p, 3), odd)
    p = O.pack_i4([-8, 7, 0, 1])
    assert p.size == 2 and O.unpack_i4(p, 4).tolist() == [-8, 7, 0, 1]
    # low nibble first: byte = (hi & 0xF) << 4 | (lo & 0xF)
    assert p.tolist() == [0x78, 0x10]


def test_i4_sign_extension():
    # quant.rs:274-279
    vals = np.array([-8, -1, 0, 7], np.int8)
    assert np.array_equal(O.unpack_i4(O.pack_i4(vals), 4), vals)


def test_i4_quant_roundtrip_loose():
    # quant.rs:281-290
    data = np.array([i / 20.0 for i in range(-20, 21)], np.float32)
    p, s = O.quantize_i4_symmetric(data)
    q = O.unpack_i4(p, data.size)
    assert np.all(np.abs(q.astype(np.float32) * s - data) < 0.1)
    assert q.min() >= -7  # -8 is never produced (quant.rs:182)


def test_pack_i4_rejects_out_of_range():
    # quant.rs:292-296 (panics in the reference)
    with pytest.raises(O.OracleError) as e:
        O.pack_i4([8])
    assert e.value.code == O.INVALID


# ---------------------------------------------------------------- dequant.rs tests
def test_dequant_symmetric_roundtrip():
    # dequant.rs:77-85 and the doc example :9-12
    data = np.array([0.0, 1.0, -1.0, 0.5], np.float32)
    q, s = O.quantize_i8_symmetric(data)
    assert np.all(np.abs(O.dequantize_i8_symmetric(q, s) - data) < 0.01)
    assert abs(O.dequantize_i8_symmetric([0, 127], np.float32(1.0 / 127.0))[1] - 1.0) < 1e-6


def test_dequant_asymmetric_roundtrip():
    # dequant.rs:87-95
    data = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    q, s, zp = O.quantize_i8_asymmetric(data)
    assert np.all(np.abs(O.dequantize_i8_asymmetric(q, s, zp) - data) < 0.01)


def test_dequant_per_channel_roundtrip():
    # dequant.rs:97-106 ((i as f32).sin())
    data = np.sin(np.arange(64, dtype=np.float32)).astype(np.float32)
    q, sc = O.quantize_i8_symmetric_per_channel(data, 4)
    d = O.dequantize_i8_symmetric_per_channel(q, sc)
    assert d.size == 64 and np.all(np.abs(d - data) < 0.02)


def test_dequant_i4_roundtrip():
    # dequant.rs:108-117
    data = np.array([i / 16.0 for i in range(-16, 17)], np.float32)
    p, s = O.quantize_i4_symmetric(data)
    d = O.dequantize_i4_symmetric(p, data.size, s)
    assert d.size == data.size and np.all(np.abs(d - data) < 0.1)


def test_dequant_i4_per_channel_roundtrip():
    # dequant.rs:119-134
    data = np.zeros(64, np.float32)
    data[:32] = np.arange(32, dtype=np.float32) / np.float32(31.0)
    data[32:] = (np.arange(32, 64, dtype=np.float32) - np.float32(32.0)) / np.float32(31.0) * np.float32(0.5)
    p, sc = O.quantize_i4_symmetric_per_channel(data, 2)
    d = O.dequantize_i4_symmetric_per_channel(p, 32, sc)
    assert d.size == 64 and np.all(np.abs(d - data) < 0.1)


# ---------------------------------------------------------------- ptq.rs tests
def _ptq_weights():
    # ptq.rs:349: (i as f32 / 32.0) - 0.5 for a [4, 8] initializer
    return (np.arange(32, dtype=np.float32) / np.float32(32.0) - np.float32(0.5)).astype(np.float32)


def test_ptq_quantizes_matmul_weights():
    # ptq.rs:358-375: per-channel over axis 0 -> 4 scales, 32 bytes, round trip < 0.01
    w = _ptq_weights()
    q, sc = O.quantize_i8_symmetric_per_channel(w, 4)
    assert sc.size == 4 and q.size == 32
    assert np.all(np.abs(O.dequantize_i8_symmetric_per_channel(q, sc) - w) < 0.01)


def test_ptq_int4_path():
    # ptq.rs:377-391: 32 elements -> 16 bytes; dequantize back to 32 values
    p, sc = O.quantize_i4_symmetric_per_channel(_ptq_weights(), 4)
    assert p.size == 16
    assert O.dequantize_i4_symmetric_per_channel(p, 8, sc).size == 32


def test_quantized_matmul_matches_f32_approx():
    # ptq.rs:409-436
    m, k, n = 4, 8, 4
    a = (np.sin(np.arange(m * k, dtype=np.float32)) * np.float32(0.5)).astype(np.float32)
    b = (np.cos(np.arange(k * n, dtype=np.float32)) * np.float32(0.5)).astype(np.float32)
    ref = O.matmul_naive(a, (m, k), b, (k, n))
    aq, sa = O.quantize_i8_symmetric(a)
    bq, sb = O.quantize_i8_symmetric(b)
    q = O.quantized_matmul_i8(aq, (m, k), sa, bq, (k, n), [sb])
    assert np.all(np.abs(ref - q) < 0.05)


def test_per_channel_w8a8_reduces_to_reference_for_uniform_scale():
    # The per-output-channel extension equals ptq.rs:293-324 when every
    # channel shares the scale and there is no bias.
    m, k, n = 5, 33, 7
    a = O.lcg_sym(m * k, 11)
    b = O.lcg_sym(k * n, 12)
    aq, sa = O.quantize_i8_symmetric(a)
    bq, sb = O.quantize_i8_symmetric(b)
    want = O.quantized_matmul_i8(aq, (m, k), sa, bq, (k, n), [sb])
    wt = bq.reshape(k, n).T.copy()
    got = O.w8a8_gemm(aq, wt, m, n, k, sa, np.full(n, sb, np.float32))
    assert np.array_equal(got, want)
    got_ref = O.w8a8_gemm_refloop(aq, bq, m, n, k, sa, np.full(n, sb, np.float32), None, m, 2)
    assert np.array_equal(got_ref, want)


# ---------------------------------------------------------------- runtime kernels.rs
def test_max_pool_known_values():
    # crates/tpt-infer-runtime/src/kernels.rs:648-663: 4x4 arange, 2x2 s2 -> [5,7,13,15]
    out = O.max_pool2d(np.arange(16, dtype=np.float32), 1, 1, 4, 4, (2, 2), (2, 2), (0, 0))
    assert out.tolist() == [5.0, 7.0, 13.0, 15.0]


def test_max_pool_padding_is_neg_inf_and_avgpool_excludes_pad():
    # kernels.rs:271-325 / :335-390 semantics
    x = -np.ones(4, np.float32)
    assert np.all(O.max_pool2d(x, 1, 1, 2, 2, (3, 3), (1, 1), (1, 1)) == -1.0)
    x = np.ones(4, np.float32)
    assert np.all(O.average_pool2d(x, 1, 1, 2, 2, (3, 3), (1, 1), (1, 1)) == 1.0)


def test_conv_plus_bias_exact():
    # crates/tpt-infer-runtime/src/tests.rs:294-322: conv [1,0,0,-1] over 1..=9
    # gives [-4]*4, then the runtime's broadcast bias add (+5) gives [1]*4
    y = O.conv2d(np.arange(1, 10), (1, 1, 3, 3), [1, 0, 0, -1], (1, 1, 2, 2))
    y = O.add_bias_nchw(y, 1, 1, 4, [5.0])
    assert y.tolist() == [1.0, 1.0, 1.0, 1.0]


def test_layernorm_definition():
    x = O.lcg_sym(3 * 16, 9)
    g, b = np.ones(16, np.float32), np.zeros(16, np.float32)
    y = O.layernorm(x, 3, 16, g, b).reshape(3, 16)
    assert np.allclose(y.mean(1), 0, atol=1e-6)
    assert np.allclose((y * y).mean(1), 1, atol=1e-3)


def test_normal_generator_moments():
    z = O.normal(200000, 1234, 0.0, 1.0)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01
    u = O.lcg_uniform(100000, 5)
    assert u.min() >= 0.0 and u.max() < 1.0 and abs(float(u.mean()) - 0.5) < 0.01


def test_requant_rule():
    # quant.rs:35-36 rule applied to one value: half away from zero, clamp
    assert O.requant_i8(2.5, 1.0) == 3 and O.requant_i8(-2.5, 1.0) == -3
    assert O.requant_i8(1e9, 1.0) == 127 and O.requant_i8(-1e9, 1.0) == -127
    assert O.requant_i8(math.nan, 1.0) == 0


def test_product_synth_matches_oracle_generators():
    # tpt_infer_b200.synth restates the same LCG stream (bit-identical uniform)
    # and Box-Muller (same formula; numpy vs libm transcendental last bits only)
    from tpt_infer_b200 import synth

    for n, seed in ((1, 3), (17, 4), (100001, 5)):
        assert np.array_equal(synth.uniform(n, seed), O.lcg_uniform(n, seed))
        a, b = synth.normal(n, seed, 0.5, 2.0), O.normal(n, seed, 0.5, 2.0)
        assert np.max(np.abs(a - b)) <= 1e-6 * (1 + np.max(np.abs(b)))


# ---------------------------------------------------------------- ONNX Gemm (defined here)
def test_gemm_known_values():
    # the loader maps Gemm to MatMul (registry.rs:21); the oracle states the full
    # semantics: alpha * A B^T + beta * C with C broadcast over rows
    y = O.gemm([1, 2, 3, 4], 2, 2, [5, 6, 7, 8], 2, c=[1, 2], alpha=2.0, beta=0.5, trans_b=True)
    assert y.tolist() == [34.5, 47.0, 78.5, 107.0]
    # no C, no transposes, alpha = 1: MatMul (naive.rs:212-219)
    assert O.gemm([1, 2, 3, 4], 2, 2, [5, 6, 7, 8], 2).tolist() == [19.0, 22.0, 43.0, 50.0]
    # trans_a: A stored [k, m]
    assert O.gemm([1, 3, 2, 4], 2, 2, [5, 6, 7, 8], 2, trans_a=True).tolist() == [19.0, 22.0, 43.0, 50.0]


def test_gemm_errors():
    with pytest.raises(O.OracleError) as e:
        O.gemm(np.ones(5), 2, 3, np.ones(9), 3)
    assert e.value.code == O.SIZE_MISMATCH
    with pytest.raises(O.OracleError) as e:
        O.gemm(np.ones(6), 2, 3, np.ones(9), 3, c=np.ones(4))
    assert e.value.code == O.SHAPE_MISMATCH


# ---------------------------------------------------------------- runtime kernels (kernels.rs tests)
def test_runtime_binary_kats():
    # kernels.rs:592-625: broadcast add, equal-shape mul/sub/div
    assert O.binary(O.BIN_ADD, [1, 2], [2, 1], [10, 20, 30], [1, 3]).tolist() == [11, 21, 31, 12, 22, 32]
    assert O.binary(O.BIN_MUL, [1, 4], [2], [3, 2], [2]).tolist() == [3, 8]
    assert O.binary(O.BIN_SUB, [1, 4], [2], [3, 2], [2]).tolist() == [-2, 2]
    d = O.binary(O.BIN_DIV, [1, 4], [2], [3, 2], [2])
    assert abs(d[0] - 1 / 3) < 1e-6 and d[1] == 2.0
    # add_inplace_broadcast_bias (:627-632)
    assert O.binary(O.BIN_ADD, [1, 2, 3, 4, 5, 6], [2, 3], [10, 20], [2, 1]).tolist() == [11, 12, 13, 24, 25, 26]
    assert O.broadcast_shape([3], [4]) is None  # binary_incompatible_broadcast_errors


def test_runtime_pool_batchnorm_transpose_concat_kats():
    assert O.max_pool2d(np.arange(16, dtype=np.float32), 1, 1, 4, 4, (2, 2), (2, 2), (0, 0)).tolist() == \
        [5, 7, 13, 15]
    g = O.average_pool2d([1, 2, 3, 6], 1, 1, 2, 2, (2, 2), (1, 1), (0, 0))
    assert abs(g[0] - 3.0) < 1e-6
    # batch_norm_channel_mode (kernels.rs:698-717)
    y = O.batch_norm([1, 2, 3, 4], [1, 2, 1, 2], [2, 1], [0, 10], [1, 3], [1, 1], 0.0)
    assert y.tolist() == [0, 2, 10, 11]
    # transpose_swaps_axes (:729-735)
    assert O.transpose([1, 2, 3, 4, 5, 6], [2, 3], [1, 0]).tolist() == [1, 4, 2, 5, 3, 6]
    # concat_streams_operands (:745-755): two [1,1,2] on axis 1
    out, od = O.concat([[1, 2], [3, 4]], [[1, 1, 2], [1, 1, 2]], 1)
    assert out.tolist() == [1, 2, 3, 4] and od == [1, 2, 2]


def test_runtime_sqrt_through_batch_norm():
    # sqrt_f32_matches_known_values (kernels.rs:719-727), seen through the
    # element mode of batch_norm (:468-473): x = 1, mean = 0, scale = 1,
    # bias = 0, eps = 0 gives out = 1 / sqrt_f32(var)
    var = np.array([0.0, 1.0, 4.0, 2.0, -1.0, np.inf], np.float32)
    y = O.batch_norm(np.ones(6), [6], np.ones(6), np.zeros(6), np.zeros(6), var, 0.0)
    assert y[0] == np.inf                      # sqrt_f32(0) == 0
    assert abs(y[1] - 1.0) < 1e-6              # sqrt_f32(1) ~ 1
    assert abs(y[2] - 0.5) < 1e-5 / 4          # sqrt_f32(4) ~ 2
    assert abs(1.0 / y[3] - np.sqrt(2.0)) < 1e-5  # sqrt_f32(2) ~ SQRT_2
    assert np.isnan(y[4])                      # sqrt_f32(-1) is NaN
    assert y[5] == 0.0                         # sqrt_f32(inf) == inf


def test_runtime_dispatch_coverage_graph_kats():
    # crates/tpt-infer-runtime/src/tests.rs:209-260 (dispatch_operator_coverage),
    # replayed through the oracle's graph executor
    from oracle import graph_exec
    from tpt_infer_b200 import lowering as L

    g = L.ComputationGraph()
    x = g.add_input([1, 1, 4, 4], "x")
    mp = g.add_node(L.Operator.max_pool2d([2, 2], [2, 2], [0, 0]), [x], [1, 1, 2, 2])
    cat = g.add_node(L.Operator.concat(1), [mp, mp], [1, 2, 2, 2])
    flat = g.add_node(L.Operator.flatten(1), [cat], [1, 8])
    tr = g.add_node(L.Operator.transpose([0, 1, 3, 2]), [mp], [1, 1, 2, 2])
    outs = [flat, tr]
    for k in ("sub", "mul", "div", "sigmoid", "gelu"):
        op = getattr(L.Operator, k)()
        ins = [mp, mp] if k in ("sub", "mul", "div") else [mp]
        outs.append(g.add_node(op, ins, [1, 1, 2, 2]))
    for o in outs:
        g.mark_output(o)
    r = graph_exec.execute_graph(g, [np.arange(16, dtype=np.float32)])
    assert r[0].ravel().tolist() == [5, 7, 13, 15, 5, 7, 13, 15]
    assert r[1].ravel().tolist() == [5, 13, 7, 15]
    assert r[2].ravel().tolist() == [0, 0, 0, 0]
    mpv = np.array([5, 7, 13, 15], np.float32)
    assert np.all(np.abs(r[3].ravel() - mpv * mpv) < 1e-4) and np.all(np.abs(r[4].ravel() - 1) < 1e-5)
    assert np.all((r[5] >= 0) & (r[5] <= 1)) and np.all(np.isfinite(r[6]))


def test_runtime_conv_bias_kat():
    # tests.rs:294-322 (conv_bias_is_added): 3x3 input of ones * [[1,0],[0,-1]] + bias 1 = ones
    from oracle import graph_exec
    from tpt_infer_b200 import lowering as L

    g = L.ComputationGraph()
    x = g.add_input([1, 1, 3, 3], "x")
    w = g.add_weight("w", [1, 1, 2, 2], [1.0, 0.0, 0.0, -1.0])
    b = g.add_weight("b", [1], [1.0])
    y = g.add_node(L.Operator.conv2d([1, 1], [0, 0]), [x, w, b], [1, 1, 2, 2])
    g.mark_output(y)
    assert graph_exec.execute_graph(g, [np.ones(9, np.float32)])[0].ravel().tolist() == [1, 1, 1, 1]


def test_deterministic_exp_and_gelu_accuracy():
    # det_math.cuh restated: exp_det within 2 ulp of e^x on [-87, 88], 0 below,
    # NaN kept; gelu_det within 1e-6 (1 + |y|) of the reference tanh formula
    x = np.linspace(-87, 88, 400001).astype(np.float32)
    e = O.exp_det(x)
    ref = np.exp(x.astype(np.float64))
    assert np.max(np.abs(e - ref) / ref) < 2 * 2.0 ** -24
    assert O.exp_det([-87.5, -1000.0])[0] == 0.0 and np.isnan(O.exp_det([np.nan])[0])
    g = O.normal(200001, 5, 0.0, 4.0)
    assert np.max(np.abs(O.gelu_det(g) - O.gelu(g)) / (1 + np.abs(O.gelu(g)))) < 1e-6
    assert O.gelu_det([0.0])[0] == 0.0 and np.isnan(O.gelu_det([np.nan])[0])


def test_dispatch_softmax_and_gelu_cases():
    # softmax_matches_naive_and_rows_sum_to_one (dispatch.rs:450-467): lcg(14,
    # seed 14) as 2 rows of 7, each row summing to 1 within 1e-5
    sm = O.softmax(O.lcg_sym(14, 14), 7)
    assert np.all(np.abs(sm.reshape(2, 7).sum(axis=1) - 1.0) < 1e-5)
    # gelu_matches_scalar_reference (dispatch.rs:482-497): lcg(50, seed 16)
    # against the tanh formula in f32, with assert_close's 1e-4 (1 + |want|)
    # (dispatch.rs:284-295); the fused epilogues' deterministic GELU meets it too
    x = O.lcg_sym(50, 16)
    f = np.float32
    inner = f(0.7978846) * (x + f(0.044715) * x * x * x)
    want = f(0.5) * x * (f(1.0) + np.tanh(inner))
    for got in (O.gelu(x), O.gelu_det(x)):
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - want) <= 1e-4 * (1.0 + np.abs(want)))


def test_runtime_batch_norm_softmax_graph_kats():
    # crates/tpt-infer-runtime/src/tests.rs, replayed through the oracle's graph walk
    from oracle import graph_exec
    from tpt_infer_b200 import lowering as L

    # batch_norm_dispatches (tests.rs:323-356): parameters as initializers
    g = L.ComputationGraph()
    x = g.add_input([1, 2, 1, 2], "x")
    ps = [g.add_weight(nm, [2], v) for nm, v in (("scale", [2.0, 1.0]), ("bias", [0.0, 10.0]),
                                                ("mean", [1.0, 3.0]), ("var", [1.0, 1.0]))]
    y = g.add_node(L.Operator.batch_norm(0.0), [x] + ps, [1, 2, 1, 2])
    g.mark_output(y)
    assert graph_exec.execute_graph(g, [np.array([1, 2, 3, 4], np.float32)])[0].ravel().tolist() == [0, 2, 10, 11]
    # softmax_non_last_axis_is_unsupported (tests.rs:358-370)
    g = L.ComputationGraph()
    x = g.add_input([2, 3], "x")
    y = g.add_node(L.Operator.softmax(0), [x], [2, 3])
    g.mark_output(y)
    with pytest.raises(NotImplementedError):
        graph_exec.execute_graph(g, [np.ones(6, np.float32)])
    # selected_backend_executes (tests.rs:372-400): relu then softmax, sum 1, argmax 3
    g = L.ComputationGraph()
    x = g.add_input([1, 4], "x")
    h = g.add_node(L.Operator.relu(), [x], [1, 4])
    y = g.add_node(L.Operator.softmax(-1), [h], [1, 4])
    g.mark_output(y)
    out = graph_exec.execute_graph(g, [np.array([-1.0, 2.0, -3.0, 4.0], np.float32)])[0].ravel()
    assert abs(out.sum() - 1.0) < 1e-4 and int(np.argmax(out)) == 3 and out[0] == out[2]


def test_lowering_graph_errors_before_device_work():
    # exec.rs:833-846 (unmarked_graph_reports_no_outputs) and :848-864
    # (custom_op_is_unsupported): both reported before the lowering touches a
    # device, so no backend is needed here
    from tpt_infer_b200 import lowering as L

    g = L.ComputationGraph()
    x = g.add_input([4], "x")
    g.add_node(L.Operator.relu(), [x], [4])
    with pytest.raises(L.NoOutputs):
        L.lower(g, None)
    g = L.ComputationGraph()
    x = g.add_input([4], "x")
    g.mark_output(g.add_node(L.Operator.custom("Erf"), [x], [4]))
    with pytest.raises(L.UnsupportedOp) as e:
        L.lower(g, None)
    assert e.value.name == "Erf"


def test_graph_rank_limit_and_idempotent_outputs():
    # crates/tpt-infer-graph/src/graph.rs:538-542 (node_rank_too_large) and
    # :630-636 (mark_output_idempotent); unknown nodes are rejected
    from tpt_infer_b200 import lowering as L
    from tpt_infer_b200.backend import OpError

    g = L.ComputationGraph()
    with pytest.raises(OpError):
        g.add_input([1] * 9, "x")
    x = g.add_input([1] * 8, "x")
    r = g.add_node(L.Operator.relu(), [x], [1] * 8)
    g.mark_output(r)
    g.mark_output(r)
    assert g.outputs == [r]
    with pytest.raises(OpError):
        g.mark_output(5)
    with pytest.raises(OpError):
        g.add_node(L.Operator.relu(), [7], [1])
