"""Committed golden vectors (tests/golden/golden.npz, made by
tests/golden/make_golden.py from the oracle).

CPU: the oracle, rebuilt here, reproduces every fixture bit for bit -- inputs
(the seeded generators) and outputs -- so the checker cannot drift.
GPU: the device path, through the C ABI, matches the committed outputs: bit-exact
for integer work and for MatMul/Conv2d/W8A8; 1e-5*(1+|y|) for the transcendental
element ops; 1e-3 x max|y| / 127 for W4.
"""
import importlib.util
import os

import numpy as np
import pytest

from oracle import oracle as O

_HERE = os.path.dirname(os.path.abspath(__file__))
_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(_HERE, "golden", "make_golden.py"))
G = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(G)

GOLD = G.load()


@pytest.mark.parametrize("name", sorted(GOLD))
def test_oracle_reproduces_golden(name):
    fresh = G.cases()[name]
    assert sorted(fresh) == sorted(GOLD[name])
    for key, want in GOLD[name].items():
        got = np.asarray(fresh[key])
        assert got.dtype == want.dtype and got.shape == want.shape, key
        assert np.array_equal(got, want), f"{name}.{key} drifted"


def _close(got, want, rel=1e-5):
    assert np.all(np.abs(got - want) <= rel * (1.0 + np.abs(want)))


@pytest.mark.gpu
def test_golden_backend_ops(cuda):
    g = GOLD["matmul"]
    m, k, n = (int(v) for v in g["in_shape"])
    y = np.empty(m * n, np.float32)
    cuda.matmul(g["in_a"], (m, k), g["in_b"], (k, n), y)
    assert np.array_equal(y, g["out_y"])

    g = GOLD["gemm"]
    m, k, n = (int(v) for v in g["in_shape"])
    y = cuda.gemm(g["in_a"], m, k, g["in_b"], n, c=g["in_c"], alpha=0.5, beta=2.0, trans_b=True)
    assert np.array_equal(y, g["out_y"])

    from tpt_infer_b200 import Conv2dOptions
    g = GOLD["conv2d"]
    bn, c, h, w, co, kh, kw, sh, sw, ph, pw = (int(v) for v in g["in_shape"])
    y = np.empty(g["out_y"].size, np.float32)
    cuda.conv2d(g["in_x"], (bn, c, h, w), g["in_w"], (co, c, kh, kw), y,
                Conv2dOptions.with_stride_padding(sh, sw, ph, pw))
    assert np.array_equal(y, g["out_y"])

    g = GOLD["eltwise"]
    out = np.empty(g["in_a"].size, np.float32)
    cuda.elementwise_add(g["in_a"], g["in_b"], out)
    assert np.array_equal(out, g["out_add"])
    cuda.relu(g["in_a"], out)
    assert np.array_equal(out, g["out_relu"])
    cuda.sigmoid(g["in_a"], out)
    _close(out, g["out_sigmoid"])
    cuda.gelu(g["in_a"], out)
    _close(out, g["out_gelu"])

    g = GOLD["softmax"]
    out = np.empty(g["in_x"].size, np.float32)
    cuda.softmax(g["in_x"], out, int(g["in_row_len"][0]))
    _close(out, g["out_y"])


@pytest.mark.gpu
def test_golden_quantize(cuda):
    g = GOLD["quant_i8"]
    q, s = cuda.quantize_i8_symmetric(g["in_sym"])
    assert np.array_equal(q, g["out_sym_q"]) and s == g["out_sym_scale"][0]
    q, s, z = cuda.quantize_i8_asymmetric(g["in_asym"])
    assert np.array_equal(q, g["out_asym_q"]) and s == g["out_asym_scale"][0] and z == g["out_asym_zp"][0]
    q, s = cuda.quantize_i8_symmetric_per_channel(g["in_pc"], int(g["in_pc_rows"][0]))
    assert np.array_equal(q, g["out_pc_q"]) and np.array_equal(s, g["out_pc_scales"])

    g = GOLD["quant_i4"]
    assert np.array_equal(cuda.pack_i4(g["in_vals"]), g["out_packed"])
    assert np.array_equal(cuda.unpack_i4(g["out_packed"], g["in_vals"].size), g["in_vals"])
    p, s = cuda.quantize_i4_symmetric_per_channel(g["in_pc"], int(g["in_pc_rows"][0]))
    assert np.array_equal(p, g["out_pc_packed"]) and np.array_equal(s, g["out_pc_scales"])
    d = cuda.dequantize_i4_symmetric_per_channel(g["out_pc_packed"], g["in_pc"].size // s.size, s)
    assert np.array_equal(d, g["out_pc_dequant"])


@pytest.mark.gpu
def test_golden_gemms(cuda):
    g = GOLD["qmatmul_i8"]
    m, k, n = (int(v) for v in g["in_shape"])
    y = np.empty(m * n, np.float32)
    cuda.quantized_matmul_i8(g["in_a"], (m, k), g["in_scales"][0], g["in_b"], (k, n), [g["in_scales"][1]], y)
    assert np.array_equal(y, g["out_y"])

    g = GOLD["w8a8"]
    m, n, k = (int(v) for v in g["in_shape"])
    w = cuda.upload_i8(g["in_w"], g["in_w_scales"], n, k)
    y = cuda.w8a8_gemm(g["in_a"], m, k, g["in_a_scale"][0], w, g["in_bias"], O.ACT_RELU)
    w.free()
    assert np.array_equal(y, g["out_y"])

    g = GOLD["w4"]
    m, n, k = (int(v) for v in g["in_shape"])
    w = cuda.upload_i4(g["in_w"], g["in_w_scales"], n, k)
    y = cuda.w4_gemm(g["in_x"], m, k, w, g["in_bias"], O.ACT_GELU)
    w.free()
    want = g["out_y"]
    assert np.max(np.abs(y - want)) <= max(1e-3 * np.max(np.abs(want)) / 127.0, 1e-6)
