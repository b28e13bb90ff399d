"""Generates tests/golden/golden.npz: seeded inputs and the oracle's outputs for
the Backend/quantize entry points, at sizes small enough to commit.

The oracle is pinned to tpt-infer's own known-answer tests in
tests/test_oracle_kat.py; these fixtures freeze its outputs on larger seeded
inputs so that (a) any drift in the oracle build shows up on CPU
(tests/test_golden.py re-runs it and compares bit for bit) and (b) the device
path is compared against committed vectors, not only against a live oracle.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402


def cases():
    """name -> dict of arrays. Inputs are prefixed ``in_``, outputs ``out_``."""
    c = {}
    # f32 MatMul (naive.rs:13-33), ragged shape
    a = O.lcg_sym(17 * 31, 101)
    b = O.lcg_sym(31 * 23, 102)
    c["matmul"] = dict(in_a=a, in_b=b, in_shape=np.array([17, 31, 23]),
                       out_y=O.matmul_naive(a, (17, 31), b, (31, 23)))
    # ONNX Gemm (the semantics the loader drops, registry.rs:21): alpha A B^T + beta C[n]
    ga, gb, gc = O.lcg_sym(9 * 20, 121), O.lcg_sym(13 * 20, 122), O.lcg_sym(13, 123)
    c["gemm"] = dict(in_a=ga, in_b=gb, in_c=gc, in_shape=np.array([9, 20, 13]),
                     out_y=O.gemm(ga, 9, 20, gb, 13, c=gc, alpha=0.5, beta=2.0, trans_b=True))
    # Conv2d (naive.rs:36-92), stride 2, pad 1
    x = O.lcg_sym(2 * 3 * 9 * 9, 103)
    w = O.lcg_sym(4 * 3 * 3 * 3, 104)
    c["conv2d"] = dict(in_x=x, in_w=w, in_shape=np.array([2, 3, 9, 9, 4, 3, 3, 2, 2, 1, 1]),
                       out_y=O.conv2d(x, (2, 3, 9, 9), w, (4, 3, 3, 3), (2, 2), (1, 1)))
    # element ops (naive.rs:95-125)
    e = O.lcg_sym(1031, 105) * np.float32(6.0)
    f = O.lcg_sym(1031, 106)
    c["eltwise"] = dict(in_a=e, in_b=f, out_add=O.elementwise_add(e, f), out_relu=O.relu(e),
                        out_sigmoid=O.sigmoid(e), out_gelu=O.gelu(e))
    s = O.lcg_sym(7 * 33, 107) * np.float32(8.0)
    c["softmax"] = dict(in_x=s, in_row_len=np.array([33]), out_y=O.softmax(s, 33))
    # quantize crate (quant.rs)
    q = O.lcg_sym(4099, 108) * np.float32(3.0)
    qs, ss = O.quantize_i8_symmetric(q)
    qa, sa, za = O.quantize_i8_asymmetric(O.lcg_uniform(1000, 109) * np.float32(5.0) - np.float32(1.0))
    qc, sc = O.quantize_i8_symmetric_per_channel(O.lcg_sym(37 * 53, 110), 37)
    c["quant_i8"] = dict(in_sym=q, out_sym_q=qs, out_sym_scale=np.array([ss], np.float32),
                         in_asym=O.lcg_uniform(1000, 109) * np.float32(5.0) - np.float32(1.0),
                         out_asym_q=qa, out_asym_scale=np.array([sa], np.float32), out_asym_zp=np.array([za]),
                         in_pc=O.lcg_sym(37 * 53, 110), in_pc_rows=np.array([37]), out_pc_q=qc, out_pc_scales=sc)
    v = (np.floor(O.lcg_uniform(101, 111) * np.float32(16.0)) - 8).astype(np.int8)
    p4, s4 = O.quantize_i4_symmetric_per_channel(O.lcg_sym(24 * 64, 112), 24)
    c["quant_i4"] = dict(in_vals=v, out_packed=O.pack_i4(v), in_pc=O.lcg_sym(24 * 64, 112),
                         in_pc_rows=np.array([24]), out_pc_packed=p4, out_pc_scales=s4,
                         out_pc_dequant=O.dequantize_i4_symmetric_per_channel(p4, 64, s4))
    # quantized_matmul_i8 (ptq.rs:293-324): B [k, n], per-tensor scale
    ai = (np.floor(O.lcg_uniform(9 * 40, 113) * np.float32(255.0)) - 127).astype(np.int8)
    bi = (np.floor(O.lcg_uniform(40 * 11, 114) * np.float32(255.0)) - 127).astype(np.int8)
    c["qmatmul_i8"] = dict(in_a=ai, in_b=bi, in_shape=np.array([9, 40, 11]),
                           in_scales=np.array([0.0125, 0.03], np.float32),
                           out_y=O.quantized_matmul_i8(ai, (9, 40), np.float32(0.0125), bi, (40, 11),
                                                       np.array([0.03], np.float32)))
    # W8A8 GEMM, per-channel weight scale, bias, ReLU (ragged M, N, K)
    m, n, k = 33, 50, 96
    xa = O.lcg_sym(m * k, 115) * np.float32(2.0)
    aq, a_scale = O.quantize_i8_symmetric(xa)
    wq, wsc = O.quantize_i8_symmetric_per_channel(O.lcg_sym(n * k, 116) * np.float32(0.1), n)
    bias = O.lcg_sym(n, 117)
    c["w8a8"] = dict(in_a=aq, in_a_scale=np.array([a_scale], np.float32), in_w=wq, in_w_scales=wsc, in_bias=bias,
                     in_shape=np.array([m, n, k]),
                     out_y=O.w8a8_gemm(aq, wq, m, n, k, a_scale, wsc, bias, O.ACT_RELU))
    # W4 GEMM (dequant.rs:56-71 + matmul), bias, GELU
    m, n, k = 5, 40, 64
    x4 = O.lcg_sym(m * k, 118)
    w4, w4s = O.quantize_i4_symmetric_per_channel(O.lcg_sym(n * k, 119) * np.float32(0.1), n)
    b4 = O.lcg_sym(n, 120)
    c["w4"] = dict(in_x=x4, in_w=w4, in_w_scales=w4s, in_bias=b4, in_shape=np.array([m, n, k]),
                   out_y=O.w4_gemm(x4, w4, w4s, m, n, k, b4, O.ACT_GELU))
    return c


def flatten(c):
    return {f"{name}.{key}": np.asarray(arr) for name, d in c.items() for key, arr in d.items()}


def load(path=os.path.join(HERE, "golden.npz")):
    """golden.npz -> {case: {key: array}}."""
    out = {}
    with np.load(path) as z:
        for full in z.files:
            name, key = full.split(".", 1)
            out.setdefault(name, {})[key] = z[full]
    return out


if __name__ == "__main__":
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **flatten(cases()))
    print("wrote", os.path.join(HERE, "golden.npz"))
