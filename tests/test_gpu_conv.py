"""The implicit-GEMM INT8 convolution (IM2COL -> LINEAR fused inside a plan).

A plan runs QUANTIZE (static scale) -> IM2COL -> LINEAR_W8A8 (+bias, act)
[-> QUANTIZE]. Fetching only the conv output lets the plan replace the two ops
by one implicit-GEMM launch; fetching the im2col rows as well forces the
separate im2col + GEMM. Both must equal the oracle (its im2col restatement
and W8A8 GEMM) bit for bit, f32 and requantized int8 outputs alike, over
ragged shapes, strides, padding, 1x1 kernels and output-channel counts that
are not tile multiples, in both ways of loading the activation tiles (cp.async
gathers for small inputs, TMA im2col for inputs of 128 KB and more).
"""
import numpy as np
import pytest

from oracle import models as OM
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = [  # N, H, W, C, OC, k, stride, pad
    (3, 13, 11, 32, 48, 3, 1, 1),
    (2, 9, 9, 64, 64, 3, 2, 1),
    (2, 16, 16, 16, 200, 1, 2, 0),
    (1, 7, 7, 128, 512, 3, 1, 1),
    (2, 10, 12, 64, 130, 3, 1, 1),
    (4, 20, 20, 64, 64, 3, 1, 1),
    # inputs of 128 KB and more: the activation tiles come from TMA im2col loads
    (2, 40, 40, 64, 64, 3, 1, 1),
    (2, 32, 32, 128, 128, 3, 2, 1),
    (3, 24, 24, 128, 256, 1, 2, 0),
    (3, 30, 26, 64, 130, 3, 1, 1),
    (1, 20, 20, 512, 512, 3, 1, 1),
    # a 128-wide tile with TMA operands (eight epilogue warps) and a ragged last chunk
    (2, 40, 40, 64, 100, 3, 1, 1),
]


@pytest.mark.parametrize("N,H,W,C,OC,k,s,pad", CASES)
@pytest.mark.parametrize("requant", [False, True])
def test_conv_implicit_gemm_bit_exact(cuda, N, H, W, C, OC, k, s, pad, requant):
    from tpt_infer_b200 import graphs

    OH, OW = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    M, K = N * OH * OW, k * k * C
    seed = 7000 + N * 131 + C + OC + k
    x = O.normal(N * H * W * C, seed)
    sx = np.float32(O.sym_scale(O.absmax(x)))
    wq, ws = O.quantize_i8_symmetric_per_channel(O.normal(OC * K, seed + 1, 0.0, 0.05), OC)
    bias = O.normal(OC, seed + 2, 0.0, 0.1)
    p = graphs.Plan(cuda)
    w = cuda.upload_i8(wq, ws, OC, K)
    p.weights.append(w)
    tx, txq = p.tensor(graphs.F32, x.size), p.tensor(graphs.I8, x.size)
    col, ty = p.tensor(graphs.I8, M * K), p.tensor(graphs.F32, M * OC)
    p.op(graphs.OP_QUANTIZE, tx, txq, f0=float(sx), dims=(x.size,))
    p.op(graphs.OP_IM2COL, txq, col, dims=(N, H, W, C, k, k, s, s, pad, pad, OH, OW, K))
    p.op(graphs.OP_LINEAR, col, ty, in1=p.const(bias), w=w, act=graphs.ACT_RELU, dims=(M,))
    sy = np.float32(0.05)
    if requant:
        tyq = p.tensor(graphs.I8, M * OC)
        p.op(graphs.OP_QUANTIZE, ty, tyq, f0=float(sy), dims=(M * OC,))
    p.finalize()

    xq = O.quantize_i8_static(x, sx).reshape(N, H, W, C)
    col_o, _, _ = OM._im2col(xq, k, s, pad, K)
    want = O.w8a8_gemm(col_o, wq, M, OC, K, sx, ws, bias, O.ACT_RELU, threads=8)
    if requant:
        want_q = O.quantize_i8_static(want, sy)
        fused = p.run({tx: x}, [tyq])[0]                    # implicit GEMM with the requantizing epilogue
        split = p.run({tx: x}, [col, tyq])[1]               # im2col rows fetched: separate ops
        for got in (fused, split):
            assert np.array_equal(np.frombuffer(got.tobytes()[:M * OC], np.int8), want_q)
    else:
        fused = p.run({tx: x}, [ty])[0]
        got_col, split = p.run({tx: x}, [col, ty])
        assert np.array_equal(np.frombuffer(got_col.tobytes()[:M * K], np.int8), col_o.ravel())
        assert np.array_equal(fused, want)
        assert np.array_equal(split, want)
    p.close()


@pytest.mark.parametrize("N,H,W,C,OC,k,s,pad", [CASES[i] for i in (0, 2, 4, 7, 9, 11)])
@pytest.mark.parametrize("requant", [False, True])
@pytest.mark.parametrize("res_first", [False, True])
def test_conv_residual_epilogue_bit_exact(cuda, N, H, W, C, OC, k, s, pad, requant, res_first):
    # IM2COL -> LINEAR -> ADD_ACT(relu) with a residual [-> QUANTIZE of the sum]:
    # with the conv output not fetched the residual add folds into the conv
    # epilogue (the sum, and its int8 copy, from one launch); fetching the conv
    # output keeps the separate ADD_ACT. Both equal the oracle's conv plus a
    # float32 add and ReLU, bit for bit, with the residual as either input.
    from tpt_infer_b200 import graphs

    OH, OW = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    M, K = N * OH * OW, k * k * C
    seed = 7500 + N * 131 + C + OC + k
    x = O.normal(N * H * W * C, seed)
    r = O.normal(M * OC, seed + 3)
    sx = np.float32(O.sym_scale(O.absmax(x)))
    wq, ws = O.quantize_i8_symmetric_per_channel(O.normal(OC * K, seed + 1, 0.0, 0.05), OC)
    bias = O.normal(OC, seed + 2, 0.0, 0.1)
    p = graphs.Plan(cuda)
    w = cuda.upload_i8(wq, ws, OC, K)
    p.weights.append(w)
    tx, txq = p.tensor(graphs.F32, x.size), p.tensor(graphs.I8, x.size)
    col, ty = p.tensor(graphs.I8, M * K), p.tensor(graphs.F32, M * OC)
    tr, ts = p.tensor(graphs.F32, M * OC), p.tensor(graphs.F32, M * OC)
    p.op(graphs.OP_QUANTIZE, tx, txq, f0=float(sx), dims=(x.size,))
    p.op(graphs.OP_IM2COL, txq, col, dims=(N, H, W, C, k, k, s, s, pad, pad, OH, OW, K))
    p.op(graphs.OP_LINEAR, col, ty, in1=p.const(bias), w=w, act=graphs.ACT_NONE, dims=(M,))
    a0, a1 = (tr, ty) if res_first else (ty, tr)
    p.op(graphs.OP_ADD_ACT, a0, ts, in1=a1, act=graphs.ACT_RELU, dims=(M * OC,))
    sy = np.float32(0.05)
    tsq = p.tensor(graphs.I8, M * OC)
    if requant:
        p.op(graphs.OP_QUANTIZE, ts, tsq, f0=float(sy), dims=(M * OC,))
    p.finalize()

    xq = O.quantize_i8_static(x, sx).reshape(N, H, W, C)
    col_o, _, _ = OM._im2col(xq, k, s, pad, K)
    conv = O.w8a8_gemm(col_o, wq, M, OC, K, sx, ws, bias, O.ACT_NONE, threads=8)
    want = np.maximum(conv + r, np.float32(0.0)).astype(np.float32)
    outs = [ts, tsq] if requant else [ts]
    fused = p.run({tx: x, tr: r}, outs)
    split = p.run({tx: x, tr: r}, [ty] + outs)
    assert np.array_equal(split[0], conv)
    for got in (fused, split[1:]):
        assert np.array_equal(got[0], want)
        if requant:
            assert np.array_equal(np.frombuffer(got[1].tobytes()[:M * OC], np.int8), O.quantize_i8_static(want, sy))
    p.close()


@pytest.mark.parametrize("N,H,W,C,k,s,pad", [(2, 17, 15, 64, 3, 2, 1), (3, 8, 8, 16, 3, 1, 1), (2, 12, 10, 8, 2, 2, 0)])
def test_maxpool_op_bit_exact(cuda, N, H, W, C, k, s, pad):
    # the plan's NHWC MAXPOOL (the 3x3 window compiled in, others generic)
    # against the oracle's NCHW max_pool2d, bit for bit, with signed zeros and
    # NaN among the inputs; a QUANTIZE of the pooled tensor runs inside the
    # pool's pass (its int8 copy) and must equal the oracle's quantizer
    from tpt_infer_b200 import graphs

    OH, OW = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    x = O.normal(N * H * W * C, 9100 + H + C).reshape(N, H, W, C)
    x.ravel()[::37] = 0.0
    x.ravel()[5::41] = -0.0
    x.ravel()[11::997] = np.nan
    p = graphs.Plan(cuda)
    tx, ty = p.tensor(graphs.F32, x.size), p.tensor(graphs.F32, N * OH * OW * C)
    tq = p.tensor(graphs.I8, N * OH * OW * C)
    p.op(graphs.OP_MAXPOOL, tx, ty, dims=(N, H, W, C, k, k, s, s, pad, pad, OH, OW))
    sq = np.float32(0.02)
    p.op(graphs.OP_QUANTIZE, ty, tq, f0=float(sq), dims=(N * OH * OW * C,))
    p.finalize()
    got, gq = p.run({tx: x}, [ty, tq])
    got = got.reshape(N, OH, OW, C)
    p.close()
    want = O.max_pool2d(np.ascontiguousarray(x.transpose(0, 3, 1, 2)), N, C, H, W, (k, k), (s, s), (pad, pad))
    want = np.ascontiguousarray(want.reshape(N, C, OH, OW).transpose(0, 2, 3, 1))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    n = want.size
    assert np.array_equal(np.frombuffer(gq.tobytes()[:n], np.int8), O.quantize_i8_static(want, sq))
