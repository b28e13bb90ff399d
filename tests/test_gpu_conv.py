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


@pytest.mark.parametrize("N,H,W,pad,oh,ow", [(2, 112, 112, 2, 112, 112), (3, 32, 48, 2, 33, 49), (1, 16, 16, 1, 15, 15),
                                               (2, 20, 32, 3, 20, 30)])
@pytest.mark.parametrize("quant", [False, True])
def test_stem_pool_fused_bit_exact(cuda, N, H, W, pad, oh, ow, quant):
    # IM2COL -> LINEAR (+bias, ReLU) -> MAXPOOL 3x3/2/1 [-> QUANTIZE] of a
    # 16-channel 4x4 stride-1 conv with 64 outputs (the ResNet stem in its
    # space-to-depth form; the output size may be cut below the full one, as the
    # stem's is) runs as one fused stem + pool launch that never writes the conv
    # output: the pooled f32 tensor and its int8 copy equal the oracle's conv,
    # ReLU, max pool and quantizer bit for bit, at the stem's own shape and at
    # odd / ragged ones
    from tpt_infer_b200 import graphs

    C, OC, k = 16, 64, 4
    PH, PW = (oh - 1) // 2 + 1, (ow - 1) // 2 + 1
    M, K = N * oh * ow, k * k * C
    seed = 9300 + H + W + pad
    x = O.normal(N * H * W * C, seed)
    sx = np.float32(O.sym_scale(O.absmax(x)))
    wq, ws = O.quantize_i8_symmetric_per_channel(O.normal(OC * K, seed + 1, 0.0, 0.05), OC)
    bias = O.normal(OC, seed + 2, 0.0, 0.1)
    p = graphs.Plan(cuda)
    w = cuda.upload_i8(wq, ws, OC, K)
    p.weights.append(w)
    tx, txq = p.tensor(graphs.F32, x.size), p.tensor(graphs.I8, x.size)
    col, ty = p.tensor(graphs.I8, M * K), p.tensor(graphs.F32, M * OC)
    tp, tq = p.tensor(graphs.F32, N * PH * PW * OC), p.tensor(graphs.I8, N * PH * PW * OC)
    p.op(graphs.OP_QUANTIZE, tx, txq, f0=float(sx), dims=(x.size,))
    p.op(graphs.OP_IM2COL, txq, col, dims=(N, H, W, C, k, k, 1, 1, pad, pad, oh, ow, K))
    p.op(graphs.OP_LINEAR, col, ty, in1=p.const(bias), w=w, act=graphs.ACT_RELU, dims=(M,))
    p.op(graphs.OP_MAXPOOL, ty, tp, dims=(N, oh, ow, OC, 3, 3, 2, 2, 1, 1, PH, PW))
    sq = np.float32(0.03)
    if quant:
        p.op(graphs.OP_QUANTIZE, tp, tq, f0=float(sq), dims=(N * PH * PW * OC,))
    p.finalize()
    outs = p.run({tx: x}, [tp, tq] if quant else [tp])
    l0 = cuda.launch_count()
    p.run_device()
    cuda.sync()
    assert cuda.launch_count() - l0 == 2  # the input's QUANTIZE and the fused stem + pool (+ its int8 copy)
    p.close()

    xq = O.quantize_i8_static(x, sx).reshape(N, H, W, C)
    # the oracle's full conv output, cut to oh x ow like the op's dims
    full_oh, full_ow = H + 2 * pad - k + 1, W + 2 * pad - k + 1
    col_o, _, _ = OM._im2col(xq, k, 1, pad, K)
    y = O.w8a8_gemm(col_o, wq, N * full_oh * full_ow, OC, K, sx, ws, bias, O.ACT_RELU, threads=8)
    y = np.ascontiguousarray(y.reshape(N, full_oh, full_ow, OC)[:, :oh, :ow, :])
    want = O.max_pool2d(np.ascontiguousarray(y.transpose(0, 3, 1, 2)), N, OC, oh, ow, (3, 3), (2, 2), (1, 1))
    want = np.ascontiguousarray(want.reshape(N, OC, PH, PW).transpose(0, 2, 3, 1))
    got = outs[0].reshape(N, PH, PW, OC)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if quant:
        assert np.array_equal(np.frombuffer(outs[1].tobytes()[:want.size], np.int8), O.quantize_i8_static(want, sq))
