"""GPU parity of the quantized GEMMs against the oracle.

W8A8: the i32 accumulators are bit-exact, and so is the f32 output
y = (float)acc * (a_scale * w_scale[n]) + bias[n] (two roundings, no FMA, in
the oracle's order). Shapes cover the W8A8 sweep (M in {1, 16, 256, 4096},
K = N = 4096) plus ragged ones; at M = 4096 the oracle checks a sample of rows.

W4: the reference computes dequant -> f32 matmul; the device factors the
channel scale out of the sum, so outputs match to rounding. Tolerance, per
the spec: max-abs error <= 1e-3 x output scale, with the output scale read
strictly as the symmetric INT8 quantisation step of the output,
max|y| / 127.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def w8a8_case(m, n, k, seed=100, with_bias=True):
    w = O.normal(k * n, seed, 0.0, 0.02).reshape(k, n)          # W [K, N]
    wt = np.ascontiguousarray(w.T)                              # W^T [N, K]
    wq, ws = O.quantize_i8_symmetric_per_channel(wt, n)          # per output channel
    x = O.normal(m * k, seed + 1, 0.0, 1.0)
    aq, sa = O.quantize_i8_symmetric(x)                          # per tensor
    bias = O.normal(n, seed + 2, 0.0, 0.01) if with_bias else None
    return aq, sa, wq, ws, bias


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (16, 4096, 4096), (256, 4096, 4096),
                                   (3, 100, 48), (9, 33, 16), (130, 200, 64), (1, 10, 512),
                                   (128, 256, 128), (300, 512, 256), (1000, 768, 768), (160, 203, 96),
                                   (4097, 300, 128), (33, 300, 256), (64, 512, 784), (48, 4096, 4096),
                                   (17, 4097, 4112), (65, 512, 256), (100, 1000, 1024), (2, 300, 8192),
                                   (4, 257, 4160), (16, 1024, 4096), (64, 2048, 2048), (5, 200, 384),
                                   # the small-batch MMA kernel: 1, 2 and 4 activation tiles
                                   (3, 4096, 4096), (8, 1000, 1024), (12, 130, 512), (24, 500, 2048),
                                   (32, 4096, 4096), (20, 17, 256),
                                   # the resident-K kernel (M <= 64, K <= 1536): K at its maximum,
                                   # a 10-channel head
                                   (40, 1000, 1536), (64, 10, 512)])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_w8a8_bit_exact(cuda, m, n, k, act):
    if act and m * n * k > 1 << 26:
        pytest.skip("activations covered at the smaller shapes")
    aq, sa, wq, ws, bias = w8a8_case(m, n, k)
    w = cuda.upload_i8(wq, ws, n, k)
    y = cuda.w8a8_gemm(aq, m, k, sa, w, bias, act)
    want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, act, threads=8)
    assert np.array_equal(y, want)  # GELU too: the epilogue's deterministic GELU has an exact CPU restatement
    w.free()


@pytest.mark.parametrize("m,n,k", [(1024, 3072, 768), (640, 768, 3072)])
def test_w8a8_gelu_bert_shapes_bit_exact(cuda, m, n, k):
    # the encoder's FFN shapes on the SM-pair kernel with the GELU epilogue
    aq, sa, wq, ws, bias = w8a8_case(m, n, k)
    w = cuda.upload_i8(wq, ws, n, k)
    y = cuda.w8a8_gemm(aq, m, k, sa, w, bias, 2)
    want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, 2, threads=8)
    assert np.array_equal(y, want)
    w.free()


@pytest.mark.parametrize("m", [1, 16, 30, 256, 4096])
def test_w8a8_accumulators_bit_exact(cuda, m):
    import torch

    n = k = 4096
    aq, sa, wq, ws, _ = w8a8_case(m, n, k, seed=200)
    w = cuda.upload_i8(wq, ws, n, k)
    a_dev = torch.from_numpy(aq).cuda()
    acc = torch.empty(m * n, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    cuda.w8a8_gemm_acc_dev(a_dev, m, w, acc)
    cuda.sync()
    got = acc.cpu().numpy().reshape(m, n)
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(m).integers(0, m, 48)]))
    want = O.i8_gemm_acc(aq.reshape(m, k)[rows].ravel(), wq, rows.size, n, k, threads=8).reshape(rows.size, n)
    assert np.array_equal(got[rows], want)
    w.free()


def test_w8a8_pinned_host_buffers_pipelined(cuda):
    """Page-locked host buffers with a large output take the chunked path (H2D,
    GEMM and D2H of row chunks overlapped): the same bits, on two calls in a row."""
    import torch

    m, n, k = 1024, 4096, 1024  # 16 MB of f32 output: four row chunks
    aq, sa, wq, ws, bias = w8a8_case(m, n, k, seed=900)
    w = cuda.upload_i8(wq, ws, n, k)
    a_pin = torch.from_numpy(aq).pin_memory()
    y_pin = torch.empty(m * n, dtype=torch.float32).pin_memory()
    want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, 1, threads=8)
    for _ in range(2):
        y_pin.zero_()
        cuda.w8a8_gemm(a_pin.numpy(), m, k, sa, w, bias, 1, out=y_pin.numpy())
        assert np.array_equal(y_pin.numpy(), want)
    w.free()


def test_w8a8_small_m_back_to_back(cuda):
    # the stream-K path combines partial tiles in a workspace that must be
    # clean again after every launch: run several shapes back to back on the
    # stream without a host sync in between and check every result
    import torch

    cases = []
    for i, (m, n, k) in enumerate([(1, 4096, 4096), (16, 4096, 4096), (64, 512, 784), (1, 4096, 4096),
                                   (40, 1000, 2048)]):
        aq, sa, wq, ws, bias = w8a8_case(m, n, k, seed=400 + 10 * i)
        w = cuda.upload_i8(wq, ws, n, k)
        a_dev = torch.from_numpy(aq).cuda()
        b_dev = torch.from_numpy(bias).cuda()
        y_dev = torch.empty(m * n, dtype=torch.float32, device="cuda")
        cases.append((m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev))
    torch.cuda.synchronize()
    for m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev in cases:
        cuda.w8a8_gemm_dev(a_dev, m, sa, w, b_dev, 1, y_dev)
    cuda.sync()
    for m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev in cases:
        want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, 1, threads=8)
        assert np.array_equal(y_dev.cpu().numpy(), want), (m, n, k)
        w.free()


def test_small_m_and_w4_share_the_split_workspace(cuda):
    # the split-K small-batch W8A8 kernel and the stream-K W4 kernel keep their
    # partial sums in the same context workspace (counters zero between
    # launches, slots overwritten): interleave them on the stream with no host
    # sync in between and check every result
    import torch

    w8, w4 = [], []
    for i, (m, n, k) in enumerate([(16, 4096, 4096), (5, 1000, 1024), (32, 768, 768)]):
        aq, sa, wq, ws, bias = w8a8_case(m, n, k, seed=700 + 10 * i)
        w = cuda.upload_i8(wq, ws, n, k)
        y_dev = torch.empty(m * n, dtype=torch.float32, device="cuda")
        w8.append((m, n, k, aq, sa, wq, ws, bias, w, torch.from_numpy(aq).cuda(), torch.from_numpy(bias).cuda(), y_dev))
    for i, (m, n, k) in enumerate([(64, 11008, 4096), (24, 1000, 1024)]):
        x, p, s = w4_case(m, n, k, seed=800 + 10 * i)
        w = cuda.upload_i4(p, s, n, k)
        w4.append((m, n, k, x, p, s, w, torch.from_numpy(x).cuda(), torch.empty(m * n, dtype=torch.float32,
                                                                                  device="cuda")))
    torch.cuda.synchronize()
    for rep in range(2):
        for j in range(3):
            m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev = w8[j]
            cuda.w8a8_gemm_dev(a_dev, m, sa, w, b_dev, 0, y_dev)
            if j < 2:
                m4, n4, k4, x, p, s, w4h, x_dev, y4 = w4[j]
                cuda.w4_gemm_dev(x_dev, m4, w4h, None, 0, y4)
    cuda.sync()
    for m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev in w8:
        want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, 0, threads=8)
        assert np.array_equal(y_dev.cpu().numpy(), want), (m, n, k)
        w.free()
    for m, n, k, x, p, s, w, x_dev, y4 in w4:
        want = O.w4_gemm(x, p, s, m, n, k, threads=8)
        assert np.max(np.abs(y4.cpu().numpy() - want)) <= w4_tol(want)
        w.free()


def test_w8a8_large_m_back_to_back(cuda):
    # SM-pair launches of several shapes and tile widths queued back to back
    # on the stream (twice) with no host sync in between, every result checked
    import torch

    cases = []
    for i, (m, n, k) in enumerate([(256, 4096, 4096), (1000, 768, 768), (8192, 768, 3072), (300, 512, 256),
                                   (256, 4096, 4096), (2048, 1000, 1024)]):
        aq, sa, wq, ws, bias = w8a8_case(m, n, k, seed=600 + 10 * i)
        w = cuda.upload_i8(wq, ws, n, k)
        a_dev = torch.from_numpy(aq).cuda()
        b_dev = torch.from_numpy(bias).cuda()
        y_dev = torch.empty(m * n, dtype=torch.float32, device="cuda")
        cases.append((m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev))
    torch.cuda.synchronize()
    for _ in range(2):
        for m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev in cases:
            cuda.w8a8_gemm_dev(a_dev, m, sa, w, b_dev, 0, y_dev)
    cuda.sync()
    for m, n, k, aq, sa, wq, ws, bias, w, a_dev, b_dev, y_dev in cases:
        got = y_dev.cpu().numpy().reshape(m, n)
        rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(m + n).integers(0, m, 64)]))
        want = O.w8a8_gemm(aq.reshape(m, k)[rows].ravel(), wq, rows.size, n, k, sa, ws, bias, 0,
                           threads=8).reshape(rows.size, n)
        assert np.array_equal(got[rows], want), (m, n, k)
        w.free()


def test_w8a8_full_m4096_sampled_rows(cuda):
    m = n = k = 4096
    aq, sa, wq, ws, bias = w8a8_case(m, n, k, seed=300)
    w = cuda.upload_i8(wq, ws, n, k)
    y = cuda.w8a8_gemm(aq, m, k, sa, w, bias, 0).reshape(m, n)
    rows = np.unique(np.concatenate([[0, 127, 128, m - 1], np.random.default_rng(7).integers(0, m, 40)]))
    want = O.w8a8_gemm(aq.reshape(m, k)[rows].ravel(), wq, rows.size, n, k, sa, ws, bias, 0,
                       threads=8).reshape(rows.size, n)
    assert np.array_equal(y[rows], want)
    w.free()


@pytest.mark.parametrize("m,k,n", [(4, 8, 4), (3, 17, 5), (64, 784, 10), (33, 100, 257)])
def test_quantized_matmul_i8_reference_contract(cuda, m, k, n):
    # ptq.rs:293-324 as is: B [k, n], per-tensor scale, no bias
    a, b = O.lcg_sym(m * k, 301), O.lcg_sym(k * n, 302)
    aq, sa = O.quantize_i8_symmetric(a)
    bq, sb = O.quantize_i8_symmetric(b)
    out = np.empty(m * n, np.float32)
    cuda.quantized_matmul_i8(aq, (m, k), sa, bq, (k, n), [sb], out)
    assert np.array_equal(out, O.quantized_matmul_i8(aq, (m, k), sa, bq, (k, n), [sb]))


def test_quantized_matmul_i8_kat_and_errors(cuda):
    from tpt_infer_b200 import OpError

    # ptq.rs:409-436
    m, k, n = 4, 8, 4
    a = (np.sin(np.arange(m * k, dtype=np.float32)) * np.float32(0.5)).astype(np.float32)
    b = (np.cos(np.arange(k * n, dtype=np.float32)) * np.float32(0.5)).astype(np.float32)
    ref = O.matmul_naive(a, (m, k), b, (k, n))
    aq, sa = cuda.quantize_i8_symmetric(a)
    bq, sb = cuda.quantize_i8_symmetric(b)
    out = np.empty(m * n, np.float32)
    cuda.quantized_matmul_i8(aq, (m, k), sa, bq, (k, n), [sb], out)
    assert np.all(np.abs(ref - out) < 0.05)
    with pytest.raises(OpError) as e:
        cuda.quantized_matmul_i8(aq, (m, k), sa, bq, (k + 1, n), [sb], out)
    assert e.value.kind == "ShapeMismatch"
    with pytest.raises(OpError) as e:
        cuda.quantized_matmul_i8(aq[:-1], (m, k), sa, bq, (k, n), [sb], out)
    assert e.value.kind == "SizeMismatch"


def w4_case(m, n, k, seed=400):
    w = O.normal(k * n, seed, 0.0, 0.02).reshape(k, n)
    wt = np.ascontiguousarray(w.T)
    p, s = O.quantize_i4_symmetric_per_channel(wt, n)
    x = O.normal(m * k, seed + 1, 0.0, 1.0)
    return x, p, s


def w4_tol(want):
    return 1e-3 * (np.max(np.abs(want)) / 127.0)


@pytest.mark.parametrize("m,n,k", [(1, 11008, 4096), (8, 11008, 4096), (64, 11008, 4096), (2, 100, 64),
                                   (5, 40, 96), (1, 8, 32), (24, 1000, 1024), (40, 300, 2048), (130, 300, 512),
                                   (300, 129, 4096),
                                   # decode GEMV: ragged groups, 3 / 11 / 12 K-slices, K beyond the ring
                                   (2, 1001, 4096), (1, 4096, 11008), (2, 4096, 11008), (1, 77, 3072),
                                   (2, 300, 12288), (1, 64, 16384), (1, 200, 8192), (2, 72, 6144),
                                   # small batches on the digit-plane kernel: 1, 2 and 3 column tiles
                                   (3, 500, 4096), (4, 1000, 2048), (6, 300, 1024), (7, 129, 3072), (8, 40, 256)])
def test_w4_gemm(cuda, m, n, k):
    x, p, s = w4_case(m, n, k)
    w = cuda.upload_i4(p, s, n, k)
    y = cuda.w4_gemm(x, m, k, w)
    want = O.w4_gemm(x, p, s, m, n, k, threads=8)
    assert np.max(np.abs(y - want)) <= w4_tol(want)
    w.free()


def test_w4_gemm_m512_sampled(cuda):
    m, n, k = 512, 11008, 4096
    x, p, s = w4_case(m, n, k, seed=500)
    w = cuda.upload_i4(p, s, n, k)
    y = cuda.w4_gemm(x, m, k, w).reshape(m, n)
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(3).integers(0, m, 14)]))
    want = O.w4_gemm(x.reshape(m, k)[rows].ravel(), p, s, rows.size, n, k, threads=8).reshape(rows.size, n)
    assert np.max(np.abs(y[rows] - want)) <= w4_tol(want)
    w.free()


@pytest.mark.parametrize("m", [2, 5])
def test_w4_gemv_non_finite(cuda, m):
    """inf / NaN activations propagate as in the reference's f32 matmul."""
    n, k = 300, 4096
    x, p, s = w4_case(m, n, k, seed=700)
    x[5] = np.inf
    x[k + 100] = np.nan
    w = cuda.upload_i4(p, s, n, k)
    y = cuda.w4_gemm(x, m, k, w)
    want = O.w4_gemm(x, p, s, m, n, k)
    assert np.array_equal(np.isnan(y), np.isnan(want))
    assert np.array_equal(np.isposinf(y), np.isposinf(want)) and np.array_equal(np.isneginf(y), np.isneginf(want))
    assert np.isnan(want[n:2 * n]).all() and np.isinf(want[:n]).any()
    if m > 2:  # the rows without non-finite inputs stay within the usual tolerance
        assert np.max(np.abs(y[2 * n:] - want[2 * n:])) <= w4_tol(want[2 * n:])
    w.free()


@pytest.mark.parametrize("act", [1, 2])
def test_w4_bias_act(cuda, act):
    m, n, k = 3, 64, 128
    x, p, s = w4_case(m, n, k, seed=600)
    bias = O.normal(n, 601, 0.0, 0.01)
    w = cuda.upload_i4(p, s, n, k)
    y = cuda.w4_gemm(x, m, k, w, bias, act)
    want = O.w4_gemm(x, p, s, m, n, k, bias, act)
    assert np.max(np.abs(y - want)) <= max(w4_tol(want), 1e-6)
    w.free()


def test_handles_outlive_context():
    # weights and plans may be freed after the context they were made through
    # has been destroyed (garbage collection order is not under the caller's
    # control); freeing them must touch only their device
    from tpt_infer_b200 import CudaBackend
    from tpt_infer_b200.graphs import Plan

    be = CudaBackend.new(0)
    aq, sa, wq, ws, bias = w8a8_case(4, 256, 128, seed=700)
    w = be.upload_i8(wq, ws, 256, 128)
    p = Plan(be)
    be.close()
    w.free()
    p.close()
