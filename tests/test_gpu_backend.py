"""GPU parity of the Backend-trait ops against the oracle, in the style of the
reference's cross-backend harness (crates/tpt-infer-ops/src/dispatch.rs:270-512):
the same LCG inputs and shapes, every op through the C ABI.

MatMul and Conv2d are bit-identical to the reference (sequential k, separately
rounded multiply and add). Softmax/Sigmoid/GELU use CUDA's expf/tanhf, which
differ from libm by a few ulp: checked at 1e-5*(1+|want|), ten times tighter
than the reference harness's 1e-4*(1+|want|).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_TRANSCENDENTAL = 1e-5


def _close(got, want, rel=TOL_TRANSCENDENTAL):
    tol = rel * (1.0 + np.abs(want))
    assert np.all(np.isfinite(got))
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"max err {np.abs(got - want).max()} at {np.argmax(bad)}"


@pytest.mark.parametrize("m,k,n,sa,sb", [
    (3, 4, 5, 1, 2),        # dispatch.rs:318-330
    (1, 784, 10, 3, 4),     # dispatch.rs:328 (MLP head)
    (13, 17, 19, 5, 6),     # odd shapes
    (32, 64, 48, 7, 8),     # dispatch.rs:501-511
    (64, 784, 512, 9, 10),  # MLP layer 1
    (257, 129, 300, 11, 12),
    # the resident-K small-output kernel: K at its 1536 maximum (24 chunks), one
    # past it (the tiled kernels), a ragged last chunk with 16-byte rows
    (48, 1536, 40, 13, 14),
    (20, 1537, 36, 15, 16),
    (16, 100, 16, 17, 18),
])
def test_matmul_bit_identical(cuda, m, k, n, sa, sb):
    a, b = O.lcg_sym(m * k, sa), O.lcg_sym(k * n, sb)
    want = O.matmul(a, (m, k), b, (k, n), threads=4)
    got = np.empty(m * n, np.float32)
    cuda.matmul(a, (m, k), b, (k, n), got)
    assert np.array_equal(got, want)


def test_matmul_known_values(cuda):
    out = np.zeros(4, np.float32)
    cuda.matmul([1, 2, 3, 4], (2, 2), [5, 6, 7, 8], (2, 2), out)
    assert out.tolist() == [19.0, 22.0, 43.0, 50.0]  # naive.rs:212-219


def test_matmul_errors_match_reference(cuda):
    from tpt_infer_b200 import OpError

    with pytest.raises(OpError) as e:  # naive.rs:221-228
        cuda.matmul(np.ones(6), (2, 3), np.ones(12), (4, 3), np.zeros(6, np.float32))
    assert e.value.kind == "ShapeMismatch"
    with pytest.raises(OpError) as e:  # naive.rs:230-243
        cuda.matmul(np.ones(5), (2, 3), np.ones(9), (3, 3), np.zeros(6, np.float32))
    assert (e.value.kind, e.value.expected, e.value.actual) == ("SizeMismatch", 6, 5)


def test_matmul_empty_and_k0(cuda):
    out = np.empty(0, np.float32)
    cuda.matmul(np.empty(0), (0, 5), np.ones(10), (5, 2), out)
    out = np.full(6, 7.0, np.float32)
    cuda.matmul(np.empty(0), (2, 0), np.empty(0), (0, 3), out)
    assert np.all(out == 0.0)


@pytest.mark.parametrize("ishape,wshape,stride,pad", [
    ((1, 1, 3, 3), (1, 1, 2, 2), (1, 1), (0, 0)),
    ((1, 2, 9, 7), (3, 2, 3, 3), (2, 2), (1, 1)),   # dispatch.rs conv pad1/stride2 case
    ((2, 3, 16, 16), (8, 3, 3, 3), (1, 1), (1, 1)),
    ((1, 3, 32, 32), (8, 3, 7, 7), (2, 2), (3, 3)),  # stem-shaped
    ((2, 16, 14, 14), (32, 16, 1, 1), (2, 2), (0, 0)),  # 1x1 s2 projection
])
def test_conv2d_bit_identical(cuda, ishape, wshape, stride, pad):
    from tpt_infer_b200 import Conv2dOptions

    x = O.lcg_sym(int(np.prod(ishape)), 21)
    w = O.lcg_sym(int(np.prod(wshape)), 22)
    want = O.conv2d(x, ishape, w, wshape, stride, pad, threads=4)
    got = np.empty(want.size, np.float32)
    cuda.conv2d(x, ishape, w, wshape, got, Conv2dOptions(stride[0], stride[1], pad[0], pad[1]))
    assert np.array_equal(got, want)


def test_conv2d_known_values_and_errors(cuda):
    from tpt_infer_b200 import Conv2dOptions, OpError

    out = np.zeros(4, np.float32)
    cuda.conv2d(np.arange(1, 10), (1, 1, 3, 3), [1, 0, 0, -1], (1, 1, 2, 2), out)
    assert out.tolist() == [-4.0] * 4  # naive.rs:245-260
    out = np.zeros(9, np.float32)
    cuda.conv2d(np.ones(64), (1, 1, 8, 8), np.ones(9), (1, 1, 3, 3), out, Conv2dOptions(2, 2, 0, 0))
    assert np.all(out == 9.0)  # naive.rs:262-282
    with pytest.raises(OpError) as e:  # naive.rs:284-300
        cuda.conv2d(np.zeros(8), (1, 2, 2, 2), np.zeros(6), (1, 3, 2, 2), np.zeros(4, np.float32))
    assert e.value.kind == "ShapeMismatch"
    with pytest.raises(OpError) as e:  # naive.rs:302-321
        cuda.conv2d(np.zeros(16), (1, 1, 4, 4), np.zeros(9), (1, 1, 3, 3), np.zeros(16, np.float32),
                    Conv2dOptions(0, 1, 0, 0))
    assert e.value.kind == "Invalid"


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 1 << 20, (1 << 20) + 3])
def test_add_relu_exact(cuda, n):
    a, b = O.lcg_sym(n, 31), O.lcg_sym(n, 32)
    out = np.empty(n, np.float32)
    cuda.elementwise_add(a, b, out)
    assert np.array_equal(out, O.elementwise_add(a, b))
    cuda.relu(a, out)
    assert np.array_equal(out, O.relu(a))


@pytest.mark.parametrize("n", [3, 1000, 65536 + 5])
def test_sigmoid_gelu(cuda, n):
    a = O.lcg_sym(n, 33) * np.float32(6.0)
    out = np.empty(n, np.float32)
    cuda.sigmoid(a, out)
    _close(out, O.sigmoid(a))
    cuda.gelu(a, out)
    _close(out, O.gelu(a))


def test_unary_known_values(cuda):
    out = np.zeros(4, np.float32)
    cuda.relu([-1.0, 0.0, 1.0, 0.5], out)
    assert out.tolist() == [0.0, 0.0, 1.0, 0.5]  # naive.rs:323-329
    out = np.zeros(1, np.float32)
    cuda.sigmoid([0.0], out)
    assert abs(out[0] - 0.5) < 1e-6  # naive.rs:331-337
    out = np.ones(3, np.float32)
    cuda.gelu([0.0, -1.0, 1.0], out)
    assert out[0] == 0.0 and out[1] < 0 and out[2] > 0  # naive.rs:339-347


@pytest.mark.parametrize("rows,row_len", [(2, 3), (64, 10), (1024, 128), (7, 3000), (3, 1)])
def test_softmax(cuda, rows, row_len):
    a = O.lcg_sym(rows * row_len, 41) * np.float32(8.0)
    out = np.empty(a.size, np.float32)
    cuda.softmax(a, out, row_len)
    _close(out, O.softmax(a, row_len))


def test_softmax_reference_cases(cuda):
    from tpt_infer_b200 import OpError

    out = np.zeros(6, np.float32)
    cuda.softmax([1.0, 2.0, 3.0, 1000.0, 1000.0, 1000.0], out, 3)  # naive.rs:349-359
    assert abs(out[:3].sum() - 1) < 1e-5 and abs(out[3:].sum() - 1) < 1e-5 and 0.3 < out[3] < 0.34
    for rl in (0, 2):  # naive.rs:361-367
        with pytest.raises(OpError) as e:
            cuda.softmax([1.0, 2.0, 3.0], np.zeros(3, np.float32), rl)
        assert e.value.kind == "Invalid"


def test_add_length_check(cuda):
    from tpt_infer_b200 import OpError

    with pytest.raises(OpError) as e:  # naive.rs:369-380
        cuda.elementwise_add([1.0, 2.0], [1.0], np.zeros(2, np.float32))
    assert (e.value.expected, e.value.actual) == (2, 1)


def test_backend_name(cuda):
    assert cuda.name() == "cuda"


@pytest.mark.parametrize("m,k,n", [(3, 4, 5), (64, 784, 512), (129, 70, 33)])
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("cmode", [0, 1, 2])
def test_gemm_onnx_bit_exact(cuda, m, k, n, ta, tb, cmode):
    a = O.lcg_sym(m * k, 91)
    b = O.lcg_sym(k * n, 92)
    c = None if cmode == 0 else O.lcg_sym(n if cmode == 1 else m * n, 93)
    got = cuda.gemm(a, m, k, b, n, c=c, alpha=1.5, beta=-0.75, trans_a=ta, trans_b=tb)
    want = O.gemm(a, m, k, b, n, c=c, alpha=1.5, beta=-0.75, trans_a=ta, trans_b=tb)
    assert np.array_equal(got, want)


def test_gemm_onnx_errors(cuda):
    from tpt_infer_b200 import OpError
    with pytest.raises(OpError) as e:
        cuda.gemm(np.ones(5), 2, 3, np.ones(9), 3)
    assert (e.value.kind, e.value.expected, e.value.actual) == ("SizeMismatch", 6, 5)
    with pytest.raises(OpError) as e:
        cuda.gemm(np.ones(6), 2, 3, np.ones(9), 3, c=np.ones(4))
    assert e.value.kind == "ShapeMismatch"
