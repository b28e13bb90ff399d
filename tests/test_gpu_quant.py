"""GPU parity of the tpt-infer-quantize path: every quantizer, packer and
dequantizer through the C ABI is bit-exact with the oracle (which the KAT
suite pins to crates/tpt-infer-quantize's own tests), including the edge
cases the domain has: empty and odd-length inputs, all-zero tensors (scale 1),
NaN and infinities, values at the clamp limits, and the full config-sized
tensors."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _edge_vectors():
    return {
        "kat": np.array([-1.0, 0.0, 1.0], np.float32),  # quant.rs:18-24
        "zeros": np.zeros(37, np.float32),
        "one": np.array([0.3], np.float32),
        "halfway": np.array([-2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 127.0, -127.0], np.float32),
        "nan": np.array([np.nan, 1.0, -3.0, 0.25], np.float32),
        "inf": np.array([np.inf, 1.0, -2.0], np.float32),
        "lcg_odd": O.lcg_sym(1001, 51),
        "normal": O.normal(1 << 16, 52),
        "big": O.normal(4096 * 4096, 53),  # W8A8 sweep activations [4096, 4096]
    }


EDGE = _edge_vectors()


@pytest.mark.parametrize("name", list(EDGE))
def test_quantize_i8_symmetric_bit_exact(cuda, name):
    x = EDGE[name]
    q, s = cuda.quantize_i8_symmetric(x)
    qw, sw = O.quantize_i8_symmetric(x)
    assert np.array_equal(q, qw) and s.tobytes() == sw.tobytes()


def test_quantize_i8_symmetric_kat_and_empty(cuda):
    q, s = cuda.quantize_i8_symmetric([-1.0, 0.0, 1.0])
    assert q.tolist() == [-127, 0, 127] and abs(s - 1 / 127) < 1e-6
    q, s = cuda.quantize_i8_symmetric(np.zeros(0, np.float32))
    assert q.size == 0 and s == 1.0


@pytest.mark.parametrize("rows,cols", [(1, 7), (4, 8), (2, 32), (37, 101), (4096, 4096), (11008, 64)])
def test_quantize_i8_per_channel_bit_exact(cuda, rows, cols):
    x = O.normal(rows * cols, 61, 0.0, 0.02)
    if rows > 1:
        x[: cols // 2] = 0.0  # a partly zero row
        x[cols: 2 * cols] = 0.0  # an all-zero row -> scale 1.0
    q, s = cuda.quantize_i8_symmetric_per_channel(x, rows)
    qw, sw = O.quantize_i8_symmetric_per_channel(x, rows)
    assert np.array_equal(q, qw) and np.array_equal(s, sw)


def test_quantize_i8_per_channel_invalid(cuda):
    from tpt_infer_b200 import OpError

    for rows in (0, 3):
        with pytest.raises(OpError) as e:
            cuda.quantize_i8_symmetric_per_channel(np.zeros(8, np.float32), rows)
        assert e.value.kind == "Invalid"


@pytest.mark.parametrize("name", ["kat", "zeros", "one", "halfway", "nan", "inf", "lcg_odd", "normal"])
def test_quantize_i8_asymmetric_bit_exact(cuda, name):
    x = EDGE[name]
    q, s, z = cuda.quantize_i8_asymmetric(x)
    qw, sw, zw = O.quantize_i8_asymmetric(x)
    assert np.array_equal(q, qw) and s.tobytes() == sw.tobytes() and z == zw


@pytest.mark.parametrize("data", [[0.0, 0.25, 0.5, 1.0, 2.0], [1.0, 2.0, 3.0, 4.0], [-5.0, -4.0, -1.0],
                                  [3.0, 3.0, 3.0], [-1e-3, 100.0]])
def test_quantize_i8_asymmetric_zero_point_branches(cuda, data):
    # quant.rs:56-74: flat range, in-range zp, and both pinned-zp branches
    x = np.array(data, np.float32)
    q, s, z = cuda.quantize_i8_asymmetric(x)
    qw, sw, zw = O.quantize_i8_asymmetric(x)
    assert np.array_equal(q, qw) and s.tobytes() == sw.tobytes() and z == zw


@pytest.mark.parametrize("n", [0, 1, 2, 3, 16, 1001, 1 << 20])
def test_pack_unpack_i4_bit_exact(cuda, n):
    v = ((O.lcg_uniform(n, 71) * 16).astype(np.int32) - 8).astype(np.int8)
    p = cuda.pack_i4(v)
    assert np.array_equal(p, O.pack_i4(v))
    assert np.array_equal(cuda.unpack_i4(p, n), v)
    # unpack of more than 2*len values stops at the data (quant.rs:145-157)
    assert np.array_equal(cuda.unpack_i4(p, n + 5), O.unpack_i4(p, n + 5))


def test_pack_i4_kats_and_rejects(cuda):
    from tpt_infer_b200 import OpError

    p = cuda.pack_i4([-8, 7, 0, 1])  # quant.rs:116-122
    assert p.size == 2 and cuda.unpack_i4(p, 4).tolist() == [-8, 7, 0, 1]
    vals = np.arange(-8, 8, dtype=np.int8)  # quant.rs:261-272
    assert np.array_equal(cuda.unpack_i4(cuda.pack_i4(vals), 16), vals)
    with pytest.raises(OpError) as e:  # quant.rs:292-296 (panics in the reference)
        cuda.pack_i4([8])
    assert e.value.kind == "Invalid"
    with pytest.raises(OpError):
        cuda.pack_i4([0, -9, 1])


@pytest.mark.parametrize("name", ["kat", "zeros", "one", "halfway", "nan", "inf", "lcg_odd", "normal"])
def test_quantize_i4_symmetric_bit_exact(cuda, name):
    x = EDGE[name]
    p, s = cuda.quantize_i4_symmetric(x)
    pw, sw = O.quantize_i4_symmetric(x)
    assert np.array_equal(p, pw) and s.tobytes() == sw.tobytes()


@pytest.mark.parametrize("rows,cols", [(2, 32), (4, 8), (3, 7), (11008, 4096)])
def test_quantize_i4_per_channel_bit_exact(cuda, rows, cols):
    # the W4 workload: W^T [N=11008, K=4096] ~ N(0, 0.02), nibbles along K
    x = O.normal(rows * cols, 81, 0.0, 0.02)
    p, s = cuda.quantize_i4_symmetric_per_channel(x, rows)
    pw, sw = O.quantize_i4_symmetric_per_channel(x, rows)
    assert np.array_equal(p, pw) and np.array_equal(s, sw)
    q = O.unpack_i4(p[: (cols + 1) // 2], cols)
    assert q.min() >= -7 and q.max() <= 7


@pytest.mark.parametrize("rows,cols", [(1, 5), (4, 8), (64, 1000)])
def test_dequantize_bit_exact(cuda, rows, cols):
    x = O.normal(rows * cols, 91)
    q, s = O.quantize_i8_symmetric_per_channel(x, rows)
    assert np.array_equal(cuda.dequantize_i8_symmetric_per_channel(q, s), O.dequantize_i8_symmetric_per_channel(q, s))
    assert np.array_equal(cuda.dequantize_i8_symmetric(q, s[0]), O.dequantize_i8_symmetric(q, s[0]))
    p, s4 = O.quantize_i4_symmetric_per_channel(x, rows)
    assert np.array_equal(cuda.dequantize_i4_symmetric_per_channel(p, cols, s4),
                          O.dequantize_i4_symmetric_per_channel(p, cols, s4))


@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
def test_dequantize_asymmetric_and_i4_per_tensor_bit_exact(cuda, n):
    # dequantize_i8_asymmetric (dequant.rs:18-22) on the reference quantizer's
    # own (scale, zero_point), including the pinned-zero-point branches (all
    # positive, all negative), and per-tensor dequantize_i4_symmetric
    # (dequant.rs:45-50) with short packed buffers (unpack_i4 stops early)
    for x in (O.normal(n, 95), np.abs(O.normal(n, 96)) + 0.5, -np.abs(O.normal(n, 97)) - 0.5):
        x = x.astype(np.float32)
        q, s, zp = O.quantize_i8_asymmetric(x)
        got = cuda.dequantize_i8_asymmetric(q, s, zp)
        assert np.array_equal(got, O.dequantize_i8_asymmetric(q, s, zp))
    p, s4 = O.quantize_i4_symmetric(O.normal(n, 98))
    for plen in sorted({p.size, (n + 1) // 2, n // 3, 0}):
        got = cuda.dequantize_i4_symmetric(p[:plen], n, s4)
        want = O.dequantize_i4_symmetric(p[:plen], n, s4)
        assert got.size == min(n, 2 * plen) and np.array_equal(got, want)


def test_dequantize_asymmetric_kat(cuda):
    # dequant.rs:87-95: the asymmetric round trip of [1, 2, 3, 4] within 0.01
    data = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    q, s, zp = cuda.quantize_i8_asymmetric(data)
    d = cuda.dequantize_i8_asymmetric(q, s, zp)
    assert np.all(np.abs(d - data) < 0.01)


def test_ptq_roundtrip_kats(cuda):
    # ptq.rs:358-391 on the device quantizers
    w = (np.arange(32, dtype=np.float32) / np.float32(32.0) - np.float32(0.5)).astype(np.float32)
    q, s = cuda.quantize_i8_symmetric_per_channel(w, 4)
    assert s.size == 4 and q.size == 32
    assert np.all(np.abs(cuda.dequantize_i8_symmetric_per_channel(q, s) - w) < 0.01)
    p, s4 = cuda.quantize_i4_symmetric_per_channel(w, 4)
    assert p.size == 16 and cuda.dequantize_i4_symmetric_per_channel(p, 8, s4).size == 32
