"""Requantization without a division: clamp(roundf(y / s), -127, 127).

The int8 epilogues (quantize, implicit-GEMM conv, W8A8 GEMM) form y / s from
s's correctly rounded reciprocal with two FMA residual steps (the second is
Markstein's correction step) for scales in [2^-40, 2^40], and divide for
others. The QUANTIZE op runs the same per-value function; here it is fed the
values where a quotient one ulp off would change the int8 result — every
half-integer multiple of the scale, rounded to f32, and 8 ulps either side —
plus signed zeros, subnormals, huge values, infinities and NaN, for scales
with awkward significands and scales outside the fast range. Expected: the
oracle's C quantizer (an IEEE division and roundf), byte for byte.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SCALES = [1.0, 0.5, np.nextafter(np.float32(1.0), np.float32(2.0)), np.nextafter(np.float32(1.0), np.float32(0.0)),
          0.0123, 3.0, 1.0 / 127.0, 7.3e-5, 2.0 ** -39, 1.7 * 2.0 ** 39,
          2.0 ** -45, 3.1 * 2.0 ** 44]  # the last two take the dividing path


def _crafted(s):
    s = np.float32(s)
    k = np.arange(-140, 141, dtype=np.float32)
    centres = ((k + np.float32(0.5)) * s).astype(np.float32)
    u = centres.view(np.int32)[:, None] + np.arange(-8, 9, dtype=np.int32)[None, :]
    vals = [u.ravel().view(np.float32)]
    vals.append((k * s).astype(np.float32))
    vals.append(np.array([0.0, -0.0, 1e-45, -1e-45, 1e-40, -3e-39, 1.5e-38, 2.0 ** 80, -(2.0 ** 80), 2.0 ** 81,
                          3e38, -3e38, np.inf, -np.inf, np.nan, -np.nan], np.float32))
    rng = np.random.default_rng(int(s.view(np.int32)) & 0xFFFF)
    vals.append((rng.standard_normal(4096) * 60 * s).astype(np.float32))
    vals.append(rng.integers(0, 2 ** 32, 4096, dtype=np.uint64).astype(np.uint32).view(np.float32))
    x = np.concatenate(vals).astype(np.float32)
    pad = (-x.size) % 16
    return np.concatenate([x, np.zeros(pad, np.float32)])


@pytest.mark.parametrize("s", SCALES)
def test_quantize_requant_ties_bit_exact(cuda, s):
    from tpt_infer_b200 import graphs

    x = _crafted(s)
    p = graphs.Plan(cuda)
    tx, tq = p.tensor(graphs.F32, x.size), p.tensor(graphs.I8, x.size)
    p.op(graphs.OP_QUANTIZE, tx, tq, f0=float(np.float32(s)), dims=(x.size,))
    p.finalize()
    got = p.run({tx: x}, [tq])[0]
    p.close()
    got = np.frombuffer(got.tobytes()[:x.size], np.int8)
    want = O.quantize_i8_static(x, np.float32(s))
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(float(x[i]), int(got[i]), int(want[i])) for i in bad[:8]]
