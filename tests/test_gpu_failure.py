"""Failure detection without a GPU fault.

- Bounded device waits: with the context's wait limit cut to a few hundred SM
  cycles (tpt_cuda_ctx_set_wait_limit), a normal launch of the TMA-ring W8A8
  kernel runs out of its waits; the kernel leaves its loops, waits (with the
  full bound) for its own copies in flight and returns, the host sees
  TPT_TIMEOUT, and with the default limit restored the next call on the same
  context is correct.
- NCCL set-up deadline: a communicator of two ranks whose second rank never
  joins ends in TPT_NCCL_ERROR after the (shortened) deadline, not a hang; run
  in a child process on one GPU.
"""
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TPT_TIMEOUT, TPT_NCCL_ERROR = 7, 8


def test_bounded_wait_selftest(cuda):
    # a barrier nothing arrives on: the bounded wait runs out (the default ~1 s
    # bound, then a 1000-cycle limit), the host reads TPT_TIMEOUT, and the
    # context keeps working
    import ctypes as C

    from tpt_infer_b200._capi import lib

    out = C.c_uint(0)
    for limit in (0, 1000):
        assert lib.tpt_cuda_ctx_set_wait_limit(cuda.ctx, limit) == 0
        t0 = time.time()
        assert lib.tpt_cuda_selftest_bounded_wait(cuda.ctx, C.byref(out)) == TPT_TIMEOUT
        assert out.value == 2  # not satisfied; the CTA's abort raised
        assert time.time() - t0 < 10
    assert lib.tpt_cuda_ctx_set_wait_limit(cuda.ctx, 0) == 0
    x = O.normal(1000, 5)
    q, s = cuda.quantize_i8_symmetric(x)
    assert np.array_equal(q, O.quantize_i8_symmetric(x)[0])


def test_wait_limit_timeout_then_recovers(cuda):
    import torch

    from tpt_infer_b200._capi import lib
    from tpt_infer_b200.backend import OpError

    m, n, k = 16, 32768, 4096  # the TMA-ring small-batch kernel, its ring cycling over HBM loads
    w = O.normal(n * k, 300, 0.0, 0.02)
    wq, ws = O.quantize_i8_symmetric_per_channel(w, n)
    aq, sa = O.quantize_i8_symmetric(O.normal(m * k, 301))
    bias = O.normal(n, 302, 0.0, 0.01)
    wh = cuda.upload_i8(wq, ws, n, k)
    a = torch.from_numpy(aq).cuda()
    b = torch.from_numpy(bias).cuda()
    y = torch.empty(m * n, dtype=torch.float32, device="cuda")
    want = O.w8a8_gemm(aq, wq, m, n, k, sa, ws, bias, 0, threads=8)
    try:
        assert lib.tpt_cuda_ctx_set_wait_limit(cuda.ctx, 100) == 0
        cuda.w8a8_gemm_dev(a, m, sa, wh, b, 0, y)
        with pytest.raises(OpError) as e:
            cuda.sync()
        assert e.value.code == TPT_TIMEOUT
    finally:
        assert lib.tpt_cuda_ctx_set_wait_limit(cuda.ctx, 0) == 0
    for _ in range(2):  # the context is usable and correct again
        cuda.w8a8_gemm_dev(a, m, sa, wh, b, 0, y)
        cuda.sync()
        assert np.array_equal(y.cpu().numpy(), want)
    wh.free()


_NCCL_CHILD = r"""
import ctypes as C, sys, time
sys.path.insert(0, sys.argv[1])
from tpt_infer_b200 import CudaBackend
from tpt_infer_b200._capi import lib
be = CudaBackend.new(0)
uid = (C.c_ubyte * 128)()
st = lib.tpt_cuda_comm_unique_id(uid, 128)
if st != 0:
    print("NOID", st); sys.exit(0)
assert lib.tpt_cuda_comm_set_timeout(3.0) == 0
h = C.c_void_p()
t0 = time.time()
st = lib.tpt_cuda_comm_create(be.ctx, uid, 128, 2, 0, C.byref(h))
print("STATUS", st, round(time.time() - t0, 1), flush=True)
"""


def test_nccl_setup_deadline_when_a_rank_never_joins():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    t0 = time.time()
    r = subprocess.run([sys.executable, "-c", _NCCL_CHILD, ROOT], capture_output=True, text=True, timeout=240,
                       env=env)
    line = [ln for ln in r.stdout.splitlines() if ln.startswith(("STATUS", "NOID"))]
    assert line, r.stdout + r.stderr
    if line[0].startswith("NOID"):
        pytest.skip("NCCL not available")
    st, secs = int(line[0].split()[1]), float(line[0].split()[2])
    assert st == TPT_NCCL_ERROR
    assert secs < 60 and time.time() - t0 < 200
