"""Recorded launch sequences (CUDA graphs) of device-pointer calls and plans.

A replay must give bit-identical results to the direct calls (it launches the
same kernels with the same arguments), count its kernels in the context's
launch counter, refuse a recording that would grow a workspace, and refuse a
replay once a workspace has moved.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _w8a8_case(be, m, n, k, seed):
    import torch

    wq, ws = O.quantize_i8_symmetric_per_channel(O.normal(n * k, seed, 0.0, 0.02), n)
    w = be.upload_i8(wq, ws, n, k)
    aq, sa = O.quantize_i8_symmetric(O.normal(m * k, seed + 1))
    a = torch.from_numpy(aq).cuda()
    bias = torch.from_numpy(O.normal(n, seed + 2, 0.0, 0.01)).cuda()
    return w, a, float(sa), bias


def test_graph_replay_matches_direct_calls():
    import torch

    from tpt_infer_b200 import CudaBackend

    be = CudaBackend.new(0)
    n, k = 1024, 2048
    cases = [(m,) + _w8a8_case(be, m, n, k, 300 + m) for m in (1, 16, 200)]
    outs = [torch.empty(m * n, dtype=torch.float32, device="cuda") for m, *_ in cases]
    torch.cuda.synchronize()

    def calls():
        for (m, w, a, sa, bias), y in zip(cases, outs):
            be.w8a8_gemm_dev(a, m, sa, w, bias, 0, y)

    calls()
    be.sync()
    want = [y.cpu().numpy().copy() for y in outs]
    for y in outs:
        y.fill_(float("nan"))
    torch.cuda.synchronize()
    g = be.capture(calls)
    assert g.kernels >= 3
    be.sync()
    assert all(torch.isnan(y).all().item() for y in outs)  # recording runs nothing
    l0 = be.launch_count()
    for _ in range(3):
        g.launch()
    be.sync()
    assert be.launch_count() - l0 == 3 * g.kernels
    for y, wnt in zip(outs, want):
        assert np.array_equal(y.cpu().numpy(), wnt)
    g.close()
    for _, w, *_ in cases:
        w.free()
    be.close()


def test_recording_refuses_workspace_growth_and_stale_replay():
    import torch

    from tpt_infer_b200 import CudaBackend
    from tpt_infer_b200.backend import OpError

    be = CudaBackend.new(0)
    K4, N4 = 4096, 256
    pk, s4 = O.quantize_i4_symmetric_per_channel(O.normal(N4 * K4, 411, 0.0, 0.02), N4)
    w4 = be.upload_i4(pk, s4, N4, K4)
    # M = 16 runs on the tensor-core kernel, whose split activations live in the
    # context workspace
    xs = {m: torch.from_numpy(O.normal(m * K4, 412 + m)).cuda() for m in (16, 512)}
    ys = {m: torch.empty(m * N4, dtype=torch.float32, device="cuda") for m in (16, 512)}
    torch.cuda.synchronize()
    call = lambda m: be.w4_gemm_dev(xs[m], m, w4, None, 0, ys[m])  # noqa: E731
    # a fresh context: the launch workspace for the split activations does not exist yet
    with pytest.raises(OpError):
        be.capture(lambda: call(16))
    # once sized, the same call records and replays
    call(16)
    be.sync()
    want = ys[16].cpu().numpy().copy()
    g = be.capture(lambda: call(16))
    ys[16].zero_()
    torch.cuda.synchronize()
    g.launch()
    be.sync()
    assert np.array_equal(ys[16].cpu().numpy(), want)
    # a larger M needs a larger workspace: it moves, and the recording is stale
    call(512)
    be.sync()
    with pytest.raises(OpError):
        g.launch()
    g.close()
    w4.free()
    be.close()


def test_plan_graph_replay_bit_identical():
    from tpt_infer_b200 import CudaBackend, graphs, synth

    be = CudaBackend.new(0)
    W = graphs.mlp_weights()
    p, x, y, z, _ = graphs.build_mlp_int8(be, 64, W)
    p.calibrate(True)
    for i in range(4):
        p.run({x: synth.uniform(64 * 784, 1000 + i)}, [y])
    p.freeze()
    xin = synth.uniform(64 * 784, 77)
    want_y, want_z = p.run({x: xin}, [y, z])
    p.set_graph(True)
    for _ in range(3):  # direct + record, then replays
        got_y, got_z = p.run({x: xin}, [y, z])
        assert np.array_equal(got_y, want_y) and np.array_equal(got_z, want_z)
    (only_y,) = p.run({x: xin}, [y])  # another output set records again
    assert np.array_equal(only_y, want_y)
    p.set_scales(p.scales())  # new scales drop the recording
    got_y, = p.run({x: xin}, [y])
    assert np.array_equal(got_y, want_y)
    p.close()
    be.close()
