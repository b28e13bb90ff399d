"""Host logic of the multi-GPU paths, on CPU.

- batch and column shard arithmetic;
- the column-sharded FFN composition, run as world-size 2 and 4 ``gloo``
  process groups over the oracle: each rank computes GELU(X W1_r + b1_r) for its
  output channels, quantizes with the max over the ranks (all_reduce MAX), the
  int8 panels are all-gathered and relaid out to rows, and FFN2 runs on the
  full rows. The result must equal the unsharded oracle FFN bit for bit, which
  is what the device plan (ALLGATHER + PANELS_TO_ROWS ops) relies on.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from tpt_infer_b200 import sharding as S


@pytest.mark.parametrize("total,world", [(256, 8), (64, 8), (10, 4), (3, 8), (0, 2), (257, 2)])
def test_batch_shard_covers(total, world):
    seen = []
    for r in range(world):
        a, n = S.batch_shard(total, world, r)
        seen.extend(range(a, a + n))
    assert seen == list(range(total))
    counts = [S.batch_shard(total, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_column_shard():
    assert [S.column_shard(3072, 8, r) for r in (0, 7)] == [(0, 384), (2688, 384)]
    with pytest.raises(ValueError):
        S.column_shard(100, 8, 0)
    with pytest.raises(ValueError):
        S.batch_shard(10, 2, 2)


def test_panels_to_rows():
    P, T, Cc = 3, 5, 4
    panels = np.arange(P * T * Cc, dtype=np.int8)
    rows = S.panels_to_rows(panels, P, T, Cc)
    for t in range(T):
        for p in range(P):
            assert np.array_equal(rows[t, p * Cc:(p + 1) * Cc], panels.reshape(P, T, Cc)[p, t])


# ----------------------------------------------------------------- sharded FFN over gloo
T_, HID, FFN = 24, 64, 256


def _ffn_data():
    x = O.normal(T_ * HID, 900, 0.0, 1.0)
    xq, xs = O.quantize_i8_symmetric(x)
    w1q, w1s = O.quantize_i8_symmetric_per_channel(O.normal(FFN * HID, 901, 0.0, 0.02), FFN)
    b1 = O.normal(FFN, 902, 0.0, 0.02)
    w2q, w2s = O.quantize_i8_symmetric_per_channel(O.normal(HID * FFN, 903, 0.0, 0.02), HID)
    b2 = O.normal(HID, 904, 0.0, 0.02)
    return xq, xs, w1q.reshape(FFN, HID), w1s, b1, w2q, w2s, b2


def _ffn_full():
    xq, xs, w1q, w1s, b1, w2q, w2s, b2 = _ffn_data()
    f = O.w8a8_gemm(xq, w1q, T_, FFN, HID, xs, w1s, b1, O.ACT_GELU)
    s = O.sym_scale(O.absmax(f))
    return O.w8a8_gemm(O.quantize_i8_static(f, s), w2q, T_, HID, FFN, s, w2s, b2, O.ACT_NONE)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        xq, xs, w1q, w1s, b1, w2q, w2s, b2 = _ffn_data()
        c0, cn = S.column_shard(FFN, world, rank)
        f = O.w8a8_gemm(xq, np.ascontiguousarray(w1q[c0:c0 + cn]), T_, cn, HID, xs, w1s[c0:c0 + cn],
                        b1[c0:c0 + cn], O.ACT_GELU)
        m = torch.tensor([float(O.absmax(f))], dtype=torch.float32)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)  # the rank-global calibration max
        s = O.sym_scale(np.float32(m.item()))
        fq = torch.from_numpy(O.quantize_i8_static(f, s).astype(np.int8))
        g = torch.empty(world * fq.numel(), dtype=torch.int8)
        dist.all_gather_into_tensor(g, fq)
        rows = S.panels_to_rows(g.numpy(), world, T_, cn)
        y = O.w8a8_gemm(rows, w2q, T_, HID, FFN, s, w2s, b2, O.ACT_NONE)
        q.put((rank, y.tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ffn_column_shard_gloo_bit_identical(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = _ffn_full()
    for r in range(world):
        assert np.array_equal(np.frombuffer(out[r], np.float32), want), r


# ----------------------------------------------------------------- a rank that leaves
def _leaver(rank, world, port, q):
    # rank 1 leaves between steps (after the first collective, before the
    # second); the others learn of it when their next collective ends with an
    # error within the short process-group timeout, not by hanging
    import datetime
    import time

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # step 1: every rank
    if rank == 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()  # the message is out before the process vanishes
        os._exit(0)  # gone without a word
    t0 = time.time()
    try:
        dist.all_reduce(t)  # step 2: the peer never arrives
        q.put((rank, "completed", time.time() - t0))
    except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError / DistBackendError)
        q.put((rank, "error:" + type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_that_leaves_is_detected_by_the_others():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (what, dt) for r, what, dt in (q.get(timeout=120) for _ in range(2))}
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] == "left"
    assert res[0][0].startswith("error"), res
    assert res[0][1] < 30
