"""The allocation-free quantize entry point, checked against the regular one.

tpt_cuda_quantize_i8_symmetric_noalloc exists for callers that cannot allocate
device memory (engines that own the whole GPU memory budget, real-time paths
that cannot take cudaMalloc's implicit synchronisation, code that must not
fail for lack of memory midway); its scratch is a fixed array in the library.
This file is collected last on purpose so that a stop-at-first-failure run has
already run every other test. It passes alone in a fresh process too.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _max_elems():
    src = open(os.path.join(ROOT, "include", "tpt_cuda.h")).read()
    return int(re.search(r"#define TPT_NOALLOC_QUANT_MAX_ELEMS (\d+)", src).group(1))


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_quantize_matches_context_entry_point_on_two_calls(cuda):
    import torch

    from tpt_infer_b200._capi import lib

    stream = torch.cuda.current_stream()
    # Two calls in a row; the second is smaller and has a smaller max|x|, so
    # any stale partial left in the shared scratch by the first would show.
    for n, seed, std in ((3_000_001, 11, 2.0), (70_000, 12, 0.5)):
        x = torch.from_numpy(O.normal(n, seed, 0.0, std)).cuda()
        q_na = torch.empty(n, dtype=torch.int8, device="cuda")
        s_na = torch.empty(1, dtype=torch.float32, device="cuda")
        q_ref = torch.empty(n, dtype=torch.int8, device="cuda")
        s_ref = torch.empty(1, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        st = lib.tpt_cuda_quantize_i8_symmetric_noalloc(_p(x), n, _p(q_na), _p(s_na), C.c_void_p(stream.cuda_stream))
        assert st == 0
        torch.cuda.synchronize()
        cuda.quantize_i8_symmetric_dev(x, q_ref, s_ref)
        cuda.sync()
        # bit-exact, the tolerance the quantize tests use
        assert s_na.view(torch.int32).item() == s_ref.view(torch.int32).item()
        assert torch.equal(q_na, q_ref)


@pytest.mark.parametrize("n,special", [(3 * 8192, False), (3 * 8192 + 1, False), (8192, False), (40_000, True)])
def test_noalloc_quantize_tile_edges_and_non_finite(cuda, n, special):
    # n an exact multiple of the 8192-element reduction tile (the last tile
    # full) and one past it (a one-element last tile); an input holding NaN and
    # +-Inf, where both entry points must ignore NaN in the max and agree on the
    # resulting scale and codes bit for bit
    import torch

    from tpt_infer_b200._capi import lib

    h = O.normal(n, 21, 0.0, 1.0)
    if special:
        h[5], h[777], h[n - 1] = np.nan, np.inf, -np.inf
    x = torch.from_numpy(h).cuda()
    for _ in range(2):
        q_na = torch.empty(n, dtype=torch.int8, device="cuda")
        s_na = torch.empty(1, dtype=torch.float32, device="cuda")
        q_ref = torch.empty(n, dtype=torch.int8, device="cuda")
        s_ref = torch.empty(1, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        st = lib.tpt_cuda_quantize_i8_symmetric_noalloc(_p(x), n, _p(q_na), _p(s_na), None)
        assert st == 0
        torch.cuda.synchronize()
        cuda.quantize_i8_symmetric_dev(x, q_ref, s_ref)
        cuda.sync()
        assert s_na.view(torch.int32).item() == s_ref.view(torch.int32).item()
        assert torch.equal(q_na, q_ref)


def test_noalloc_quantize_edge_sizes(cuda):
    import torch

    from tpt_infer_b200._capi import lib

    s = torch.empty(1, dtype=torch.float32, device="cuda")
    q = torch.empty(8, dtype=torch.int8, device="cuda")
    x = torch.zeros(8, dtype=torch.float32, device="cuda")
    # empty input: scale 1.0, nothing else touched
    assert lib.tpt_cuda_quantize_i8_symmetric_noalloc(_p(x), 0, _p(q), _p(s), None) == 0
    torch.cuda.synchronize()
    assert s.item() == 1.0
    # beyond the scratch's maximum: rejected up front (TPT_INVALID), nothing enqueued
    assert lib.tpt_cuda_quantize_i8_symmetric_noalloc(_p(x), _max_elems() + 1, _p(q), _p(s), None) == 4
    # the documented KAT of quant.rs:18-24
    x3 = torch.tensor([-1.0, 0.0, 1.0], dtype=torch.float32, device="cuda")
    assert lib.tpt_cuda_quantize_i8_symmetric_noalloc(_p(x3), 3, _p(q), _p(s), None) == 0
    torch.cuda.synchronize()
    assert q[:3].tolist() == [-127, 0, 127] and abs(s.item() - 1 / 127) < 1e-6
