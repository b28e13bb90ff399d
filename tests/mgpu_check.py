"""Multi-GPU check, one process per GPU (launched by tests/test_gpu_multi.py):

  python -m torch.distributed.run --nnodes 1 --nproc-per-node P \
      --master-addr 127.0.0.1 --master-port PORT tests/mgpu_check.py

1. FFN column sharding: a 2-layer BERT-shaped plan built unsharded and with
   FFN1 column-sharded over the ranks (ALLGATHER + PANELS_TO_ROWS inside the
   plan) calibrates to the same scales and gives bit-identical outputs.
2. Batch sharding: each rank's slice of the batch through the unsharded plan
   equals the same rows of the full batch.
Rank 0 prints one JSON line; any mismatch raises (non-zero exit).
"""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from tpt_infer_b200 import CudaBackend, graphs, sharding, synth  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    be = CudaBackend.new(local)
    comm = sharding.Comm.create(be, world, rank, sharding.torch_broadcast)
    B, S, L, H = 2 * world, 64, 2, 768
    layers = graphs.bert_weights(be, layers=L)
    cal = synth.normal(B * S * H, 41)
    xin = synth.normal(B * S * H, 42)

    ref, xr, hr = graphs.build_bert(be, B, S, layers)
    shd, xs, hs = graphs.build_bert(be, B, S, layers, ffn_shard=comm)
    for p, x, h in ((ref, xr, hr), (shd, xs, hs)):
        p.calibrate(True)
        p.run({x: cal}, [h])
        p.freeze()
    assert np.array_equal(ref.scales(), shd.scales()), "rank-global scales differ"
    yr = ref.run({xr: xin}, [hr])[0]
    ys = shd.run({xs: xin}, [hs])[0]
    assert np.array_equal(yr, ys), f"ffn-sharded output differs: max {np.max(np.abs(yr - ys))}"
    shd.set_graph(True)  # recorded with its NCCL all-gathers (first run), then replayed
    for _ in range(2):
        yg = shd.run({xs: xin}, [hs])[0]
        assert np.array_equal(yr, yg), "graph-replayed ffn-sharded output differs"

    b0, bn = sharding.batch_shard(B, world, rank)
    part, xp, hp = graphs.build_bert(be, bn, S, layers)
    part.set_scales(ref.scales())  # the batch slice runs with the full batch's frozen scales
    yp = part.run({xp: xin[b0 * S * H:(b0 + bn) * S * H]}, [hp])[0]
    assert np.array_equal(yp, yr[b0 * S * H:(b0 + bn) * S * H]), "batch shard differs"

    ok = torch.tensor([1], device="cuda")
    dist.all_reduce(ok)
    if rank == 0:
        print(json.dumps({"ok": True, "world": world, "ranks_ok": int(ok.item()),
                          "ffn_shard": "bit-identical (direct and graph-replayed)",
                          "batch_shard": "bit-identical"}), flush=True)
    for p in (part, shd, ref):
        p.close()
    comm.close()
    be.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
