"""Head-sharded layer on two GPUs whose output is reassembled without an NCCL
all-gather: by the prefill's own peer stores (PeerOutputs + attention_scatter),
or by copy-engine peer copies of each finished head block (attention_copied).
Every rank's copy of the layer output equals the single-GPU layer bit for bit.
Needs two visible GPUs (skipped otherwise); NCCL's NVLS is off, the transfers
are plain peer stores and copies."""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADS, GRID, PAGES, SEED = 4, (2, 16, 40), 2, 9


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path, mode):
    import torch.distributed as dist

    from ab_attention_b200 import apply_plan, build_plan, shard
    from ab_attention_b200.synthetic import smooth_field

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    peers = None
    try:
        chunks = 2 if mode == "copy" else 1
        heads = shard.rank_heads(HEADS, world, rank, chunks)
        q, k, v = (x.reshape(1, len(heads), -1, 128)
                   for x in smooth_field(HEADS, *GRID, seed=SEED, device=device, heads=heads))
        tokens = q.shape[2]
        layer = shard.layer_offsets(HEADS, tokens, SEED, device)
        offsets = shard.shard_offsets(layer, tokens, heads)
        out = torch.zeros((HEADS, tokens, 128), dtype=torch.bfloat16, device=device)
        peers = shard.PeerOutputs(out)
        for _ in range(2):  # the second step overwrites the first's output in every copy
            if mode == "copy":
                shard.attention_copied(q, k, v, offsets, peers, rank=rank, world=world, chunks=chunks,
                                       sample_pages=PAGES)
            else:
                shard.attention_scatter(q, k, v, offsets, peers, rank=rank, world=world, sample_pages=PAGES)
        torch.cuda.synchronize()
        fq, fk, fv = (x.reshape(1, HEADS, -1, 128) for x in smooth_field(HEADS, *GRID, seed=SEED, device=device))
        want = apply_plan(fq, fk, fv, build_plan(fq, fk, sample_pages=PAGES, offsets=layer))[0]
        ok = torch.tensor([float(torch.equal(out, want))], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if rank == 0:
            torch.save({"equal": bool(ok.item())}, path)
    finally:
        if peers is not None:
            torch.cuda.synchronize()
            dist.barrier()
            peers.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["scatter", "copy"])
def test_peer_output_equals_single_gpu_layer(tmp_path, mode):
    import torch.multiprocessing as mp

    path = str(tmp_path / "result.pt")
    mp.start_processes(_worker, args=(2, _free_port(), path, mode), nprocs=2, join=True, start_method="spawn")
    assert torch.load(path)["equal"]
