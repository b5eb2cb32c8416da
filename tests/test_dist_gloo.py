"""Head-sharded execution across ranks, on CPU with the gloo backend.

The per-head computation is replaced by a deterministic CPU stand-in (the
kernels need a GPU); what is tested is the sharding contract: contiguous head
slices, offsets drawn for the whole layer then sliced (so plans do not depend
on the number of ranks), and one all-gather in rank order. A rank that fails
before the collective makes the others error out within the process-group
timeout instead of hanging.
"""
import math
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ab_attention_b200 import shard

BH, TOKENS, SEED = 8, 600, 5


def _per_head(x: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """Stand-in for one head's layer: depends on the head's input and its rows' offsets."""
    qb = math.ceil(x.shape[0] / 128)
    scale = offsets.reshape(qb).repeat_interleave(128)[: x.shape[0]]
    return x * scale[:, None] + x.sum()


def _reference():
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(BH, TOKENS, 4, generator=gen)
    offsets = shard.layer_offsets(BH, TOKENS, SEED, "cpu")
    qb = math.ceil(TOKENS / 128)
    out = torch.stack([_per_head(x[h], offsets[h * qb:(h + 1) * qb]) for h in range(BH)])
    return x, out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        x, _ = _reference()
        heads = shard.head_slice(BH, world, rank)
        offsets = shard.shard_offsets(shard.layer_offsets(BH, TOKENS, SEED, "cpu"), TOKENS, heads)
        qb = math.ceil(TOKENS / 128)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the all-gather")
        local = torch.stack([_per_head(x[h], offsets[i * qb:(i + 1) * qb])
                             for i, h in enumerate(range(heads.start, heads.stop))])
        try:
            full = shard.gather_heads(local, world)
            status = "ok"
        except Exception as exc:  # noqa: BLE001
            full, status = None, f"error: {type(exc).__name__}"
        if rank == 0:
            torch.save({"status": status, "full": full}, result_path)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _block_worker(rank, world, port, result_path, chunks):
    """Block-interleaved heads, each block all-gathered asynchronously into place."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        x, _ = _reference()
        heads = shard.rank_heads(BH, world, rank, chunks)
        offsets = shard.shard_offsets(shard.layer_offsets(BH, TOKENS, SEED, "cpu"), TOKENS, heads)
        qb = math.ceil(TOKENS / 128)
        ch = len(heads) // chunks
        out = torch.empty_like(x)
        works = []
        for c in range(chunks):
            block = torch.stack([_per_head(x[h], offsets[i * qb:(i + 1) * qb])
                                 for i, h in enumerate(heads) if c * ch <= i < (c + 1) * ch])
            works.append(shard.gather_block(out, block, world, c, async_op=True))
        for w in works:
            w.wait()
        if rank == 0:
            torch.save({"status": "ok", "full": out}, result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunks", [(2, 2), (4, 2), (2, 4)])
def test_block_interleaved_gather_matches_single_process(tmp_path, world, chunks):
    path = str(tmp_path / "out.pt")
    mp.start_processes(_block_worker, args=(world, _free_port(), path, chunks), nprocs=world, join=True,
                       start_method="spawn")
    _, want = _reference()
    assert torch.equal(torch.load(path)["full"], want)


def test_rank_heads_partition_every_head_once():
    for world, chunks in [(1, 1), (2, 4), (4, 2), (8, 1)]:
        owned = sorted(h for r in range(world) for h in shard.rank_heads(BH, world, r, chunks))
        assert owned == list(range(BH))
    assert shard.chunk_count(80, 8) == 5 and shard.chunk_count(80, 2) == 8 and shard.chunk_count(24, 8) == 3
    assert shard.chunk_count(80, 8, max_chunks=4) == 2
    with pytest.raises(ValueError):
        shard.rank_heads(BH, 3, 0)


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_layer_matches_single_process(tmp_path, world):
    path = str(tmp_path / "out.pt")
    mp.start_processes(_worker, args=(world, _free_port(), path, -1), nprocs=world, join=True,
                       start_method="spawn")
    result = torch.load(path)
    _, want = _reference()
    assert result["status"] == "ok"
    assert torch.equal(result["full"], want)


def test_plan_offsets_do_not_depend_on_world_size():
    full = shard.layer_offsets(BH, TOKENS, SEED, "cpu")
    qb = math.ceil(TOKENS / 128)
    for world in (1, 2, 4, 8):
        parts = [shard.shard_offsets(full, TOKENS, shard.head_slice(BH, world, r)) for r in range(world)]
        assert torch.equal(torch.cat(parts), full)
        assert all(p.numel() == BH // world * qb for p in parts)
    with pytest.raises(ValueError):
        shard.head_slice(BH, 3, 0)


def test_failed_rank_surfaces_as_error_not_hang(tmp_path):
    path = str(tmp_path / "out.pt")
    ctx = mp.start_processes(_worker, args=(2, _free_port(), path, 1), nprocs=2, join=False,
                             start_method="spawn")
    with pytest.raises(Exception):
        while not ctx.join(timeout=60):
            pass
    # rank 0 either recorded an error from the collective or never wrote a result
    if os.path.exists(path):
        assert torch.load(path)["status"].startswith("error")


def test_taper_sizes_end_with_one_head_and_cover_the_rank():
    for per in (1, 2, 3, 5, 10, 12, 20, 40, 80):
        sizes = shard.taper_sizes(per)
        assert sum(sizes) == per and len(sizes) <= 8
        assert sizes == sorted(sizes, reverse=True)
        if per <= 36:
            assert sizes[-1] == 1
    assert shard.taper_sizes(10) == [4, 3, 2, 1]


@pytest.mark.parametrize("world,sizes", [(2, [2, 1, 1]), (4, [1, 1])])
def test_uneven_blocks_partition_and_gather_in_place(tmp_path, world, sizes):
    owned = sorted(h for r in range(world) for h in shard.rank_heads(BH, world, r, sizes))
    assert owned == list(range(BH))
    path = str(tmp_path / "out.pt")
    mp.start_processes(_uneven_worker, args=(world, _free_port(), path, sizes), nprocs=world, join=True,
                       start_method="spawn")
    _, want = _reference()
    assert torch.equal(torch.load(path)["full"], want)


def _uneven_worker(rank, world, port, result_path, sizes):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        x, _ = _reference()
        heads = shard.rank_heads(BH, world, rank, sizes)
        offsets = shard.shard_offsets(shard.layer_offsets(BH, TOKENS, SEED, "cpu"), TOKENS, heads)
        qb = math.ceil(TOKENS / 128)
        out = torch.empty_like(x)
        works, local, first = [], 0, 0
        for c, b in enumerate(sizes):
            block = torch.stack([_per_head(x[heads[i]], offsets[i * qb:(i + 1) * qb])
                                 for i in range(local, local + b)])
            works.append(shard.gather_block(out, block, world, c, async_op=True, start=first))
            local += b
            first += world * b
        for w in works:
            w.wait()
        if rank == 0:
            torch.save({"status": "ok", "full": out}, result_path)
    finally:
        dist.destroy_process_group()


def _copy_streams_worker(rank, world, port, result_path, count):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        try:
            shard.PeerOutputs(torch.empty(4, 8), copy_streams=count)
            status = "accepted"
        except ValueError:
            status = "ValueError"
        if rank == 0:
            torch.save({"status": status}, result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("count", [0, 2])
def test_peer_outputs_rejects_copy_stream_counts_outside_one_to_world_minus_one(tmp_path, count):
    # With 2 ranks a block has one peer to copy to: one copy stream at most.
    path = str(tmp_path / "out.pt")
    mp.start_processes(_copy_streams_worker, args=(2, _free_port(), path, count), nprocs=2, join=True,
                       start_method="spawn")
    assert torch.load(path)["status"] == "ValueError"
