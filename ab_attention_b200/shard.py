"""Head sharding across the GPUs of one node.

Every AB-attention row (head, 128-query block) depends only on its own head's
Q/K/V and its own uniform offset, so heads split across ranks with no
communication during compute. The per-row offsets are drawn once for the whole
layer from the seed (as the reference draws them before chunking,
ab_attention/attention.py:56-57) and sliced, so the plan is bit-identical for
any number of GPUs. The output is reassembled with NCCL all-gathers.

Heads are dealt to ranks in blocks so that the all-gathers overlap compute: the
layer's heads form consecutive blocks, block c holding world * b_c heads, of
which rank r owns [start_c + r * b_c, start_c + (r + 1) * b_c). The blocks are
either even (`chunks` blocks of the same size) or tapered (`taper_sizes`: the
largest first and one head per rank last, so the all-gather left exposed after
the last prefill is the smallest). A rank builds the plan for all its heads at
once, then runs the sparse prefill block by block and all-gathers block c
(straight into its place in the [BH, S, 128] output) while block c + 1
computes. Consecutive blocks' prefills can also alternate between streams
(`block_streams`), so that a block's launch fills the SMs the previous block's
last wave leaves idle; measured on 8 B200s this starves NCCL's all-gather
kernels of SMs (the gathers then queue behind the prefills), so one stream is
the default.

Two alternatives to the NCCL all-gather share every rank's copy of the output
through CUDA IPC (`PeerOutputs`): `attention_copied` pushes each finished head
block to the other ranks with copy engines, and `attention_scatter` has the
prefill store every output row into all copies itself.
"""
from __future__ import annotations

import ctypes
import math

import torch


def chunk_count(batch_heads: int, world: int, max_chunks: int = 8) -> int:
    """Largest number of head blocks <= max_chunks that divides the heads evenly.

    More blocks shorten the exposed all-gather of the last block; 8 keeps each
    block's prefill launch at several waves of CTAs at the Wan shapes."""
    if batch_heads % world:
        raise ValueError(f"{batch_heads} heads do not split evenly over {world} ranks")
    for chunks in range(max_chunks, 0, -1):
        if batch_heads % (world * chunks) == 0:
            return chunks
    return 1


def taper_sizes(per_rank: int, max_blocks: int = 8) -> list[int]:
    """Heads per rank in each block, non-increasing and ending with one head:
    1, 2, ..., n from the end (n(n + 1)/2 <= per_rank, n <= max_blocks), the
    remainder as one more block or, at the block limit, one head more on each of
    the largest blocks. Each block's all-gather then hides under the next,
    smaller block's prefill (a head's gather over NVLink takes well under half
    its prefill) and the gather left exposed at the end is one head per rank."""
    if per_rank <= 0 or max_blocks <= 0:
        raise ValueError("a rank needs at least one head and one block")
    n = 1
    while n + 1 <= max_blocks and (n + 1) * (n + 2) // 2 <= per_rank:
        n += 1
    sizes = list(range(n, 0, -1))
    rest = per_rank - n * (n + 1) // 2
    if rest and n < max_blocks:
        sizes.append(rest)
    else:
        for i in range(rest):
            sizes[i % n] += 1
    return sorted(sizes, reverse=True)


def block_sizes(batch_heads: int, world: int, chunks) -> list[int]:
    """Heads per rank in each block: `chunks` is a block count (even blocks) or
    the list of sizes itself."""
    if batch_heads % world:
        raise ValueError(f"{batch_heads} heads do not split evenly over {world} ranks")
    per = batch_heads // world
    if isinstance(chunks, int):
        if per % chunks:
            raise ValueError(f"{batch_heads} heads do not split into {chunks} blocks over {world} ranks")
        return [per // chunks] * chunks
    sizes = [int(c) for c in chunks]
    if any(c <= 0 for c in sizes) or sum(sizes) != per:
        raise ValueError(f"block sizes {sizes} do not cover the {per} heads of a rank")
    return sizes


def rank_heads(batch_heads: int, world: int, rank: int, chunks=1) -> list[int]:
    """The flattened heads rank `rank` owns, in its local (block-major) order.
    `chunks`: a block count (even blocks) or the per-rank block sizes."""
    sizes = block_sizes(batch_heads, world, chunks)
    heads, start = [], 0
    for b in sizes:
        heads.extend(start + rank * b + i for i in range(b))
        start += world * b
    return heads


def head_slice(batch_heads: int, world: int, rank: int) -> slice:
    """Contiguous heads of `rank` (the one-block layout)."""
    heads = rank_heads(batch_heads, world, rank, 1)
    return slice(heads[0], heads[-1] + 1)


def layer_offsets(batch_heads: int, tokens: int, seed: int, device) -> torch.Tensor:
    """The whole layer's per-row uniforms (rows = BH * ceil(tokens/128))."""
    rows = batch_heads * math.ceil(tokens / 128)
    generator = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(rows, device=device, generator=generator)


def shard_offsets(offsets: torch.Tensor, tokens: int, heads) -> torch.Tensor:
    """Rows of `heads` (a slice or a list of heads) in that order."""
    qb = math.ceil(tokens / 128)
    if isinstance(heads, slice):
        return offsets[heads.start * qb:heads.stop * qb].contiguous()
    return torch.cat([offsets[h * qb:(h + 1) * qb] for h in heads]).contiguous()


def gather_heads(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather [BH/G, ...] shards into [BH, ...] (rank order = head order)."""
    import torch.distributed as dist

    if world == 1:
        return local
    out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def gather_block(out: torch.Tensor, local_block: torch.Tensor, world: int, block: int, group=None,
                 async_op: bool = False, start: int | None = None):
    """All-gather block `block` (each rank's [ch, ...] heads) into its place in
    `out` [BH, ...]: heads [start, start + world * ch), start = block * world * ch
    for even blocks (pass `start` for uneven ones)."""
    import torch.distributed as dist

    ch = local_block.shape[0]
    first = block * world * ch if start is None else start
    dst = out[first:first + world * ch]
    if world == 1:
        dst.copy_(local_block)
        return None
    return dist.all_gather_into_tensor(dst, local_block.contiguous(), group=group, async_op=async_op)


def attention_sharded(q, k, v, offsets, out, *, world: int, chunks, sample_pages: int = 64,
                      text_kv=None, group=None, timing: dict | None = None, block_streams: int = 1):
    """This rank's part of a head-sharded AB-attention layer.

    q, k, v: [1, per, S, 128] bf16, the rank's heads in `rank_heads(BH, world,
    rank, chunks)` order (`chunks`: a block count or the per-rank block sizes);
    offsets: their rows of `layer_offsets` (see `shard_offsets`); out: [BH, S,
    128] bf16, receives every rank's output. The plan covers all the rank's
    heads in one call; the prefill runs block by block, consecutive blocks on
    `block_streams` alternating streams, and block c is all-gathered on NCCL's
    stream while block c + 1 computes. Returns when `out` is complete on the
    current stream.

    `timing` (a dict, optional) receives CUDA events recorded on the current
    stream: "plan" (start, end), "blocks" [(start, end)] around each block's
    prefill, and "tail" (after the last prefill, after the last all-gather
    has landed), whose span is the all-gather time left exposed.
    """
    from .attention import SamplePlan, apply_plan, build_plan

    per, tokens = q.shape[1], q.shape[2]
    sizes = block_sizes(per * world, world, chunks)
    qb = math.ceil(tokens / 128)
    main = torch.cuda.current_stream(q.device)
    streams = [main] + [torch.cuda.Stream(q.device) for _ in range(max(1, block_streams) - 1)]

    def event(stream=None):
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream or main)
        return e

    if timing is not None:
        timing["blocks"] = []
        plan_start = event()
    plan = build_plan(q, k, sample_pages=sample_pages, offsets=offsets)
    planned = event()
    if timing is not None:
        timing["plan"] = (plan_start, planned)
    works = []
    first = local = 0
    for c, ch in enumerate(sizes):
        stream = streams[c % len(streams)]
        heads = slice(local, local + ch)
        rows = slice(local * qb, (local + ch) * qb)
        block_plan = SamplePlan(plan.descriptor[rows], plan.log_weights[rows])
        block_text = None if text_kv is None else tuple(t[:, heads] for t in text_kv)
        stream.wait_event(planned)
        with torch.cuda.stream(stream):
            start = event(stream) if timing is not None else None
            o = apply_plan(q[:, heads], k[:, heads], v[:, heads], block_plan, text_kv=block_text)
            if timing is not None:
                timing["blocks"].append((start, event(stream)))
            # issued from the block's stream, so NCCL waits for this block only
            works.append(gather_block(out, o.reshape(ch, tokens, q.shape[3]), world, c, group=group,
                                      async_op=True, start=first))
        first += world * ch
        local += ch
    for stream in streams[1:]:
        main.wait_stream(stream)
    tail_start = event() if timing is not None else None
    for work in works:
        if work is not None:
            work.wait()
    if timing is not None:
        timing["tail"] = (tail_start, event())
    return out


def attention_sharded_host(q, k, v, offsets, out, host_out, *, world: int, chunks: int, sample_pages: int = 64,
                           text_kv=None, group=None):
    """`attention_sharded` for Q/K/V in host memory, with the copies overlapped.

    q, k, v: pinned host [1, per, S, 128] bf16, the rank's heads in
    `rank_heads(BH, world, rank, chunks)` order (`chunks`: a block count or the
    per-rank block sizes); offsets: their rows of
    `layer_offsets` on the device; out: [BH, S, 128] bf16 on the device,
    receives every rank's output; host_out: pinned host [1, per, S, 128],
    receives this rank's heads. text_kv (optional): the rank's prompt keys and
    values on the device, [1, per, T, 128] each.

    Head block c + 1 is copied in on a side stream while block c is planned,
    attended and all-gathered, and block c's own heads are copied out on a
    third stream, so the layer costs about its host transfers rather than their
    sum with the compute. The plan of each block is built from its rows of the
    layer's offsets, so it is bit-identical to `attention_sharded`'s. Every
    rank issues the same all-gathers in the same order. Returns when `out` and
    host_out are complete on the current stream.
    """
    from .attention import apply_plan, build_plan

    per, tokens, dim = q.shape[1], q.shape[2], q.shape[3]
    sizes = block_sizes(per * world, world, chunks)
    if q.device.type != "cpu" or k.device.type != "cpu" or v.device.type != "cpu" or host_out.device.type != "cpu":
        raise ValueError("q, k, v and host_out must be host tensors")
    if host_out.shape != q.shape or host_out.dtype != q.dtype:
        raise ValueError("host_out must be shaped like q")
    ch = max(sizes)
    starts = [sum(sizes[:c]) for c in range(len(sizes))]
    qb = math.ceil(tokens / 128)
    device = out.device
    main = torch.cuda.current_stream(device)
    copy_in = torch.cuda.Stream(device)
    copy_out = torch.cuda.Stream(device)
    copy_in.wait_stream(main)  # work the caller queued before this call comes first
    # two device slots per input so block c + 1 lands while block c computes
    slots = [[torch.empty((1, ch, tokens, dim), dtype=q.dtype, device=device) for _ in range(3)] for _ in range(2)]
    landed = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def load(c):
        s, b, h0 = c % 2, sizes[c], starts[c]
        with torch.cuda.stream(copy_in):
            if c >= 2:
                copy_in.wait_event(freed[s])  # the slot's previous block has been consumed
            for dst, src in zip(slots[s], (q, k, v)):
                dst[:, :b].copy_(src[:, h0:h0 + b], non_blocking=True)
            landed[s].record(copy_in)

    works = []
    load(0)
    for c, b in enumerate(sizes):
        if c + 1 < len(sizes):
            load(c + 1)
        s, h0 = c % 2, starts[c]
        main.wait_event(landed[s])
        qs, ks, vs = (x[:, :b] for x in slots[s])
        plan = build_plan(qs, ks, sample_pages=sample_pages, offsets=offsets[h0 * qb:(h0 + b) * qb])
        block_text = None if text_kv is None else tuple(t[:, h0:h0 + b] for t in text_kv)
        o = apply_plan(qs, ks, vs, plan, text_kv=block_text)
        freed[s].record(main)
        works.append(gather_block(out, o.reshape(b, tokens, dim), world, c, group=group, async_op=True,
                                  start=world * h0))
        done = torch.cuda.Event()
        done.record(main)
        with torch.cuda.stream(copy_out):
            copy_out.wait_event(done)
            host_out[:, h0:h0 + b].copy_(o, non_blocking=True)
            o.record_stream(copy_out)
    for work in works:
        if work is not None:
            work.wait()
    main.wait_stream(copy_out)
    return out


# ---- output scatter over peer memory --------------------------------------------------------

class PeerOutputs:
    """Every rank's [BH, S, 128] layer output, mapped into this process.

    Each rank allocates its own copy of the layer output; the ranks exchange CUDA
    IPC handles (abx_ipc_handle) over the process group and map the others'
    copies for this rank's device (abx_ipc_open, peer access enabled), so one
    kernel can store its rows into all of them over NVLink. `pointers` lists the
    device addresses in rank order (this rank's own copy at its rank).
    `copy_streams` (1 to world - 1) are the streams `attention_copied` pushes
    finished head blocks on; peers are spread over them, so with world - 1
    streams every peer's copy runs on its own stream. Call `close()` before the
    process group is destroyed.
    """

    def __init__(self, out: torch.Tensor, group=None, copy_streams: int = 1):
        import torch.distributed as dist

        from . import _lib

        self.out = out
        self._lib = _lib.load()
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if not 1 <= copy_streams <= max(1, world - 1):
            raise ValueError(f"copy_streams must be in [1, {max(1, world - 1)}], got {copy_streams}")
        # peer copies of finished head blocks
        self.copy_streams = [torch.cuda.Stream(out.device) for _ in range(copy_streams)]
        self.copy_stream = self.copy_streams[0]
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_size_t(0)
        with torch.cuda.device(out.device):
            _lib.check(self._lib.abx_ipc_handle(_lib.ptr(out), handle, ctypes.byref(offset)), "abx_ipc_handle")
        shared = [None] * world
        dist.all_gather_object(shared, (bytes(handle.raw), offset.value), group=group)
        self._opened = []
        self.pointers = []
        with torch.cuda.device(out.device):
            for r, (raw, off) in enumerate(shared):
                if r == rank:
                    self.pointers.append(out.data_ptr())
                    continue
                base = ctypes.c_void_p(0)
                _lib.check(self._lib.abx_ipc_open(ctypes.create_string_buffer(raw, 64), ctypes.byref(base)),
                           "abx_ipc_open")
                self._opened.append(base.value)
                self.pointers.append(base.value + off)

    def close(self) -> None:
        from . import _lib

        with torch.cuda.device(self.out.device):
            for base in self._opened:
                _lib.check(self._lib.abx_ipc_close(ctypes.c_void_p(base)), "abx_ipc_close")
        self._opened = []
        self.pointers = []


def attention_scatter(q, k, v, offsets, peers: PeerOutputs, *, rank: int, world: int, sample_pages: int = 64,
                      text_kv=None, group=None, timing: dict | None = None):
    """This rank's part of a head-sharded AB-attention layer whose output needs no
    all-gather: the rank plans its contiguous heads (`head_slice(BH, world,
    rank)`), and one paired-prefill launch writes every output row into all
    ranks' copies of the layer output (`peers`) through peer stores over NVLink.

    Two one-element all-reduces on the current stream bracket the launch: the
    first orders it after every rank's earlier readers of the output (the
    buffers are overwritten), the second tells every rank that all rows have
    landed. Returns when `peers.out` is complete on the current stream.
    """
    import torch.distributed as dist

    from . import ops
    from .attention import build_plan

    per, tokens, dim = q.shape[1], q.shape[2], q.shape[3]
    bh = per * world
    flag = torch.zeros(1, dtype=torch.float32, device=q.device)

    def event():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    dist.all_reduce(flag, group=group)
    start = event() if timing is not None else None
    plan = build_plan(q, k, sample_pages=sample_pages, offsets=offsets)
    planned = event() if timing is not None else None
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    tk = tv = None
    if text_kv is not None:
        tk, tv = (t.reshape(per, -1, dim).contiguous() for t in text_kv)
    ops.sparse_prefill_scatter(q.reshape(per, tokens, dim).contiguous(), k.reshape(per, tokens, dim).contiguous(),
                               v.reshape(per, tokens, dim).contiguous(), ids, logw, peers.pointers,
                               head_base=rank * per, out_heads=bh, text_k=tk, text_v=tv)
    attended = event() if timing is not None else None
    dist.all_reduce(flag, group=group)
    if timing is not None:
        timing["plan"] = (start, planned)
        timing["blocks"] = [(planned, attended)]
        timing["tail"] = (attended, event())
    return peers.out


def attention_copied(q, k, v, offsets, peers: PeerOutputs, *, rank: int, world: int, chunks, sample_pages: int = 64,
                     text_kv=None, group=None, timing: dict | None = None):
    """`attention_sharded` with the all-gather done by copy engines.

    Same block-interleaved heads and plan as `attention_sharded`; each block's
    prefill writes its rows straight into this rank's copy of the layer output
    (at the block's global heads), and as soon as it finishes, the copy streams
    push that slice into every other rank's copy (`abx_peer_copy` through the
    `peers` mappings: copy engines over NVLink, no SMs), so the next block's
    prefill keeps every SM. Rank g visits its peers in the order g + 1, g + 2, ...
    (mod world), dealt round-robin over `peers.copy_streams`, so the ranks start
    on different destinations. Two one-element all-reduces bracket the step, as
    in `attention_scatter`. Returns when `peers.out` is complete on the current
    stream.
    """
    import torch.distributed as dist

    from . import _lib, ops
    from .attention import build_plan

    per, tokens, dim = q.shape[1], q.shape[2], q.shape[3]
    sizes = block_sizes(per * world, world, chunks)
    bh = per * world
    qb = math.ceil(tokens / 128)
    head_bytes = tokens * dim * q.element_size()
    lib = _lib.load()
    main = torch.cuda.current_stream(q.device)
    streams = peers.copy_streams
    targets = [(rank + i) % world for i in range(1, world)]
    own = peers.pointers[rank]
    flag = torch.zeros(1, dtype=torch.float32, device=q.device)

    def event():
        e = torch.cuda.Event(enable_timing=True)
        e.record(main)
        return e

    dist.all_reduce(flag, group=group)  # every rank is done with the buffers this step overwrites
    if timing is not None:
        timing["blocks"] = []
        plan_start = event()
    plan = build_plan(q, k, sample_pages=sample_pages, offsets=offsets)
    if timing is not None:
        timing["plan"] = (plan_start, event())
    rows_all = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows_all, -1).contiguous()
    logw = plan.log_weights.reshape(rows_all, -1).contiguous()
    q3, k3, v3 = (x.reshape(per, tokens, dim) for x in (q, k, v))
    text3 = None if text_kv is None else tuple(t.reshape(per, -1, dim) for t in text_kv)
    first = local = 0
    for b in sizes:
        heads = slice(local, local + b)
        rows = slice(local * qb, (local + b) * qb)
        head0 = first + rank * b  # this rank's first head of the block, in the layer's order
        start = event() if timing is not None else None
        ops.sparse_prefill_scatter(q3[heads], k3[heads], v3[heads], ids[rows], logw[rows], [own], head_base=head0,
                                   out_heads=bh, text_k=None if text3 is None else text3[0][heads],
                                   text_v=None if text3 is None else text3[1][heads])
        done = event()
        if timing is not None:
            timing["blocks"].append((start, done))
        for s in streams:
            s.wait_event(done)
        for i, r in enumerate(targets):
            s = streams[i % len(streams)]
            _lib.check(lib.abx_peer_copy(ctypes.c_void_p(peers.pointers[r] + head0 * head_bytes),
                                         ctypes.c_void_p(own + head0 * head_bytes), b * head_bytes,
                                         ctypes.c_void_p(s.cuda_stream)), "abx_peer_copy")
        first += world * b
        local += b
    tail_start = event() if timing is not None else None
    for s in streams:
        main.wait_stream(s)
    dist.all_reduce(flag, group=group)  # every rank's rows have landed in every copy
    if timing is not None:
        timing["tail"] = (tail_start, event())
    return peers.out

