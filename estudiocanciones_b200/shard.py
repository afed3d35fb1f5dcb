"""Take sharding over the GPUs of one box (one process per GPU).

The reference generates its takes as rows of one batch on one device
(``app/engine.py:374-448``, ``n`` takes = ``2n`` CFG rows).  Takes are
independent, so on a box with several B200s they are partitioned across ranks:
each rank runs the unchanged single-GPU decode path on its own takes (its own
KV cache, its own frame graph) with no collective on the hot path, and the
finished token streams are gathered once at the end (NCCL over NVLink on the
GPUs, gloo on CPU for the tests).  Scaling is weak in takes: per-GPU work is
fixed as the number of GPUs grows.

* :func:`partition` - which takes a rank owns (contiguous blocks, the first
  ``n % world`` ranks take one more).
* :func:`gather_streams` - every rank's variable-length ``[8, T]`` streams to
  rank 0 (or to all ranks), in global take order.
* :func:`generate_sharded` - ``generate_ids`` over a rank's takes + the gather.
"""
from __future__ import annotations

import torch


def partition(n_takes: int, world: int, rank: int) -> range:
    """Global take indices owned by ``rank`` out of ``world`` ranks."""
    if n_takes < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad partition request: n={n_takes} world={world} rank={rank}")
    base, extra = divmod(n_takes, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def _dist():
    import torch.distributed as dist
    return dist


def gather_streams(streams: list[torch.Tensor], n_takes: int, world: int, rank: int, *, device=None,
                   to_all: bool = False) -> list[torch.Tensor] | None:
    """Collect the ``[n_cb, T_i]`` int64 streams of every rank's takes.

    Each rank passes the streams of its own takes (``partition`` order).  Lengths
    differ per take (EOS), so every rank sends ``[n_local, n_cb, T_max]`` padded
    blocks plus the lengths; one ``all_gather`` of sizes and one of the padded
    blocks (fixed shapes on every rank, as NCCL needs).  Returns the ``n_takes``
    streams in global order on rank 0 (on every rank with ``to_all``), else None.
    """
    mine = partition(n_takes, world, rank)
    if len(streams) != len(mine):
        raise ValueError(f"rank {rank} owns {len(mine)} takes but passed {len(streams)} streams")
    if world == 1:  # one process: nothing to exchange, no process group needed
        return list(streams)
    dist = _dist()
    device = device or (streams[0].device if streams else torch.device("cpu"))
    n_cb = streams[0].shape[0] if streams else 0
    # sizes: (n_cb, T_max) of every rank
    t_local = max((s.shape[1] for s in streams), default=0)
    meta = torch.tensor([n_cb, t_local], dtype=torch.int64, device=device)
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta)
    n_cb = max(int(m[0]) for m in metas)
    t_max = max(int(m[1]) for m in metas)
    n_max = len(partition(n_takes, world, 0))  # rank 0 owns the most takes
    block = torch.full((n_max, n_cb, max(t_max, 1)), -1, dtype=torch.int64, device=device)
    lens = torch.zeros(n_max, dtype=torch.int64, device=device)
    for i, s in enumerate(streams):
        block[i, :, :s.shape[1]] = s.to(device)
        lens[i] = s.shape[1]
    blocks = [torch.empty_like(block) for _ in range(world)]
    all_lens = [torch.empty_like(lens) for _ in range(world)]
    dist.all_gather(all_lens, lens)
    dist.all_gather(blocks, block)
    if rank != 0 and not to_all:
        return None
    out = []
    for r in range(world):
        for i, _ in enumerate(partition(n_takes, world, r)):
            out.append(blocks[r][i, :, :int(all_lens[r][i])].clone())
    return out


def generate_sharded(model, text, muq_idx, n_takes: int, *, world: int, rank: int, seed: int = 0, to_all=False,
                     **kw):
    """``HeartMuLaLite.generate_ids`` for this rank's takes (seeded by the first take
    index, so a take's stream does not depend on the number of GPUs it ran on when
    each rank holds one take), then :func:`gather_streams`."""
    mine = partition(n_takes, world, rank)
    streams = []
    if len(mine):
        res = model.generate_ids(text, muq_idx, n=len(mine), seed=seed + mine.start, **kw)
        streams = [res] if len(mine) == 1 else list(res)
    return gather_streams(streams, n_takes, world, rank, device=model.dev, to_all=to_all)
