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

from .checkpoint import FRAME_MS


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
                   to_all: bool = False, t_cap: int | None = None, n_cb: int | None = None) -> list[torch.Tensor] | None:
    """Collect the ``[n_cb, T_i]`` int64 streams of every rank's takes.

    Each rank passes the streams of its own takes (``partition`` order).  Lengths differ
    per take (EOS); every rank sends one fixed-shape block ``[n_max, 1 + n_cb * t_cap]``
    (per take: its length, then its padded ``[n_cb, t_cap]`` ids), so the exchange is a
    single ``gather`` to rank 0 (``all_gather`` with ``to_all``).  ``t_cap`` (an upper
    bound of T, e.g. the frame budget) and ``n_cb`` make the block shape known to every
    rank up front; without them one small ``all_gather`` of the sizes comes first.
    Returns the ``n_takes`` streams in global order on rank 0 (on every rank with
    ``to_all``), else None.
    """
    mine = partition(n_takes, world, rank)
    if len(streams) != len(mine):
        raise ValueError(f"rank {rank} owns {len(mine)} takes but passed {len(streams)} streams")
    if world == 1:  # one process: nothing to exchange, no process group needed
        return list(streams)
    dist = _dist()
    device = device or (streams[0].device if streams else torch.device("cpu"))
    t_local = max((s.shape[1] for s in streams), default=0)
    if t_cap is not None and t_local > t_cap:
        raise ValueError(f"a stream of {t_local} frames is longer than t_cap={t_cap}")
    if t_cap is None or n_cb is None:
        meta = torch.tensor([streams[0].shape[0] if streams else 0, t_local], dtype=torch.int64, device=device)
        metas = [torch.empty_like(meta) for _ in range(world)]
        dist.all_gather(metas, meta)
        n_cb = max(int(m[0]) for m in metas) if n_cb is None else n_cb
        t_cap = max(int(m[1]) for m in metas) if t_cap is None else t_cap
    t_cap = max(t_cap, 1)
    n_max = len(partition(n_takes, world, 0))  # rank 0 owns the most takes
    block = torch.full((n_max, 1 + n_cb * t_cap), -1, dtype=torch.int64, device=device)
    for i, st in enumerate(streams):
        if st.shape[0] != n_cb:
            raise ValueError(f"stream {i} has {st.shape[0]} codebooks, expected {n_cb}")
        block[i, 0] = st.shape[1]
        block[i, 1:].view(n_cb, t_cap)[:, :st.shape[1]] = st.to(device)
    if to_all:
        blocks = [torch.empty_like(block) for _ in range(world)]
        dist.all_gather(blocks, block)
    else:
        blocks = [torch.empty_like(block) for _ in range(world)] if rank == 0 else None
        dist.gather(block, blocks, dst=0)
        if rank != 0:
            return None
    out = []
    for r in range(world):
        for i, _ in enumerate(partition(n_takes, world, r)):
            T = int(blocks[r][i, 0])
            out.append(blocks[r][i, 1:].view(n_cb, t_cap)[:, :T].clone())
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
    t_cap = kw.get("max_ms", 60_000) // FRAME_MS + 1  # generate_ids never returns more frames
    return gather_streams(streams, n_takes, world, rank, device=model.dev, to_all=to_all, t_cap=t_cap,
                          n_cb=model.n_cb)
