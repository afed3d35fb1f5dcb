"""Take sharding across ranks (host logic, CPU): the partition of takes over GPUs and
the gather of the finished variable-length token streams, run as two gloo ranks.
The same code path runs over NCCL on a multi-GPU box (bench.py --gpus N)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from estudiocanciones_b200.shard import gather_streams, partition


@pytest.mark.parametrize("n,world", [(0, 1), (1, 1), (4, 1), (1, 2), (4, 2), (5, 2), (7, 3), (64, 8), (3, 8)])
def test_partition_covers_every_take_once_in_order(n, world):
    parts = [partition(n, world, r) for r in range(world)]
    flat = [t for p in parts for t in p]
    assert flat == list(range(n))                      # contiguous, in order, each take once
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1                # balanced
    assert sizes == sorted(sizes, reverse=True)        # the larger blocks go to the first ranks


def test_partition_rejects_bad_requests():
    for args in [(-1, 2, 0), (4, 0, 0), (4, 2, 2), (4, 2, -1)]:
        with pytest.raises(ValueError):
            partition(*args)


def _stream(take: int, n_cb: int = 8) -> torch.Tensor:
    """A deterministic [n_cb, T] stream whose length depends on the take (EOS at different frames)."""
    T = 3 + 2 * take
    return (torch.arange(n_cb * T, dtype=torch.int64).reshape(n_cb, T) * 7 + take * 1000) % 8197


def _worker(rank, world, port, n_takes, to_all, errq, known_shape=False):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mine = partition(n_takes, world, rank)
        kw = {"t_cap": 3 + 2 * n_takes, "n_cb": 8} if known_shape else {}
        calls = []
        for name in ("all_gather", "gather"):
            fn = getattr(dist, name)
            setattr(dist, name, lambda *a, _fn=fn, _n=name, **k: (calls.append(_n), _fn(*a, **k))[1])
        out = gather_streams([_stream(t) for t in mine], n_takes, world, rank, to_all=to_all, **kw)
        # one collective when the block shape is known up front, sizes + blocks otherwise
        assert len(calls) == (1 if known_shape else 2), calls
        if rank == 0 or to_all:
            assert out is not None and len(out) == n_takes
            for t, s in enumerate(out):
                assert torch.equal(s, _stream(t)), f"take {t}"
        else:
            assert out is None
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n_takes,to_all,known_shape", [(4, False, False), (5, True, False), (1, True, False),
                                                       (4, False, True), (1, False, True), (3, True, True)])
def test_gather_streams_two_gloo_ranks(n_takes, to_all, known_shape):
    """known_shape: the frame cap and codebook count are passed, so the exchange is one
    fixed-shape gather (all_gather with to_all); otherwise the sizes go first."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_takes, to_all, errq, known_shape)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_gather_streams_single_process_needs_no_process_group():
    import torch.distributed as dist
    assert not dist.is_initialized()
    streams = [_stream(t) for t in range(3)]
    out = gather_streams(streams, 3, 1, 0)
    assert len(out) == 3 and all(torch.equal(a, b) for a, b in zip(out, streams))
    with pytest.raises(ValueError):
        gather_streams(streams[:2], 3, 1, 0)
