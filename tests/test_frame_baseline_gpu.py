"""Whole-frame parity at the BASELINE shape (28 x 3072 backbone, 4 x 1024 decoder,
8 codebooks of 8197) for the benchmark configurations.

For each configuration the static KV caches are filled with N(0, 1) values up to
the decode position (the benchmark's setup; a CPU prefill of this model would take
hours), then one teacher-forced frame -- backbone step at that position, c0 head, 7
local-decoder passes and 7 audio heads -- runs through the B200 engine and through
the CPU oracle (the reference fast path's arithmetic, ``mode="fast"``) with the same
forced ids.  The north-star rule per head and row: logits within 2e-2 max-abs, KL
<= 1e-3, identical argmax (except at exact ties: then within 4e-3 of the best), and
identical top-50 sets where the 50th and 51st logits differ by more than 4e-3; the
K/V written at the decode position match the oracle's.

configs: 0 = 1 row, CFG off, KV 512; 1 = 4 takes x CFG = 8 rows at KV 975 (the
middle of the 60 s song); 3 = 8 rows at KV 4024 (the end of the 4-minute song).
"""
import os

import pytest
import torch

from oracle import heartmula_oracle as O
from estudiocanciones_b200.checkpoint import BASELINE_SHAPE, synthetic_tensors

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE = 4e-3


@pytest.fixture(scope="module")
def models():
    from estudiocanciones_b200 import build
    from estudiocanciones_b200.engine import HeartMuLaLite
    build.build()
    torch.set_num_threads(os.cpu_count() or 1)
    t = synthetic_tensors(BASELINE_SHAPE, seed=0, device=DEV, gamma_one=True)
    m = HeartMuLaLite(t, device=DEV)
    tc = {k: v.cpu() for k, v in t.items()}
    del t
    o = O.OracleModel(tc, mode="fast")
    yield m, o
    m.release()


def check_heads(got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    d = (got - ref).abs().max().item()
    assert d <= 2e-2, f"max abs {d}"
    p = torch.log_softmax(ref, -1)
    q = torch.log_softmax(got, -1)
    kl = (p.exp() * (p - q)).sum(-1).max().item()
    assert kl <= 1e-3, f"KL {kl}"
    top = ref.topk(51, -1)
    clear1 = (top.values[..., 0] - top.values[..., 1]) > TIE
    assert torch.equal(got.argmax(-1)[clear1], ref.argmax(-1)[clear1])
    picked = ref.gather(-1, got.argmax(-1).unsqueeze(-1)).squeeze(-1)
    assert bool((picked >= top.values[..., 0] - TIE).all())
    clear50 = (top.values[..., 49] - top.values[..., 50]) > TIE
    gs = got.topk(50, -1).indices.sort(-1).values
    rs = top.indices[..., :50].sort(-1).values
    assert torch.equal(gs[clear50], rs[clear50])
    return d, kl


@pytest.mark.parametrize("cfg_id,takes,cfg_on,kv", [(0, 1, False, 512), (1, 4, True, 975), (3, 4, True, 4024)])
def test_baseline_shape_frame_matches_oracle(models, cfg_id, takes, cfg_on, kv):
    m, o = models
    N = takes
    B = 2 * N if cfg_on else N
    L = kv + 2 + 256
    m.alloc(N, B, L)
    gen = torch.Generator(device=DEV).manual_seed(100 + cfg_id)
    for blk in m.backbone.blocks:
        blk.kc[:, :, :kv].normal_(generator=gen)
        blk.vc[:, :, :kv].normal_(generator=gen)
    g = torch.Generator().manual_seed(200 + cfg_id)
    tok = torch.randint(0, 8192, (N, 8), generator=g)
    force = torch.randint(0, 8192, (N, 8), generator=g)
    if cfg_on:
        tok, force = tok.repeat(2, 1), force.repeat(2, 1)
    pos = torch.full((B,), kv, dtype=torch.long)
    got = m.teacher_frame(force.to(DEV), with_backbone=True, tok=tok.to(DEV), pos=pos.to(DEV),
                          cfg=1.5 if cfg_on else 1.0)
    # the oracle on the same caches (copied), ids and positions
    o.alloc(B, L)
    for ob, mb in zip(o.bb, m.backbone.blocks):
        ob.kc.copy_(mb.kc.cpu())
        ob.vc.copy_(mb.vc.cpu())
        ob.kc[:, :, kv:] = 0
        ob.vc[:, :, kv:] = 0
    rec = []
    o.step(tok, pos.reshape(B, 1), N, 1.5 if cfg_on else 1.0, 50, 1.0, force=force, record=rec,
           noise=[torch.ones(N, o.vocab)] * o.n_cb)
    ref = torch.stack(rec)
    assert got.shape == ref.shape
    check_heads(got, ref)
    # the K/V the qkv epilogue wrote at the decode position (first and last layer)
    for ob, mb in ((o.bb[0], m.backbone.blocks[0]), (o.bb[-1], m.backbone.blocks[-1])):
        torch.testing.assert_close(mb.kc[:, :, kv].float().cpu(), ob.kc[:, :, kv].float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(mb.vc[:, :, kv].float().cpu(), ob.vc[:, :, kv].float(), atol=1e-2, rtol=1e-2)
        assert int(mb.kc[:, :, kv + 1:].abs().sum()) == 0
