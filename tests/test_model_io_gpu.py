"""Model I/O on the GPU: ``HeartMuLaLite.to(device)`` (the reference moves the weights to
the host while its codec uses the GPU, ``app/engine.py:267-288``) and checkpoints with
plain fp weights (``app/engine.py:235-260``: fp16/bf16 ``Linear`` weights, a bf16
``audio_head [heads, D, V]``, plain embedding tables), which the loader quantises as
the converter would."""
import pytest
import torch

from estudiocanciones_b200.checkpoint import TINY_SHAPE, synthetic_tensors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _frame(m, seed=0):
    N, B, L = 2, 4, 64
    m.alloc(N, B, L)
    g = torch.Generator(device=DEV).manual_seed(seed)
    for blk in m.backbone.blocks:
        blk.kc[:, :, :20].normal_(generator=g)
        blk.vc[:, :, :20].normal_(generator=g)
    gc = torch.Generator().manual_seed(seed)
    tok = torch.randint(0, 8192, (N, 8), generator=gc).repeat(2, 1).to(DEV)
    force = torch.randint(0, 8192, (N, 8), generator=gc).repeat(2, 1).to(DEV)
    pos = torch.full((B,), 20, dtype=torch.long, device=DEV)
    out = m.teacher_frame(force, with_backbone=True, tok=tok, pos=pos, cfg=1.5).clone()
    kv = m.backbone.blocks[-1].kc[:, :, 20].clone()
    return out, kv


@pytest.fixture(scope="module")
def built():
    from estudiocanciones_b200 import build
    build.build()


def test_to_host_and_back_gives_identical_frames(built):
    from estudiocanciones_b200._lib import HMError
    from estudiocanciones_b200.engine import HeartMuLaLite
    m = HeartMuLaLite(synthetic_tensors(TINY_SHAPE, seed=3, gamma_one=False), device=DEV,
                      bb_heads=TINY_SHAPE.bb_heads, dec_heads=TINY_SHAPE.dec_heads)
    ref, kv = _frame(m)
    free0 = torch.cuda.mem_get_info()[0]
    m.to("cpu")
    assert m.backbone.blocks[0].qkv.q8.device.type == "cpu" and m.audio_head[0].s8.device.type == "cpu"
    assert m.backbone.blocks[0].kc is None and m._rt is None
    assert torch.cuda.mem_get_info()[0] > free0  # the weights and caches left the GPU
    with pytest.raises(HMError):
        m.alloc(2, 4, 64)
    m.to("cuda")
    assert m.backbone.blocks[0].qkv.q8.is_cuda and m.text_emb.q8.is_cuda
    got, kv2 = _frame(m)
    assert torch.equal(got, ref) and torch.equal(kv2, kv)
    m.release()


def _plain(t):
    """The same weights in the plain layout: every q8/s8 Linear as bf16 ``[N, K]``, the
    audio heads as one bf16 ``[heads, D, V]``, the embedding tables as bf16."""
    out = {}
    heads = sorted(k for k in t if k.startswith("audio_head.") and k.endswith(".q8"))
    for k, v in t.items():
        if k.startswith("audio_head."):
            continue
        if k.endswith(".q8"):
            base = k[:-3]
            out[base] = (v.float() * t[base + ".s8"].float()[:, None]).to(torch.bfloat16)
        elif not k.endswith(".s8"):
            out[k] = v
    out["audio_head"] = torch.stack([
        (t[h].float() * t[h[:-3] + ".s8"].float()[:, None]).t() for h in heads]).to(torch.bfloat16)
    return out


def test_plain_weight_checkpoint_runs_as_its_int8_conversion(built):
    from estudiocanciones_b200.convert import quantize_plain
    from estudiocanciones_b200.engine import HeartMuLaLite
    plain = {k: v.to(DEV) for k, v in _plain(synthetic_tensors(TINY_SHAPE, seed=4, gamma_one=False)).items()}
    assert plain["audio_head"].dim() == 3 and "backbone.layers.0.attn.q_proj.weight" in plain
    kw = dict(device=DEV, bb_heads=TINY_SHAPE.bb_heads, dec_heads=TINY_SHAPE.dec_heads)
    a = HeartMuLaLite(plain, **kw)
    b = HeartMuLaLite(quantize_plain(plain), **kw)
    fa, ka = _frame(a, seed=1)
    fb, kb = _frame(b, seed=1)
    assert torch.equal(fa, fb) and torch.equal(ka, kb)
    assert len(a.audio_head) == TINY_SHAPE.n_cb - 1
    a.release()
    b.release()


def test_graph_capture_keeps_the_allocator_cache(built):
    """``_lib.capture_graph`` captures like ``torch.cuda.graph`` but does not empty torch's
    allocator cache first (which sent every later allocation back to cudaMalloc: up to
    ~1 s per song with an NCCL group): freed blocks stay reserved across a capture, and
    the captured work replays correctly."""
    from estudiocanciones_b200._lib import capture_graph
    x = torch.empty(256 << 20, dtype=torch.uint8, device=DEV)
    del x  # 256 MB now cached, not in use
    reserved = torch.cuda.memory_reserved()
    a = torch.arange(1024, dtype=torch.float32, device=DEV)
    b = torch.empty_like(a)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with capture_graph(g, s):
        b.copy_(a * 2)
    torch.cuda.current_stream().wait_stream(s)
    assert torch.cuda.memory_reserved() >= reserved
    a.fill_(3)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(b, torch.full_like(b, 6))
    # torch.cuda.graph itself returns the cached blocks to the device
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        b.copy_(a + 1)
    assert torch.cuda.memory_reserved() < reserved
