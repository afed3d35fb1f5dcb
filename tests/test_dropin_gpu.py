"""The reference's per-layer decode loop, written with its own call-site shapes
(``Stack.decode``, ``app/engine.py:180-211``: an RMSNorm, the fused qkv linear, the
``_rope_cache[grid]`` launch, split partial buffers for ``_attn[grid]`` and
``_attn_combine[grid]``, the residual linears and ``_silu_mul[grid]``), driven through
this package's drop-in names, must give what the package's own fused ``Stack.decode``
gives, and the ``torch.library`` operators must give what ``kernels`` gives.

The two loops round at the same points but split the work differently (separate
RMSNorm launches against the fused RMSNorm prologue, and their own attention split
counts), so they agree within fp16 rounding, not bit for bit."""
import math

import pytest
import torch

from estudiocanciones_b200.checkpoint import ModelShape, synthetic_tensors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference_style_decode(K, stack, x, pos, S):
    """Written anew after the reference's loop: same launches, same argument lists."""
    R = x.shape[0]
    ns = 16
    for b in stack.blocks:
        Hq, Hk, HD, L = b.h, b.kvh, b.hd, b.kc.shape[2]
        qkv = b.qkv(K.rms(x, b.n1))
        q = torch.empty(R, Hq * HD, device=x.device, dtype=x.dtype)
        K._rope_cache[(R, Hq + Hk)](qkv, stack.rope, pos, q, b.kc, b.vc, S, Hq, Hk, L, HD=HD, HALF=HD // 2)
        o = torch.empty_like(q)
        pm = torch.empty(R * Hq * ns, device=x.device)
        pl = torch.empty_like(pm)
        pa = torch.empty(R * Hq * ns, HD, device=x.device)
        K._attn[(R, Hk, ns)](q, b.kc, b.vc, pos, o, pm, pl, pa, S, Hq, Hk, L, 1.0 / math.sqrt(HD),
                             HD=HD, HDP=HD, G=Hq // Hk, BLK=64, NSPLIT=ns, num_warps=4)
        K._attn_combine[(R * Hq,)](pm, pl, pa, o, HD=HD, HDP=HD, NSPLIT=ns)
        x = b.o(o, res=x)
        a = b.w13(K.rms(x, b.n2))
        Fd = a.shape[1] // 2
        mm = torch.empty(R, Fd, device=x.device, dtype=x.dtype)
        K._silu_mul[(R, (Fd + 1023) // 1024)](a, mm, Fd, BLOCK=1024)
        x = b.w2(mm, res=x)
    return K.rms(x, stack.norm)


@pytest.fixture(scope="module")
def model():
    from estudiocanciones_b200 import build
    from estudiocanciones_b200.engine import HeartMuLaLite
    build.build()
    shape = ModelShape(bb_layers=2, bb_dim=1024, bb_heads=8, bb_kv_heads=2, bb_ffn=2048, dec_layers=1,
                       dec_dim=256, dec_heads=2, dec_kv_heads=1, dec_ffn=512, text_vocab=512)
    t = synthetic_tensors(shape, seed=31, gamma_one=False)
    return HeartMuLaLite(t, device=DEV, bb_heads=8, dec_heads=2)


@pytest.mark.parametrize("R,S,L,p", [(8, 1, 640, 517), (4, 2, 96, 40)])
def test_reference_loop_through_standins_matches_stack_decode(model, R, S, L, p):
    from estudiocanciones_b200 import kernels as K
    st = model.backbone
    B = R // S
    st.alloc(B, L, torch.device(DEV))
    gen = torch.Generator(device=DEV).manual_seed(R + L)
    for b in st.blocks:
        b.kc[:, :, :p].normal_(generator=gen)
        b.vc[:, :, :p].normal_(generator=gen)
    kv0 = [(b.kc.clone(), b.vc.clone()) for b in st.blocks]
    x = (torch.randn(R, st.dim, generator=gen, device=DEV) * 0.5).half()
    pos = torch.full((R,), p, dtype=torch.long, device=DEV) + (torch.arange(R, device=DEV) % S)
    ours = st.decode(x, pos, S)
    kv_ours = [(b.kc.clone(), b.vc.clone()) for b in st.blocks]
    for b, (kc, vc) in zip(st.blocks, kv0):
        b.kc.copy_(kc)
        b.vc.copy_(vc)
    theirs = reference_style_decode(K, st, x, pos, S)
    torch.cuda.synchronize()
    assert K.read_errors(DEV) == 0
    torch.testing.assert_close(theirs.float(), ours.float(), atol=2e-2, rtol=2e-2)
    for (kc, vc), b in zip(kv_ours, st.blocks):
        torch.testing.assert_close(b.kc.float(), kc.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(b.vc.float(), vc.float(), atol=1e-2, rtol=1e-2)
    st.free()


def test_torch_library_operators_match_kernels():
    from estudiocanciones_b200 import kernels as K
    from estudiocanciones_b200 import ops  # noqa: F401
    O = torch.ops.heartmula_b200
    gen = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(8, 1024, generator=gen, device=DEV).half()
    w = torch.randint(-127, 128, (512, 1024), generator=gen, device=DEV, dtype=torch.int8)
    s = (torch.rand(512, generator=gen, device=DEV) * 1e-3).half()
    r = torch.randn(8, 512, generator=gen, device=DEV).half()
    assert torch.equal(O.int8_mm(x, w, s, r), K.int8_mm(x, w, s, r))
    g = (1 + 0.1 * torch.randn(1024, generator=gen, device=DEV)).half()
    assert torch.equal(O.rms(x, g), K.rms(x, g))
    a = torch.randn(8, 2048, generator=gen, device=DEV).half()
    assert torch.equal(O.silu_mul(a), K.silu_mul(a))
    # in-place attention through the operator and through kernels
    q = torch.randn(4, 8 * 128, generator=gen, device=DEV).half()
    kc = torch.randn(4, 2, 200, 128, generator=gen, device=DEV).half()
    vc = torch.randn_like(kc)
    pos = torch.tensor([10, 50, 120, 199], device=DEV)
    o1, o2 = torch.empty_like(q), torch.empty_like(q)
    O.attn(q, kc, vc, pos, o1, 1, 8, 2, 200, 1.0 / math.sqrt(128), 4)
    K.attn(q, kc, vc, pos, o2, 1, 8, 2, 200, 1.0 / math.sqrt(128), nsplit=4)
    assert torch.equal(o1, o2)


def test_stack_decode_reuses_its_plan_with_new_inputs(model):
    """Stack.decode keeps its launch plan per shape: a second call with other rows and
    positions (copied into the plan's buffers) gives what the reference loop gives."""
    from estudiocanciones_b200 import kernels as K
    st = model.backbone
    R, S, L, p = 8, 1, 640, 300
    st.alloc(R, L, torch.device(DEV))
    gen = torch.Generator(device=DEV).manual_seed(77)
    for b in st.blocks:
        b.kc[:, :, :p + 8].normal_(generator=gen)
        b.vc[:, :, :p + 8].normal_(generator=gen)
    x1 = (torch.randn(R, st.dim, generator=gen, device=DEV) * 0.5).half()
    st.decode(x1, torch.full((R,), p, dtype=torch.long, device=DEV), S)
    assert len(st._decode_plans) == 1
    kv0 = [(b.kc.clone(), b.vc.clone()) for b in st.blocks]
    x2 = (torch.randn(R, st.dim, generator=gen, device=DEV) * 0.5).half()
    pos2 = torch.arange(R, device=DEV) + p - 3
    ours = st.decode(x2, pos2, S)
    assert len(st._decode_plans) == 1
    for b, (kc, vc) in zip(st.blocks, kv0):
        b.kc.copy_(kc)
        b.vc.copy_(vc)
    theirs = reference_style_decode(K, st, x2, pos2, S)
    torch.cuda.synchronize()
    assert K.read_errors(DEV) == 0
    torch.testing.assert_close(theirs.float(), ours.float(), atol=2e-2, rtol=2e-2)
    st.free()
    assert not st._decode_plans
