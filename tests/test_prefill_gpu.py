"""Prompt-prefill kernels on the GPU: the tcgen05 int8-weight GEMM and the causal
GQA prefill attention, each against a plain PyTorch fp32 computation of the same
op with the reference's rounding points, and the whole tensor-core prefill
against the position-by-position decode path."""
import math

import pytest
import torch

from oracle import heartmula_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _built():
    from estudiocanciones_b200 import build
    build.build()


def _gemm_case(seed, M, N, K, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) * 0.5).half()
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = (torch.rand(N, generator=g) * scale / 127 + 1e-5).half()
    return a, w, s


def _ref_acc(a, w):
    return a.double() @ w.double().t()


def _assert_fp16_close(out, ref_f64, bound):
    """out fp16 vs an exact value: within 1 fp16 ulp of the rounded result plus
    the fp32 accumulation-order bound."""
    out = out.double().cpu()
    ulp = torch.finfo(torch.float16).eps * ref_f64.abs().clamp_min(6.1e-5)
    err = (out - ref_f64).abs()
    lim = 1.01 * ulp + bound
    bad = err > lim
    assert not bad.any(), f"{int(bad.sum())} values off; worst {float((err - lim).max())}"


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (37, 512, 1024), (128, 256, 3072), (300, 5120, 512),
                                   (129, 400, 128), (64, 3072, 8192)])
def test_gemm_i8w_store(M, N, K):
    from estudiocanciones_b200 import kernels
    a, w, s = _gemm_case(M * 7 + N, M, N, K)
    out = kernels.gemm_i8w(a.to(DEV), w.to(DEV), s.to(DEV))
    acc = _ref_acc(a, w)
    ref = acc * s.double()[None, :]
    # fp32 accumulation of K products, each exact in fp32: |error| <= K * 2^-24 * sum|a*w|
    bound = K * 2.0 ** -24 * (a.double().abs() @ w.double().abs().t()) * s.double()[None, :]
    _assert_fp16_close(out, ref, bound)


def test_gemm_i8w_residual_in_place():
    from estudiocanciones_b200 import kernels
    M, N, K = 200, 768, 1024
    a, w, s = _gemm_case(5, M, N, K)
    x = (torch.randn(M, N, generator=torch.Generator().manual_seed(6))).half()
    xd = x.to(DEV)
    kernels.gemm_i8w(a.to(DEV), w.to(DEV), s.to(DEV), res=xd, out=xd)
    y = (_ref_acc(a, w) * s.double()[None, :]).half().double()   # rounded GEMM output
    ref = y + x.double()
    bound = K * 2.0 ** -24 * (a.double().abs() @ w.double().abs().t()) * s.double()[None, :] + \
        torch.finfo(torch.float16).eps * y.abs()
    _assert_fp16_close(xd, ref, bound)


@pytest.mark.parametrize("M,F,K", [(5, 128, 64), (200, 1024, 512), (130, 8192, 3072)])
def test_gemm_i8w_silu(M, F, K):
    from estudiocanciones_b200 import kernels
    a, w, s = _gemm_case(M + F, M, 2 * F, K, scale=0.5)
    out = kernels.gemm_i8w(a.to(DEV), w.to(DEV), s.to(DEV), silu=True).cpu()
    acc = (a.float() @ w.float().t())
    y = (acc * s.float()[None, :]).half()
    ref = O.silu_mul(y)
    # the two operands are rounded GEMM outputs: compare within 2 fp16 ulp after the
    # products, plus a small absolute term for accumulation-order flips of a rounding
    d = (out.float() - ref.float()).abs()
    lim = 2 * torch.finfo(torch.float16).eps * ref.float().abs() + 2e-3 * ref.float().abs().max()
    assert (d <= lim).all(), float((d - lim).max())


def _sdpa_ref(q, kc, vc, B, P, Hq, Hk):
    hd = kc.shape[-1]
    G = Hq // Hk
    qh = q.float().reshape(B, P, Hq, hd).transpose(1, 2)                      # B Hq P hd
    k = kc[:, :, :P].float().repeat_interleave(G, 1)
    v = vc[:, :, :P].float().repeat_interleave(G, 1)
    sc = qh @ k.transpose(-1, -2) / math.sqrt(hd)
    mask = torch.ones(P, P, dtype=torch.bool).tril()
    sc = sc.masked_fill(~mask, float("-inf"))
    return (sc.softmax(-1) @ v).transpose(1, 2).reshape(B * P, Hq * hd)


@pytest.mark.parametrize("B,P,Hq,Hk,L", [(1, 1, 4, 4, 64), (2, 63, 6, 2, 128), (2, 64, 24, 8, 100),
                                         (1, 200, 8, 2, 300), (3, 129, 3, 3, 129), (1, 300, 10, 2, 300),
                                         (2, 1024, 24, 8, 1100), (1, 777, 8, 8, 800)])
def test_prefill_attn(B, P, Hq, Hk, L):
    from estudiocanciones_b200 import kernels
    gen = torch.Generator().manual_seed(P * 31 + Hq)
    hd = 128
    q = torch.randn(B * P, Hq * hd, generator=gen).half()
    kc = torch.randn(B, Hk, L, hd, generator=gen).half()
    vc = torch.randn(B, Hk, L, hd, generator=gen).half()
    # cache slots past the prompt hold garbage that must not leak into the result
    kc[:, :, P:] = float("nan")
    vc[:, :, P:] = float("inf")
    o = kernels.prefill_attn(q.to(DEV), kc.to(DEV), vc.to(DEV), P).cpu()
    ref = _sdpa_ref(q, kc, vc, B, P, Hq, Hk)
    torch.testing.assert_close(o.float(), ref, atol=2e-3, rtol=5e-3)
    assert kernels.read_errors(DEV) == 0


def test_prefill_rejects_unsupported_shapes():
    from estudiocanciones_b200 import _lib
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.empty(64, 100, dtype=torch.float16, device=DEV)
    w = torch.empty(64, 100, dtype=torch.int8, device=DEV)
    s = torch.empty(64, dtype=torch.float16, device=DEV)
    # K = 100 is not a multiple of 64
    assert L.hm_gemm_i8w(x.data_ptr(), 100, w.data_ptr(), s.data_ptr(), None, 0, x.data_ptr(), 100, 64, 64, 100, 0,
                         None, st) == -1
    q = torch.empty(8, 5 * 128, dtype=torch.float16, device=DEV)
    kv = torch.empty(1, 1, 8, 128, dtype=torch.float16, device=DEV)
    # head dim 64 is not supported; neither is a query head count that is not a multiple of Hk
    assert L.hm_prefill_attn(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), q.data_ptr(), 1, 8, 10, 1, 64, 8, 0.1,
                             None, st) == -1
    assert L.hm_prefill_attn(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), q.data_ptr(), 1, 8, 5, 2, 128, 8, 0.1,
                             None, st) == -1
    # a prompt longer than the cache
    assert L.hm_prefill_attn(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), q.data_ptr(), 1, 9, 5, 1, 128, 8, 0.1,
                             None, st) == -1


def test_tensor_core_prefill_matches_decode_path_prefill():
    """Both GPU prefill paths over the same prompt: caches and the last hidden state
    agree (different rounding orders, fp16 tolerance)."""
    from estudiocanciones_b200.checkpoint import TINY_SHAPE, synthetic_tensors
    from estudiocanciones_b200.engine import HeartMuLaLite
    from estudiocanciones_b200.prefill import prefill_backbone, prefill_backbone_steps
    t = synthetic_tensors(TINY_SHAPE, seed=5, gamma_one=False)
    m = HeartMuLaLite(t, device=DEV, bb_heads=TINY_SHAPE.bb_heads, dec_heads=TINY_SHAPE.dec_heads)
    N, B, P = 2, 4, 70
    L = P + 64
    m.alloc(N, B, L)
    gen = torch.Generator().manual_seed(9)
    h = (torch.randn(B, P, TINY_SHAPE.bb_dim, generator=gen) * 0.05).half().to(DEV)
    prefill_backbone(m, h)
    kc = [b.kc.clone() for b in m.backbone.blocks]
    x = m._rt.x_bb.clone()
    for b in m.backbone.blocks:
        b.kc.zero_()
        b.vc.zero_()
    prefill_backbone_steps(m, h)
    for a, b in zip(kc, (b.kc for b in m.backbone.blocks)):
        torch.testing.assert_close(a.float(), b.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(x.float(), m._rt.x_bb.float(), atol=5e-2, rtol=2e-2)


def test_dequant_i8_is_exact():
    from estudiocanciones_b200 import kernels
    g = torch.Generator().manual_seed(17)
    w = torch.randint(-128, 128, (384, 1040), generator=g, dtype=torch.int8)
    wh = kernels.dequant_i8(w.to(DEV)).cpu()
    assert wh.dtype == torch.float16 and torch.equal(wh.float(), w.float())


@pytest.mark.parametrize("M,N,K,mode", [(37, 512, 1024, "store"), (128, 256, 3072, "store"), (300, 5120, 512, "res"),
                                        (200, 2048, 512, "silu"), (130, 16384, 3072, "silu"),
                                        (64, 3072, 8192, "res")])
def test_gemm_f16w_equals_gemm_i8w(M, N, K, mode):
    """Weights converted once (exact) then read as fp16 tiles: the same MMA sequence over
    the same values, so the results equal the int8-weight GEMM's bit for bit."""
    from estudiocanciones_b200 import kernels
    a, w, s = _gemm_case(M * 3 + N + K, M, N, K, scale=0.5 if mode == "silu" else 0.02)
    a, w, s = a.to(DEV), w.to(DEV), s.to(DEV)
    wh = kernels.dequant_i8(w)
    if mode == "silu":
        x = kernels.gemm_i8w(a, w, s, silu=True)
        y = kernels.gemm_f16w(a, wh, s, silu=True)
    elif mode == "res":
        r = torch.randn(M, N, generator=torch.Generator(device=DEV).manual_seed(2), device=DEV).half()
        x, y = r.clone(), r.clone()
        kernels.gemm_i8w(a, w, s, res=x, out=x)
        kernels.gemm_f16w(a, wh, s, res=y, out=y)
    else:
        x = kernels.gemm_i8w(a, w, s)
        y = kernels.gemm_f16w(a, wh, s)
    torch.cuda.synchronize()
    assert kernels.read_errors(DEV) == 0
    assert torch.equal(x, y)
