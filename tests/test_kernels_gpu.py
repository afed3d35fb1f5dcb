"""Kernel-level parity of the sm_100a library against the CPU oracle and the
reference's golden vectors.  Every call goes through the C ABI."""
import math

import numpy as np
import pytest
import torch

from oracle import heartmula_oracle as O
from estudiocanciones_b200._lib import HM_EPI_ROPE_KV, HM_EPI_SILU

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _built():
    from estudiocanciones_b200 import build, kernels
    build.build()
    kernels.read_errors(DEV)
    yield
    assert kernels.read_errors(DEV) == 0, "a kernel reported an error bit"


def g(a):
    return torch.from_numpy(np.array(a))


def close16(out, ref, ulps=2, frac_exact=0.95, slack=None):
    """fp16 results equal up to `ulps` fp16 ulps (of the reference value), most of them exactly.
    `slack`: extra absolute tolerance per element (fp32 accumulation-order bound)."""
    o, r = out.float().cpu(), ref.float().cpu()
    ulp = torch.clamp(2.0 ** (torch.floor(torch.log2(r.abs().clamp_min(2.0 ** -14))) - 10), min=2.0 ** -24)
    tol = ulps * ulp + (0 if slack is None else slack)
    bad = (o - r).abs() > tol
    assert int(bad.sum()) == 0, f"{int(bad.sum())} values off by > {ulps} ulp; max abs {float((o - r).abs().max())}"
    assert (o == r).float().mean().item() >= frac_exact


def acc_slack(x, w, s):
    """Bound on the difference two fp32 accumulation orders can make in x.w*s:
    about K*2^-24 relative to sum |x_k w_k|."""
    return (x.float().abs() @ w.float().abs().t()) * s.float() * (x.shape[-1] * 2.0 ** -24)


def rms_slack(xn, w, s, ref):
    """Accumulation-order slack plus the effect of the normalised input differing by
    one fp16 ulp in a few places (the 1/rms sum is accumulated in another order)."""
    return acc_slack(xn, w, s) + 1e-3 * ref.float().abs() + 1e-4


def rand_lin(N, K, gen):
    w = torch.randint(-127, 128, (N, K), generator=gen, dtype=torch.int8)
    s = (torch.randn(N, generator=gen).abs() * 0.02 / 127).half()
    return w, s


# ----------------------------------------------------------------------------- GEMV
@pytest.mark.parametrize("i", range(5))
def test_gemv_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("kernels")
    x, w, s, y = g(z[f"gemv{i}_x"]), g(z[f"gemv{i}_w"]), g(z[f"gemv{i}_s"]), g(z[f"gemv{i}_y"])
    r = g(z[f"gemv{i}_r"]).to(DEV) if f"gemv{i}_r" in z else None
    out = kernels.int8_mm(x.to(DEV), w.to(DEV), s.to(DEV), r)
    close16(out, y, ulps=2, frac_exact=0.9)


@pytest.mark.parametrize("M,N,K,kspan,res", [
    (1, 64, 128, 0, False), (3, 200, 512, 0, True), (8, 5120, 3072, 0, False), (8, 3072, 8192, 1024, True),
    (9, 1536, 1024, 512, False), (16, 8197, 3072, 0, False), (20, 1024, 3072, 512, True), (32, 3072, 1024, 0, True),
    (8, 8197, 1024, 0, False), (1, 16384, 3072, 1024, False), (32, 1024, 8192, 0, True), (5, 2048, 8192, 0, False),
    (8, 3072, 8192, 0, True), (8, 1024, 8192, 0, True), (8, 1024, 3072, 0, False), (7, 5120, 3072, 0, True)])
def test_gemv_matches_oracle(M, N, K, kspan, res):
    from estudiocanciones_b200 import kernels
    gen = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=gen).half()
    w, s = rand_lin(N, K, gen)
    r = torch.randn(M, N, generator=gen).half() if res else None
    out = kernels.int8_mm(x.to(DEV), w.to(DEV), s.to(DEV), r.to(DEV) if res else None, kspan=kspan)
    # the oracle's M > 16 branch rounds w*s to fp16 first (the reference's cuBLAS path);
    # the kernel keeps the exact int8 x fp16 product for every M, so compare with that
    acc = x.float() @ w.float().t()
    ref = (acc * s.float()).half()
    if res:
        ref = (ref.float() + r.float()).half()
    slack = acc_slack(x, w, s)
    close16(out, ref, ulps=2, frac_exact=0.9, slack=slack)
    if M <= 16:
        close16(out, O.gemv_i8(x, w, s, r), ulps=2, frac_exact=0.9, slack=slack)


def test_gemv_is_deterministic():
    from estudiocanciones_b200 import kernels
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(8, 3072, generator=gen).half().to(DEV)
    w, s = rand_lin(3072, 3072, gen)
    w, s = w.to(DEV), s.to(DEV)
    a = kernels.int8_mm(x, w, s, kspan=512)
    b = kernels.int8_mm(x, w, s, kspan=512)
    assert torch.equal(a, b)


# ----------------------------------------------------------------------------- fused GEMV prologues/epilogues
def _plan():
    from estudiocanciones_b200.engine import FramePlan, _Ctx
    return FramePlan(_Ctx(DEV, 64 << 20, 1 << 20), pdl=False)


def _ss(x):
    R, D = x.shape
    return (x.float() ** 2).reshape(R, D // 16, 16).sum(-1).t().contiguous()


def test_gemv_rms_prologue_and_residual_ss():
    from estudiocanciones_b200.engine import Linear
    gen = torch.Generator().manual_seed(11)
    M, D, N = 8, 3072, 3072
    x = (torch.randn(M, D, generator=gen) * 2).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half()
    w, s = rand_lin(N, D, gen)
    res = torch.randn(M, N, generator=gen).half()
    lin = Linear(w.to(DEV), s.to(DEV))
    xd, yd = x.to(DEV), res.to(DEV).clone()
    ss_in = _ss(xd)
    ss_out = torch.zeros(N // 16, M, device=DEV)
    p = _plan()
    p._gemv(lin, M, p.src_rms(xd, ss_in, gamma.to(DEV)), y=yd, res=yd, ss_out=ss_out)
    p.run()
    xn = O.rmsnorm(x, gamma)
    ref = O.gemv_i8(xn, w, s, res)
    close16(yd, ref, ulps=2, frac_exact=0.9, slack=rms_slack(xn, w, s, ref))
    torch.testing.assert_close(ss_out.cpu(), _ss(yd).cpu(), rtol=1e-5, atol=1e-4)


def test_gemv_emb_interleave_prologue():
    """Decoder pass 0 input: rows (2b, 2b+1) = (rms(x_b), emb(c0_b))."""
    from estudiocanciones_b200.engine import Emb, Linear
    gen = torch.Generator().manual_seed(12)
    B, D, N, V = 4, 3072, 1024, 8197
    x = torch.randn(B, D, generator=gen).half()
    gamma = torch.ones(D).half()
    tq = torch.randint(-127, 128, (8 * V, D), generator=gen, dtype=torch.int8)
    ts = (torch.rand(8 * V, generator=gen) * 0.01).half()
    tok = torch.randint(0, V, (B, 8), generator=gen)
    w, s = rand_lin(N, D, gen)
    lin, emb = Linear(w.to(DEV), s.to(DEV)), Emb(tq.to(DEV), ts.to(DEV))
    xd, tokd = x.to(DEV), tok.to(DEV)
    y = torch.empty(2 * B, N, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, 2 * B, p.src_rms(xd, _ss(xd), gamma.to(DEV)), p.src_emb(emb, tokd, 0, 0), y=y)
    p._gemv(lin, B, p.src_emb(emb, tokd, 3, 3 * V), y=y[:B])  # codebook 3 rows -> y[:B]
    p.run()
    e0 = O.emb_i8(tok[:, 0], tq, ts)
    xin = torch.stack([O.rmsnorm(x, gamma), e0], 1).reshape(2 * B, D)
    ref = O.gemv_i8(xin, w, s)
    close16(y[B:], ref[B:], ulps=2, frac_exact=0.9, slack=rms_slack(xin[B:], w, s, ref[B:]))
    close16(y[:B], O.gemv_i8(O.emb_i8(tok[:, 3] + 3 * V, tq, ts), w, s), ulps=2, frac_exact=0.9)


@pytest.mark.parametrize("S,Hq,Hk", [(1, 24, 8), (2, 8, 2)])
def test_gemv_rope_kv_epilogue(S, Hq, Hk):
    from estudiocanciones_b200.engine import Block, Linear
    gen = torch.Generator().manual_seed(13)
    hd, D, L = 128, 1024, 64
    R = 4
    B = R // S
    x = torch.randn(R, D, generator=gen).half()
    gamma = torch.ones(D).half()
    N = (Hq + 2 * Hk) * hd
    w, s = rand_lin(N, D, gen)
    pos = torch.tensor([5, 63, 0, 17][:R]) if S == 1 else torch.tensor([0, 1, 0, 1])
    rope = O.rope_table(hd, L)
    kc0 = torch.randn(B, Hk, L, hd, generator=gen).half()
    vc0 = torch.randn(B, Hk, L, hd, generator=gen).half()
    blk = Block.__new__(Block)
    blk.h, blk.kvh, blk.hd = Hq, Hk, hd
    blk.kc, blk.vc = kc0.clone().to(DEV), vc0.clone().to(DEV)
    lin = Linear(w.to(DEV), s.to(DEV))
    xd = x.to(DEV)
    q = torch.empty(R, Hq * hd, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, R, p.src_rms(xd, _ss(xd), gamma.to(DEV)), epi=HM_EPI_ROPE_KV, rope=rope.to(DEV), pos=pos.to(DEV), S=S,
            blk=blk, q_out=q)
    p.run()
    xn = O.rmsnorm(x, gamma)
    qkv = O.gemv_i8(xn, w, s)
    kc, vc = kc0.clone(), vc0.clone()
    qr = O.rope_kv_write(qkv, rope, pos, kc, vc, S, Hq, Hk)
    sl = rms_slack(xn, w, s, qkv).float().abs().reshape(R, -1)
    qsl = sl[:, : Hq * 128]
    qsl = torch.maximum(qsl, qsl.reshape(R, Hq, 64, 2).flip(-1).reshape(R, -1))  # rotation mixes pairs
    close16(q, qr, ulps=2, frac_exact=0.9, slack=qsl)
    close16(blk.kc, kc, ulps=2, frac_exact=0.95, slack=1e-3 * kc.float().abs() + 2e-4)
    close16(blk.vc, vc, ulps=2, frac_exact=0.95, slack=1e-3 * vc.float().abs() + 2e-4)
    # slots other than the written positions are untouched (bit-exact)
    mask = torch.ones(B, L, dtype=torch.bool)
    for r in range(R):
        mask[r // S, int(pos[r])] = False
    idx = mask.nonzero(as_tuple=True)      # (batch, position) pairs nobody wrote
    assert torch.equal(blk.kc.cpu().permute(0, 2, 1, 3)[idx], kc0.permute(0, 2, 1, 3)[idx])
    assert torch.equal(blk.vc.cpu().permute(0, 2, 1, 3)[idx], vc0.permute(0, 2, 1, 3)[idx])


def test_gemv_silu_epilogue():
    from estudiocanciones_b200.engine import Linear
    gen = torch.Generator().manual_seed(14)
    M, D, F = 8, 1024, 8192
    x = torch.randn(M, D, generator=gen).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half()
    w, s = rand_lin(2 * F, D, gen)
    lin = Linear(w.to(DEV), s.to(DEV))
    xd = x.to(DEV)
    y = torch.empty(M, F, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, M, p.src_rms(xd, _ss(xd), gamma.to(DEV)), epi=HM_EPI_SILU, y=y)
    p.run()
    xn = O.rmsnorm(x, gamma)
    a = O.gemv_i8(xn, w, s)
    ref = O.silu_mul(a)
    sl = rms_slack(xn, w, s, a)
    close16(y, ref, ulps=3, frac_exact=0.9, slack=2 * (sl[:, :F] * a[:, F:].float().abs() + sl[:, F:]))


# ----------------------------------------------------------------------------- small kernels
@pytest.mark.parametrize("i", range(2))
def test_rms_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("kernels")
    out = kernels.rms(g(z[f"rms{i}_x"]).to(DEV), g(z[f"rms{i}_w"]).to(DEV))
    close16(out, g(z[f"rms{i}_y"]), ulps=1, frac_exact=0.99)


@pytest.mark.parametrize("i", range(2))
def test_rope_cache_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("kernels")
    R, S, Hq, Hk, L = (int(v) for v in z[f"rope{i}_cfg"])
    kc, vc = g(z[f"rope{i}_kc0"]).to(DEV), g(z[f"rope{i}_vc0"]).to(DEV)
    q = torch.empty(R, Hq * 128, dtype=torch.float16, device=DEV)
    kernels.rope_cache(g(z[f"rope{i}_qkv"]).to(DEV), g(z[f"rope{i}_table"]).to(DEV), g(z[f"rope{i}_pos"]).to(DEV), q,
                       kc, vc, S, Hq, Hk, L)
    close16(q, g(z[f"rope{i}_q"]), ulps=1, frac_exact=0.98)
    close16(kc, g(z[f"rope{i}_kc"]), ulps=1, frac_exact=0.98)
    assert torch.equal(vc.cpu(), g(z[f"rope{i}_vc"]))


@pytest.mark.parametrize("i", range(2))
def test_silu_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("kernels")
    out = kernels.silu_mul(g(z[f"silu{i}_a"]).to(DEV))
    # CUDA's expf and Triton's tl.exp differ in the last fp32 bits, which can move
    # the rounded silu by one fp16 ulp and the product by one more
    close16(out, g(z[f"silu{i}_y"]), ulps=2, frac_exact=0.99)


def test_emb_gather_and_sum():
    from estudiocanciones_b200 import kernels
    from estudiocanciones_b200.engine import Emb, FramePlan
    gen = torch.Generator().manual_seed(15)
    V, D, B = 8197, 3072, 8
    tq = torch.randint(-127, 128, (8 * V, D), generator=gen, dtype=torch.int8)
    ts = (torch.rand(8 * V, generator=gen) * 0.01).half()
    tok = torch.randint(0, V, (B, 8), generator=gen)
    out = kernels.emb_i8(tok[:, 2].to(DEV) + 2 * V, tq.to(DEV), ts.to(DEV))
    assert torch.equal(out.cpu(), O.emb_i8(tok[:, 2] + 2 * V, tq, ts))
    x = torch.empty(B, D, dtype=torch.float16, device=DEV)
    ss = torch.empty(D // 16, B, device=DEV)
    p = _plan()
    p.emb_sum(Emb(tq.to(DEV), ts.to(DEV)), tok.to(DEV), B, 8, V, x, ss)
    p.run()
    assert torch.equal(x.cpu(), O.emb_sum(tok, tq, ts, V))
    torch.testing.assert_close(ss.cpu(), _ss(x).cpu(), rtol=1e-5, atol=1e-4)


def test_bad_token_sets_error_bit_without_fault():
    from estudiocanciones_b200 import kernels
    tq = torch.zeros(10, 64, dtype=torch.int8, device=DEV)
    ts = torch.ones(10, dtype=torch.float16, device=DEV)
    out = kernels.emb_i8(torch.tensor([3, 12], device=DEV), tq, ts)
    assert kernels.read_errors(DEV) == 2
    assert torch.all(out[1] == 0)


# ----------------------------------------------------------------------------- attention
@pytest.mark.parametrize("i", range(3))
def test_attn_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("kernels")
    R, S, Hq, Hk, L, ns = (int(v) for v in z[f"attn{i}_cfg"])
    o = torch.empty(R, Hq * 128, dtype=torch.float16, device=DEV)
    kernels.attn(g(z[f"attn{i}_q"]).to(DEV), g(z[f"attn{i}_kc"]).to(DEV), g(z[f"attn{i}_vc"]).to(DEV),
                 g(z[f"attn{i}_pos"]).to(DEV), o, S, Hq, Hk, L, nsplit=ns)
    torch.testing.assert_close(o.cpu().float(), g(z[f"attn{i}_o"]).float(), atol=2e-3, rtol=5e-3)


@pytest.mark.parametrize("R,S,Hq,Hk,hd,L,pos,ns", [
    (8, 1, 24, 8, 128, 1350, [0, 1, 31, 32, 599, 975, 1348, 1349], 5),
    (1, 1, 24, 8, 128, 512, [511], 37),
    (16, 2, 8, 2, 128, 8, [0, 1] * 8, 1),
    (4, 1, 8, 2, 128, 8, [7, 6, 5, 2], 1),
    (4, 1, 8, 2, 128, 64, [15, 16, 17, 63], 1),
    (4, 1, 8, 4, 384, 40, [3, 39, 0, 20], 3),
    (2, 1, 24, 8, 128, 4282, [4281, 4023], 16),
    # 2..8 splits merge inside a thread-block cluster (DSMEM); rows whose later splits are empty
    (8, 1, 24, 8, 128, 1350, [0, 1, 63, 64, 200, 975, 1348, 1349], 2),
    (8, 1, 24, 8, 128, 1350, [0, 5, 64, 130, 700, 975, 1100, 1349], 4),
    (8, 1, 24, 8, 128, 1350, [0, 2, 65, 127, 512, 974, 1200, 1349], 8),
    (16, 2, 8, 2, 128, 300, [0, 1] * 4 + [100, 101] * 2 + [298, 299] * 2, 4)])
def test_attn_matches_oracle(R, S, Hq, Hk, hd, L, pos, ns):
    from estudiocanciones_b200 import kernels
    gen = torch.Generator().manual_seed(R + L + ns)
    B = R // S
    q = torch.randn(R, Hq * hd, generator=gen).half()
    kc = torch.randn(B, Hk, L, hd, generator=gen).half()
    vc = torch.randn(B, Hk, L, hd, generator=gen).half()
    pos_t = torch.tensor(pos)
    o = torch.empty(R, Hq * hd, dtype=torch.float16, device=DEV)
    kernels.attn(q.to(DEV), kc.to(DEV), vc.to(DEV), pos_t.to(DEV), o, S, Hq, Hk, L, nsplit=ns)
    ref = O.decode_attn(q, kc, vc, pos_t, S, Hq, Hk)
    torch.testing.assert_close(o.cpu().float(), ref.float(), atol=2e-3, rtol=5e-3)


# ----------------------------------------------------------------------------- sampler
@pytest.mark.parametrize("i", range(5))
def test_sampler_golden(golden, i):
    from estudiocanciones_b200 import kernels
    z = golden("sampler")
    rows, n_takes, topk, temp, cfg = z[f"s{i}_cfg"]
    rows, n_takes, topk = int(rows), int(n_takes), int(topk)
    out = torch.full((rows, 8), -1, dtype=torch.long, device=DEV)
    kernels.sample(g(z[f"s{i}_logits"]).to(DEV), n_takes, float(cfg), topk, float(temp),
                   g(z[f"s{i}_noise"]).to(DEV), out, 3)
    assert torch.equal(out[:, 3:4].cpu(), g(z[f"s{i}_ids"]))


@pytest.mark.parametrize("seed", range(8))
def test_sampler_matches_oracle(seed):
    from estudiocanciones_b200 import kernels
    gen = torch.Generator().manual_seed(100 + seed)
    N, V = 4, 8197
    # temp 3.7 / 0.7: the fp32 division merges or separates neighbouring fp16 values
    cfg, topk, temp = [(1.5, 50, 1.0), (1.0, 50, 1.0), (3.0, 5, 0.5), (1.5, 1, 1.0), (1.5, 8197, 1.2),
                       (1.5, 50, 1.0), (1.5, 50, 3.7), (1.0, 200, 0.7)][seed]
    B = 2 * N if cfg != 1.0 else N
    logits = (torch.randn(B, V, generator=gen) * 4).half()
    if seed == 5:
        logits[:, 200:260] = 0.5   # a plateau of equal values straddling the top-k boundary
    noise = torch.empty(N, V).exponential_(1, generator=gen)
    out = torch.full((B, 8), -1, dtype=torch.long, device=DEV)
    kernels.sample(logits.to(DEV), N, cfg, topk, temp, noise.to(DEV), out, 0)
    ref = O.guided_sample(logits, N, cfg, topk, temp, noise)
    assert torch.equal(out[:, :1].cpu(), ref)


@pytest.mark.parametrize("N,cfg,topk,temp", [(8, 1.5, 50, 1.0), (1, 1.0, 50, 1.0), (3, 2.0, 100, 0.9)])
def test_sampler_cluster_shapes_match_oracle(N, cfg, topk, temp):
    """The sampler's cluster split at other take counts: config 4's 8 takes x CFG (64 CTAs),
    one take without CFG, an odd count; vocabularies that do not divide by the cluster."""
    from estudiocanciones_b200 import kernels
    for V in (8197, 4099):
        gen = torch.Generator().manual_seed(N * 1000 + V)
        B = 2 * N if cfg != 1.0 else N
        logits = (torch.randn(B, V, generator=gen) * 4).half()
        noise = torch.empty(N, V).exponential_(1, generator=gen)
        out = torch.full((B, 8), -1, dtype=torch.long, device=DEV)
        kernels.sample(logits.to(DEV), N, cfg, topk, temp, noise.to(DEV), out, 5)
        ref = O.guided_sample(logits, N, cfg, topk, temp, noise)
        assert torch.equal(out[:, 5:6].cpu(), ref), V
    assert kernels.read_errors(DEV) == 0


def test_rms_apply_equals_fused_rms_prologue():
    """hm_rms_apply (RMSNorm from the producer's sum-of-squares partials, one launch)
    gives exactly the rows the GEMV's fused RMSNorm prologue feeds its MMAs: a GEMV on
    its output equals the GEMV with the fused prologue bit for bit."""
    import ctypes as C
    from estudiocanciones_b200 import _lib, kernels
    from estudiocanciones_b200._lib import GemvDesc, RowSrc, HM_SRC_F16, HM_SRC_RMS
    gen = torch.Generator().manual_seed(21)
    R, D, N = 8, 3072, 1024
    x = torch.randn(R, D, generator=gen).half().to(DEV)
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half().to(DEV)
    ss = (x.float() ** 2).reshape(R, D // 16, 16).sum(-1).t().contiguous()
    w, s = rand_lin(N, D, gen)
    w, s = w.to(DEV), s.to(DEV)
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    err = kernels.error_word(DEV)
    xn = torch.empty_like(x)
    assert L.hm_rms_apply(x.data_ptr(), D, ss.data_ptr(), D // 16, R, gamma.data_ptr(), 1e-5, D, xn.data_ptr(), D,
                          R, D, 0, st) == 0
    ref = O.rmsnorm(x.cpu(), gamma.cpu())
    close16(xn, ref, ulps=1, frac_exact=0.99)

    def run(src):
        d = GemvDesc()
        d.w, d.s, d.N, d.K, d.M = w.data_ptr(), s.data_ptr(), N, D, R
        d.src[0] = src
        y = torch.empty(R, N, dtype=torch.float16, device=DEV)
        d.y, d.ldy, d.err = y.data_ptr(), N, err.data_ptr()
        assert L.hm_gemv_i8_fused(C.byref(d), st) == 0
        return y
    s_rms = RowSrc()
    s_rms.mode, s_rms.row_mul, s_rms.x, s_rms.ldx = HM_SRC_RMS, 1, x.data_ptr(), D
    s_rms.ss, s_rms.ss_tiles, s_rms.ss_ld, s_rms.gamma, s_rms.eps, s_rms.dim = ss.data_ptr(), D // 16, R, \
        gamma.data_ptr(), 1e-5, D
    s_f16 = RowSrc()
    s_f16.mode, s_f16.row_mul, s_f16.x, s_f16.ldx = HM_SRC_F16, 1, xn.data_ptr(), D
    torch.testing.assert_close(run(s_rms), run(s_f16), rtol=0, atol=0)
    assert kernels.read_errors(DEV) == 0


# ----------------------------------------------------------------------------- GEMV split over a cluster
@pytest.mark.parametrize("M,N,K,epi,src,csplit", [
    (8, 1024, 8192, "store_res", "f16", 4),    # decoder w2 shape
    (8, 3072, 8192, "store_res", "f16", 2),    # backbone w2 shape
    (8, 1024, 8192, "store_res", "f16", 8),
    (5, 3072, 3072, "store_res", "rms", 2),    # RMS prologue, padding rows
    (8, 4096, 3072, "silu", "rms", 2),
    (16, 1024, 4096, "store", "f16", 4),       # two MMA row groups
    (8, 1536, 1024, "rope", "rms", 2)])
def test_gemv_cluster_split_equals_workspace_split(M, N, K, epi, src, csplit):
    """kspan = -s splits K over the s CTAs of a thread-block cluster (partials summed
    in DSMEM by rank 0); it must give exactly the workspace split with kspan = K / s
    (same partials, same split order), including the residual, the sum-of-squares
    partials of the next RMSNorm and the RoPE / KV-cache and SiLU epilogues."""
    from estudiocanciones_b200.engine import Block, Linear
    gen = torch.Generator().manual_seed(M * 7 + N + K + csplit)
    x = torch.randn(M, K, generator=gen).half().to(DEV)
    gamma = (1 + 0.1 * torch.randn(K, generator=gen)).half().to(DEV)
    w, s = rand_lin(N, K, gen)
    lin = Linear(w.to(DEV), s.to(DEV))
    res0 = torch.randn(M, N, generator=gen).half().to(DEV)
    ss_x = _ss(x)  # a row source holds pointers only: keep its tensors alive until the launch
    kspan_ws = K // csplit
    outs = []
    for kspan in (-csplit, kspan_ws):
        p = _plan()
        srcx = p.src_rms(x, ss_x, gamma) if src == "rms" else p.src_f16(x)
        if epi == "store_res":
            y = res0.clone()
            ss_out = torch.zeros(N // 16, M, device=DEV)
            p._gemv(lin, M, srcx, y=y, res=y, ss_out=ss_out, kspan=kspan)
            p.run()
            outs.append((y, ss_out))
        elif epi == "store":
            y = torch.empty(M, N, dtype=torch.float16, device=DEV)
            p._gemv(lin, M, srcx, y=y, kspan=kspan)
            p.run()
            outs.append((y,))
        elif epi == "silu":
            y = torch.empty(M, N // 2, dtype=torch.float16, device=DEV)
            p._gemv(lin, M, srcx, epi=HM_EPI_SILU, y=y, kspan=kspan)
            p.run()
            outs.append((y,))
        else:
            Hq, Hk, hd, L = 8, 2, 128, 16
            blk = Block.__new__(Block)
            blk.h, blk.kvh, blk.hd = Hq, Hk, hd
            blk.kc = torch.zeros(M, Hk, L, hd, dtype=torch.float16, device=DEV)
            blk.vc = torch.zeros_like(blk.kc)
            q = torch.empty(M, Hq * hd, dtype=torch.float16, device=DEV)
            pos = torch.arange(M, device=DEV) % L
            p._gemv(lin, M, srcx, epi=HM_EPI_ROPE_KV, rope=O.rope_table(hd, L).to(DEV), pos=pos, S=1, blk=blk,
                    q_out=q, kspan=kspan)
            p.run()
            outs.append((q, blk.kc, blk.vc))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert kernels_errors() == 0


def kernels_errors():
    from estudiocanciones_b200 import kernels
    return kernels.read_errors(DEV)


# ----------------------------------------------------------------------------- wide GEMV kernel (backbone shapes)
@pytest.mark.parametrize("M", [8, 5, 16, 12])
def test_gemv_wide_silu_backbone_shape(M):
    """w1|w3 of the backbone (N 2 x 8192, K 3072: 512 tiles, more than the narrow kernel
    has CTAs) runs on the wide kernel (four consumer groups at 8 rows, three at 16):
    RMSNorm prologue + SiLU epilogue vs the oracle."""
    from estudiocanciones_b200.engine import Linear
    gen = torch.Generator().manual_seed(31 + M)
    D, F = 3072, 8192
    x = torch.randn(M, D, generator=gen).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half()
    w, s = rand_lin(2 * F, D, gen)
    lin = Linear(w.to(DEV), s.to(DEV))
    xd, gd = x.to(DEV), gamma.to(DEV)
    ss = _ss(xd)
    y = torch.empty(M, F, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, M, p.src_rms(xd, ss, gd), epi=HM_EPI_SILU, y=y)
    p.run()
    xn = O.rmsnorm(x, gamma)
    a = O.gemv_i8(xn, w, s)
    ref = O.silu_mul(a)
    sl = rms_slack(xn, w, s, a)
    close16(y, ref, ulps=3, frac_exact=0.9, slack=2 * (sl[:, :F] * a[:, F:].float().abs() + sl[:, F:]))


@pytest.mark.parametrize("R", [8, 16])
def test_gemv_wide_rope_backbone_shape(R):
    """qkv of the backbone (N 5120, K 3072: 320 tiles) on the wide kernel: RoPE + KV-cache
    write epilogue vs the oracle; cache slots nobody writes stay untouched."""
    from estudiocanciones_b200.engine import Block, Linear
    gen = torch.Generator().manual_seed(41 + R)
    Hq, Hk, hd, D, L = 24, 8, 128, 3072, 64
    x = torch.randn(R, D, generator=gen).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half()
    N = (Hq + 2 * Hk) * hd
    w, s = rand_lin(N, D, gen)
    pos = torch.tensor([0, 1, 5, 17, 33, 62, 63, 40, 2, 9, 61, 30, 3, 44, 12, 50][:R])
    rope = O.rope_table(hd, L)
    kc0 = torch.randn(R, Hk, L, hd, generator=gen).half()
    vc0 = torch.randn(R, Hk, L, hd, generator=gen).half()
    blk = Block.__new__(Block)
    blk.h, blk.kvh, blk.hd = Hq, Hk, hd
    blk.kc, blk.vc = kc0.clone().to(DEV), vc0.clone().to(DEV)
    lin = Linear(w.to(DEV), s.to(DEV))
    xd, gd, rd, pd = x.to(DEV), gamma.to(DEV), rope.to(DEV), pos.to(DEV)
    ss = _ss(xd)
    q = torch.empty(R, Hq * hd, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, R, p.src_rms(xd, ss, gd), epi=HM_EPI_ROPE_KV, rope=rd, pos=pd, S=1, blk=blk, q_out=q)
    p.run()
    xn = O.rmsnorm(x, gamma)
    qkv = O.gemv_i8(xn, w, s)
    kc, vc = kc0.clone(), vc0.clone()
    qr = O.rope_kv_write(qkv, rope, pos, kc, vc, 1, Hq, Hk)
    sl = rms_slack(xn, w, s, qkv).float().abs()
    qsl = sl[:, : Hq * hd]
    qsl = torch.maximum(qsl, qsl.reshape(R, Hq, hd // 2, 2).flip(-1).reshape(R, -1))
    close16(q, qr, ulps=2, frac_exact=0.9, slack=qsl)
    close16(blk.kc, kc, ulps=2, frac_exact=0.95, slack=2e-3 * kc.float().abs() + 5e-4)
    close16(blk.vc, vc, ulps=2, frac_exact=0.95, slack=2e-3 * vc.float().abs() + 5e-4)
    mask = torch.ones(R, L, dtype=torch.bool)
    for r in range(R):
        mask[r, int(pos[r])] = False
    idx = mask.nonzero(as_tuple=True)
    assert torch.equal(blk.kc.cpu().permute(0, 2, 1, 3)[idx], kc0.permute(0, 2, 1, 3)[idx])
    assert torch.equal(blk.vc.cpu().permute(0, 2, 1, 3)[idx], vc0.permute(0, 2, 1, 3)[idx])


def test_gemv_wide_store_codebook0_head_16_rows():
    """The codebook-0 head at 16 rows (N 8197, K 3072: 513 tiles, the last one ragged)
    on the three-group wide kernel: RMSNorm prologue, plain store."""
    from estudiocanciones_b200.engine import Linear
    gen = torch.Generator().manual_seed(47)
    M, D, N = 16, 3072, 8197
    x = torch.randn(M, D, generator=gen).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half()
    w, s = rand_lin(N, D, gen)
    lin = Linear(w.to(DEV), s.to(DEV))
    xd, gd = x.to(DEV), gamma.to(DEV)
    y = torch.empty(M, N, dtype=torch.float16, device=DEV)
    p = _plan()
    p._gemv(lin, M, p.src_rms(xd, _ss(xd), gd), y=y)
    p.run()
    xn = O.rmsnorm(x, gamma)
    ref = O.gemv_i8(xn, w, s)
    close16(y, ref, ulps=2, frac_exact=0.9, slack=rms_slack(xn, w, s, ref))


def test_gemv_wide_store_residual_backbone_w2_shape():
    """w2 of the backbone (N 3072, K 8192: one narrow CTA per SM, 192 tiles) on the wide
    kernel: residual + sum-of-squares partials vs the oracle."""
    from estudiocanciones_b200.engine import Linear
    gen = torch.Generator().manual_seed(43)
    M, D, N = 8, 8192, 3072
    x = (torch.randn(M, D, generator=gen) * 0.5).half()
    w, s = rand_lin(N, D, gen)
    res = torch.randn(M, N, generator=gen).half()
    lin = Linear(w.to(DEV), s.to(DEV))
    xd, yd = x.to(DEV), res.to(DEV).clone()
    ss_out = torch.zeros(N // 16, M, device=DEV)
    p = _plan()
    p._gemv(lin, M, p.src_f16(xd), y=yd, res=yd, ss_out=ss_out)
    p.run()
    ref = O.gemv_i8(x, w, s, res)
    close16(yd, ref, ulps=2, frac_exact=0.9, slack=acc_slack(x, w, s))
    torch.testing.assert_close(ss_out.cpu(), _ss(yd).cpu(), rtol=1e-5, atol=1e-4)
