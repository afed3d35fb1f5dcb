"""HeartCodec detokenize on the B200: every kernel against a torch fp64/fp32 reference of the
same op, then the whole codec against the goldens of the unmodified reference
(tests/golden/codec.npz) and, at the full codec's layer widths, against the CPU oracle.

Tolerances (fp16 operands, fp32 accumulation on the tensor cores):
* a GEMM/conv with fp16 output: max |err| <= 2e-3 max |ref| (one fp16 rounding, 2^-11,
  plus fp32 accumulation order); fp32 output: <= 2e-5 max |ref|;
* attention: max |err| <= 4e-3 max |ref| (probabilities rounded to fp16 for the PV product);
* whole estimator / decoder / detokenize: the bounds stated at each test, set by the fp16
  activations between layers (the reference's own GPU mode computes in fp16 too).
"""
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = Path(__file__).parent / "golden" / "codec.npz"


@pytest.fixture(scope="module")
def L():
    from estudiocanciones_b200 import build
    build.build()
    from estudiocanciones_b200 import _lib
    return _lib


def stream():
    return torch.cuda.current_stream().cuda_stream


def ref_conv(x, w, off0, dil, T):
    """x [B, tin, cin], w [taps, N, cin] -> [B, T, N] in fp64 (rows outside [0, tin) are zero)."""
    B, tin, _ = x.shape
    out = torch.zeros(B, T, w.shape[1], dtype=torch.float64, device=x.device)
    xd, wd = x.double(), w.double()
    for j in range(w.shape[0]):
        src = torch.arange(T, device=x.device) + off0 + j * dil
        ok = (src >= 0) & (src < tin)
        xs = torch.zeros(B, T, x.shape[2], dtype=torch.float64, device=x.device)
        xs[:, ok] = xd[:, src[ok]]
        out += xs @ wd[j].t()
    return out


def run_conv(L, x, w, *, T=None, off0=0, dil=1, bias=None, scale=1.0, act=0, prelu=1.0, epi=0, res=None,
             gate=None, gate_ld=0, rope=None, rope_cols=0, hd=0, y_f32=False, bn=0, N=None, y=None, y_ld=None):
    B, tin, cin = x.shape
    taps, npad, _ = w.shape
    N = N or npad
    T = T or tin
    out_cols = N // 2 if epi == L.HM_CEPI_SILU else N
    if y is None:
        y = torch.zeros(B * T, out_cols, dtype=torch.float32 if y_f32 else torch.float16, device=DEV)
    d = L.ConvDesc()
    d.x, d.x_ld, d.x_bstride = x.data_ptr(), cin, tin * cin
    d.w, d.bias = w.data_ptr(), 0 if bias is None else bias.data_ptr()
    d.y, d.y_ld = y.data_ptr(), y_ld or out_cols
    d.res, d.res_ld = (0, 0) if res is None else (res.data_ptr(), res.shape[-1])
    d.gate, d.gate_ld = (0 if gate is None else gate.data_ptr()), gate_ld
    d.rope = 0 if rope is None else rope.data_ptr()
    d.err = 0
    d.B, d.T, d.tin, d.cin, d.N, d.npad, d.taps, d.off0, d.dil = B, T, tin, cin, N, npad, taps, off0, dil
    d.scale, d.prelu, d.act, d.epi, d.y_f32, d.rope_cols, d.hd, d.bn = scale, prelu, act, epi, int(y_f32), \
        rope_cols, hd, bn
    L.check(L.lib().hm_conv1d_gemm(d, stream()), "hm_conv1d_gemm")
    torch.cuda.synchronize()
    return y


def rnd(*shape, s=1.0, dtype=torch.float16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * s).to(dtype)


def close(got, ref, rel):
    err = (got.double() - ref.double()).abs().max().item()
    return err <= rel * ref.abs().max().item(), err


@pytest.mark.parametrize("B,T,tin,cin,N,taps,off0,dil", [
    (1, 300, 300, 192, 320, 1, 0, 1),      # linear, N not a multiple of 128
    (2, 250, 250, 128, 64, 7, -18, 3),     # causal dilated residual conv
    (2, 200, 200, 576, 128, 3, -1, 1),     # ProjectLayer conv (centered, k=3)
    (2, 150, 150, 256, 256, 2, 0, -1),     # causal transposed conv as taps (stride 4, 64 channels)
    (2, 130, 130, 64, 128, 4, -3, 1),      # PostProcessor repeat + conv folded into taps
    (3, 129, 129, 64, 192, 5, -2, 1),      # ragged rows, three items
])
def test_conv_matches_fp64(L, B, T, tin, cin, N, taps, off0, dil):
    x = rnd(B, tin, cin, seed=1)
    w = rnd(taps, N, cin, s=(taps * cin) ** -0.5, seed=2)
    bias = rnd(N, s=0.1, dtype=torch.float32, seed=3)
    ref = (ref_conv(x, w, off0, dil, T) + bias.double()) * 0.7
    ref = torch.where(ref >= 0, ref, 0.2 * ref)
    y16 = run_conv(L, x, w, T=T, off0=off0, dil=dil, bias=bias, scale=0.7, act=L.HM_ACT_PRELU, prelu=0.2)
    ok, err = close(y16.view(B, T, N), ref, 2e-3)
    assert ok, err
    y32 = run_conv(L, x, w, T=T, off0=off0, dil=dil, bias=bias, scale=0.7, act=L.HM_ACT_PRELU, prelu=0.2, y_f32=True)
    ok, err = close(y32.view(B, T, N), ref, 2e-5)
    assert ok, err


def test_conv_tile_widths_agree(L):
    """bn 64 / 128 / 256 accumulate each element over k in the same order: identical results."""
    x = rnd(2, 333, 256, seed=4)
    w = rnd(3, 512, 256, s=0.05, seed=5)
    outs = [run_conv(L, x, w, off0=-1, bn=bn, y_f32=True) for bn in (64, 128, 256)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    ok, err = close(outs[0].view(2, 333, 512), ref_conv(x, w, -1, 1, 333), 2e-5)
    assert ok, err


def test_conv_epilogues(L):
    B, T, cin, N = 2, 200, 128, 256
    x = rnd(B, T, cin, seed=6)
    w = rnd(1, N, cin, s=cin ** -0.5, seed=7)
    acc = ref_conv(x, w, 0, 1, T)
    # gated residual in place: h = h + gate[b] * acc
    h = rnd(B * T, N, dtype=torch.float32, seed=8)
    gate = rnd(B, N, dtype=torch.float32, seed=9)
    want = h.double().view(B, T, N) + gate.double()[:, None] * acc
    run_conv(L, x, w, epi=L.HM_CEPI_GATED, res=h, gate=gate, gate_ld=N, y_f32=True, y=h)
    ok, err = close(h.view(B, T, N), want, 2e-5)
    assert ok, err
    # residual add (fp16, in place) after PReLU
    r = rnd(B * T, N, seed=10)
    pre = torch.where(acc >= 0, acc, 0.3 * acc)
    want = pre + r.double().view(B, T, N)
    run_conv(L, x, w, act=L.HM_ACT_PRELU, prelu=0.3, epi=L.HM_CEPI_RES, res=r, y=r)
    ok, err = close(r.view(B, T, N), want, 2e-3)
    assert ok, err
    # SiLU act
    y = run_conv(L, x, w, act=L.HM_ACT_SILU)
    ok, err = close(y.view(B, T, N), F.silu(acc), 2e-3)
    assert ok, err


def test_conv_silu_mul(L):
    B, T, cin, Fh = 1, 300, 192, 256  # two 256-row blocks: 128 gate rows then 128 up rows each
    x = rnd(B, T, cin, seed=11)
    gate = rnd(Fh, cin, s=cin ** -0.5, seed=12)
    up = rnd(Fh, cin, s=cin ** -0.5, seed=13)
    w = torch.stack([gate.view(2, 128, cin), up.view(2, 128, cin)], 1).reshape(1, 2 * Fh, cin)
    y = run_conv(L, x, w, epi=L.HM_CEPI_SILU)
    a = ref_conv(x, gate[None], 0, 1, T)
    u = ref_conv(x, up[None], 0, 1, T)
    ok, err = close(y.view(B, T, Fh), F.silu(a) * u, 2e-3)
    assert ok, err


@pytest.mark.parametrize("hd", [64, 128])
def test_conv_rope(L, hd):
    B, T, D = 2, 200, 2 * hd
    x = rnd(B, T, D, seed=14)
    w = rnd(1, 3 * D, D, s=D ** -0.5, seed=15)
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32, device=DEV) / hd))
    fr = torch.arange(T, dtype=torch.float32, device=DEV)[:, None] * inv[None]
    rope = torch.stack([fr.cos(), fr.sin()], -1).contiguous()
    y = run_conv(L, x, w, epi=L.HM_CEPI_ROPE, rope=rope, rope_cols=2 * D, hd=hd)
    acc = ref_conv(x, w, 0, 1, T)
    qk = acc[..., :2 * D].reshape(B, T, 2 * D // hd, hd // 2, 2)
    c, s = fr.cos().double()[None, :, None], fr.sin().double()[None, :, None]
    rot = torch.stack([qk[..., 0] * c - qk[..., 1] * s, qk[..., 0] * s + qk[..., 1] * c], -1).reshape(B, T, 2 * D)
    want = torch.cat([rot, acc[..., 2 * D:]], -1)
    ok, err = close(y.view(B, T, 3 * D), want, 2e-3)
    assert ok, err


def test_conv_single_output_column_and_small_m(L):
    x = rnd(2, 500, 64, seed=16)
    w = torch.zeros(7, 64, 64, dtype=torch.float16, device=DEV)
    w[:, :1] = rnd(7, 1, 64, s=0.05, seed=17)
    y = torch.zeros(2 * 500, dtype=torch.float32, device=DEV)
    run_conv(L, x, w, N=1, off0=-6, y_f32=True, y=y, y_ld=1)
    ok, err = close(y.view(2, 500, 1), ref_conv(x, w[:, :1], -6, 1, 500), 2e-5)
    assert ok, err
    # 3 output rows from a zero-padded 128-row input
    xs = torch.zeros(1, 128, 128, dtype=torch.float16, device=DEV)
    xs[0, :3] = rnd(3, 128, seed=18)
    w2 = rnd(1, 192, 128, s=0.1, seed=19)
    y2 = run_conv(L, xs, w2, T=3, y_f32=True)
    ok, err = close(y2.view(1, 3, 192), ref_conv(xs, w2, 0, 1, 3), 2e-5)
    assert ok, err


def test_conv_rejects_bad_arguments(L):
    x = rnd(1, 64, 96)  # cin % 64 != 0
    w = rnd(1, 64, 96)
    with pytest.raises(L.HMError):
        run_conv(L, x, w)
    x = rnd(1, 64, 128)
    w = rnd(1, 256, 128)
    with pytest.raises(L.HMError):  # SiLU needs N % 256 == 0 and its own tile width
        run_conv(L, x, w[:, :128].contiguous(), epi=L.HM_CEPI_SILU)


@pytest.mark.parametrize("B,T,H,hd", [(2, 200, 2, 64), (2, 744, 24, 64), (2, 744, 24, 128), (1, 100, 3, 128),
                                      (2, 300, 2, 128)])
def test_codec_attention_matches_sdpa(L, B, T, H, hd):
    D = H * hd
    qkv = rnd(B * T, 3 * D, seed=20)
    o = torch.zeros(B * T, D, dtype=torch.float16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.check(L.lib().hm_codec_attn(qkv.data_ptr(), qkv[:, D:].data_ptr(), qkv[:, 2 * D:].data_ptr(), o.data_ptr(), B, T,
                                  H, hd, 3 * D, D, hd ** -0.5, err.data_ptr(), stream()), "hm_codec_attn")
    torch.cuda.synchronize()
    q, k, v = (qkv.float().view(B, T, 3, H, hd)[:, :, i].transpose(1, 2) for i in range(3))
    want = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B * T, D)
    ok, e = close(o, want, 4e-3)
    assert ok, e
    assert int(err) == 0


@pytest.mark.parametrize("layer_norm", [0, 1])
def test_norm_mod(L, layer_norm):
    B, T, D = 2, 150, 1536
    x = rnd(B * T, D, s=3.0, dtype=torch.float32, seed=21) + 1.5
    w = rnd(D, s=0.1, dtype=torch.float32, seed=22) + 1
    shift = rnd(B, D, s=0.1, dtype=torch.float32, seed=23)
    scale = rnd(B, D, s=0.1, dtype=torch.float32, seed=24)
    out = torch.zeros(B * T, D + 64, dtype=torch.float16, device=DEV)
    L.check(L.lib().hm_codec_norm_mod(x.data_ptr(), D, 0 if layer_norm else w.data_ptr(), shift.data_ptr(),
                                      scale.data_ptr(), D, out.data_ptr(), D + 64, B, T, D, 1e-6, layer_norm,
                                      stream()), "norm_mod")
    torch.cuda.synchronize()
    xd = x.double()
    if layer_norm:
        n = F.layer_norm(xd, (D,), eps=1e-6)
    else:
        n = w.double() * (xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-6))
    want = (n.view(B, T, D) * (1 + scale.double()[:, None]) + shift.double()[:, None]).view(B * T, D)
    ok, e = close(out[:, :D], want, 2e-3)
    assert ok, e


def test_vq_embed_and_upsample(L):
    nq, n, K, cd, dim = 8, 50, 64, 8, 128
    g = torch.Generator().manual_seed(25)
    codes = torch.randint(0, K, (nq, n), generator=g)
    codes[0, 3], codes[5, 7] = -4, K + 9  # clamped into the codebook like codec_lite.decode's clamp
    cb = torch.randn(nq, K, cd, generator=g)
    pw, pb = torch.randn(dim, cd, generator=g), torch.randn(dim, generator=g)
    out = torch.zeros(n, dim, dtype=torch.float16, device=DEV)
    cdev, cbd, pwd, pbd = codes.to(DEV), cb.to(DEV), pw.to(DEV), pb.to(DEV)
    L.check(L.lib().hm_codec_vq_embed(cdev.data_ptr(), n, nq, n, cbd.data_ptr(), K, cd, pwd.data_ptr(), pbd.data_ptr(),
                                      out.data_ptr(), dim, dim, stream()), "vq")
    cl = codes.clamp(0, K - 1)
    want = sum(cb[q][cl[q]] for q in range(nq)) @ pw.t() + pb
    ok, e = close(out.cpu(), want, 2e-3)
    assert ok, e
    up = torch.zeros(2 * n, dim + 64, dtype=torch.float16, device=DEV)
    L.check(L.lib().hm_codec_upsample_rows(out.data_ptr(), dim, n, dim, 2, up[:, 64:].data_ptr(), dim + 64, stream()),
            "up")
    torch.cuda.synchronize()
    assert torch.equal(up[:, 64:], out.repeat_interleave(2, 0)) and not up[:, :64].any()


def test_euler_steps(L):
    T, C, L_in, nb = 300, 256, 40, 2
    XW = 2 * C + 64
    v = rnd(nb * T, C, dtype=torch.float32, seed=26)
    x = rnd(T, C, dtype=torch.float32, seed=27)
    noise = rnd(T, C, dtype=torch.float32, seed=28)
    inc = rnd(L_in, C, dtype=torch.float32, seed=29)
    xin = torch.zeros(nb, T, XW, dtype=torch.float16, device=DEV)
    lib = L.lib()
    # first call: x = noise, in-context blend at t = 0, inc columns written
    x0 = x.clone()
    L.check(lib.hm_codec_euler(0, nb, x0.data_ptr(), noise.data_ptr(), inc.data_ptr(), T, C, L_in, 0.0, 0.0, 0.0, 0,
                               xin.data_ptr(), XW, T * XW, stream()), "euler")
    torch.cuda.synchronize()
    assert torch.allclose(x0, noise)
    want_inc = torch.zeros(T, C, device=DEV)
    want_inc[:L_in] = inc
    for b in range(nb):
        assert torch.equal(xin[b, :, :C], noise.half()) and torch.equal(xin[b, :, C:2 * C], want_inc.half())
    # an update step
    dt, gs, tn = 0.1, 1.25, 0.3
    x1 = x.clone()
    L.check(lib.hm_codec_euler(v.data_ptr(), nb, x1.data_ptr(), noise.data_ptr(), inc.data_ptr(), T, C, L_in, dt, gs,
                               tn, 0, xin.data_ptr(), XW, T * XW, stream()), "euler")
    torch.cuda.synchronize()
    u, c = v[:T], v[T:]
    want = x + dt * (u + gs * (c - u))
    want[:L_in] = (1 - (1 - 1e-6) * tn) * noise[:L_in] + tn * inc
    assert (x1 - want).abs().max() < 1e-5
    assert torch.equal(xin[1, :, :C], x1.half())
    # last step: rows < L_in take the in-context latents
    x2 = x.clone()
    L.check(lib.hm_codec_euler(v.data_ptr(), nb, x2.data_ptr(), noise.data_ptr(), inc.data_ptr(), T, C, L_in, dt, gs,
                               tn, 1, 0, XW, T * XW, stream()), "euler")
    torch.cuda.synchronize()
    assert torch.equal(x2[:L_in], inc) and (x2[L_in:] - want[L_in:]).abs().max() < 1e-5


def test_band_quant_and_overlap_add(L):
    T, Cb = 300, 128
    x = rnd(T, 2 * Cb, dtype=torch.float32, seed=30)
    x[0, :8] = torch.tensor([0.5, 1.5, 2.5, -0.5, 1 / 18, 3 / 18, -5 / 18, 0.0], device=DEV) / 9 * 9 / 9
    q = torch.zeros(2, T, Cb, dtype=torch.float16, device=DEV)
    L.check(L.lib().hm_codec_band_quant(x.data_ptr(), T, Cb, 2, q.data_ptr(), stream()), "bq")
    torch.cuda.synchronize()
    want = (torch.round(9 * x) / 9).view(T, 2, Cb).permute(1, 0, 2).half()
    assert torch.equal(q, want)
    n, ovlp, total = 1000, 300, 1700
    out = rnd(2, total, dtype=torch.float32, seed=31)
    cur = rnd(2, n, dtype=torch.float32, seed=32)
    start = total - n
    before = out.clone()
    L.check(L.lib().hm_codec_overlap_add(cur.data_ptr(), n, out.data_ptr(), total, 2, start, n, ovlp, stream()), "ola")
    torch.cuda.synchronize()
    w = torch.from_numpy(np.linspace(0, 1, ovlp))[None].to(DEV)
    blend = (before[:, start:start + ovlp].double() * (1 - w) + cur[:, :ovlp].double() * w).float()
    assert torch.equal(out[:, :start], before[:, :start])
    assert (out[:, start:start + ovlp] - blend).abs().max() <= 1e-6
    assert torch.equal(out[:, start + ovlp:], cur[:, ovlp:])


# ---------------------------------------------------------------- whole codec
@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def tiny(L, gold):
    from estudiocanciones_b200.checkpoint import tensors_sha
    from estudiocanciones_b200.codec import HeartCodecB200
    from estudiocanciones_b200.codec_checkpoint import TINY_CODEC, synthetic_codec_tensors
    sd = synthetic_codec_tensors(TINY_CODEC, 4321)
    assert bytes(gold["sha"]).hex() == tensors_sha(sd)
    return HeartCodecB200(sd, TINY_CODEC, device=DEV)


def rel_l2(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_estimator_matches_reference_golden(tiny, gold):
    from estudiocanciones_b200.codec_checkpoint import TINY_CODEC
    x = torch.randn(2, 200, TINY_CODEC.in_channels, generator=torch.Generator().manual_seed(5))
    got = tiny.estimator(x.to(DEV), float(gold["est_t"][0]))
    ref = torch.from_numpy(gold["est_out"])
    e = rel_l2(got, ref)
    assert e < 5e-3, e


def test_scalar_decode_matches_reference_golden(tiny, gold):
    lat = torch.from_numpy(gold["dec_in"])  # [2 bands, C, T]
    T = lat.shape[2]
    got = tiny.scalar_decode(lat.permute(2, 0, 1).reshape(T, -1).to(DEV))
    ref = torch.from_numpy(gold["dec_out"])[:, 0]
    e = rel_l2(got, ref)
    assert e < 5e-3, e


@pytest.mark.parametrize("case", [0, 1, 2])
def test_detokenize_matches_reference_golden(tiny, gold, case):
    n, steps, gs, seed = gold[f"detok{case}_cfg"]
    g = torch.Generator().manual_seed(int(seed))
    wav = tiny.detokenize(torch.from_numpy(gold[f"detok{case}_codes"]), num_steps=int(steps),
                          guidance_scale=float(gs), randn=lambda shape, where: torch.randn(shape, generator=g))
    ref = torch.from_numpy(gold[f"detok{case}_wav"])
    assert wav.shape == ref.shape
    e = rel_l2(wav, ref)
    assert e < 3e-2, e


@pytest.fixture(scope="module")
def wide(L):
    """The full codec's layer widths (24 heads x 64, 1536 / 3072, FFN 4096 / 8192, decoder
    2048 -> 64 over strides 5/4/4/4/3) with fewer layers, against the CPU oracle."""
    import dataclasses
    from estudiocanciones_b200.codec import HeartCodecB200
    from estudiocanciones_b200.codec_checkpoint import FULL_CODEC, synthetic_codec_tensors
    from oracle.heartcodec_oracle import OracleCodec
    cfg = dataclasses.replace(FULL_CODEC, num_layers=2, num_layers_2=1)
    sd = synthetic_codec_tensors(cfg, 99)
    return HeartCodecB200(sd, cfg, device=DEV), OracleCodec(sd, cfg), cfg


def test_full_width_estimator_matches_oracle(wide):
    ours, orc, cfg = wide
    x = torch.randn(2, 744, cfg.in_channels, generator=torch.Generator().manual_seed(3))
    with torch.inference_mode():
        ref = orc.estimator(x, torch.tensor([0.45, 0.45]))
    got = ours.estimator(x.to(DEV), 0.45)
    e = rel_l2(got, ref)
    assert e < 5e-3, e


def test_full_width_decoder_matches_oracle(wide):
    ours, orc, cfg = wide
    T = 24
    lat = torch.randn(T, cfg.out_channels, generator=torch.Generator().manual_seed(4)) * 0.5
    with torch.inference_mode():
        ref = orc.scalar_decode(lat.view(T, 2, -1).permute(1, 2, 0))[:, 0]
    got = ours.scalar_decode(lat.to(DEV))
    assert got.shape == ref.shape == (2, T * cfg.hop)
    e = rel_l2(got, ref)
    assert e < 5e-3, e


def test_graph_replay_equals_eager(L, gold):
    """detokenize's window solves and decoder run as CUDA graphs after their first use: the
    same noise gives the same audio, bit for bit, as a codec that never captures."""
    from estudiocanciones_b200.codec import HeartCodecB200
    from estudiocanciones_b200.codec_checkpoint import TINY_CODEC, synthetic_codec_tensors
    sd = synthetic_codec_tensors(TINY_CODEC, 4321)
    codes = torch.from_numpy(gold["detok2_codes"])

    def run(c):
        g = torch.Generator().manual_seed(13)
        return c.detokenize(codes, num_steps=2, guidance_scale=1.5,
                            randn=lambda shape, where: torch.randn(shape, generator=g)).clone()

    eager = HeartCodecB200(sd, TINY_CODEC, device=DEV, graphs=False)
    graphed = HeartCodecB200(sd, TINY_CODEC, device=DEV)
    a = run(eager)
    run(graphed)  # first use of each plan: eager run + capture
    b = run(graphed)  # replays
    assert all("graph" in p for k, p in graphed._plans.items() if k[0] in ("flow", "dec"))
    assert torch.equal(a, b)


def test_conv_sm_pairs_equal_single_sm(L):
    """The SM-pair variant (bn -128 / -256: 256-row tiles over two SMs, cta_group::2) gives the
    single-SM results bit for bit: same products, same k order per element.  Ragged rows (333:
    the second pair's upper half lies past the item), three taps, two items, and the SiLU-mul,
    RoPE and gated-residual epilogues."""
    x = rnd(2, 333, 256, seed=40)
    w = rnd(3, 512, 256, s=0.05, seed=41)
    bias = rnd(512, s=0.1, dtype=torch.float32, seed=42)
    ref = run_conv(L, x, w, off0=-1, bias=bias, bn=256, y_f32=True)
    for bn in (-128, -256):
        assert torch.equal(run_conv(L, x, w, off0=-1, bias=bias, bn=bn, y_f32=True), ref), bn
    ok, err = close(ref.view(2, 333, 512), ref_conv(x, w, -1, 1, 333) + bias.double(), 2e-5)
    assert ok, err
    # SiLU-mul (pair tiles of 256: 128 gate rows on one SM, the 128 up rows on the other)
    xs = rnd(1, 300, 192, seed=43)
    ws = rnd(1, 512, 192, s=0.07, seed=44)
    assert torch.equal(run_conv(L, xs, ws, epi=L.HM_CEPI_SILU, bn=-256), run_conv(L, xs, ws, epi=L.HM_CEPI_SILU))
    # RoPE of q and k
    hd, D = 64, 128
    xr = rnd(2, 200, D, seed=45)
    wr = rnd(1, 3 * D, D, s=D ** -0.5, seed=46)
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32, device=DEV) / hd))
    fr = torch.arange(200, dtype=torch.float32, device=DEV)[:, None] * inv[None]
    rope = torch.stack([fr.cos(), fr.sin()], -1).contiguous()
    kw = dict(epi=L.HM_CEPI_ROPE, rope=rope, rope_cols=2 * D, hd=hd)
    assert torch.equal(run_conv(L, xr, wr, bn=-128, **kw), run_conv(L, xr, wr, bn=128, **kw))
    # gated residual into an fp32 stream, in place
    h1 = rnd(2 * 333, 512, dtype=torch.float32, seed=47)
    h2 = h1.clone()
    gate = rnd(2, 512, dtype=torch.float32, seed=48)
    run_conv(L, x, w, off0=-1, epi=L.HM_CEPI_GATED, res=h1, gate=gate, gate_ld=512, y_f32=True, y=h1, bn=256)
    run_conv(L, x, w, off0=-1, epi=L.HM_CEPI_GATED, res=h2, gate=gate, gate_ld=512, y_f32=True, y=h2, bn=-256)
    assert torch.equal(h1, h2)


def test_codec_api_surface(L, gold, tmp_path):
    """load_codec(path) + decode(codec, frames) as app/codec_lite.py calls them: the same audio as
    the codec built from the tensors; codes outside the codebook are clamped like the reference's
    decode; abort_signal returns None; a non-default duration runs its own window shape."""
    import json

    from safetensors.torch import save_file

    from estudiocanciones_b200 import codec as codec_lite
    from estudiocanciones_b200.codec import HeartCodecB200
    from estudiocanciones_b200.codec_checkpoint import TINY_CODEC, synthetic_codec_tensors
    sd = synthetic_codec_tensors(TINY_CODEC, 4321)
    f = tmp_path / "codec.safetensors"
    save_file(sd, str(f))
    f.with_suffix(".json").write_text(json.dumps(TINY_CODEC.to_dict()))
    c = codec_lite.load_codec(f, torch.float16, device=DEV)
    ref = HeartCodecB200(sd, TINY_CODEC, device=DEV)
    codes = torch.from_numpy(gold["detok1_codes"]).clone()
    torch.manual_seed(12)
    a = codec_lite.decode(c, codes, steps=2, guidance=1.0).clone()
    torch.manual_seed(12)
    b = ref.detokenize(codes, num_steps=2, guidance_scale=1.0).clone()
    assert torch.equal(a, b)
    bad = codes.clone()
    bad[0, 5], bad[3, 9] = -7, TINY_CODEC.codebook_size + 100
    clamped = bad.clamp(0, TINY_CODEC.codebook_size - 1)
    torch.manual_seed(12)
    x = codec_lite.decode(c, bad, steps=2, guidance=1.0).clone()
    torch.manual_seed(12)
    y = ref.detokenize(clamped, num_steps=2, guidance_scale=1.0).clone()
    assert torch.equal(x, y)
    assert ref.detokenize(codes, abort_signal=lambda: True) is None
    short = ref.detokenize(codes[:, :100], duration=10.24, num_steps=1, guidance_scale=1.25)
    assert short.shape == (2, int(100 / 12.5 * TINY_CODEC.sample_rate)) and torch.isfinite(short).all()
