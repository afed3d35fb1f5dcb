"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden`` were made by ``tests/golden/make_golden.py``
from the reference's unmodified ``app/kernels.py`` (Triton, interpreter mode)
and ``app/engine.py`` (CPU path and fast path).  These tests need no GPU.
"""
import numpy as np
import pytest
import torch

from oracle import heartmula_oracle as O
from estudiocanciones_b200.checkpoint import TINY_SHAPE, synthetic_tensors, tensors_sha


def t(a):
    return torch.from_numpy(np.array(a))


def ulp_close(a, b, max_abs=2e-3, rel=2e-3):
    a, b = a.float(), b.float()
    return torch.all((a - b).abs() <= max_abs + rel * b.abs()).item()


def test_rope_table_bit_identical(golden):
    z = golden("kernels")
    for i in range(2):
        tab = t(z[f"rope{i}_table"])
        assert torch.equal(O.rope_table(128, tab.shape[0]), tab)


@pytest.mark.parametrize("i", range(5))
def test_gemv_matches_reference_kernel(golden, i):
    z = golden("kernels")
    x, w, s, y = t(z[f"gemv{i}_x"]), t(z[f"gemv{i}_w"]), t(z[f"gemv{i}_s"]), t(z[f"gemv{i}_y"])
    r = t(z[f"gemv{i}_r"]) if f"gemv{i}_r" in z else None
    out = O.gemv_i8(x, w, s, r)
    # same rounding points; only the fp32 accumulation order differs -> 1 fp16 ulp
    diff = (out.float() - y.float()).abs()
    assert diff.max().item() <= 2 * 2.0 ** -10 * max(1.0, y.float().abs().max().item())
    assert (out == y).float().mean().item() > 0.97


@pytest.mark.parametrize("i", range(2))
def test_rmsnorm_matches_reference_kernel(golden, i):
    z = golden("kernels")
    out = O.rmsnorm(t(z[f"rms{i}_x"]), t(z[f"rms{i}_w"]))
    y = t(z[f"rms{i}_y"])
    assert ulp_close(out, y, 1e-3, 1e-3)
    assert (out == y).float().mean().item() > 0.99


@pytest.mark.parametrize("i", range(2))
def test_rope_cache_matches_reference_kernel(golden, i):
    z = golden("kernels")
    R, S, Hq, Hk, L = (int(v) for v in z[f"rope{i}_cfg"])
    kc, vc = t(z[f"rope{i}_kc0"]).clone(), t(z[f"rope{i}_vc0"]).clone()
    q = O.rope_kv_write(t(z[f"rope{i}_qkv"]), t(z[f"rope{i}_table"]), t(z[f"rope{i}_pos"]), kc, vc, S, Hq, Hk)
    assert ulp_close(q, t(z[f"rope{i}_q"]), 1e-3, 1e-3)
    assert ulp_close(kc, t(z[f"rope{i}_kc"]), 1e-3, 1e-3)
    # v is copied untouched and untouched slots keep their values: bit-exact
    assert torch.equal(vc, t(z[f"rope{i}_vc"]))


@pytest.mark.parametrize("i", range(3))
def test_decode_attention_matches_reference_kernel(golden, i):
    z = golden("kernels")
    R, S, Hq, Hk, L, ns = (int(v) for v in z[f"attn{i}_cfg"])
    o = O.decode_attn(t(z[f"attn{i}_q"]), t(z[f"attn{i}_kc"]), t(z[f"attn{i}_vc"]), t(z[f"attn{i}_pos"]), S, Hq, Hk)
    assert ulp_close(o, t(z[f"attn{i}_o"]), 2e-3, 5e-3)


@pytest.mark.parametrize("i", range(2))
def test_silu_mul_matches_reference_kernel(golden, i):
    z = golden("kernels")
    out = O.silu_mul(t(z[f"silu{i}_a"]))
    y = t(z[f"silu{i}_y"])
    assert ulp_close(out, y, 1e-3, 1e-3)
    assert (out == y).float().mean().item() > 0.99


@pytest.mark.parametrize("i", range(5))
def test_sampler_matches_reference(golden, i):
    z = golden("sampler")
    rows, n_takes, topk, temp, cfg = z[f"s{i}_cfg"]
    rows, n_takes, topk = int(rows), int(n_takes), int(topk)
    ids = O.guided_sample(t(z[f"s{i}_logits"]), n_takes, float(cfg), topk, float(temp), t(z[f"s{i}_noise"]))
    assert torch.equal(ids, t(z[f"s{i}_ids"]))


def _tiny_model(golden, name, mode):
    z = golden(name)
    tensors = synthetic_tensors(TINY_SHAPE, seed=int(z["seed"]), gamma_one=False)
    assert tensors_sha(tensors) == str(z["sha"]), "synthetic checkpoint drifted from the fixture"
    return z, O.OracleModel(tensors, bb_heads=TINY_SHAPE.bb_heads, dec_heads=TINY_SHAPE.dec_heads,
                            mode=mode, dtype=torch.float16)


def _run_teacher_forced(z, m):
    N, B, P, muq_idx, n_frames = (int(v) for v in z["meta"])
    cfg, topk, temp = z["cfg"]
    force = t(z["force"])
    m.alloc(B, P + n_frames + 2 + 256)
    h = m.prompt_embed(t(z["text"]), N, muq_idx)
    hb = m.prefill(h)
    rec = []
    tok = m.frame(hb[:, -1], N, float(cfg), int(topk), float(temp), force=force[0], record=rec,
                  noise=[torch.ones(N, m.vocab)] * m.n_cb)
    for f in range(n_frames):
        pos = torch.full((B, 1), P + f, dtype=torch.long)
        tok = m.step(tok, pos, N, float(cfg), int(topk), float(temp), force=force[f + 1], record=rec,
                     noise=[torch.ones(N, m.vocab)] * m.n_cb)
    return hb, torch.stack(rec)


@pytest.mark.parametrize("name,mode", [("model_fast", "fast"), ("model_cpu", "cpu")])
def test_teacher_forced_frame_matches_reference_engine(golden, name, mode):
    """Whole frames (prefill + 1 decode frame) under teacher forcing: per-head
    logits within 2e-2 max-abs, and identical argmax / top-50 sets."""
    z, m = _tiny_model(golden, name, mode)
    hb, logits = _run_teacher_forced(z, m)
    ref = t(z["logits"])
    assert logits.shape == ref.shape
    d = (logits.float() - ref.float()).abs().max().item()
    assert d <= 2e-2, d
    assert torch.equal(logits.float().argmax(-1), ref.float().argmax(-1))
    assert ulp_close(hb[:, -1], t(z["hb_last"]), 1e-2, 1e-2)
    # KV cache slots: prefill tail and the decode frame's slot
    P = int(z["meta"][2])
    for j, ly in enumerate((m.bb[0], m.bb[-1])):
        assert ulp_close(ly.kc[:, :, P - 3:P], t(z[f"kc_pre{j}"]), 1e-2, 1e-2)
        assert ulp_close(ly.vc[:, :, P - 3:P], t(z[f"vc_pre{j}"]), 1e-2, 1e-2)
        assert ulp_close(ly.kc[:, :, P:P + 1], t(z[f"kc_dec{j}"]), 1e-2, 1e-2)
        assert ulp_close(ly.vc[:, :, P:P + 1], t(z[f"vc_dec{j}"]), 1e-2, 1e-2)


def assert_argmax_except_ties(got, ref, tie=4e-3):
    """Identical argmax wherever the reference's best logit leads its second by more than
    ``tie``; where it does not (the 10-frame golden holds exact fp16 ties), the chosen id
    must be within ``tie`` of the reference's best."""
    top2 = ref.topk(2, -1).values
    clear = (top2[..., 0] - top2[..., 1]) > tie
    a, b = got.argmax(-1), ref.argmax(-1)
    assert torch.equal(a[clear], b[clear])
    picked = ref.gather(-1, a.unsqueeze(-1)).squeeze(-1)
    assert bool((picked >= top2[..., 0] - tie).all())


def test_forced_generate_golden_matches_oracle_steps(golden):
    """The reference ``generate`` golden (teacher-forced, 10 frames) against the oracle
    stepped at positions P, P+1, ...: logits of every head within the parity rule and
    the backbone cache slots P-1 .. P+10 (the last one untouched).  Pins the fixture that
    the GPU ``generate`` test compares with, including its position bookkeeping."""
    from dataclasses import replace
    z = golden("generate")
    sh = replace(TINY_SHAPE, text_vocab=128256)
    tensors = synthetic_tensors(sh, seed=int(z["seed"]), gamma_one=False)
    assert tensors_sha(tensors) == str(z["sha"])
    m = O.OracleModel(tensors, bb_heads=sh.bb_heads, dec_heads=sh.dec_heads, mode="cpu", dtype=torch.float16)
    N, B, P, muq_idx, n_frames = (int(v) for v in z["meta"])
    force = t(z["force"])
    m.alloc(B, P + n_frames + 2 + 256)
    hb = m.prefill(m.prompt_embed(t(z["text"]), N, muq_idx))
    rec = []
    ones = [torch.ones(N, m.vocab)] * m.n_cb
    tok = m.frame(hb[:, -1], N, 1.5, 50, 1.0, force=force[0], record=rec, noise=ones)
    for f in range(n_frames):
        tok = m.step(tok, torch.full((B, 1), P + f, dtype=torch.long), N, 1.5, 50, 1.0, force=force[f + 1],
                     record=rec, noise=ones)
    got, ref = torch.stack(rec).float(), t(z["logits"]).float()
    assert got.shape == ref.shape
    assert (got - ref).abs().max().item() <= 2e-2
    assert_argmax_except_ties(got, ref)
    for j, ly in enumerate((m.bb[0], m.bb[-1])):
        assert ulp_close(ly.kc[:, :, P - 1:P + n_frames + 1], t(z[f"kc{j}"]), 1e-2, 1e-2)
        assert ulp_close(ly.vc[:, :, P - 1:P + n_frames + 1], t(z[f"vc{j}"]), 1e-2, 1e-2)
    assert float(t(z["kc0"])[:, :, -1].abs().sum()) == 0.0     # slot P + n_frames untouched
    assert float(t(z["kc0"])[:, :, 1].abs().sum()) > 0.0       # slot P written by the first step
    # streams: frame 0 .. end, cut at take 0's first EOS frame (4); take 1 runs to the end
    assert t(z["stream0"]).shape == (8, 4) and t(z["stream1"]).shape == (8, n_frames + 1)
    assert torch.equal(t(z["stream1"]), force[:, 1].t())
