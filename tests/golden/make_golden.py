"""Generate golden vectors from the reference implementation itself.

Run where the reference source tree is available (it is not on the GPU box):

    python tests/golden/make_golden.py --ref <path to the reference's app/ dir>

It imports the reference's ``kernels.py`` and ``engine.py`` unmodified and

* runs every Triton kernel of the decode path under ``TRITON_INTERPRET=1``
  (``_gemv8`` through ``.fn`` with fixed tile sizes, because the autotuner
  needs a driver) on seeded inputs -> ``kernels.npz``;
* runs the reference ``_sample`` / ``_guided`` with a seeded torch generator and
  records the exponential noise it drew -> ``sampler.npz``;
* builds a tiny synthetic checkpoint in the reference format, loads it with
  ``HeartMuLaLite(device="cpu", dtype=float16)`` and records, under teacher
  forcing, every codebook head's logits and selected KV-cache slots for the
  prompt prefill plus decode frames, once through the CPU path and once through
  the Triton fast path (interpreter) -> ``model_cpu.npz`` / ``model_fast.npz``.

* runs the checkpoint converter's ``q8_rows`` (``convert_final.py``) on seeded and
  hand-made rows (ties, zero and tiny rows, bf16 / fp16 inputs, an ``audio_head``
  block) -> ``q8_rows.npz``.  It calls ``.cuda()`` on its input; with no GPU in
  the generating container that call is made an identity for the duration, so
  the same fp32 arithmetic runs on the CPU.

The fixtures hold inputs and outputs; the tiny checkpoint is regenerated in the
tests from its seed, and its SHA-256 is stored to catch any drift.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from estudiocanciones_b200.checkpoint import (TINY_SHAPE, synthetic_tensors, save_checkpoint,  # noqa: E402
                                              tensors_sha)

TINY_SEED = 1234


def np16(t):
    return t.detach().cpu().numpy()


# ----------------------------------------------------------------------------- kernels
def gen_kernels(K):
    import triton
    g = torch.Generator().manual_seed(7)
    out = {}
    # int8 GEMV: (M, N, K, residual)
    for i, (M, N, Kd, res) in enumerate([(1, 96, 256, False), (3, 200, 512, True), (8, 128, 1024, True),
                                         (16, 64, 256, False), (5, 8197, 64, False)]):
        x = torch.randn(M, Kd, generator=g).half()
        w = torch.randint(-127, 128, (N, Kd), generator=g, dtype=torch.int8)
        s = (torch.randn(N, generator=g).abs() * 0.02 / 127).half()
        r = torch.randn(M, N, generator=g).half() if res else None
        y = torch.empty(M, N, dtype=torch.float16)
        BN, BK = 32, 128
        K._gemv8.fn[(triton.cdiv(N, BN),)](x, w, s, r if res else y, y, M, N, Kd, MP=16, RES=res, BN=BN, BK=BK)
        out.update({f"gemv{i}_x": np16(x), f"gemv{i}_w": np16(w), f"gemv{i}_s": np16(s), f"gemv{i}_y": np16(y)})
        if res:
            out[f"gemv{i}_r"] = np16(r)
    # RMSNorm
    for i, (R, D) in enumerate([(3, 512), (2, 3072)]):
        x = (torch.randn(R, D, generator=g) * 2).half()
        w = (1 + 0.1 * torch.randn(D, generator=g)).half()
        out.update({f"rms{i}_x": np16(x), f"rms{i}_w": np16(w), f"rms{i}_y": np16(K.rms(x, w))})
    # RoPE + cache write, S=1 and S=2
    from engine import rope_cache
    for i, (R, S, Hq, Hk, L, pos) in enumerate([(4, 1, 4, 2, 32, [3, 0, 17, 31]), (4, 2, 6, 2, 16, [0, 1, 0, 1])]):
        HD = 128
        B = R // S
        qkv = torch.randn(R, (Hq + 2 * Hk) * HD, generator=g).half()
        rope = rope_cache(HD, max(L, 16))
        pos_t = torch.tensor(pos, dtype=torch.long)
        q = torch.empty(R, Hq * HD, dtype=torch.float16)
        kc = torch.randn(B, Hk, L, HD, generator=g).half()
        vc = torch.randn(B, Hk, L, HD, generator=g).half()
        kc0, vc0 = kc.clone(), vc.clone()
        K._rope_cache[(R, Hq + Hk)](qkv, rope, pos_t, q, kc, vc, S, Hq, Hk, L, HD=HD, HALF=64)
        out.update({f"rope{i}_qkv": np16(qkv), f"rope{i}_pos": pos_t.numpy(), f"rope{i}_kc0": np16(kc0),
                    f"rope{i}_vc0": np16(vc0), f"rope{i}_q": np16(q), f"rope{i}_kc": np16(kc),
                    f"rope{i}_vc": np16(vc), f"rope{i}_cfg": np.array([R, S, Hq, Hk, L]),
                    f"rope{i}_table": rope.numpy()})
    # decode attention + combine
    for i, (R, S, Hq, Hk, L, pos, ns) in enumerate([(3, 1, 6, 2, 300, [0, 130, 299], 16),
                                                    (4, 2, 8, 2, 8, [0, 1, 0, 1], 16),
                                                    (2, 1, 4, 1, 64, [5, 63], 1)]):
        HD, G = 128, Hq // Hk
        B = R // S
        q = torch.randn(R, Hq * HD, generator=g).half()
        kc = torch.randn(B, Hk, L, HD, generator=g).half()
        vc = torch.randn(B, Hk, L, HD, generator=g).half()
        pos_t = torch.tensor(pos, dtype=torch.long)
        o = torch.empty(R, Hq * HD, dtype=torch.float16)
        if ns > 1:
            pm = torch.empty(R * Hq * ns)
            pl = torch.empty_like(pm)
            pa = torch.empty(R * Hq * ns, HD)
        else:
            pm = pl = pa = o
        K._attn[(R, Hk, ns)](q, kc, vc, pos_t, o, pm, pl, pa, S, Hq, Hk, L, 1.0 / (HD ** 0.5),
                             HD=HD, HDP=HD, G=G, BLK=64, NSPLIT=ns, num_warps=4)
        if ns > 1:
            K._attn_combine[(R * Hq,)](pm, pl, pa, o, HD=HD, HDP=HD, NSPLIT=ns)
        out.update({f"attn{i}_q": np16(q), f"attn{i}_kc": np16(kc), f"attn{i}_vc": np16(vc),
                    f"attn{i}_pos": pos_t.numpy(), f"attn{i}_o": np16(o),
                    f"attn{i}_cfg": np.array([R, S, Hq, Hk, L, ns])})
    # SiLU * mul
    for i, (R, F_) in enumerate([(3, 300), (2, 8192)]):
        a = (torch.randn(R, 2 * F_, generator=g) * 3).half()
        y = torch.empty(R, F_, dtype=torch.float16)
        K._silu_mul[(R, triton.cdiv(F_, 1024))](a, y, F_, BLOCK=1024)
        out.update({f"silu{i}_a": np16(a), f"silu{i}_y": np16(y)})
    return out


# ----------------------------------------------------------------------------- sampler
def gen_sampler(E):
    out = {}
    g = torch.Generator().manual_seed(11)
    V = 8197
    cases = [(3, 50, 1.0, 1.0), (2, 50, 0.7, 1.0), (4, 5, 1.3, 1.0), (4, 50, 1.0, 1.5), (2, 1, 1.0, 1.5)]
    for i, (rows, topk, temp, cfg) in enumerate(cases):
        logits16 = (torch.randn(rows, V, generator=g) * 3).half()
        if i == 0:     # plant ties at the top-k boundary
            logits16[0, 100:110] = logits16[0].max()
        seed = 100 + i
        if cfg == 1.0:
            torch.manual_seed(seed)
            ids = E.HeartMuLaLite._sample(logits16.float(), topk, temp)
            n_takes = rows
        else:
            n_takes = rows // 2
            obj = E.HeartMuLaLite.__new__(E.HeartMuLaLite)
            obj.N, obj.B = n_takes, rows
            torch.manual_seed(seed)
            ids = obj._guided(logits16, cfg, topk, temp)
        torch.manual_seed(seed)
        noise = torch.empty(n_takes, V).exponential_(1)
        out.update({f"s{i}_logits": np16(logits16), f"s{i}_noise": noise.numpy(), f"s{i}_ids": ids.numpy(),
                    f"s{i}_cfg": np.array([rows, n_takes, topk, temp, cfg], dtype=np.float64)})
    return out


# ----------------------------------------------------------------------------- whole model
class _DimPatch:
    """Give each Stack the width its checkpoint needs (the reference reads the
    module constant DIM at construction, app/engine.py:116,161)."""

    def __init__(self, E, shape):
        self.E, self.shape = E, shape

    def __enter__(self):
        E, sh = self.E, self.shape
        self.saved = (E.DIM, E.BACKBONE, E.DECODER, E.Stack.__init__)
        E.BACKBONE = dict(layers=sh.bb_layers, heads=sh.bb_heads, kv_heads=sh.bb_kv_heads, max_seq=8192)
        E.DECODER = dict(layers=sh.dec_layers, heads=sh.dec_heads, kv_heads=sh.dec_kv_heads, max_seq=2048)
        orig = self.saved[3]

        def init(st, p, prefix, cfg):
            E.DIM = sh.bb_dim if prefix == "backbone" else sh.dec_dim
            orig(st, p, prefix, cfg)
        E.Stack.__init__ = init
        return self

    def __exit__(self, *a):
        E = self.E
        E.DIM, E.BACKBONE, E.DECODER, E.Stack.__init__ = self.saved


def _to_int8_fast(E, m, t):
    """Turn a CPU-loaded model into the int8 fast path with the reference's own
    Linear/fuse classes (what ``HeartMuLaLite.__init__`` builds when CUDA is present)."""
    def lin(k):
        return E.Linear(q8=t[k + ".q8"], s8=t[k + ".s8"].to(torch.float16))

    for pre, st in (("backbone", m.backbone), ("decoder", m.decoder)):
        for i, b in enumerate(st.blocks):
            p = f"{pre}.layers.{i}."
            b.qkv = E.fuse([lin(p + f"attn.{n}_proj.weight") for n in ("q", "k", "v")])
            b.o = lin(p + "attn.output_proj.weight")
            b.w13 = E.fuse([lin(p + "mlp.w1.weight"), lin(p + "mlp.w3.weight")])
            b.w2 = lin(p + "mlp.w2.weight")
    m.projection = lin("projection.weight")
    m.c0_head = lin("codebook0_head.weight")
    m.audio_head = [lin(f"audio_head.{i}") for i in range(len(m.audio_head))]
    m.fast = True


def _interp_int8_mm(K):
    import triton
    orig = K.int8_mm

    def int8_mm(x, w, s, res=None):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).contiguous()
        M, Kd = x2.shape
        if M > 16:
            return orig(x, w, s, res)
        N = w.shape[0]
        y = torch.empty(M, N, dtype=x.dtype)
        r = res.reshape(M, N).contiguous() if res is not None else y
        K._gemv8.fn[(triton.cdiv(N, 64),)](x2, w, s, r, y, M, N, Kd, MP=16, RES=res is not None, BN=64, BK=128)
        return y.reshape(*shp[:-1], N)
    return int8_mm


def gen_model(E, K, fast: bool, n_frames: int = 1):
    sh = TINY_SHAPE
    t = synthetic_tensors(sh, seed=TINY_SEED, gamma_one=False)
    sha = tensors_sha(t)
    path = Path("/tmp/heartmula_tiny.safetensors")
    save_checkpoint(t, path)
    with _DimPatch(E, sh):
        m = E.HeartMuLaLite(path, device="cpu", dtype=torch.float16)
    if fast:
        _to_int8_fast(E, m, t)
        K.int8_mm = _interp_int8_mm(K)
    N, B, P, muq_idx, cfg, topk, temp = 2, 4, 12, 4, 1.5, 50, 1.0
    g = torch.Generator().manual_seed(5)
    text = torch.randint(0, sh.text_vocab, (P,), generator=g)
    force = torch.randint(0, 8192, (n_frames + 1, B // 2, sh.n_cb), generator=g)
    force = torch.cat([force, force], 1)       # both CFG halves carry the same ids
    rec = []
    fidx = [0]

    def guided(self, logits, cfg_, topk_, temp_):
        rec.append(logits.clone())
        i = len(rec) - 1
        f, c = divmod(i, sh.n_cb)
        return force[f, :, c:c + 1].clone()

    E.HeartMuLaLite._guided = guided
    m.N, m.B = N, B
    L = P + n_frames + 2
    m._ar = torch.arange(L + 256)
    m.backbone.alloc(B, L + 256, m.dev, m.dt)
    m.decoder.alloc(B, sh.n_cb, m.dev, m.dt)
    te = m.text_emb(text)
    h = te.unsqueeze(0).repeat(B, 1, 1)
    h[:N, muq_idx] = m.muq_b
    h[N:] = m.uncond[0]
    pos = torch.arange(P).unsqueeze(0).expand(B, P)
    hb = m.backbone(h, pos, P, None)
    tok = m._frame_from_h(hb[:, -1], cfg, topk, temp)
    assert torch.equal(tok, force[0])
    kv_pre = [(b.kc[:, :, :P].clone(), b.vc[:, :, :P].clone()) for b in (m.backbone.blocks[0], m.backbone.blocks[-1])]
    for f in range(n_frames):
        p_t = torch.full((B, 1), P + f, dtype=torch.long)
        tok = m._step(tok, p_t, L + 256, cfg, topk, temp)
        assert torch.equal(tok, force[f + 1])
    out = {"sha": np.array(sha), "seed": np.array(TINY_SEED), "text": text.numpy(), "force": force.numpy(),
           "meta": np.array([N, B, P, muq_idx, n_frames]), "cfg": np.array([cfg, topk, temp]),
           "logits": np.stack([np16(x) for x in rec]), "hb_last": np16(hb[:, -1])}
    for j, (kk, vv) in enumerate(kv_pre):
        out[f"kc_pre{j}"], out[f"vc_pre{j}"] = np16(kk[:, :, -3:]), np16(vv[:, :, -3:])
    for j, b in enumerate((m.backbone.blocks[0], m.backbone.blocks[-1])):
        out[f"kc_dec{j}"] = np16(b.kc[:, :, P:P + n_frames])
        out[f"vc_dec{j}"] = np16(b.vc[:, :, P:P + n_frames])
    del fidx
    return out


# ----------------------------------------------------------------------------- generate
GEN_LYRICS = "La luna canta sobre el mar\nY el viento baila sin parar"
GEN_TAGS = "Pop, Acoustic, Female vocal"


def gen_generate(E, n_frames: int = 10):
    """The reference's own ``generate`` (``app/engine.py:374-448``, CPU path, fp16) on a
    tiny checkpoint with the real text vocabulary, 2 takes x CFG, with every sampled id
    replaced by a fixed table (teacher forcing through ``_guided``).  Take 0 emits an EOS
    id at frame 4, so its stream is cut there by the reference's EOS scan; take 1 runs to
    the end.  Records the prompt ids, the returned streams, every head's logits in call
    order, and the backbone cache slots around the prompt end (captured when ``generate``
    releases its buffers)."""
    from dataclasses import replace
    from wordtok import WordTokenizer
    sh = replace(TINY_SHAPE, text_vocab=128256)
    t = synthetic_tensors(sh, seed=TINY_SEED + 1, gamma_one=False)
    sha = tensors_sha(t)
    path = Path("/tmp/heartmula_tiny_gen.safetensors")
    save_checkpoint(t, path)
    with _DimPatch(E, sh):
        m = E.HeartMuLaLite(path, device="cpu", dtype=torch.float16)
    N, B = 2, 4
    g = torch.Generator().manual_seed(21)
    force = torch.randint(0, 8192, (n_frames + 1, N, sh.n_cb), generator=g)
    force[4, 0, 3] = E.AUDIO_EOS          # take 0 ends at frame 4
    force[7, 0, 5] = E.AUDIO_EOS + 2      # a later EOS-range id does not move the end
    force = torch.cat([force, force], 1)  # both CFG halves carry the same ids
    rec = []

    def guided(self, logits, cfg_, topk_, temp_):
        rec.append(logits.clone())
        f, c = divmod(len(rec) - 1, sh.n_cb)
        return force[f, :, c:c + 1].clone()

    kv = {}
    release0 = m.release

    def release():
        for j, b in enumerate((m.backbone.blocks[0], m.backbone.blocks[-1])):
            kv[f"kc{j}"] = np16(b.kc[:, :, P - 1:P + n_frames + 1])
            kv[f"vc{j}"] = np16(b.vc[:, :, P - 1:P + n_frames + 1])
        release0()

    text, muq_idx = m._prompt(GEN_LYRICS, GEN_TAGS, WordTokenizer())
    P = len(text)
    guided0 = E.HeartMuLaLite._guided
    E.HeartMuLaLite._guided = guided
    m.release = release
    try:
        res = m.generate(GEN_LYRICS, GEN_TAGS, WordTokenizer(), max_ms=n_frames * 80, cfg_scale=1.5, topk=50,
                         temperature=1.0, seed=3, n=N)
    finally:
        E.HeartMuLaLite._guided = guided0
    out = {"sha": np.array(sha), "seed": np.array(TINY_SEED + 1), "text": text.numpy(),
           "meta": np.array([N, B, P, muq_idx, n_frames]), "force": force.numpy(),
           "logits": np.stack([np16(x) for x in rec]), "lyrics": np.array(GEN_LYRICS), "tags": np.array(GEN_TAGS)}
    for c, r in enumerate(res):
        out[f"stream{c}"] = r.numpy()
    out.update(kv)
    return out


# ----------------------------------------------------------------------------- converter
def q8_cases():
    """Inputs of the q8_rows fixture: name -> 2-D tensor."""
    g = torch.Generator().manual_seed(11)
    ties = torch.tensor([[127.0, 2.5, -3.5, 0.5, -0.5, 1.5, 126.5, -127.0, 0.0, -1.5, 3.5, 64.5]])
    tiny = torch.tensor([[1e-9, -3e-9, 5e-10, 0.0], [0.0, 0.0, 0.0, 0.0]])
    mixed = torch.randn(6, 37, generator=g)
    mixed[2] = 0.0
    mixed[4] *= 1e4
    return {
        "f32_ties": ties,
        "f32_tiny_zero": tiny,
        "f32_mixed": mixed,
        "f32_wide": torch.randn(3, 3072, generator=g) * 0.05,
        "bf16": (torch.randn(5, 64, generator=g) * 3).to(torch.bfloat16),
        "f16": (torch.randn(2, 48, generator=g) * 0.1).to(torch.float16),
        "audio_head": torch.randn(2, 16, 24, generator=g),  # [heads, D, V], quantised per head as [V, D]
    }


def gen_q8(C):
    cuda0 = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self  # no GPU here: the same fp32 arithmetic on the CPU
    try:
        out = {}
        for name, t in q8_cases().items():
            out[f"{name}.x"] = t.float().numpy()
            out[f"{name}.dtype"] = np.array(str(t.dtype))
            mats = [t[i].t().contiguous() for i in range(t.shape[0])] if name == "audio_head" else [t]
            for j, m in enumerate(mats):
                q, s = C.q8_rows(m)
                out[f"{name}.{j}.q"] = q.numpy()
                out[f"{name}.{j}.s"] = s.view(torch.int16).numpy()  # bf16 bits
        return out
    finally:
        torch.Tensor.cuda = cuda0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HEARTMULA_REF_APP", ""), help="reference app/ directory")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", default="", help="'q8' / 'generate': write q8_rows.npz / generate.npz only")
    a = ap.parse_args()
    if not a.ref or not Path(a.ref, "engine.py").exists():
        raise SystemExit("pass --ref <reference app dir>")
    sys.path.insert(0, a.ref)
    import convert_final as C
    np.savez_compressed(Path(a.out, "q8_rows.npz"), **gen_q8(C))
    if a.only == "q8":
        return
    import kernels as K
    import engine as E
    sys.path.insert(0, str(HERE))
    if a.only == "generate":
        np.savez_compressed(Path(a.out, "generate.npz"), **gen_generate(E))
        return
    torch.set_num_threads(8)
    np.savez_compressed(Path(a.out, "kernels.npz"), **gen_kernels(K))
    np.savez_compressed(Path(a.out, "sampler.npz"), **gen_sampler(E))
    guided0 = E.HeartMuLaLite._guided
    np.savez_compressed(Path(a.out, "model_cpu.npz"), **gen_model(E, K, fast=False, n_frames=1))
    E.HeartMuLaLite._guided = guided0
    np.savez_compressed(Path(a.out, "model_fast.npz"), **gen_model(E, K, fast=True, n_frames=1))
    np.savez_compressed(Path(a.out, "generate.npz"), **gen_generate(E))
    for f in sorted(Path(a.out).glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
