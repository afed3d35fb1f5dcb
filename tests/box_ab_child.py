"""Child process of tests/test_box_layout_gpu.py: runs a fixed set of seeded GEMV,
attention and whole-frame launches and saves every output to the file named by argv[1].

The weight and K/V requests of the kernels come in two forms that fill shared memory
identically (one 3-D / 4-D box per stage or several 2-D boxes: HM_GEMV_BOX, HM_ATTN_BOX).
Each form is chosen once per process, so the test runs this script once per form and
compares the saved outputs bit for bit."""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from estudiocanciones_b200 import _lib, kernels  # noqa: E402
from estudiocanciones_b200._lib import HM_EPI_SILU  # noqa: E402
from estudiocanciones_b200.checkpoint import TINY_SHAPE, synthetic_tensors  # noqa: E402
from estudiocanciones_b200.engine import FramePlan, HeartMuLaLite, Linear, _Ctx  # noqa: E402

DEV = "cuda"


def lin(N, K, gen):
    w = torch.randint(-127, 128, (N, K), generator=gen, dtype=torch.int8)
    s = (torch.randn(N, generator=gen).abs() * 0.02 / 127).half()
    return w.to(DEV), s.to(DEV)


def ss_of(x):
    R, D = x.shape
    return (x.float() ** 2).reshape(R, D // 16, 16).sum(-1).t().contiguous()


def main(out_path):
    out = {}
    forms = []  # the request form each launch used (1: one box per stage / tile)
    gen = torch.Generator().manual_seed(2024)
    # store epilogue: narrow and wide kernels, a split K range, rows past N (c0 head), K of one chunk
    for M, N, K, kspan, res in [(8, 5120, 3072, 0, False), (8, 3072, 8192, 1024, True), (16, 8197, 3072, 0, False),
                                (1, 64, 128, 0, False), (8, 1024, 8192, 0, True), (3, 200, 640, 0, True),
                                (8, 8197, 1024, 0, False)]:
        x = torch.randn(M, K, generator=gen).half().to(DEV)
        w, s = lin(N, K, gen)
        r = torch.randn(M, N, generator=gen).half().to(DEV) if res else None
        out[f"store_{M}_{N}_{K}_{kspan}"] = kernels.int8_mm(x, w, s, r, kspan=kspan).cpu()
        forms.append(_lib.lib().hm_gemv_box_form(w.data_ptr(), N, K, 0))
    # RMSNorm prologue + SiLU epilogue (the 4-D w1|w3 box): backbone and decoder widths, 8 and 16 rows
    for M, D, F in [(8, 3072, 8192), (16, 3072, 8192), (8, 1024, 8192), (5, 512, 1024)]:
        x = torch.randn(M, D, generator=gen).half().to(DEV)
        gamma = (1 + 0.1 * torch.randn(D, generator=gen)).half().to(DEV)
        w, s = lin(2 * F, D, gen)
        y = torch.empty(M, F, dtype=torch.float16, device=DEV)
        p = FramePlan(_Ctx(DEV, 64 << 20, 1 << 20), pdl=False)
        p._gemv(Linear(w, s), M, p.src_rms(x, ss_of(x), gamma), epi=HM_EPI_SILU, y=y)
        p.run()
        out[f"silu_{M}_{D}_{F}"] = y.cpu()
        forms.append(_lib.lib().hm_gemv_box_form(w.data_ptr(), 2 * F, D, HM_EPI_SILU))
    # decode attention (tensor-core kernel), cluster-merged and workspace-merged splits
    for R, Hq, Hk, L, pos, ns in [(8, 24, 8, 1350, [0, 1, 63, 64, 600, 975, 1348, 1349], 4),
                                  (8, 24, 8, 1350, [0, 2, 65, 127, 512, 974, 1200, 1349], 8),
                                  (2, 24, 8, 4282, [4281, 4023], 16), (4, 8, 2, 64, [15, 16, 17, 63], 1)]:
        q = torch.randn(R, Hq * 128, generator=gen).half().to(DEV)
        kc = torch.randn(R, Hk, L, 128, generator=gen).half().to(DEV)
        vc = torch.randn(R, Hk, L, 128, generator=gen).half().to(DEV)
        o = torch.empty(R, Hq * 128, dtype=torch.float16, device=DEV)
        kernels.attn(q, kc, vc, torch.tensor(pos, device=DEV), o, 1, Hq, Hk, L, nsplit=ns)
        out[f"attn_{R}_{L}_{ns}"] = o.cpu()
        forms.append(_lib.lib().hm_decode_attn_box_form(kc.data_ptr(), R * Hk * L))
    # a whole teacher-forced frame (every epilogue, RoPE / KV write included) at the tiny shape
    sh = TINY_SHAPE
    t = synthetic_tensors(sh, seed=77, gamma_one=False)
    m = HeartMuLaLite(t, device=DEV, bb_heads=sh.bb_heads, dec_heads=sh.dec_heads)
    N, B, P = 2, 4, 12
    text = torch.randint(0, sh.text_vocab, (P,), generator=gen)
    force = torch.randint(0, 8192, (2, N, sh.n_cb), generator=gen).repeat(1, 2, 1)
    m.prefill_ids(text, 4, N, B, P + 3 + 256)
    out["frame0"] = m.teacher_frame(force[0].to(DEV), with_backbone=False).cpu()
    out["frame1"] = m.teacher_frame(force[1].to(DEV), with_backbone=True, tok=force[0].to(DEV),
                                    pos=torch.full((B,), P, dtype=torch.long, device=DEV)).cpu()
    out["kc0"] = m.backbone.blocks[0].kc.cpu()
    out["errors"] = torch.tensor(kernels.read_errors(DEV))
    out["forms"] = torch.tensor(forms)
    torch.save(out, out_path)


if __name__ == "__main__":
    main(sys.argv[1])
