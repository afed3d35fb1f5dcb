"""Prompt prefill of the backbone: fills the static KV cache for positions [0, P).

The reference runs the prompt through ``Stack.__call__`` (``app/engine.py:174-178,
390-398``): per layer an RMSNorm, the dequantised fp16 GEMMs of ``int8_mm``'s
M > 16 branch (``app/kernels.py:46-49``), RoPE, ``index_copy_`` into the cache,
causal SDPA over ``repeat_interleave``d K/V, SiLU·mul and the residual adds.

Here the B*P prompt rows go through, per layer:

* ``hm_rmsnorm``                     RMSNorm of the residual stream
* ``hm_gemm_i8w``                    q|k|v projection (tcgen05 tensor cores, int8 weights)
* ``hm_rope_kv_write``               RoPE of q and k; k, v written into the cache slots
* ``hm_prefill_attn``                causal GQA attention, K/V shared by each head group
* ``hm_gemm_i8w`` (+ residual)       output projection, added in place
* ``hm_rmsnorm``, ``hm_gemm_i8w`` SiLU epilogue (w1|w3 fused, SiLU·mul in the epilogue),
  ``hm_gemm_i8w`` (+ residual)       the MLP

The unnormalised hidden state of the last position of every row is left in the
runtime's residual buffer (with its sums of squares) for the first frame.
``prefill_backbone_steps`` is the position-by-position alternative through the
decode launches (used by the tests as a second GPU path).
"""
from __future__ import annotations

import torch

from . import kernels
from ._lib import HMError, capture_graph


def _rows_to_runtime(rt, x_last: torch.Tensor) -> None:
    from .engine import SS_COLS
    B, D = x_last.shape
    rt.x_bb.copy_(x_last)
    rt.ss_bb.copy_((x_last.float() ** 2).reshape(B, D // SS_COLS, SS_COLS).sum(-1).t())


@torch.inference_mode()
def prefill_backbone(model, h: torch.Tensor, keep_f16: bool = True) -> None:
    """h ``[B, P, D]`` fp16 prompt embeddings on the device.

    keep_f16: the GEMMs read fp16 weight tiles (the exact int8 values); with True each
    backbone matrix is converted once and the copy kept for later prompts (2 bytes per
    weight: 5.6 GB at the 3B shape, ``model.drop_prefill_weights()`` frees them), with False
    every prompt converts each matrix again into one scratch buffer."""
    rt = model._rt
    if rt is None:
        raise HMError("alloc() first")
    B, P, D = h.shape
    stack = model.backbone
    L = stack.L
    if P > L:
        raise HMError(f"prompt of {P} positions does not fit the {L}-slot cache")
    dev = h.device
    M = B * P
    x = h.reshape(M, D).contiguous().clone()
    pos = torch.arange(P, device=dev, dtype=torch.long).repeat(B)
    b0 = stack.blocks[0]
    q = torch.empty(M, b0.h * b0.hd, device=dev, dtype=torch.float16)
    # each weight in fp16 (exact int8 values) so the GEMMs read their tiles as they are: kept
    # per matrix, or converted for this prompt into one scratch reused by every matrix
    wbuf = None if keep_f16 else torch.empty(max(lin.q8.numel() for lin in (b0.qkv, b0.o, b0.w13, b0.w2)),
                                             device=dev, dtype=torch.float16)

    def gemm(a, lin, **kw):
        if keep_f16:
            if lin.f16 is None:
                lin.f16 = kernels.dequant_i8(lin.q8)
            wh = lin.f16
        else:
            wh = kernels.dequant_i8(lin.q8, wbuf[:lin.q8.numel()].view(lin.q8.shape))
        return kernels.gemm_f16w(a, wh, lin.s8, **kw)

    for blk in stack.blocks:
        hn = kernels.rms(x, blk.n1)
        qkv = gemm(hn, blk.qkv)
        kernels.rope_cache(qkv, stack.rope, pos, q, blk.kc, blk.vc, P, blk.h, blk.kvh, L)
        o = kernels.prefill_attn(q, blk.kc, blk.vc, P)
        gemm(o, blk.o, res=x, out=x)
        hn = kernels.rms(x, blk.n2)
        mm = gemm(hn, blk.w13, silu=True)
        gemm(mm, blk.w2, res=x, out=x)
    _rows_to_runtime(rt, x.reshape(B, P, D)[:, P - 1])


@torch.inference_mode()
def prefill_backbone_steps(model, h: torch.Tensor) -> None:
    """The same through the decode launches: one position per replay of a captured
    backbone-step graph (fused RMSNorm/RoPE/KV-write GEMVs, decode attention over
    ``[0, p]``, which is causal attention)."""
    rt = model._rt
    if rt is None:
        raise HMError("alloc() first")
    B, P, D = h.shape
    from .engine import SS_COLS, FramePlan
    plan = rt.plans.get("prefill_step")
    if plan is None:
        plan = FramePlan(rt.ctx)
        plan.stack(model.backbone, rt.bb, rt.pos, 1, B, rt.nsplit)
        rt.plans["prefill_step"] = plan
    x_in = torch.empty(B, D, device=h.device, dtype=torch.float16)

    def load(p):
        x_in.copy_(h[:, p])
        rt.x_bb.copy_(x_in)
        rt.ss_bb.copy_((x_in.float() ** 2).reshape(B, D // SS_COLS, SS_COLS).sum(-1).t())
        rt.pos.fill_(p)

    if P <= 2:
        for p in range(P):
            load(p)
            plan.run()
        return
    # eager first position (sets kernel attributes), then a captured step graph
    load(0)
    plan.run()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=h.device)
    s.wait_stream(torch.cuda.current_stream())
    with capture_graph(g, s):
        rt.x_bb.copy_(x_in)
        rt.ss_bb.copy_((x_in.float() ** 2).reshape(B, D // SS_COLS, SS_COLS).sum(-1).t())
        plan.run()
    torch.cuda.current_stream().wait_stream(s)
    for p in range(1, P):
        x_in.copy_(h[:, p])
        rt.pos.fill_(p)
        g.replay()
    del g
