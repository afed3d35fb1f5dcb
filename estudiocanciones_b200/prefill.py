"""Prompt prefill of the backbone: fills the static KV cache for positions [0, P).

The reference runs the prompt through ``Stack.__call__`` (``app/engine.py:174-178,
390-398``): dequantised fp16 GEMMs, torch RMSNorm/RoPE, ``index_copy_`` into the
cache and causal SDPA.  Here every row of every prompt position goes through
the same sm_100a decode launches (fused RMSNorm/RoPE/KV-write GEMVs and decode
attention over ``[0, p]``, which is causal attention), one position per replay
of a captured backbone-step graph.  The unnormalised hidden state of the last
position is left in the runtime's residual buffer for the first frame.
"""
from __future__ import annotations

import torch

from ._lib import HMError


@torch.inference_mode()
def prefill_backbone(model, h: torch.Tensor) -> None:
    """h ``[B, P, D]`` fp16 prompt embeddings on the device."""
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
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            rt.x_bb.copy_(x_in)
            rt.ss_bb.copy_((x_in.float() ** 2).reshape(B, D // SS_COLS, SS_COLS).sum(-1).t())
            plan.run()
    torch.cuda.current_stream().wait_stream(s)
    for p in range(1, P):
        x_in.copy_(h[:, p])
        rt.pos.fill_(p)
        g.replay()
    del g
