"""The decode entry points as ``torch.library`` custom operators (namespace ``heartmula_b200``).

Each operator calls the same C-ABI launch as the function of the same name in
:mod:`estudiocanciones_b200.kernels` (the drop-in for ``app/kernels.py``), on the current
CUDA stream, so ``torch.cuda.graph`` captures it.  Registering them lets torch tooling
see the kernels as opaque operators with known output shapes (a fake implementation
per operator) and known in-place arguments (``mutates_args``), instead of untraceable
ctypes calls:

* ``int8_mm(x, w, s, res)`` -> ``[..., N]``       (``app/kernels.py:40-54``)
* ``rms(x, w, eps)`` -> ``[R, D]``                  (``app/kernels.py:70-74``)
* ``rope_cache(qkv, rope, pos, q_out, kc, vc, S, Hq, Hk, L)``, writes q_out / kc / vc
                                                    (``app/kernels.py:79-107``)
* ``attn(q, kc, vc, pos, o, S, Hq, Hk, L, scale, nsplit)``, writes o
                                                    (``app/kernels.py:112-167``)
* ``silu_mul(a)`` -> ``[R, F]``                     (``app/kernels.py:172-180``)
* ``gemm_i8w(a, w, s, res, silu)`` -> ``[M, N or N/2]`` (the ``M > 16`` branch of ``int8_mm``)
* ``prefill_attn(q, kc, vc, P)`` -> like ``q``      (``Block.__call__`` causal attention)

Importing this module registers them; nothing is loaded onto a GPU until an operator runs.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import kernels

NS = "heartmula_b200"


@torch.library.custom_op(f"{NS}::int8_mm", mutates_args=())
def int8_mm(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, res: Optional[torch.Tensor] = None) -> torch.Tensor:
    return kernels.int8_mm(x, w, s, res)


@int8_mm.register_fake
def _(x, w, s, res=None):
    return x.new_empty(*x.shape[:-1], w.shape[0])


@torch.library.custom_op(f"{NS}::rms", mutates_args=())
def rms(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    return kernels.rms(x, w, eps)


@rms.register_fake
def _(x, w, eps=1e-5):
    return torch.empty_like(x)


@torch.library.custom_op(f"{NS}::rope_cache", mutates_args=("q_out", "kc", "vc"))
def rope_cache(qkv: torch.Tensor, rope: torch.Tensor, pos: torch.Tensor, q_out: torch.Tensor, kc: torch.Tensor,
               vc: torch.Tensor, S: int, Hq: int, Hk: int, L: int) -> None:
    kernels.rope_cache(qkv, rope, pos, q_out, kc, vc, S, Hq, Hk, L)


@rope_cache.register_fake
def _(qkv, rope, pos, q_out, kc, vc, S, Hq, Hk, L):
    return None


@torch.library.custom_op(f"{NS}::attn", mutates_args=("o",))
def attn(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, pos: torch.Tensor, o: torch.Tensor, S: int, Hq: int,
         Hk: int, L: int, scale: float, nsplit: int = 16) -> None:
    kernels.attn(q, kc, vc, pos, o, S, Hq, Hk, L, scale, nsplit=nsplit)


@attn.register_fake
def _(q, kc, vc, pos, o, S, Hq, Hk, L, scale, nsplit=16):
    return None


@torch.library.custom_op(f"{NS}::silu_mul", mutates_args=())
def silu_mul(a: torch.Tensor) -> torch.Tensor:
    return kernels.silu_mul(a)


@silu_mul.register_fake
def _(a):
    return a.new_empty(a.shape[0], a.shape[1] // 2)


@torch.library.custom_op(f"{NS}::gemm_i8w", mutates_args=())
def gemm_i8w(a: torch.Tensor, w: torch.Tensor, s: torch.Tensor, res: Optional[torch.Tensor] = None,
             silu: bool = False) -> torch.Tensor:
    return kernels.gemm_i8w(a, w, s, res=res, silu=silu)


@gemm_i8w.register_fake
def _(a, w, s, res=None, silu=False):
    return a.new_empty(a.shape[0], w.shape[0] // 2 if silu else w.shape[0])


@torch.library.custom_op(f"{NS}::prefill_attn", mutates_args=())
def prefill_attn(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, P: int) -> torch.Tensor:
    return kernels.prefill_attn(q, kc, vc, P)


@prefill_attn.register_fake
def _(q, kc, vc, P):
    return torch.empty_like(q)
