"""Drop-in counterparts of the reference's decode kernels (``app/kernels.py``).

Same names, argument meaning and return conventions as the reference module,
backed by the sm_100a library through its C ABI:

=====================  ==========================================  ==============================
here                   reference                                   C entry point
=====================  ==========================================  ==============================
``int8_mm``            ``int8_mm`` (``app/kernels.py:40-54``)       ``hm_gemv_i8``
``rms``                ``rms`` / ``_rms`` (``:58-74``)              ``hm_rmsnorm``
``rope_cache``         ``_rope_cache`` launch (``:79-107``)         ``hm_rope_kv_write``
``attn``               ``_attn`` + ``_attn_combine`` (``:112-167``) ``hm_decode_attn``
``silu_mul``           ``_silu_mul`` launch (``:172-180``)          ``hm_silu_mul``
``gemm_i8w``           ``int8_mm`` for M > 16 (``:46-49``)           ``hm_gemm_i8w`` (tcgen05)
``prefill_attn``       causal SDPA of ``Block.__call__``            ``hm_prefill_attn``
                       (``app/engine.py:123-153``)
``_rope_cache``        ``_rope_cache[grid](...)`` (``:79-107``)      ``hm_rope_kv_write``
``_attn``              ``_attn[grid](...)`` (``:112-153``)           ``hm_decode_attn`` (merged)
``_attn_combine``      ``_attn_combine[grid](...)`` (``:157-167``)   nothing (``_attn`` merged)
``_silu_mul``          ``_silu_mul[grid](...)`` (``:172-180``)       ``hm_silu_mul``
=====================  ==========================================  ==============================

The four underscore names take the reference's own launch syntax, ``kernel[grid](*args,
**constexprs)`` as ``Stack.decode`` writes it (``app/engine.py:184-210``), so that loop
runs unchanged on top of this module: the grid and the Triton meta-parameters (``HD``,
``HALF``, ``HDP``, ``G``, ``BLK``, ``NSPLIT``, ``BLOCK``, ``num_warps``) are accepted and
not needed, because each C entry point sizes its own launch.  ``_attn`` writes the
merged output into ``o`` itself (its split count is chosen for this GPU), so the
reference's following ``_attn_combine`` launch has nothing left to do and returns.

Launches go to the current torch CUDA stream, so everything here can be
captured in a CUDA graph.  Scratch memory comes from the torch allocator (the
graph pool during capture), as in the reference; the split-K tickets live in
one zeroed int32 buffer per device that every launch leaves zeroed.
There is no CPU fallback: non-CUDA tensors raise.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import HMError, check

_TICKETS: dict[int, torch.Tensor] = {}
_ERRS: dict[int, torch.Tensor] = {}
N_TICKETS = 1 << 16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda):
            raise HMError("estudiocanciones_b200 kernels need CUDA tensors (there is no CPU path)")


def tickets(device) -> torch.Tensor:
    """The per-device zeroed ticket buffer (allocated once, outside any capture)."""
    idx = torch.device(device).index or 0
    t = _TICKETS.get(idx)
    if t is None:
        if torch.cuda.is_current_stream_capturing():
            raise HMError("first kernel call on a device happened inside graph capture; warm up first")
        t = torch.zeros(N_TICKETS, dtype=torch.int32, device=device)
        _TICKETS[idx] = t
    return t


def error_word(device) -> torch.Tensor:
    """Device int that kernels OR HM_ERR_* bits into (bounded waits, bad indices)."""
    idx = torch.device(device).index or 0
    t = _ERRS.get(idx)
    if t is None:
        if torch.cuda.is_current_stream_capturing():
            raise HMError("first kernel call on a device happened inside graph capture; warm up first")
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERRS[idx] = t
    return t


def read_errors(device, clear: bool = True) -> int:
    """Synchronising read of the device error word."""
    e = error_word(device)
    v = int(e.item())
    if clear and v:
        with torch.inference_mode():   # the word may have been created under inference mode
            e.zero_()
    return v


def int8_mm(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, res: torch.Tensor | None = None,
            *, kspan: int = 0, pdl: bool = False) -> torch.Tensor:
    """x [..., K] fp16, w [N, K] int8, s [N] fp16 -> [..., N] (+ res), for up to 32 rows."""
    _need_cuda(x, w, s, res)
    shp = x.shape
    x2 = x.reshape(-1, shp[-1]).contiguous()
    M, K = x2.shape
    N = w.shape[0]
    if M > 32:
        raise HMError("int8_mm decodes at most 32 rows; prompts go through the prefill kernels")
    y = torch.empty(M, N, device=x.device, dtype=torch.float16)
    r = res.reshape(M, N).contiguous() if res is not None else None
    L = _lib.lib()
    wsb = L.hm_gemv_workspace_bytes(M, N, K, _lib.HM_EPI_STORE, kspan)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x.device)
    tk = tickets(x.device)
    check(L.hm_gemv_i8(x2.data_ptr(), K, w.data_ptr(), s.data_ptr(), r.data_ptr() if r is not None else None, N,
                       y.data_ptr(), N, M, N, K, ws.data_ptr(), wsb, tk.data_ptr(), tk.numel(),
                       error_word(x.device).data_ptr(), kspan, int(pdl), _stream()), "hm_gemv_i8")
    return y.reshape(*shp[:-1], N)


def rms(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    _need_cuda(x, w)
    R, D = x.shape
    y = torch.empty_like(x)
    check(_lib.lib().hm_rmsnorm(x.data_ptr(), w.data_ptr(), y.data_ptr(), R, D, eps, _stream()), "hm_rmsnorm")
    return y


def rope_cache(qkv, rope, pos, q_out, kc, vc, S, Hq, Hk, L):
    """RoPE q/k of every row at ``pos[r]`` and write k, v into ``kc/vc[r // S, :, pos[r]]``."""
    _need_cuda(qkv, rope, pos, q_out, kc, vc)
    R = qkv.shape[0]
    hd = kc.shape[-1]
    check(_lib.lib().hm_rope_kv_write(qkv.data_ptr(), rope.data_ptr(), rope.shape[0], pos.data_ptr(),
                                      q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), R, S, Hq, Hk, hd, L,
                                      error_word(qkv.device).data_ptr(), _stream()), "hm_rope_kv_write")


def attn(q, kc, vc, pos, o, S, Hq, Hk, L, scale=None, nsplit: int = 16, pdl: bool = False):
    """Decode attention of every row over ``[0, pos[r]]`` of its cache; writes ``o`` in place."""
    _need_cuda(q, kc, vc, pos, o)
    R = q.shape[0]
    hd = kc.shape[-1]
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    Lb = _lib.lib()
    wsb = Lb.hm_decode_attn_workspace_bytes(R, Hq, hd, nsplit)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    tk = tickets(q.device)
    check(Lb.hm_decode_attn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), o.data_ptr(), R, S, Hq, Hk,
                            hd, L, scale, nsplit, ws.data_ptr(), wsb, tk.data_ptr(), tk.numel(),
                            error_word(q.device).data_ptr(), int(pdl), _stream()), "hm_decode_attn")


def silu_mul(a: torch.Tensor) -> torch.Tensor:
    _need_cuda(a)
    R, F2 = a.shape
    y = torch.empty(R, F2 // 2, device=a.device, dtype=a.dtype)
    return silu_mul_into(a, y)


def silu_mul_into(a: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """``y[r, j] = fp16(silu(a[r, j])) * a[r, F + j]`` into a caller's ``[R, F]`` tensor."""
    _need_cuda(a, y)
    R, F2 = a.shape
    if y.shape != (R, F2 // 2) or not a.is_contiguous() or not y.is_contiguous():
        raise HMError("silu_mul: a [R, 2F] and y [R, F], both contiguous")
    check(_lib.lib().hm_silu_mul(a.data_ptr(), y.data_ptr(), R, F2 // 2, _stream()), "hm_silu_mul")
    return y


def emb_i8(idx: torch.Tensor, q8: torch.Tensor, s8: torch.Tensor) -> torch.Tensor:
    """``Emb.__call__`` int8 branch: ``fp16(q8[idx]) * s8[idx]`` -> ``[*idx.shape, D]``."""
    _need_cuda(idx, q8, s8)
    flat = idx.reshape(-1).contiguous().long()
    D = q8.shape[1]
    out = torch.empty(flat.numel(), D, device=q8.device, dtype=torch.float16)
    check(_lib.lib().hm_emb_gather_i8(flat.data_ptr(), flat.numel(), q8.data_ptr(), s8.data_ptr(), q8.shape[0], D,
                                      out.data_ptr(), error_word(q8.device).data_ptr(), _stream()),
          "hm_emb_gather_i8")
    return out.reshape(*idx.shape, D)


def sample(logits: torch.Tensor, n_takes: int, cfg: float, topk: int, temp: float, noise: torch.Tensor,
           out: torch.Tensor, col: int, pdl: bool = False) -> None:
    """``_guided`` + ``_sample`` with the exponential noise given: writes the id of
    take n into ``out[n, col]`` (and ``out[n + N, col]`` when rows are CFG pairs)."""
    _need_cuda(logits, noise, out)
    B, V = logits.shape
    check(_lib.lib().hm_cfg_topk_sample(logits.data_ptr(), logits.stride(0), B, n_takes, V, noise.data_ptr(),
                                        noise.stride(0), cfg, topk, temp, out.data_ptr(), out.stride(0), col,
                                        error_word(logits.device).data_ptr(), int(pdl), _stream()),
          "hm_cfg_topk_sample")


def gemm_i8w(a: torch.Tensor, w: torch.Tensor, s: torch.Tensor, res: torch.Tensor | None = None,
             out: torch.Tensor | None = None, silu: bool = False) -> torch.Tensor:
    """Prompt-sized ``int8_mm``: a ``[M, K]`` fp16 times int8 ``w [N, K]`` with per-row
    scales, on the tensor cores.  ``silu``: ``w`` is the fused w1|w3 (N = 2F) and the
    result is ``fp16(silu(a1)) * a3`` ``[M, F]``.  ``res`` may be ``out`` (in-place add)."""
    _need_cuda(a, w, s, res, out)
    M, K = a.shape
    N = w.shape[0]
    nout = N // 2 if silu else N
    if out is None:
        out = torch.empty(M, nout, device=a.device, dtype=torch.float16)
    check(_lib.lib().hm_gemm_i8w(a.data_ptr(), a.stride(0), w.data_ptr(), s.data_ptr(),
                                 res.data_ptr() if res is not None else None, res.stride(0) if res is not None else 0,
                                 out.data_ptr(), out.stride(0), M, N, K,
                                 _lib.HM_EPI_SILU if silu else _lib.HM_EPI_STORE,
                                 error_word(a.device).data_ptr(), _stream()), "hm_gemm_i8w")
    return out


def dequant_i8(w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Exact int8 -> fp16 copy of a weight matrix (no scale), for :func:`gemm_f16w`."""
    _need_cuda(w, out)
    if out is None:
        out = torch.empty(w.shape, device=w.device, dtype=torch.float16)
    if out.numel() < w.numel() or not w.is_contiguous() or not out.is_contiguous():
        raise HMError("dequant_i8: contiguous w and an output of at least w's size")
    check(_lib.lib().hm_dequant_i8_f16(w.data_ptr(), out.data_ptr(), w.numel(), _stream()), "hm_dequant_i8_f16")
    return out


def gemm_f16w(a: torch.Tensor, wh: torch.Tensor, s: torch.Tensor, res: torch.Tensor | None = None,
              out: torch.Tensor | None = None, silu: bool = False) -> torch.Tensor:
    """:func:`gemm_i8w` with the weights already dequantised to fp16 (``wh [N, K]``, the exact
    int8 values): the same result, without a conversion of every weight tile per CTA."""
    _need_cuda(a, wh, s, res, out)
    M, K = a.shape
    N = wh.shape[0]
    nout = N // 2 if silu else N
    if out is None:
        out = torch.empty(M, nout, device=a.device, dtype=torch.float16)
    check(_lib.lib().hm_gemm_f16w(a.data_ptr(), a.stride(0), wh.data_ptr(), s.data_ptr(),
                                  res.data_ptr() if res is not None else None, res.stride(0) if res is not None else 0,
                                  out.data_ptr(), out.stride(0), M, N, K,
                                  _lib.HM_EPI_SILU if silu else _lib.HM_EPI_STORE,
                                  error_word(a.device).data_ptr(), _stream()), "hm_gemm_f16w")
    return out


def prefill_attn(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, P: int, o: torch.Tensor | None = None,
                 scale: float | None = None) -> torch.Tensor:
    """Causal attention of a whole prompt: q ``[B*P, Hq*hd]`` (row ``b*P + p``) over
    ``kc/vc[b, :, :P]``; returns o like q."""
    _need_cuda(q, kc, vc, o)
    B, Hk, L, hd = kc.shape
    Hq = q.shape[1] // hd
    if o is None:
        o = torch.empty_like(q)
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    check(_lib.lib().hm_prefill_attn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), B, P, Hq, Hk, hd, L,
                                     scale, error_word(q.device).data_ptr(), _stream()), "hm_prefill_attn")
    return o


# ----------------------------------------------------------------------------- raw-launch stand-ins
class _Launch:
    """A kernel name that launches with the reference's ``kernel[grid](*args, **meta)``
    syntax.  ``grid`` and the Triton meta-parameters are accepted and ignored: the C
    entry point behind ``run`` sizes its own launch."""

    def __init__(self, name: str, run):
        self.__name__ = name
        self._run = run

    def __getitem__(self, grid):
        def launch(*args, **meta):
            return self._run(*args, **meta)
        return launch

    def __call__(self, *args, **kwargs):
        raise TypeError(f"{self.__name__} launches as {self.__name__}[grid](...), like the reference's kernel")


def _rope_cache_launch(qkv, rope, pos, q_out, kc, vc, S, Hq, Hk, L, **meta):
    rope_cache(qkv, rope, pos, q_out, kc, vc, int(S), int(Hq), int(Hk), int(L))


def _attn_launch(q, kc, vc, pos, o, pm, pl, pa, S, Hq, Hk, L, scale, **meta):
    # the scratch tensors the reference passes for its split partials (pm, pl, pa) are not
    # needed: the split count is chosen for this GPU and the merge happens inside
    from .engine import default_nsplit
    del pm, pl, pa, meta
    R = q.shape[0]
    attn(q, kc, vc, pos, o, int(S), int(Hq), int(Hk), int(L), float(scale),
         nsplit=default_nsplit(R, int(Hk), int(L), sms=torch.cuda.get_device_properties(q.device).multi_processor_count))


def _attn_combine_launch(pm, pl, pa, o, **meta):
    """Nothing to do: ``_attn`` wrote the merged output into ``o``."""
    del pm, pl, pa, o, meta


def _silu_mul_launch(a, y, F_, **meta):
    if a.shape[1] != 2 * int(F_):
        raise HMError("_silu_mul: a must hold the w1 and w3 halves [R, 2F]")
    silu_mul_into(a, y)


_rope_cache = _Launch("_rope_cache", _rope_cache_launch)
_attn = _Launch("_attn", _attn_launch)
_attn_combine = _Launch("_attn_combine", _attn_combine_launch)
_silu_mul = _Launch("_silu_mul", _silu_mul_launch)
