"""ctypes binding of ``libheartmula_b200.so`` (the C ABI in include/heartmula_b200.h).

The library is built in-tree by :mod:`estudiocanciones_b200.build`.  There is
no fallback: if the library is missing or a call reports an error, this module
raises.  Device pointers are passed as integers (``tensor.data_ptr()``) and the
stream as the raw ``cudaStream_t`` handle of the current torch stream.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import gc
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libheartmula_b200.so"

HM_SRC_F16, HM_SRC_RMS, HM_SRC_EMB = 0, 1, 2
HM_EPI_STORE, HM_EPI_ROPE_KV, HM_EPI_SILU = 0, 1, 2
HM_ERR_TIMEOUT, HM_ERR_BADINDEX = 1, 2
HM_EARG = -1
HM_DT_F32, HM_DT_BF16, HM_DT_F16 = 0, 1, 2
HM_ENOSPACE = -2
HM_ACT_NONE, HM_ACT_PRELU, HM_ACT_SILU = 0, 1, 2
HM_CEPI_STORE, HM_CEPI_GATED, HM_CEPI_RES, HM_CEPI_SILU, HM_CEPI_ROPE = 0, 1, 2, 3, 4

# Every exported symbol of include/heartmula_b200.h with (restype, argtypes).
_P, _I, _I64, _F, _SZ = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t


class RowSrc(C.Structure):
    _fields_ = [("mode", C.c_int), ("row_mul", C.c_int), ("row_add", C.c_int),
                ("x", _P), ("ldx", _I64),
                ("ss", _P), ("ss_tiles", C.c_int), ("ss_ld", _I64),
                ("gamma", _P), ("eps", C.c_float), ("dim", C.c_int),
                ("etab", _P), ("escale", _P), ("erows", _I64),
                ("tok", _P), ("tok_ld", _I64), ("tok_col", C.c_int), ("tok_off", _I64)]


class GemvDesc(C.Structure):
    _fields_ = [("w", _P), ("s", _P), ("N", C.c_int), ("K", C.c_int), ("M", C.c_int),
                ("src", RowSrc * 2), ("interleave", C.c_int), ("epi", C.c_int),
                ("y", _P), ("ldy", _I64), ("res", _P), ("ldres", _I64),
                ("ss_out", _P), ("ss_out_ld", _I64),
                ("rope", _P), ("rope_rows", C.c_int), ("pos", _P),
                ("S", C.c_int), ("Hq", C.c_int), ("Hk", C.c_int), ("hd", C.c_int), ("L", C.c_int),
                ("q_out", _P), ("kc", _P), ("vc", _P),
                ("ws", _P), ("ws_bytes", C.c_size_t), ("counters", _P), ("n_counters", C.c_int),
                ("err", _P), ("kspan", C.c_int), ("pdl", C.c_int), ("l2_keep", C.c_int)]


class ConvDesc(C.Structure):
    """hm_conv_desc: one implicit-GEMM convolution / linear layer of the codec."""
    _fields_ = [("x", _P), ("x_ld", _I64), ("x_bstride", _I64), ("w", _P), ("bias", _P),
                ("y", _P), ("y_ld", _I64), ("res", _P), ("res_ld", _I64), ("gate", _P), ("gate_ld", _I64),
                ("rope", _P), ("err", _P),
                ("B", C.c_int), ("T", C.c_int), ("tin", C.c_int), ("cin", C.c_int), ("N", C.c_int),
                ("npad", C.c_int), ("taps", C.c_int), ("off0", C.c_int), ("dil", C.c_int),
                ("scale", C.c_float), ("prelu", C.c_float),
                ("act", C.c_int), ("epi", C.c_int), ("y_f32", C.c_int), ("rope_cols", C.c_int), ("hd", C.c_int),
                ("bn", C.c_int)]


SIGNATURES = {
    "hm_gemv_i8": (_I, [_P, _I64, _P, _P, _P, _I64, _P, _I64, _I, _I, _I, _P, _SZ, _P, _I, _P, _I, _I, _P]),
    "hm_gemv_i8_fused": (_I, [C.POINTER(GemvDesc), _P]),
    "hm_gemv_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "hm_gemv_counters": (_I, [_I, _I]),
    "hm_gemv_pick_kspan": (_I, [_I, _I, _I, _I, _I]),
    "hm_rmsnorm": (_I, [_P, _P, _P, _I, _I, _F, _P]),
    "hm_rms_apply": (_I, [_P, _I64, _P, _I, _I64, _P, _F, _I, _P, _I64, _I, _I, _I, _P]),
    "hm_rope_kv_write": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "hm_silu_mul": (_I, [_P, _P, _I, _I, _P]),
    "hm_emb_gather_i8": (_I, [_P, _I, _P, _P, _I64, _I, _P, _P, _P]),
    "hm_emb_sum_i8": (_I, [_P, _I64, _I, _I, _I64, _P, _P, _I64, _I, _P, _P, _I64, _P, _I, _P]),
    "hm_frame_commit": (_I, [_P, _P, _I, _I, _P, _I, _P, _P, _I64, _P, _I64, _I, _P]),
    "hm_q8_rows": (_I, [_P, _I, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "hm_decode_attn": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _I, _P, _SZ, _P, _I, _P, _I, _P]),
    "hm_decode_attn_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "hm_decode_attn_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "hm_cfg_topk_sample": (_I, [_P, _I64, _I, _I, _I, _P, _I64, _F, _I, _F, _P, _I64, _I, _P, _I, _P]),
    "hm_gemm_i8w": (_I, [_P, _I64, _P, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _P, _P]),
    "hm_gemm_f16w": (_I, [_P, _I64, _P, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _P, _P]),
    "hm_dequant_i8_f16": (_I, [_P, _P, _I64, _P]),
    "hm_prefill_attn": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P]),
    "hm_conv1d_gemm": (_I, [C.POINTER(ConvDesc), _P]),
    "hm_codec_attn": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I64, _I64, _F, _P, _P]),
    "hm_codec_norm_mod": (_I, [_P, _I64, _P, _P, _P, _I64, _P, _I64, _I, _I, _I, _F, _I, _P]),
    "hm_codec_vq_embed": (_I, [_P, _I64, _I, _I, _P, _I, _I, _P, _P, _P, _I64, _I, _P]),
    "hm_codec_upsample_rows": (_I, [_P, _I64, _I, _I, _I, _P, _I64, _P]),
    "hm_codec_euler": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _F, _F, _F, _I, _P, _I64, _I64, _P]),
    "hm_codec_band_quant": (_I, [_P, _I, _I, _I, _P, _P]),
    "hm_codec_temb_post": (_I, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "hm_codec_overlap_add": (_I, [_P, _I64, _P, _I64, _I, _I64, _I64, _I64, _P]),
    "hm_device_sm_count": (_I, [_I]),
    "hm_gemv_box_form": (_I, [_P, _I, _I, _I]),
    "hm_decode_attn_box_form": (_I, [_P, _I64]),
    "hm_abi_layout": (_SZ, [_I]),
    "hm_version": (C.c_char_p, []),
}

_lib = None


class HMError(RuntimeError):
    pass


def lib() -> C.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise HMError(f"{LIB_PATH.name} is not built; run `python -m estudiocanciones_b200.build` "
                          f"(or __graft_entry__.build())")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


@contextlib.contextmanager
def capture_no_gc():
    """Python's cyclic collector stays off while a CUDA graph is captured: a collection
    there could destroy a dead graph, whose memory pool then returns device memory
    (cudaFree), and that invalidates the capture in progress."""
    was_on = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was_on:
            gc.enable()


@contextlib.contextmanager
def capture_graph(g, stream, pool=None):
    """Capture CUDA work into ``g`` on ``stream`` as ``torch.cuda.graph`` does, minus its
    entry step that empties torch's device and pinned-host allocator caches: after that,
    every later allocation goes back to cudaMalloc, which with peer access enabled (an
    NCCL process group) took up to ~1 s per song on two B200s.  The cyclic collector is
    off meanwhile (see :func:`capture_no_gc`).  ``pool``: a graph memory pool handle to
    share between captures (its blocks are then reused instead of allocated anew)."""
    import torch
    torch.cuda.synchronize()
    with torch.cuda.stream(stream), capture_no_gc():
        if pool is None:
            g.capture_begin(capture_error_mode="global")
        else:
            g.capture_begin(pool, capture_error_mode="global")
        try:
            yield g
        finally:
            g.capture_end()


def check(rc: int, what: str) -> None:
    if rc != 0:
        kind = "bad argument" if rc < 0 else f"CUDA error {rc}"
        raise HMError(f"{what}: {kind}")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def abi_mismatches() -> list[str]:
    """Compare the ctypes struct layouts with the library's own sizeof/offsetof."""
    L = lib()
    want = {0: C.sizeof(RowSrc), 1: C.sizeof(GemvDesc), 2: GemvDesc.src.offset, 3: GemvDesc.ws.offset,
            4: GemvDesc.pdl.offset, 5: GemvDesc.l2_keep.offset, 6: C.sizeof(ConvDesc), 7: ConvDesc.B.offset,
            8: ConvDesc.scale.offset, 9: ConvDesc.bn.offset}
    return [f"layout[{k}]: C {L.hm_abi_layout(k)} vs ctypes {v}" for k, v in want.items() if L.hm_abi_layout(k) != v]
