"""HeartMuLa int8 checkpoint: model shapes, synthetic weights and loading.

The on-disk format is the reference's ``mula_int8.safetensors``
(``app/convert_final.py:17-47``):

* every 2-D tensor except ``unconditional_text_embedding.weight`` is stored as
  ``<key>.q8`` (int8 ``[N, K]``, symmetric per row) plus ``<key>.s8``
  (bf16 ``[N]``, ``amax / 127``);
* ``audio_head`` is split into ``audio_head.{i}.q8/.s8`` of shape ``[V, D_dec]``;
* norms (``*.scale``), ``muq_linear.bias`` and the unconditional embedding are bf16;
* metadata ``{"lite": "{\\"mode\\": \\"int8\\"}"}``.

Shapes are not fixed constants here: :func:`shape_from_tensors` derives layer
counts and widths from the tensors themselves (the reference reads them from
module constants, ``app/engine.py:16-24``, and computes ``head_dim = DIM // heads``,
``app/engine.py:116``). Only the query-head counts must be given.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, asdict, replace

import torch

AUDIO_VOCAB = 8197          # app/engine.py:16
N_CB = 8                    # app/engine.py:17
TEXT_BOS, TEXT_EOS, AUDIO_EOS, EMPTY_ID = 128000, 128001, 8193, 0   # app/engine.py:20
FRAME_MS = 80               # app/engine.py:21


@dataclass(frozen=True)
class ModelShape:
    """Widths of the backbone and local decoder (one HeartMuLa checkpoint)."""
    bb_layers: int = 28
    bb_dim: int = 3072
    bb_heads: int = 24
    bb_kv_heads: int = 8
    bb_ffn: int = 8192
    dec_layers: int = 4
    dec_dim: int = 1024
    dec_heads: int = 8
    dec_kv_heads: int = 2
    dec_ffn: int = 8192
    audio_vocab: int = AUDIO_VOCAB
    n_cb: int = N_CB
    text_vocab: int = 128256
    uncond_rows: int = 1

    @property
    def bb_hd(self) -> int:
        return self.bb_dim // self.bb_heads

    @property
    def dec_hd(self) -> int:
        return self.dec_dim // self.dec_heads

    def to_json(self) -> str:
        return json.dumps(asdict(self), sort_keys=True)


# BASELINE config 0 architecture: Llama-3.2-3B backbone + 4-layer 1024-wide decoder.
BASELINE_SHAPE = ModelShape()
# The reference's own module constants (app/engine.py:23-24): decoder of 3 layers,
# width DIM=3072, 8 query / 4 KV heads, so head_dim 384.
REFERENCE_SHAPE = ModelShape(dec_layers=3, dec_dim=3072, dec_heads=8, dec_kv_heads=4, dec_ffn=8192)
# Small shapes for CPU-checkable parity cases (head_dim stays 128 like the real model).
TINY_SHAPE = ModelShape(bb_layers=2, bb_dim=512, bb_heads=4, bb_kv_heads=2, bb_ffn=1024,
                        dec_layers=2, dec_dim=256, dec_heads=2, dec_kv_heads=1, dec_ffn=512,
                        text_vocab=1024)


def linear_shapes(shape: ModelShape) -> dict[str, tuple[int, int]]:
    """Every int8 matrix of the checkpoint as ``key -> (N, K)``."""
    out: dict[str, tuple[int, int]] = {}
    for pre, L, D, H, KV, F in (("backbone", shape.bb_layers, shape.bb_dim, shape.bb_heads, shape.bb_kv_heads, shape.bb_ffn),
                                 ("decoder", shape.dec_layers, shape.dec_dim, shape.dec_heads, shape.dec_kv_heads, shape.dec_ffn)):
        hd = D // H
        for i in range(L):
            p = f"{pre}.layers.{i}."
            out[p + "attn.q_proj.weight"] = (H * hd, D)
            out[p + "attn.k_proj.weight"] = (KV * hd, D)
            out[p + "attn.v_proj.weight"] = (KV * hd, D)
            out[p + "attn.output_proj.weight"] = (D, H * hd)
            out[p + "mlp.w1.weight"] = (F, D)
            out[p + "mlp.w3.weight"] = (F, D)
            out[p + "mlp.w2.weight"] = (D, F)
    out["projection.weight"] = (shape.dec_dim, shape.bb_dim)
    out["codebook0_head.weight"] = (shape.audio_vocab, shape.bb_dim)
    for i in range(shape.n_cb - 1):
        out[f"audio_head.{i}"] = (shape.audio_vocab, shape.dec_dim)
    out["audio_embeddings.weight"] = (shape.n_cb * shape.audio_vocab, shape.bb_dim)
    out["text_embeddings.weight"] = (shape.text_vocab, shape.bb_dim)
    return out


def norm_shapes(shape: ModelShape) -> dict[str, int]:
    out = {}
    for pre, L, D in (("backbone", shape.bb_layers, shape.bb_dim), ("decoder", shape.dec_layers, shape.dec_dim)):
        for i in range(L):
            out[f"{pre}.layers.{i}.sa_norm.scale"] = D
            out[f"{pre}.layers.{i}.mlp_norm.scale"] = D
        out[f"{pre}.norm.scale"] = D
    return out


def synthetic_tensors(shape: ModelShape, seed: int = 0, device="cpu", gamma_one: bool = True,
                      scale_dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init weights in the checkpoint's own key/dtype layout.

    Distributions follow the benchmark configuration: int8 weights uniform in
    [-127, 127]; per-row scales ``|N(0, 0.02)| / 127``; RMSNorm gammas 1 (or
    ``1 + N(0, 0.1)`` with ``gamma_one=False``, to exercise the gamma multiply);
    ``muq_linear.bias`` and the unconditional embedding ``N(0, 0.02)``-ish.
    Deterministic for a given ``seed`` and device type.
    """
    g = torch.Generator(device=device).manual_seed(seed)
    t: dict[str, torch.Tensor] = {}
    for k, (n, kk) in linear_shapes(shape).items():
        t[k + ".q8"] = torch.randint(-127, 128, (n, kk), generator=g, device=device, dtype=torch.int8)
        t[k + ".s8"] = (torch.randn(n, generator=g, device=device).abs() * 0.02 / 127).to(scale_dtype)
    for k, d in norm_shapes(shape).items():
        if gamma_one:
            t[k] = torch.ones(d, device=device, dtype=torch.bfloat16)
        else:
            t[k] = (1 + 0.1 * torch.randn(d, generator=g, device=device)).to(torch.bfloat16)
    t["muq_linear.bias"] = (0.02 * torch.randn(shape.bb_dim, generator=g, device=device)).to(torch.bfloat16)
    t["unconditional_text_embedding.weight"] = (
        torch.randn(shape.uncond_rows, shape.bb_dim, generator=g, device=device) * 0.5).to(torch.bfloat16)
    return t


def save_checkpoint(tensors: dict[str, torch.Tensor], path: str) -> None:
    """Write ``tensors`` as a reference-format int8 checkpoint."""
    from safetensors.torch import save_file
    save_file({k: v.contiguous().cpu() for k, v in tensors.items()}, str(path),
              metadata={"lite": json.dumps({"mode": "int8"})})


def load_tensors(path_or_dict, device="cpu") -> dict[str, torch.Tensor]:
    """Read a checkpoint file (or pass a dict through) onto ``device``."""
    if isinstance(path_or_dict, dict):
        return {k: v.to(device) for k, v in path_or_dict.items()}
    from safetensors import safe_open
    out = {}
    with safe_open(str(path_or_dict), "pt", device=str(device)) as f:
        for k in f.keys():
            out[k] = f.get_tensor(k)
    return out


def shape_from_tensors(t: dict[str, torch.Tensor], bb_heads: int = 24, dec_heads: int = 8) -> ModelShape:
    """Derive a :class:`ModelShape` from checkpoint tensors.

    Layer counts come from the key names, widths from the norm sizes, FFN
    widths from ``w1`` rows, KV heads from ``k_proj`` rows / head_dim.
    """
    def count(pre):
        n = 0
        while f"{pre}.layers.{n}.sa_norm.scale" in t:
            n += 1
        return n

    def q8(k):
        return t[k + ".q8"] if k + ".q8" in t else t[k]

    bb_dim = t["backbone.norm.scale"].numel()
    dec_dim = t["decoder.norm.scale"].numel()
    bb_hd, dec_hd = bb_dim // bb_heads, dec_dim // dec_heads
    v = q8("codebook0_head.weight").shape[0]
    n_cb = 1
    while f"audio_head.{n_cb - 1}.q8" in t:
        n_cb += 1
    return ModelShape(
        bb_layers=count("backbone"), bb_dim=bb_dim, bb_heads=bb_heads,
        bb_kv_heads=q8("backbone.layers.0.attn.k_proj.weight").shape[0] // bb_hd,
        bb_ffn=q8("backbone.layers.0.mlp.w1.weight").shape[0],
        dec_layers=count("decoder"), dec_dim=dec_dim, dec_heads=dec_heads,
        dec_kv_heads=q8("decoder.layers.0.attn.k_proj.weight").shape[0] // dec_hd,
        dec_ffn=q8("decoder.layers.0.mlp.w1.weight").shape[0],
        audio_vocab=v, n_cb=n_cb,
        text_vocab=q8("text_embeddings.weight").shape[0],
        uncond_rows=t["unconditional_text_embedding.weight"].shape[0])


def with_shape(shape: ModelShape, **kw) -> ModelShape:
    return replace(shape, **kw)


def tensors_sha(t: dict[str, torch.Tensor]) -> str:
    """SHA-256 over key names, dtypes and raw bytes (CPU tensors), in key order."""
    import hashlib
    h = hashlib.sha256()
    for k in sorted(t):
        v = t[k].contiguous().cpu()
        h.update(k.encode())
        h.update(str(v.dtype).encode())
        raw = v.view(torch.int16) if v.dtype == torch.bfloat16 else v.view(torch.uint8)
        h.update(raw.numpy().tobytes())
    return h.hexdigest()
