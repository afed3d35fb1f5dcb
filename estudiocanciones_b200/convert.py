"""Checkpoint converter: official HeartMuLa weights -> the int8 checkpoint format the
engine loads (``app/convert_final.py:24-47``, ``convert_mula``), with the per-row int8
quantisation (``q8_rows``, ``app/convert_final.py:17-21``) done by the ``hm_q8_rows``
kernel and the shards read straight onto the GPU.

Format (unchanged from the reference): every 2-D tensor except
``unconditional_text_embedding.weight`` (and, with ``keep_emb``, the embedding tables)
becomes ``<key>.q8`` int8 ``[N, K]`` + ``<key>.s8`` bf16 ``[N]``; ``audio_head``
``[heads, D, V]`` becomes ``audio_head.<i>.q8`` ``[V, D]`` / ``.s8`` per head; the RoPE
``pos_embeddings`` and ``muq_linear.weight`` are dropped (the table is recomputed, the
MuQ input is always zero so only the bias counts); everything else is stored as bf16.

    python -m estudiocanciones_b200.convert <HeartMuLa dir> <out.safetensors> [--keep-emb-bf16]
    python -m estudiocanciones_b200.convert <HeartMuLa dir> <HeartCodec dir> <out dir> [--keep-emb-bf16]

The second form is the reference's full command (``app/convert_final.py:60-66``): it
writes ``mula_int8.safetensors`` and ``codec_bf16.safetensors`` (:func:`convert_codec`)
into ``<out dir>``.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

from . import _lib
from ._lib import HMError, check

_DT = {torch.float32: _lib.HM_DT_F32, torch.bfloat16: _lib.HM_DT_BF16, torch.float16: _lib.HM_DT_F16}


def q8_rows(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric int8 quantisation of a 2-D CUDA tensor (fp32 / bf16 / fp16; other
    floating types are read as fp32) on the current stream.  Returns (int8 ``[N, K]``,
    bf16 scales ``[N]``) on the tensor's device, bit-identical to the converter's."""
    if not t.is_cuda:
        raise HMError("q8_rows runs on CUDA tensors (hm_q8_rows)")
    if t.dim() != 2 or t.shape[0] < 1 or t.shape[1] < 1:
        raise HMError(f"q8_rows wants a non-empty 2-D tensor, got {tuple(t.shape)}")
    if t.dtype not in _DT:
        t = t.float()
    if t.stride(1) != 1:
        t = t.contiguous()
    N, K = t.shape
    q = torch.empty(N, K, dtype=torch.int8, device=t.device)
    s = torch.empty(N, dtype=torch.bfloat16, device=t.device)
    st = torch.cuda.current_stream(t.device).cuda_stream
    check(_lib.lib().hm_q8_rows(t.data_ptr(), _DT[t.dtype], N, K, t.stride(0), q.data_ptr(), K, s.data_ptr(), st),
          "hm_q8_rows")
    return q, s


def shard_files(d) -> list[Path]:
    """The safetensors shards of a checkpoint directory (``app/convert_final.py:24-29``):
    those named by ``model.safetensors.index.json``, else ``model.safetensors``."""
    d = Path(d)
    idx = d / "model.safetensors.index.json"
    if idx.exists():
        return [d / name for name in sorted(set(json.loads(idx.read_text())["weight_map"].values()))]
    return [d / "model.safetensors"]


def convert_entry(k: str, t: torch.Tensor, quant, keep_emb: bool = False) -> dict[str, torch.Tensor]:
    """The converted form of one checkpoint tensor (``app/convert_final.py:30-47``): dropped
    (RoPE tables, ``muq_linear.weight``), split per head and quantised (``audio_head``
    ``[heads, D, V]`` -> ``audio_head.<i>.q8/.s8`` ``[V, D]``), quantised (other 2-D
    tensors except the unconditional embedding and, with ``keep_emb``, the embedding
    tables) or kept as bf16."""
    if "pos_embeddings" in k or k == "muq_linear.weight":
        return {}
    out = {}
    if k == "audio_head":  # [heads, D, V]: one [V, D] matrix per head
        for i in range(t.shape[0]):
            out[f"audio_head.{i}.q8"], out[f"audio_head.{i}.s8"] = quant(t[i].t().contiguous())
    elif t.dim() == 2 and k != "unconditional_text_embedding.weight" and not (keep_emb and "embeddings" in k):
        out[k + ".q8"], out[k + ".s8"] = quant(t)
    else:
        out[k] = t.to(torch.bfloat16).contiguous()
    return out


def quantize_plain(t: dict[str, torch.Tensor], quant=None) -> dict[str, torch.Tensor]:
    """A loaded checkpoint with every plain (un-quantised) weight converted as the converter
    would (the reference also loads fp16/bf16 ``Linear`` weights, a bf16 ``audio_head``
    ``[heads, D, V]`` and bf16 embedding tables: ``app/engine.py:235-260``).  Tensors
    already in the int8 format pass through; the result is what ``convert_tensors`` makes
    of the same weights, on the tensors' device."""
    quant = quant or q8_rows
    out: dict[str, torch.Tensor] = {}
    for k, v in t.items():
        if k.endswith((".q8", ".s8")) or k in ("unconditional_text_embedding.weight", "muq_linear.bias"):
            out[k] = v
        elif v.dim() == 1 and not k == "audio_head":  # norm scales, biases
            out[k] = v
        else:
            out.update(convert_entry(k, v, quant))
    return out


def convert_tensors(src, keep_emb: bool = False, device="cuda", quant=None) -> dict[str, torch.Tensor]:
    """Converted tensors (on the host) of the checkpoint directory ``src``.  ``quant``
    replaces the quantiser (default: :func:`q8_rows` on ``device``)."""
    from safetensors import safe_open
    quant = quant or q8_rows
    out: dict[str, torch.Tensor] = {}
    for sh in shard_files(src):
        with safe_open(str(sh), "pt", device=str(device)) as f:
            for k in f.keys():
                for kk, v in convert_entry(k, f.get_tensor(k), quant, keep_emb).items():
                    out[kk] = v.cpu()
    return out


def convert_mula(src, dst, keep_emb: bool = False, device="cuda", quant=None) -> list[str]:
    """Write the int8 checkpoint of ``src`` to ``dst``; returns its keys."""
    from safetensors.torch import save_file
    out = convert_tensors(src, keep_emb=keep_emb, device=device, quant=quant)
    save_file(out, str(dst), metadata={"lite": json.dumps({"mode": "int8"})})
    return sorted(out)


def convert_codec(src, dst) -> list[str]:
    """The codec's distribution file (``app/convert_final.py:50-58``): every tensor of the
    HeartCodec checkpoint except the waveform encoder (``scalar_model.encoder.*``, not used
    to generate), floating tensors cast to bf16, written to ``dst``; the codec's
    ``config.json`` is copied beside it as ``dst`` with a ``.json`` suffix.  Returns the keys."""
    import shutil
    from safetensors import safe_open
    from safetensors.torch import save_file
    out: dict[str, torch.Tensor] = {}
    for sh in shard_files(src):
        with safe_open(str(sh), "pt") as f:
            for k in f.keys():
                if k.startswith("scalar_model.encoder"):
                    continue
                t = f.get_tensor(k)
                out[k] = t.to(torch.bfloat16).contiguous() if t.is_floating_point() else t
    save_file(out, str(dst))
    shutil.copy(Path(src) / "config.json", Path(dst).with_suffix(".json"))
    return sorted(out)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) < 2:
        raise SystemExit(__doc__)
    keep = "--keep-emb-bf16" in sys.argv
    if len(args) >= 3:  # <mula dir> <codec dir> <out dir>, as app/convert_final.py
        outdir = Path(args[2])
        outdir.mkdir(parents=True, exist_ok=True)
        convert_mula(args[0], outdir / "mula_int8.safetensors", keep)
        convert_codec(args[1], outdir / "codec_bf16.safetensors")
        files = sorted(outdir.glob("*.safetensors"))
    else:
        dst = Path(args[1])
        dst.parent.mkdir(parents=True, exist_ok=True)
        convert_mula(args[0], dst, keep)
        files = [dst]
    for f in files:
        print(f.name, round(f.stat().st_size / 1e9, 2), "GB")
