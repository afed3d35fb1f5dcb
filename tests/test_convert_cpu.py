"""Checkpoint conversion on the CPU: the oracle's q8_rows against the reference
converter's own outputs (tests/golden/q8_rows.npz), and the converter's key mapping
(``app/convert_final.py:32-47``) with the oracle as its quantiser."""
import json

import numpy as np
import pytest
import torch

from oracle import heartmula_oracle as O
from estudiocanciones_b200 import convert

GOLD = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "q8_rows.npz")
DTYPES = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}


def golden_cases():
    names = sorted({k.split(".")[0] for k in GOLD.files})
    for name in names:
        x = torch.from_numpy(GOLD[f"{name}.x"]).to(DTYPES[str(GOLD[f"{name}.dtype"])])
        mats = [x[i].t().contiguous() for i in range(x.shape[0])] if name == "audio_head" else [x]
        for j, m in enumerate(mats):
            yield f"{name}.{j}", m, GOLD[f"{name}.{j}.q"], GOLD[f"{name}.{j}.s"]


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_oracle_q8_rows_equals_reference_converter(case):
    _, m, q_ref, s_ref = case
    q, s = O.q8_rows(m)
    assert np.array_equal(q.numpy(), q_ref)
    assert np.array_equal(s.view(torch.int16).numpy(), s_ref)


def test_golden_ties_round_half_to_even():
    q = GOLD["f32_ties.0.q"][0].tolist()
    # scale 1.0: 2.5 -> 2, -3.5 -> -4, 0.5 -> 0, -0.5 -> 0, 1.5 -> 2, 126.5 -> 126, -1.5 -> -2, 3.5 -> 4, 64.5 -> 64
    assert q == [127, 2, -4, 0, 0, 2, 126, -127, 0, -2, 4, 64]


def fake_official(tmp_path, sharded=True):
    """A tiny checkpoint in the official layout (fp32), split over two shards."""
    g = torch.Generator().manual_seed(3)
    t = {
        "backbone.layers.0.attn.q_proj.weight": torch.randn(8, 16, generator=g),
        "backbone.layers.0.sa_norm.scale": torch.randn(16, generator=g),
        "backbone.pos_embeddings.weight": torch.randn(4, 16, generator=g),
        "muq_linear.weight": torch.randn(16, 8, generator=g),
        "muq_linear.bias": torch.randn(16, generator=g),
        "audio_head": torch.randn(3, 16, 10, generator=g),
        "unconditional_text_embedding.weight": torch.randn(1, 16, generator=g),
        "text_embeddings.weight": torch.randn(12, 16, generator=g),
        "audio_embeddings.weight": torch.randn(20, 16, generator=g),
        "codebook0_head.weight": torch.randn(10, 16, generator=g),
    }
    from safetensors.torch import save_file
    keys = sorted(t)
    if sharded:
        parts = {"model-00001-of-00002.safetensors": keys[: len(keys) // 2],
                 "model-00002-of-00002.safetensors": keys[len(keys) // 2:]}
        for fn, ks in parts.items():
            save_file({k: t[k] for k in ks}, str(tmp_path / fn))
        wm = {k: fn for fn, ks in parts.items() for k in ks}
        (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    else:
        save_file(t, str(tmp_path / "model.safetensors"))
    return t


@pytest.mark.parametrize("sharded", [True, False])
@pytest.mark.parametrize("keep_emb", [False, True])
def test_converter_key_mapping(tmp_path, sharded, keep_emb):
    t = fake_official(tmp_path, sharded)
    out = convert.convert_tensors(tmp_path, keep_emb=keep_emb, device="cpu", quant=O.q8_rows)
    assert "backbone.pos_embeddings.weight" not in out and not any(k.startswith("muq_linear.weight") for k in out)
    assert out["muq_linear.bias"].dtype == torch.bfloat16
    assert out["backbone.layers.0.sa_norm.scale"].dtype == torch.bfloat16
    assert out["unconditional_text_embedding.weight"].dtype == torch.bfloat16
    for k in ("backbone.layers.0.attn.q_proj.weight", "codebook0_head.weight"):
        q, s = O.q8_rows(t[k])
        assert torch.equal(out[k + ".q8"], q) and torch.equal(out[k + ".s8"].view(torch.int16), s.view(torch.int16))
    for i in range(3):  # audio_head [heads, D, V] -> per head [V, D]
        q, s = O.q8_rows(t["audio_head"][i].t().contiguous())
        assert out[f"audio_head.{i}.q8"].shape == (10, 16)
        assert torch.equal(out[f"audio_head.{i}.q8"], q)
    for k in ("text_embeddings.weight", "audio_embeddings.weight"):
        if keep_emb:
            assert out[k].dtype == torch.bfloat16 and k + ".q8" not in out
        else:
            assert out[k + ".q8"].dtype == torch.int8 and out[k + ".s8"].dtype == torch.bfloat16


def test_converter_writes_the_checkpoint_format(tmp_path):
    fake_official(tmp_path / "", sharded=False)
    dst = tmp_path / "mula_int8.safetensors"
    keys = convert.convert_mula(tmp_path, dst, device="cpu", quant=O.q8_rows)
    from safetensors import safe_open
    with safe_open(str(dst), "pt") as f:
        assert json.loads(f.metadata()["lite"]) == {"mode": "int8"}
        assert sorted(f.keys()) == keys


def test_q8_rows_refuses_cpu_tensors():
    with pytest.raises(Exception, match="CUDA"):
        convert.q8_rows(torch.zeros(2, 4))


def test_plain_weights_are_quantised_on_load_as_the_converter_would(tmp_path):
    """A checkpoint with plain fp weights (the reference's Linear(w=...), bf16 audio_head
    [heads, D, V] and embedding branches) becomes, on load, what the converter makes of it;
    int8 tensors pass through unchanged."""
    t = fake_official(tmp_path, sharded=False)
    conv = convert.convert_tensors(tmp_path, device="cpu", quant=O.q8_rows)
    loaded = {k: v for k, v in t.items()}
    got = convert.quantize_plain(loaded, quant=O.q8_rows)
    for k, v in conv.items():
        if k.endswith((".q8", ".s8")):
            assert torch.equal(got[k].view(torch.int8) if got[k].dtype == torch.int8 else got[k].view(torch.int16),
                               v.view(torch.int8) if v.dtype == torch.int8 else v.view(torch.int16)), k
    assert "audio_head" not in got and "audio_head.2.q8" in got and "muq_linear.weight" not in got
    assert "backbone.pos_embeddings.weight" not in got
    assert torch.equal(got["backbone.layers.0.sa_norm.scale"], t["backbone.layers.0.sa_norm.scale"])
    again = convert.quantize_plain(got, quant=O.q8_rows)  # already converted: a pass-through
    assert sorted(again) == sorted(got) and all(again[k] is got[k] for k in got)


def test_convert_codec_drops_the_encoder_and_casts_to_bf16(tmp_path):
    """``convert_codec`` (app/convert_final.py:50-58): encoder keys dropped, floating
    tensors bf16, integer tensors unchanged, config.json copied beside the output."""
    from safetensors import safe_open
    from safetensors.torch import save_file
    src = tmp_path / "codec"
    src.mkdir()
    g = torch.Generator().manual_seed(9)
    t = {"scalar_model.encoder.conv.weight": torch.randn(4, 3, generator=g),
         "scalar_model.decoder.conv.weight": torch.randn(4, 3, generator=g),
         "flow_matching.estimator.proj.weight": torch.randn(2, 5, generator=g, dtype=torch.float64),
         "quantizer.codebook_size": torch.tensor([8192], dtype=torch.int64)}
    save_file(t, str(src / "model.safetensors"))
    (src / "config.json").write_text('{"sample_rate": 48000}')
    dst = tmp_path / "out" / "codec_bf16.safetensors"
    dst.parent.mkdir()
    keys = convert.convert_codec(src, dst)
    assert keys == sorted(k for k in t if not k.startswith("scalar_model.encoder"))
    with safe_open(str(dst), "pt") as f:
        assert f.get_tensor("scalar_model.decoder.conv.weight").dtype == torch.bfloat16
        assert torch.equal(f.get_tensor("scalar_model.decoder.conv.weight"),
                           t["scalar_model.decoder.conv.weight"].to(torch.bfloat16))
        assert f.get_tensor("flow_matching.estimator.proj.weight").dtype == torch.bfloat16
        assert torch.equal(f.get_tensor("quantizer.codebook_size"), t["quantizer.codebook_size"])
    assert (tmp_path / "out" / "codec_bf16.json").read_text() == '{"sample_rate": 48000}'
