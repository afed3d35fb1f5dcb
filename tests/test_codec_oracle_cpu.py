"""The codec oracle against the golden vectors of the unmodified reference codec
(tests/golden/codec.npz, made by tests/golden/make_codec_golden.py): estimator forward,
scalar decoder and whole detokenize runs, all fp32 on the CPU."""
from pathlib import Path

import numpy as np
import pytest
import torch

from estudiocanciones_b200.checkpoint import tensors_sha
from estudiocanciones_b200.codec_checkpoint import TINY_CODEC, synthetic_codec_tensors
from oracle.heartcodec_oracle import OracleCodec

GOLD = Path(__file__).parent / "golden" / "codec.npz"
SEED = 4321
EST_T = 200


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def oracle(gold):
    sd = synthetic_codec_tensors(TINY_CODEC, SEED)
    assert bytes(gold["sha"]).hex() == tensors_sha(sd), "synthetic codec checkpoint drifted"
    return OracleCodec(sd, TINY_CODEC)


def est_input(gold):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, EST_T, TINY_CODEC.in_channels, generator=g)
    assert bytes(gold["est_x_sha"]).hex() == tensors_sha({"x": x})
    return x


def test_estimator_matches_reference(gold, oracle):
    with torch.inference_mode():
        out = oracle.estimator(est_input(gold), torch.from_numpy(gold["est_t"]))
    ref = torch.from_numpy(gold["est_out"])
    assert (out - ref).abs().max() <= 2e-5 * ref.abs().max()


def test_scalar_decode_matches_reference(gold, oracle):
    with torch.inference_mode():
        out = oracle.scalar_decode(torch.from_numpy(gold["dec_in"]))
    ref = torch.from_numpy(gold["dec_out"])
    assert out.shape == ref.shape
    assert (out - ref).abs().max() <= 2e-5 * ref.abs().max()


def seeded_randn(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda shape, where: torch.randn(shape, generator=g)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_detokenize_matches_reference(gold, oracle, case):
    n, steps, gs, seed = gold[f"detok{case}_cfg"]
    codes = torch.from_numpy(gold[f"detok{case}_codes"])
    with torch.inference_mode():
        wav = oracle.detokenize(codes, num_steps=int(steps), guidance_scale=float(gs), randn=seeded_randn(int(seed)))
    ref = torch.from_numpy(gold[f"detok{case}_wav"])
    assert wav.shape == ref.shape == (2, int(n / 12.5 * TINY_CODEC.sample_rate))
    assert (wav - ref).abs().max() <= 1e-4 * ref.abs().max()


def test_codec_checkpoint_round_trip(tmp_path):
    """load_codec_tensors reads what the reference's load_codec reads: one .safetensors with its
    .json beside it, or a directory with config.json and model*.safetensors; the audio
    encoder's tensors are dropped (app/codec_lite.py:13-26)."""
    import json

    from safetensors.torch import save_file

    from estudiocanciones_b200.codec_checkpoint import CodecConfig, load_codec_tensors
    sd = synthetic_codec_tensors(TINY_CODEC, 1)
    sd_enc = dict(sd)
    sd_enc["scalar_model.encoder.0.bias"] = torch.zeros(64)
    f = tmp_path / "codec_bf16.safetensors"
    save_file({k: v.to(torch.bfloat16) if v.is_floating_point() else v for k, v in sd_enc.items()}, str(f))
    cfgd = dict(TINY_CODEC.to_dict(), model_type="heartcodec", unknown_key=3)
    f.with_suffix(".json").write_text(json.dumps(cfgd))
    t, cfg = load_codec_tensors(f)
    assert cfg == TINY_CODEC and set(t) == set(sd)
    assert all(torch.equal(t[k], sd[k].to(torch.bfloat16)) for k in sd)
    d = tmp_path / "dir"
    d.mkdir()
    save_file({k: v for k, v in sd_enc.items()}, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(cfgd))
    t2, cfg2 = load_codec_tensors(d)
    assert cfg2 == TINY_CODEC and set(t2) == set(sd) and torch.equal(t2[next(iter(sd))], sd[next(iter(sd))])
    assert CodecConfig.from_dict(None) == CodecConfig()
