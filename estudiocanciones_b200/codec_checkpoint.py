"""HeartCodec configuration and checkpoint format (the detokenizer that turns token streams into audio).

* :class:`CodecConfig` - the fields of the reference's ``HeartCodecConfig``
  (``app/heartcodec/configuration_heartcodec.py:9-71``), defaults included; unknown keys
  of a ``config.json`` are ignored as ``PretrainedConfig`` keeps them.
* :func:`synthetic_codec_tensors` - a seeded random checkpoint with exactly the key names and
  shapes of the reference's ``HeartCodec.state_dict()`` minus the audio encoder (which
  ``load_codec`` drops, ``app/codec_lite.py:26-28``): weight-norm parametrisations
  (``parametrizations.weight.original0/1``), PReLU slopes, the residual-VQ codebooks
  (``vq_embed.layers.{q}._codebook.embed``) and the estimator's ada-norm tables.  There is no
  network in this environment, so tests and the benchmark run on such checkpoints.
* :func:`load_codec_tensors` - the tensors of a ``codec*.safetensors`` file or a directory of
  ``model*.safetensors`` (+ ``config.json``), as ``load_codec`` reads them (``:13-26``).
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from pathlib import Path

import torch


@dataclass
class CodecConfig:
    dim: int = 512
    codebook_size: int = 8192
    codebook_dim: int = 32
    num_quantizers: int = 8
    attention_head_dim: int = 64
    in_channels: int = 1024
    norm_type: str = "ada_norm_single"
    num_attention_heads: int = 24
    num_layers: int = 24
    num_layers_2: int = 6
    out_channels: int = 256
    num_bands: int = 1
    sample_rate: int = 48000
    causal: bool = True
    num_samples: int = 2
    downsample_factors: list = field(default_factory=lambda: [3, 4, 4, 4, 5])
    downsample_kernel_sizes: list = field(default_factory=lambda: [6, 8, 8, 8, 10])
    upsample_factors: list = field(default_factory=lambda: [5, 4, 4, 4, 3])
    upsample_kernel_sizes: list = field(default_factory=lambda: [10, 8, 8, 8, 6])
    latent_hidden_dim: int = 128
    default_kernel_size: int = 7
    delay_kernel_size: int = 5
    init_channel: int = 64
    res_kernel_size: int = 7

    @classmethod
    def from_dict(cls, d: dict | None) -> "CodecConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in (d or {}).items() if k in names})

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    # derived sizes (models/transformer.py:262-265, 135-143; sq_codec.py:449-479)
    @property
    def inner(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def inner2(self) -> int:
        return 2 * self.inner

    @staticmethod
    def mlp_hidden(d: int, multiple_of: int = 256) -> int:
        h = int(2 * (4 * d) / 3)
        return multiple_of * ((h + multiple_of - 1) // multiple_of)

    def decoder_channels(self) -> list[int]:
        """Channels entering decoder stage i (0 = after decoder.0) .. the last stage's output."""
        n = len(self.upsample_factors)
        return [self.init_channel * 2 ** (n - i) for i in range(n + 1)]

    @property
    def hop(self) -> int:
        """Audio samples per latent frame."""
        h = self.num_samples
        for f in self.upsample_factors:
            h *= f
        return h


# The full-size codec and a tiny one of the same structure (every layer kind, both head
# dims of the estimator, two up-sampling stages), sized so the reference runs it on a CPU in
# seconds; its sample rate keeps 25 latent frames per second (hop 8 at 200 Hz).
FULL_CODEC = CodecConfig()
# (detokenize fixes the latent width at 256 channels, app/heartcodec/modeling_heartcodec.py:72-74,
# so out_channels and latent_hidden_dim keep their full sizes.)
TINY_CODEC = CodecConfig(dim=64, codebook_size=64, codebook_dim=8, num_quantizers=8, attention_head_dim=64,
                         in_channels=576, num_attention_heads=2, num_layers=2, num_layers_2=1, out_channels=256,
                         sample_rate=200, downsample_factors=[2, 2], downsample_kernel_sizes=[4, 4],
                         upsample_factors=[2, 2], upsample_kernel_sizes=[4, 4], latent_hidden_dim=128)


def _wn_pair(g: torch.Generator, out_shape, dim0: int, fan_in: int, pre: str, out: dict) -> None:
    """weight_norm(dim=0) parametrisation: original0 = g [dim0, 1, 1], original1 = v."""
    v = torch.randn(out_shape, generator=g) / fan_in ** 0.5
    norm = v.flatten(1).norm(dim=1).view(dim0, 1, 1)
    out[pre + ".parametrizations.weight.original0"] = norm * (1 + 0.1 * torch.randn(dim0, 1, 1, generator=g))
    out[pre + ".parametrizations.weight.original1"] = v


def synthetic_codec_tensors(cfg: CodecConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """A seeded random codec checkpoint (fp32) with the reference's keys and shapes."""
    g = torch.Generator().manual_seed(seed)
    t: dict[str, torch.Tensor] = {}

    def rnd(*shape, s=1.0):
        return torch.randn(*shape, generator=g) * s

    def lin(pre, n, k, bias=True):
        t[pre + ".weight"] = rnd(n, k, s=k ** -0.5)
        if bias:
            t[pre + ".bias"] = rnd(n, s=0.02)

    fm = "flow_matching."
    for q in range(cfg.num_quantizers):
        t[f"{fm}vq_embed.layers.{q}._codebook.embed"] = rnd(1, cfg.codebook_size, cfg.codebook_dim)
    lin(fm + "vq_embed.project_in", cfg.codebook_dim, cfg.dim)
    lin(fm + "vq_embed.project_out", cfg.dim, cfg.codebook_dim)
    lin(fm + "cond_feature_emb", cfg.dim, cfg.dim)
    t[fm + "zero_cond_embedding1"] = rnd(cfg.dim)
    est = fm + "estimator."
    D, D2, inc, out = cfg.inner, cfg.inner2, cfg.in_channels, cfg.out_channels

    def project(pre, cin, cout):
        t[pre + ".ffn_1.weight"] = rnd(cout, cin, 3, s=(3 * cin) ** -0.5)
        t[pre + ".ffn_1.bias"] = rnd(cout, s=0.02)
        lin(pre + ".ffn_2", cout, cout)

    def adaln(pre, d):
        lin(pre + ".emb.timestep_embedder.linear_1", d, 512)
        lin(pre + ".emb.timestep_embedder.linear_2", d, d)
        lin(pre + ".linear", 6 * d, d)

    def block(pre, d):
        f = CodecConfig.mlp_hidden(d)
        t[pre + ".attn_norm.weight"] = 1 + rnd(d, s=0.1)
        for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
            lin(f"{pre}.attn.{p}", d, d, bias=False)
        t[pre + ".mlp_norm.weight"] = 1 + rnd(d, s=0.1)
        lin(pre + ".mlp.gate", f, d, bias=False)
        lin(pre + ".mlp.up", f, d, bias=False)
        lin(pre + ".mlp.down", d, f, bias=False)
        t[pre + ".scale_shift_table"] = rnd(6, d, s=d ** -0.5)

    project(est + "proj_in", inc, D)
    adaln(est + "adaln_single", D)
    for i in range(cfg.num_layers):
        block(f"{est}transformer_blocks.{i}", D)
    project(est + "connection_proj", inc + D, D2)
    adaln(est + "adaln_single_2", D2)
    for i in range(cfg.num_layers_2):
        block(f"{est}transformer_blocks_2.{i}", D2)
    t[est + "scale_shift_table"] = rnd(2, D, s=D ** -0.5)
    t[est + "scale_shift_table_2"] = rnd(2, D2, s=D2 ** -0.5)
    project(est + "proj_out", D2, out)

    dec = "scalar_model.decoder."
    ch = cfg.decoder_channels()
    _wn_pair(g, (ch[0], cfg.latent_hidden_dim, cfg.delay_kernel_size), ch[0],
             cfg.latent_hidden_dim * cfg.delay_kernel_size, dec + "0", t)
    t[dec + "0.bias"] = rnd(ch[0], s=0.02)
    for i, (s, k) in enumerate(zip(cfg.upsample_factors, cfg.upsample_kernel_sizes)):
        pre = f"{dec}{i + 1}"
        cin, cout = ch[i], ch[i + 1]
        # ConvTranspose1d weight [cin, cout, k]: weight_norm(dim=0) normalises per input channel
        _wn_pair(g, (cin, cout, k), cin, cin * k // s, pre + ".up_conv.layer", t)
        t[pre + ".up_conv.layer.bias"] = rnd(cout, s=0.02)
        for j in range(5):
            u = f"{pre}.convs.{j}"
            _wn_pair(g, (cout, cout, cfg.res_kernel_size), cout, cout * cfg.res_kernel_size, u + ".conv1", t)
            t[u + ".conv1.bias"] = rnd(cout, s=0.02)
            _wn_pair(g, (cout, cout, 1), cout, cout, u + ".conv2", t)
            t[u + ".conv2.bias"] = rnd(cout, s=0.02)
            t[u + ".activation1.weight"] = 0.25 + rnd(1, s=0.05)
            t[u + ".activation2.weight"] = 0.25 + rnd(1, s=0.05)
    n = len(cfg.upsample_factors)
    if cfg.num_samples > 1:
        c = cfg.init_channel
        t[f"{dec}{n + 1}.conv.weight"] = rnd(c, c, cfg.default_kernel_size, s=(c * cfg.default_kernel_size) ** -0.5)
        t[f"{dec}{n + 1}.conv.bias"] = rnd(c, s=0.02)
        t[f"{dec}{n + 1}.activation.weight"] = 0.25 + rnd(1, s=0.05)
    last = f"{dec}{n + 2 if cfg.num_samples > 1 else n + 1}"
    _wn_pair(g, (cfg.num_bands, cfg.init_channel, cfg.default_kernel_size), cfg.num_bands,
             cfg.init_channel * cfg.default_kernel_size, last, t)
    t[last + ".bias"] = rnd(cfg.num_bands, s=0.02)
    return t


def load_codec_tensors(path) -> tuple[dict[str, torch.Tensor], CodecConfig]:
    """(tensors, config) of a codec checkpoint: a directory with ``config.json`` and
    ``model*.safetensors``, or one ``.safetensors`` file with a ``.json`` beside it
    (``app/codec_lite.py:13-26``).  Audio-encoder tensors are dropped."""
    from safetensors.torch import load_file
    path = Path(path)
    if path.is_dir():
        cfg = json.loads((path / "config.json").read_text())
        files = sorted(path.glob("model*.safetensors"))
    else:
        cfg = json.loads(path.with_suffix(".json").read_text())
        files = [path]
    t: dict[str, torch.Tensor] = {}
    for f in files:
        t.update({k: v for k, v in load_file(str(f)).items() if not k.startswith("scalar_model.encoder")})
    return t, CodecConfig.from_dict(cfg)
