"""CPU oracle of the HeartCodec detokenizer — TEST INFRASTRUCTURE ONLY.

A functional restatement, in fp32 torch on the CPU, of the reference codec that turns the
decoded ``[8, T]`` token streams into audio (``app/codec_lite.py:63-75`` ->
``HeartCodec.detokenize``, ``app/heartcodec/modeling_heartcodec.py:57-204``).  It is the
checker for the CUDA path (``estudiocanciones_b200/codec.py``), never a product code path:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import it.

Pieces, each citing the reference lines it restates:

* residual-VQ code lookup + ``project_out`` (``models/flow_matching.py:100-104``; the
  lookup itself is ``vector_quantize_pytorch.ResidualVQ.get_codes_from_indices``, a
  dependency the reference lists unpinned and that is absent here: its published
  behaviour, a per-quantizer gather, is restated), ``cond_feature_emb``, nearest
  up-sampling and the mask mix (``:105-131``);
* the LlamaTransformer estimator (``models/transformer.py:253-375``): ProjectLayer convs,
  ada-norm blocks with RoPE'd non-causal attention and SiLU-gated MLPs, output norms;
* ``solve_euler`` with classifier-free guidance (``models/flow_matching.py:161-210``);
* ``ScalarModel.decode`` (``models/sq_codec.py:506-510``): round(9x)/9, weight-normed
  convolutions, causal transposed convolutions, dilated residual units, PReLU, the
  PostProcessor's repeat;
* the window loop with in-context overlap and the linear cross-fade of ``detokenize``.

Parity of this oracle with the reference is pinned by ``tests/golden/codec.npz``, generated
by running the unmodified reference (``tests/golden/make_codec_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def weight_norm(sd: dict, pre: str) -> torch.Tensor:
    """w = g * v / ||v|| with the norm over every dim but 0 (torch weight_norm, dim=0);
    a plain ``pre.weight`` is returned as is."""
    if pre + ".weight" in sd:
        return sd[pre + ".weight"].float()
    g = sd[pre + ".parametrizations.weight.original0"].float()
    v = sd[pre + ".parametrizations.weight.original1"].float()
    n = v.flatten(1).norm(dim=1).view(-1, *([1] * (v.dim() - 1)))
    return v * (g / n)


def timestep_embedding(t: torch.Tensor, dim: int = 512, max_period: float = 10000.0, scale: float = 1000.0):
    """PixArtAlphaCombinedFlowEmbeddings.timestep_embedding (models/transformer.py:401-415)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(start=0, end=half) / half).type(t.type())
    args = t[:, None] * freqs[None] * scale
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def rope_tables(T: int, hd: int, base: float = 10000.0):
    """RotaryEmbedding.get_sin_cos in fp32 (models/transformer.py:27-40)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    t = torch.arange(T, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return freqs.sin(), freqs.cos()


class OracleCodec:
    def __init__(self, sd: dict, cfg):
        self.sd = {k: v.float() for k, v in sd.items()}
        self.cfg = cfg

    # ------------------------------------------------------------------ conditioning
    def vq_features(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [nq, n] -> cond_feature_emb(project_out(sum_q codebook_q[codes[q]])) [n, dim]
        (models/flow_matching.py:100-107)."""
        sd, fm = self.sd, "flow_matching."
        books = [sd[f"{fm}vq_embed.layers.{q}._codebook.embed"][0] for q in range(codes.shape[0])]
        s = sum(books[q][codes[q].long()] for q in range(codes.shape[0]))
        s = F.linear(s, sd[fm + "vq_embed.project_out.weight"], sd[fm + "vq_embed.project_out.bias"])
        return F.linear(s, sd[fm + "cond_feature_emb.weight"], sd[fm + "cond_feature_emb.bias"])

    # ------------------------------------------------------------------ estimator
    def _project(self, pre: str, x: torch.Tensor) -> torch.Tensor:
        """ProjectLayer: Conv1d(k=3, padding 1) * 3^-0.5 then Linear (models/transformer.py:205-220)."""
        sd = self.sd
        y = F.conv1d(x.transpose(1, 2), sd[pre + ".ffn_1.weight"], sd[pre + ".ffn_1.bias"], padding=1).transpose(1, 2)
        return F.linear(y * 3 ** -0.5, sd[pre + ".ffn_2.weight"], sd[pre + ".ffn_2.bias"])

    def _adaln(self, pre: str, t: torch.Tensor):
        """AdaLayerNormSingleFlow (models/transformer.py:420-443): (linear(silu(e)), e)."""
        sd = self.sd
        te = pre + ".emb.timestep_embedder."
        e = F.linear(timestep_embedding(t), sd[te + "linear_1.weight"], sd[te + "linear_1.bias"])
        e = F.linear(F.silu(e), sd[te + "linear_2.weight"], sd[te + "linear_2.bias"])
        return F.linear(F.silu(e), sd[pre + ".linear.weight"], sd[pre + ".linear.bias"]), e

    def _attention(self, pre: str, x: torch.Tensor, H: int, hd: int) -> torch.Tensor:
        """LlamaAttention without mask (models/transformer.py:84-146): RoPE on adjacent pairs
        of q and k, SDPA non-causal, o_proj."""
        sd = self.sd
        b, t, _ = x.shape

        def heads(w):
            return F.linear(x, sd[f"{pre}.{w}.weight"]).view(b, t, H, hd).transpose(1, 2)

        q, k, v = heads("q_proj"), heads("k_proj"), heads("v_proj")
        sin, cos = rope_tables(t, hd)

        def rope(u):
            u = u.reshape(b, H, t, hd // 2, 2)
            x1, x2 = u[..., 0], u[..., 1]
            s, c = sin.view(1, 1, t, hd // 2), cos.view(1, 1, t, hd // 2)
            return torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).view(b, H, t, hd)

        o = F.scaled_dot_product_attention(rope(q), rope(k), v)
        return F.linear(o.transpose(1, 2).reshape(b, t, H * hd), sd[f"{pre}.o_proj.weight"])

    def _block(self, pre: str, x: torch.Tensor, tmod: torch.Tensor, H: int, hd: int) -> torch.Tensor:
        """LlamaTransformerBlock with ada_norm_single (models/transformer.py:185-201)."""
        sd = self.sd
        B = x.shape[0]
        mods = (sd[pre + ".scale_shift_table"][None] + tmod.reshape(B, 6, -1)).chunk(6, dim=1)
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mods

        def rms(u, w):
            return sd[w] * (u * torch.rsqrt(u.pow(2).mean(-1, keepdim=True) + 1e-6))

        n = rms(x, pre + ".attn_norm.weight") * (1 + scale_msa) + shift_msa
        x = x + gate_msa * self._attention(pre + ".attn", n, H, hd)
        n = rms(x, pre + ".mlp_norm.weight") * (1 + scale_mlp) + shift_mlp
        m = F.silu(F.linear(n, sd[pre + ".mlp.gate.weight"])) * F.linear(n, sd[pre + ".mlp.up.weight"])
        return x + gate_mlp * F.linear(m, sd[pre + ".mlp.down.weight"])

    def estimator(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """LlamaTransformer.forward (models/transformer.py:300-375): x [B, T, in], t [B] -> [B, T, out]."""
        sd, cfg, est = self.sd, self.cfg, "flow_matching.estimator."
        H, hd = cfg.num_attention_heads, cfg.attention_head_dim
        s = self._project(est + "proj_in", x)
        tmod, e = self._adaln(est + "adaln_single", t)
        for i in range(cfg.num_layers):
            s = self._block(f"{est}transformer_blocks.{i}", s, tmod, H, hd)
        shift, scale = (sd[est + "scale_shift_table"][None] + e[:, None]).chunk(2, dim=1)
        s = F.layer_norm(s, (s.shape[-1],), eps=1e-6) * (1 + scale) + shift
        y = self._project(est + "connection_proj", torch.cat([x, s], dim=-1))
        tmod2, e2 = self._adaln(est + "adaln_single_2", t)
        for i in range(cfg.num_layers_2):
            y = self._block(f"{est}transformer_blocks_2.{i}", y, tmod2, H, 2 * hd)
        shift2, scale2 = (sd[est + "scale_shift_table_2"][None] + e2[:, None]).chunk(2, dim=1)
        y = F.layer_norm(y, (y.shape[-1],), eps=1e-6) * (1 + scale2) + shift2
        return self._project(est + "proj_out", y)

    # ------------------------------------------------------------------ flow matching
    def inference_codes(self, codes, true_latents, latent_length, incontext_length, guidance_scale, num_steps, randn):
        """FlowMatching.inference_codes with scenario "other_seg" + solve_euler
        (models/flow_matching.py:72-210).  codes [1, nq, n]; true_latents [1, T, out]."""
        cfg = self.cfg
        mu = self.vq_features(codes[0])  # [n, dim]
        mu = mu.repeat_interleave(2, dim=0)[None]  # F.interpolate(scale 2, nearest) along time
        T = mu.shape[1]
        latents = randn((1, T, cfg.out_channels), "device").float()
        masks = torch.zeros(1, T, dtype=torch.int64)
        masks[:, :latent_length] = 2
        masks[:, :incontext_length] = 1
        zero_cond = self.sd["flow_matching.zero_cond_embedding1"]
        mu = (masks > 0.5).unsqueeze(-1) * mu + (masks < 0.5).unsqueeze(-1) * zero_cond[None]
        inc_mask = ((masks > 0.5) * (masks < 1.5)).unsqueeze(-1).float()
        inc = true_latents.float() * inc_mask
        L_in = int(((masks > 0.5) * (masks < 1.5)).sum(-1)[0])
        t_span = torch.linspace(0, 1, num_steps + 1)
        x = latents.clone()
        noise = x.clone()
        t, dt = t_span[0], t_span[1] - t_span[0]
        for step in range(1, len(t_span)):
            x[:, :L_in] = (1 - (1 - 1e-6) * t) * noise[:, :L_in] + t * inc[:, :L_in]
            if guidance_scale > 1.0:
                inp = torch.cat([torch.cat([x, x]), torch.cat([inc, inc]), torch.cat([torch.zeros_like(mu), mu])], 2)
                d = self.estimator(inp, t.unsqueeze(-1).repeat(2))
                u, c = d.chunk(2, 0)
                d = u + guidance_scale * (c - u)
            else:
                d = self.estimator(torch.cat([x, inc, mu], 2), t.unsqueeze(-1))
            x = x + dt * d
            t = t + dt
            if step < len(t_span) - 1:
                dt = t_span[step + 1] - t
        x[:, :L_in] = inc[:, :L_in]
        return x

    # ------------------------------------------------------------------ waveform decoder
    def scalar_decode(self, x: torch.Tensor) -> torch.Tensor:
        """ScalarModel.decode (models/sq_codec.py:506-510): x [B, C, T] -> [B, bands, T * hop]."""
        sd, cfg, dec = self.sd, self.cfg, "scalar_model.decoder."
        x = torch.round(9 * x.float()) / 9
        k0 = cfg.delay_kernel_size
        x = F.conv1d(x, weight_norm(sd, dec + "0"), sd[dec + "0.bias"], padding=(k0 - 1) // 2)

        def causal(u, w, b, dil=1):
            return F.conv1d(F.pad(u, (dil * (w.shape[-1] - 1), 0)), w, b, dilation=dil)

        def prelu(u, a):
            return F.prelu(u, sd[a])

        n = len(cfg.upsample_factors)
        for i, s in enumerate(cfg.upsample_factors):
            pre = f"{dec}{i + 1}"
            x = F.conv_transpose1d(x, weight_norm(sd, pre + ".up_conv.layer"), sd[pre + ".up_conv.layer.bias"],
                                   stride=s)[:, :, :-s]
            for j, dil in enumerate((1, 3, 5, 7, 9)):
                u = f"{pre}.convs.{j}"
                y = prelu(causal(x, weight_norm(sd, u + ".conv1"), sd[u + ".conv1.bias"], dil), u + ".activation1.weight")
                y = prelu(causal(y, weight_norm(sd, u + ".conv2"), sd[u + ".conv2.bias"]), u + ".activation2.weight")
                x = y + x
        if cfg.num_samples > 1:
            pre = f"{dec}{n + 1}"
            b, c, t = x.shape
            x = x.transpose(1, 2).repeat(1, 1, cfg.num_samples).view(b, -1, c).transpose(1, 2)
            x = prelu(causal(x, sd[pre + ".conv.weight"], sd[pre + ".conv.bias"]), pre + ".activation.weight")
        last = f"{dec}{n + 2 if cfg.num_samples > 1 else n + 1}"
        return causal(x, weight_norm(sd, last), sd[last + ".bias"])

    # ------------------------------------------------------------------ detokenize
    def detokenize(self, codes: torch.Tensor, duration: float = 29.76, num_steps: int = 10,
                   guidance_scale: float = 1.25, randn=None) -> torch.Tensor:
        """HeartCodec.detokenize (modeling_heartcodec.py:57-204): codes [nq, n] -> [2, samples].
        ``randn(shape, where)`` draws the noise ("host" / "device" as the reference draws it)."""
        cfg = self.cfg
        randn = randn or (lambda shape, where: torch.randn(shape))
        codes = codes.unsqueeze(0).long()
        first_latent = randn((codes.shape[0], int(duration * 25), 256), "host")
        min_samples = int(duration * 12.5)
        hop_samples = min_samples // 93 * 80
        ovlp_samples = min_samples - hop_samples
        ovlp_frames = ovlp_samples * 2
        codes_len = codes.shape[-1]
        target_len = int(codes_len / 12.5 * cfg.sample_rate)
        if codes_len < min_samples:
            while codes.shape[-1] < min_samples:
                codes = torch.cat([codes, codes], -1)
            codes = codes[:, :, :min_samples]
        codes_len = codes.shape[-1]
        if (codes_len - ovlp_frames) % hop_samples > 0:
            len_codes = math.ceil((codes_len - ovlp_samples) / float(hop_samples)) * hop_samples + ovlp_samples
            while codes.shape[-1] < len_codes:
                codes = torch.cat([codes, codes], -1)
            codes = codes[:, :, :len_codes]
        latent_length = int(duration * 25)
        latents_list = []
        for sinx in range(0, codes.shape[-1] - hop_samples + 1, hop_samples):
            win = codes[:, :, sinx:sinx + min_samples]
            if sinx == 0 or ovlp_frames == 0:
                lat = self.inference_codes(win, first_latent, latent_length, 0, guidance_scale, num_steps, randn)
            else:
                true = latents_list[-1][:, -ovlp_frames:, :]
                extra = randn((true.shape[0], latent_length - true.shape[1], true.shape[-1]), "device").float()
                true = torch.cat([true, extra], 1)
                lat = self.inference_codes(win, true, latent_length, true.shape[1] - extra.shape[1],
                                           guidance_scale, num_steps, randn)
            latents_list.append(lat)
        min_audio = int(duration * cfg.sample_rate)
        hop_audio = min_audio // 93 * 80
        ovlp_audio = min_audio - hop_audio
        output = None
        for lat in latents_list:
            b, t, c = lat.shape
            z = lat.reshape(b, t, 2, c // 2).permute(0, 2, 1, 3).reshape(b * 2, t, c // 2)
            cur = self.scalar_decode(z.transpose(1, 2)).squeeze(0).squeeze(1)[:, :min_audio]
            if output is None:
                output = cur
            elif ovlp_audio == 0:
                output = torch.cat([output, cur], -1)
            else:
                w = torch.from_numpy(np.linspace(0, 1, ovlp_audio)[None, :])  # fp64, as the reference
                output[:, -ovlp_audio:] = (output[:, -ovlp_audio:].double() * (1 - w)
                                           + cur[:, :ovlp_audio].double() * w).float()
                output = torch.cat([output, cur[:, ovlp_audio:]], -1)
        return output[:, :target_len]
