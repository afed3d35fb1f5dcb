"""HeartCodec detokenize on the B200: the step after token generation, the codec that turns
the ``[8, T]`` token streams into audio.

Mirrors the reference's codec surface (``app/codec_lite.py``):

* :func:`load_codec` (``codec_lite.load_codec``, ``:13-33``) -> :class:`HeartCodecB200`;
* :meth:`HeartCodecB200.detokenize` (``HeartCodec.detokenize``,
  ``app/heartcodec/modeling_heartcodec.py:57-204``): windows of 29.76 s with an in-context
  overlap, each a flow-matching Euler solve (``models/flow_matching.py:72-210``) over the
  LlamaTransformer estimator (``models/transformer.py:253-375``), then the ScalarModel
  waveform decoder (``models/sq_codec.py:506-510``) and a linear cross-fade;
* :func:`decode` (``codec_lite.decode``, ``:63-75``): codes clamped to the codebook, default
  10 steps and guidance 1.25.

Every GEMM-shaped layer (linear, ProjectLayer conv, decoder conv, causal transposed conv,
the PostProcessor's repeat + conv) runs through ``hm_conv1d_gemm``, the implicit-GEMM
convolution on the 5th-generation tensor cores, with its bias / scale / PReLU / SiLU /
RoPE / gated-residual / residual epilogue fused; attention through ``hm_codec_attn``
(tcgen05, non-causal, head dims 64 and 128); norms, the VQ lookup, the Euler update, the
band quantiser and the cross-fade through the small kernels of ``csrc/codec.cu``.  The
weights are converted once at load: weight norms folded, q|k|v and gate|up fused, the
transposed and repeat convolutions laid out as taps, the per-block ada-norm tables folded
into the biases of their timestep projections.  Activations are fp16 with fp32
accumulation; the residual streams of the estimator and the latents are fp32.

Host work per window: the noise draws (the reference's ``torch.randn`` calls, in its order
and shapes, so a seeded run draws the same noise), a few device copies and the replay of a
prebuilt list of kernel calls (optionally one CUDA graph).  No step runs on the CPU and
there is no fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import _lib as L
from .codec_checkpoint import CodecConfig, load_codec_tensors

_DIL = (1, 3, 5, 7, 9)  # ResidualUnit dilations of a ResDecoderBlock (sq_codec.py:212-244)


def _ptr(t) -> int:
    return t if isinstance(t, int) else t.data_ptr()


def _wn(sd: dict, pre: str) -> torch.Tensor:
    """Weight-norm fold w = g v / ||v|| (norm over every dim but 0), fp32; plain weights pass."""
    if pre + ".weight" in sd:
        return sd[pre + ".weight"].float()
    if pre + ".weight_g" in sd:
        g, v = sd[pre + ".weight_g"].float(), sd[pre + ".weight_v"].float()
    else:
        g = sd[pre + ".parametrizations.weight.original0"].float()
        v = sd[pre + ".parametrizations.weight.original1"].float()
    n = v.flatten(1).norm(dim=1).view(-1, *([1] * (v.dim() - 1)))
    return v * (g / n)


class _Layer:
    """One layer in hm_conv1d_gemm's layout: fp16 weights [taps, npad, cin], fp32 bias."""

    def __init__(self, w_taps: torch.Tensor, bias, dev, off0: int = 0, dil: int = 1):
        taps, n, cin = w_taps.shape
        if cin % 64:
            raise ValueError(f"layer input width {cin} is not a multiple of 64")
        npad = (n + 63) // 64 * 64
        w = torch.zeros(taps, npad, cin, dtype=torch.float16, device=dev)
        w[:, :n] = w_taps.to(dev, torch.float32).to(torch.float16)
        self.w, self.N, self.npad, self.cin, self.taps, self.off0, self.dil = w, n, npad, cin, taps, off0, dil
        self.bias = None if bias is None else bias.to(dev, torch.float32).contiguous()

    @classmethod
    def linear(cls, w, b, dev):
        return cls(w.float()[None], b, dev)

    @classmethod
    def conv(cls, w, b, dev, pad_left: int, dil: int = 1):
        """Conv1d weight [Cout, Cin, k]; input row of tap j = t - pad_left + j*dil."""
        return cls(w.float().permute(2, 0, 1), b, dev, off0=-pad_left, dil=dil)

    def desc(self, x, x_ld, B, T, tin, y, y_ld, *, x_bstride=None, scale=1.0, act=L.HM_ACT_NONE, prelu=1.0,
             epi=L.HM_CEPI_STORE, res=None, res_ld=0, gate=None, gate_ld=0, rope=None, rope_cols=0, hd=0,
             y_f32=False, bn=0, err=None) -> L.ConvDesc:
        d = L.ConvDesc()
        d.x, d.x_ld = _ptr(x), x_ld
        d.x_bstride = tin * x_ld if x_bstride is None else x_bstride
        d.w = self.w.data_ptr()
        d.bias = 0 if self.bias is None else self.bias.data_ptr()
        d.y, d.y_ld = _ptr(y), y_ld
        d.res, d.res_ld = (0 if res is None else _ptr(res)), res_ld
        d.gate, d.gate_ld = (0 if gate is None else _ptr(gate)), gate_ld
        d.rope = 0 if rope is None else _ptr(rope)
        d.err = 0 if err is None else _ptr(err)
        d.B, d.T, d.tin, d.cin, d.N, d.npad = B, T, tin, self.cin, self.N, self.npad
        d.taps, d.off0, d.dil = self.taps, self.off0, self.dil
        d.scale, d.prelu = scale, prelu
        d.act, d.epi, d.y_f32, d.rope_cols, d.hd, d.bn = act, epi, int(y_f32), rope_cols, hd, bn
        return d


class _Plan:
    """A prebuilt list of library calls (pointers and sizes bound), replayed on a stream."""

    def __init__(self):
        self.calls: list = []
        self.keep: list = []

    def conv(self, layer: _Layer, *args, **kw):
        d = layer.desc(*args, **kw)
        self.keep.append(d)
        self.calls.append(("hm_conv1d_gemm", (C.byref(d),)))

    def add(self, name: str, *args):
        self.calls.append((name, tuple(_ptr(a) if isinstance(a, torch.Tensor) else a for a in args)))

    def run(self, stream: int) -> None:
        lib = L.lib()
        for name, args in self.calls:
            L.check(getattr(lib, name)(*args, stream), name)


def _block_layers(sd: dict, pre: str, d: int, dev):
    """Fused q|k|v, o, gate|up (blocks of 128 features: 128 gate rows then the same 128
    features' up rows) and down projections of one LlamaTransformerBlock."""
    qkv = torch.cat([sd[f"{pre}.attn.{p}.weight"].float() for p in ("q_proj", "k_proj", "v_proj")])
    gate, up = sd[pre + ".mlp.gate.weight"].float(), sd[pre + ".mlp.up.weight"].float()
    f = gate.shape[0]
    if f % 128:
        raise ValueError(f"MLP width {f} is not a multiple of 128")
    gu = torch.stack([gate.view(f // 128, 128, d), up.view(f // 128, 128, d)], 1).reshape(2 * f, d)
    return dict(qkv=_Layer.linear(qkv, None, dev), o=_Layer.linear(sd[pre + ".attn.o_proj.weight"], None, dev),
                gu=_Layer.linear(gu, None, dev), down=_Layer.linear(sd[pre + ".mlp.down.weight"], None, dev),
                attn_norm=sd[pre + ".attn_norm.weight"].to(dev, torch.float32).contiguous(),
                mlp_norm=sd[pre + ".mlp_norm.weight"].to(dev, torch.float32).contiguous(),
                table=sd[pre + ".scale_shift_table"].float().reshape(-1), f=f)


class _Stage:
    """One transformer stage of the estimator: its timestep embedding, blocks and output norm."""

    def __init__(self, sd: dict, est: str, suffix: str, nlayers: int, d: int, heads: int, hd: int, dev):
        ada = f"{est}adaln_single{suffix}"
        te = ada + ".emb.timestep_embedder."
        self.d, self.heads, self.hd = d, heads, hd
        self.lin1 = _Layer.linear(sd[te + "linear_1.weight"], sd[te + "linear_1.bias"], dev)
        self.lin2 = _Layer.linear(sd[te + "linear_2.weight"], sd[te + "linear_2.bias"], dev)
        blocks = "transformer_blocks" + suffix
        self.blocks = [_block_layers(sd, f"{est}{blocks}.{i}", d, dev) for i in range(nlayers)]
        w_ada, b_ada = sd[ada + ".linear.weight"].float(), sd[ada + ".linear.bias"].float()
        # per block: linear(silu(e)) + bias + the block's scale_shift_table (transformer.py:185-189)
        self.ada = [_Layer.linear(w_ada, b_ada + blk["table"], dev) for blk in self.blocks]
        self.out_table = sd[f"{est}scale_shift_table{suffix}"].to(dev, torch.float32).contiguous()
        self.f = self.blocks[0]["f"] if self.blocks else 0


def _rope_table(T: int, hd: int, dev) -> torch.Tensor:
    """(cos, sin) pairs [T, hd/2] in fp32 (RotaryEmbedding.get_sin_cos, transformer.py:27-40)."""
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32, device=dev) / hd))
    freqs = torch.einsum("i,j->ij", torch.arange(T, dtype=torch.float32, device=dev), inv_freq)
    return torch.stack([freqs.cos(), freqs.sin()], -1).contiguous()


def _timestep_embedding(t: torch.Tensor, dim: int = 512) -> torch.Tensor:
    """PixArtAlphaCombinedFlowEmbeddings.timestep_embedding (transformer.py:401-415), fp32 on
    the host: the sinusoid of the solver's timesteps, the input of the timestep projections."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000) * torch.arange(start=0, end=half) / half).type(t.type())
    args = t[:, None] * freqs[None] * 1000
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def euler_schedule(num_steps: int):
    """(t_k, dt_k) of solve_euler's loop in fp32 (flow_matching.py:172-207): t_span = linspace(0, 1,
    n + 1); dt re-derived from t_span each step, t accumulated."""
    t_span = torch.linspace(0, 1, num_steps + 1)
    t, dt = t_span[0], t_span[1] - t_span[0]
    ts, dts = [], []
    for step in range(1, num_steps + 1):
        ts.append(float(t))
        dts.append(float(dt))
        t = t + dt
        if step < num_steps:
            dt = t_span[step + 1] - t
    ts.append(float(t))
    return ts, dts


class HeartCodecB200:
    """The codec on one B200 (``HeartCodec`` minus its audio encoder)."""

    def __init__(self, tensors: dict, config, device="cuda", graphs: bool = True):
        self.cfg = config if isinstance(config, CodecConfig) else CodecConfig.from_dict(config)
        self.use_graphs = graphs
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise L.HMError("HeartCodecB200 runs on a CUDA device; there is no CPU path")
        L.lib()
        cfg, dev, sd = self.cfg, self.dev, tensors
        if cfg.in_channels != 2 * cfg.out_channels + cfg.dim:
            raise ValueError("in_channels must be 2 * out_channels + dim (latents, in-context latents, features)")
        if cfg.out_channels != 2 * cfg.latent_hidden_dim:
            raise ValueError("the latents split into two bands of latent_hidden_dim channels")
        self.sample_rate = cfg.sample_rate
        self.dtype = torch.float16
        fm, est = "flow_matching.", "flow_matching.estimator."
        nq = cfg.num_quantizers
        self.codebooks = torch.stack([sd[f"{fm}vq_embed.layers.{q}._codebook.embed"].float().reshape(
            cfg.codebook_size, cfg.codebook_dim) for q in range(nq)]).to(dev).contiguous()
        self.proj_w = sd[fm + "vq_embed.project_out.weight"].to(dev, torch.float32).contiguous()
        self.proj_b = sd[fm + "vq_embed.project_out.bias"].to(dev, torch.float32).contiguous()
        self.cond = _Layer.linear(sd[fm + "cond_feature_emb.weight"], sd[fm + "cond_feature_emb.bias"], dev)
        self.zero_cond = sd[fm + "zero_cond_embedding1"].to(dev, torch.float16).reshape(1, -1).contiguous()

        def project(pre):
            return (_Layer.conv(sd[pre + ".ffn_1.weight"], sd[pre + ".ffn_1.bias"], dev, pad_left=1),
                    _Layer.linear(sd[pre + ".ffn_2.weight"], sd[pre + ".ffn_2.bias"], dev))

        self.proj_in = project(est + "proj_in")
        self.connection = project(est + "connection_proj")
        self.proj_out = project(est + "proj_out")
        H, hd = cfg.num_attention_heads, cfg.attention_head_dim
        self.st1 = _Stage(sd, est, "", cfg.num_layers, cfg.inner, H, hd, dev)
        self.st2 = _Stage(sd, est, "_2", cfg.num_layers_2, cfg.inner2, H, 2 * hd, dev)
        self._prep_decoder(sd)
        self._plans: dict = {}
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    # ------------------------------------------------------------------ decoder weights
    def _prep_decoder(self, sd: dict) -> None:
        cfg, dev, dec = self.cfg, self.dev, "scalar_model.decoder."
        if not cfg.causal:
            raise ValueError("only the causal waveform decoder (the released codec's) is supported")
        k0 = cfg.delay_kernel_size
        self.dec0 = _Layer.conv(_wn(sd, dec + "0"), sd[dec + "0.bias"], dev, pad_left=(k0 - 1) // 2)
        self.stages = []
        ch = cfg.decoder_channels()
        for i, (s, k) in enumerate(zip(cfg.upsample_factors, cfg.upsample_kernel_sizes)):
            pre = f"{dec}{i + 1}"
            if k != 2 * s:
                raise ValueError("a causal ConvTranspose1d has kernel 2 * stride")
            w = _wn(sd, pre + ".up_conv.layer")  # [cin, cout, 2s]
            cin, cout = w.shape[0], w.shape[1]
            # output phase j of input row t: x[t] w[:, :, j] + x[t - 1] w[:, :, j + s]
            taps = torch.stack([w[:, :, :s].permute(2, 1, 0).reshape(s * cout, cin),
                                w[:, :, s:].permute(2, 1, 0).reshape(s * cout, cin)])
            up = _Layer(taps, sd[pre + ".up_conv.layer.bias"].float().repeat(s), dev, off0=0, dil=-1)
            units = []
            for j, dil in enumerate(_DIL):
                u = f"{pre}.convs.{j}"
                c1 = _Layer.conv(_wn(sd, u + ".conv1"), sd[u + ".conv1.bias"], dev,
                                 pad_left=dil * (cfg.res_kernel_size - 1), dil=dil)
                c2 = _Layer.conv(_wn(sd, u + ".conv2"), sd[u + ".conv2.bias"], dev, pad_left=0)
                units.append((c1, float(sd[u + ".activation1.weight"].reshape(-1)[0]),
                              c2, float(sd[u + ".activation2.weight"].reshape(-1)[0])))
            self.stages.append((s, cout, up, units))
        n = len(cfg.upsample_factors)
        self.post = None
        if cfg.num_samples > 1:
            pre, r, kk = f"{dec}{n + 1}", cfg.num_samples, cfg.default_kernel_size
            w = sd[pre + ".conv.weight"].float()  # [c, c, k] on the r-times repeated rows
            c = w.shape[0]
            # out[r u + phi] = sum_k w_k x[u + floor((phi + k - (k - 1)) / r)]: taps over the unrepeated rows
            dmin = -((kk - 1) // r) - (1 if (kk - 1) % r else 0)
            taps = torch.zeros(1 - dmin, r * c, w.shape[1])
            for phi in range(r):
                for k in range(kk):
                    dd = (phi + k - (kk - 1)) // r
                    taps[dd - dmin, phi * c:(phi + 1) * c] += w[:, :, k]
            self.post = (_Layer(taps, sd[pre + ".conv.bias"].float().repeat(r), dev, off0=dmin, dil=1), r, c,
                         float(sd[pre + ".activation.weight"].reshape(-1)[0]))
        last = f"{dec}{n + 2 if cfg.num_samples > 1 else n + 1}"
        kk = cfg.default_kernel_size
        self.final = _Layer.conv(_wn(sd, last), sd[last + ".bias"], dev, pad_left=kk - 1)

    # ------------------------------------------------------------------ plans
    def _flow_plan(self, n_codes: int, nb: int, latent_length: int, L_in: int, steps: int, g: float) -> dict:
        """Buffers and the call list of one window's solve: VQ features, then per Euler step
        the estimator and the update."""
        key = ("flow", n_codes, nb, latent_length, L_in, steps, g)
        if key in self._plans:
            return self._plans[key]
        cfg, dev = self.cfg, self.dev
        T, Cl, dim = 2 * n_codes, cfg.out_channels, cfg.dim
        D1, D2, inch = cfg.inner, cfg.inner2, cfg.in_channels
        XW = inch + D1  # estimator input + the first stage's normed output (connection_proj's input)
        R = nb * T
        f16, f32 = torch.float16, torch.float32
        b = dict(codes=torch.zeros(cfg.num_quantizers, n_codes, dtype=torch.int64, device=dev),
                 pq=torch.empty(n_codes, dim, dtype=f16, device=dev),
                 cf=torch.empty(n_codes, dim, dtype=f16, device=dev),
                 xin=torch.zeros(nb, T, XW, dtype=f16, device=dev),
                 x=torch.zeros(T, Cl, dtype=f32, device=dev), noise=torch.zeros(T, Cl, dtype=f32, device=dev),
                 inc=torch.zeros(max(L_in, 1), Cl, dtype=f32, device=dev),
                 s16=torch.empty(R, D2, dtype=f16, device=dev), h=torch.empty(R, D2, dtype=f32, device=dev),
                 hn=torch.empty(R, D2, dtype=f16, device=dev),
                 qkv=torch.empty(R, 3 * D2, dtype=f16, device=dev), att=torch.empty(R, D2, dtype=f16, device=dev),
                 mlp=torch.empty(R, max(self.st1.f, self.st2.f), dtype=f16, device=dev),
                 p16=torch.empty(R, Cl, dtype=f16, device=dev), v=torch.empty(R, Cl, dtype=f32, device=dev),
                 rope1=_rope_table(T, self.st1.hd, dev), rope2=_rope_table(T, self.st2.hd, dev))
        ts, dts = euler_schedule(steps)
        mods = self._mod_tables(tuple(ts[:steps]))
        P = _Plan()
        xin = b["xin"]
        # conditioning features (flow_matching.py:100-131): VQ sum + project_out, cond_feature_emb,
        # nearest x2 along time into the conditional item's feature columns; frames past
        # latent_length take zero_cond
        P.add("hm_codec_vq_embed", b["codes"], n_codes, cfg.num_quantizers, n_codes, self.codebooks,
              cfg.codebook_size, cfg.codebook_dim, self.proj_w, self.proj_b, b["pq"], dim, dim)
        P.conv(self.cond, b["pq"], dim, 1, n_codes, n_codes, b["cf"], dim)
        mu = xin[nb - 1, :, 2 * Cl:2 * Cl + dim]
        P.add("hm_codec_upsample_rows", b["cf"], dim, n_codes, dim, 2, mu, XW)
        if latent_length < T:
            P.add("hm_codec_upsample_rows", self.zero_cond, dim, 1, dim, T - latent_length,
                  xin[nb - 1, latent_length:, 2 * Cl:], XW)
        inc_ptr = b["inc"] if L_in > 0 else 0
        P.add("hm_codec_euler", 0, nb, b["x"], b["noise"], inc_ptr, T, Cl, L_in, 0.0, 0.0, ts[0], 0, xin, XW, T * XW)
        for k in range(steps):
            self._estimator_calls(P, b, mods, k, nb, T)
            final = int(k == steps - 1)
            P.add("hm_codec_euler", b["v"], nb, b["x"], b["noise"], inc_ptr, T, Cl, L_in, dts[k], g, ts[k + 1],
                  final, xin, XW, T * XW)
        plan = dict(P=P, b=b, mods=mods, T=T)
        self._plans[key] = plan
        return plan

    def _mod_tables(self, ts: tuple) -> dict:
        """The modulation vectors of every block at each timestep of ``ts`` (fp32 [steps, 6D] per
        block) and the output norms' shift/scale (the same for every window of a call)."""
        key = ("mods", ts)
        if key in self._plans:
            return self._plans[key]
        dev, steps = self.dev, len(ts)
        rows = max(steps, 128)  # the GEMM inputs hold a whole 128-row tile (zero rows past steps)
        emb = torch.zeros(rows, 512, dtype=torch.float16, device=dev)
        emb[:steps] = _timestep_embedding(torch.tensor(ts, dtype=torch.float32)).to(dev, torch.float16)
        out = dict(emb=emb)
        P = _Plan()
        for name, st in (("st1", self.st1), ("st2", self.st2)):
            d = st.d
            a = torch.zeros(rows, d, dtype=torch.float16, device=dev)
            E = torch.empty(steps, d, dtype=torch.float32, device=dev)
            se = torch.zeros(rows, d, dtype=torch.float16, device=dev)
            shift = torch.empty(steps, d, dtype=torch.float32, device=dev)
            scale = torch.empty(steps, d, dtype=torch.float32, device=dev)
            P.conv(st.lin1, emb, 512, 1, steps, rows, a, d, act=L.HM_ACT_SILU)
            P.conv(st.lin2, a, d, 1, steps, rows, E, d, y_f32=True)
            P.add("hm_codec_temb_post", E, steps, d, st.out_table, se, shift, scale)
            mods = []
            for lay in st.ada:
                m = torch.empty(steps, 6 * d, dtype=torch.float32, device=dev)
                P.conv(lay, se, d, 1, steps, rows, m, 6 * d, y_f32=True)
                mods.append(m)
            out[name] = dict(tmp=(a, E, se), shift=shift, scale=scale, mods=mods)
        P.run(torch.cuda.current_stream(dev).cuda_stream)
        self._plans[key] = out
        return out

    def _estimator_calls(self, P: _Plan, b: dict, mods: dict, k: int, nb: int, T: int) -> None:
        """LlamaTransformer.forward (transformer.py:300-375) at timestep index k on the nb items."""
        cfg = self.cfg
        Cl, inch, D1 = cfg.out_channels, cfg.in_channels, cfg.inner
        XW = inch + D1
        R = nb * T
        xin = b["xin"]
        c1, l1 = self.proj_in
        P.conv(c1, xin, XW, nb, T, T, b["s16"], D1, x_bstride=T * XW, scale=3 ** -0.5)
        P.conv(l1, b["s16"], D1, 1, R, R, b["h"], D1, y_f32=True)
        self._stage_calls(P, b, self.st1, mods["st1"], k, nb, T, b["rope1"])
        m1 = mods["st1"]
        P.add("hm_codec_norm_mod", b["h"], D1, 0, m1["shift"][k], m1["scale"][k], 0, xin[:, :, inch:], XW, nb, T,
              D1, 1e-6, 1)
        D2 = cfg.inner2
        c2, l2 = self.connection
        P.conv(c2, xin, XW, nb, T, T, b["s16"], D2, x_bstride=T * XW, scale=3 ** -0.5)
        P.conv(l2, b["s16"], D2, 1, R, R, b["h"], D2, y_f32=True)
        self._stage_calls(P, b, self.st2, mods["st2"], k, nb, T, b["rope2"])
        m2 = mods["st2"]
        P.add("hm_codec_norm_mod", b["h"], D2, 0, m2["shift"][k], m2["scale"][k], 0, b["hn"], D2, nb, T, D2, 1e-6, 1)
        c3, l3 = self.proj_out
        P.conv(c3, b["hn"], D2, nb, T, T, b["p16"], Cl, scale=3 ** -0.5)
        P.conv(l3, b["p16"], Cl, 1, R, R, b["v"], Cl, y_f32=True)

    def _stage_calls(self, P: _Plan, b: dict, st: _Stage, m: dict, k: int, nb: int, T: int, rope) -> None:
        """The ada-norm blocks of one stage (transformer.py:185-201)."""
        d, H, hd, R = st.d, st.heads, st.hd, nb * T
        h, hn, qkv, att, mlp = b["h"], b["hn"], b["qkv"], b["att"], b["mlp"]
        for blk, mod in zip(st.blocks, m["mods"]):
            row = mod[k]  # [6d]: shift/scale/gate of attention, shift/scale/gate of the MLP
            P.add("hm_codec_norm_mod", h, d, blk["attn_norm"], row[0:d], row[d:2 * d], 0, hn, d, nb, T, d, 1e-6, 0)
            # per item (RoPE angle of the row's position in its item)
            P.conv(blk["qkv"], hn, d, nb, T, T, qkv, 3 * d, x_bstride=T * d, epi=L.HM_CEPI_ROPE, rope=rope,
                   rope_cols=2 * d, hd=hd)
            P.add("hm_codec_attn", qkv, qkv[:, d:], qkv[:, 2 * d:], att, nb, T, H, hd, 3 * d, d, hd ** -0.5,
                  self.err)
            P.conv(blk["o"], att, d, 1, R, R, h, d, epi=L.HM_CEPI_GATED, res=h, res_ld=d, gate=row[2 * d:3 * d],
                   y_f32=True)
            P.add("hm_codec_norm_mod", h, d, blk["mlp_norm"], row[3 * d:4 * d], row[4 * d:5 * d], 0, hn, d, nb, T, d,
                  1e-6, 0)
            P.conv(blk["gu"], hn, d, 1, R, R, mlp, blk["f"], epi=L.HM_CEPI_SILU)
            P.conv(blk["down"], mlp, blk["f"], 1, R, R, h, d, epi=L.HM_CEPI_GATED, res=h, res_ld=d,
                   gate=row[5 * d:6 * d], y_f32=True)

    def _decoder_plan(self, T: int) -> dict:
        """Buffers and calls of ScalarModel.decode (sq_codec.py:506-510) on the two latent
        bands of one window (T latent frames): x [T, 2 Cb] fp32 -> wave [2, T * hop] fp32."""
        key = ("dec", T)
        if key in self._plans:
            return self._plans[key]
        cfg, dev = self.cfg, self.dev
        Cb = cfg.latent_hidden_dim
        nband = cfg.out_channels // Cb
        sizes = [T * self.dec0.N]
        t = T
        for s, cout, _, _ in self.stages:
            t *= s
            sizes.append(t * cout)
        if self.post is not None:
            sizes.append(t * self.post[1] * self.post[2])
        big = max(sizes) * nband
        bufs = [torch.empty(big, dtype=torch.float16, device=dev) for _ in range(3)]
        S = T * cfg.hop
        b = dict(xin=torch.empty(T, cfg.out_channels, dtype=torch.float32, device=dev),
                 q=torch.empty(nband, T, Cb, dtype=torch.float16, device=dev),
                 wave=torch.empty(nband, S, dtype=torch.float32, device=dev), bufs=bufs)
        P = _Plan()
        P.add("hm_codec_band_quant", b["xin"], T, Cb, nband, b["q"])
        X, Y, Tm = bufs
        c0 = self.dec0.N
        P.conv(self.dec0, b["q"], Cb, nband, T, T, X, c0)
        t, c = T, c0
        for s, cout, up, units in self.stages:
            # causal ConvTranspose1d: rows t of s*cout columns = rows s t .. s t + s - 1 of cout
            P.conv(up, X, c, nband, t, t, Y, s * cout)
            t, c = t * s, cout
            for c1, a1, c2, a2 in units:
                P.conv(c1, Y, c, nband, t, t, Tm, c, act=L.HM_ACT_PRELU, prelu=a1)
                P.conv(c2, Tm, c, nband, t, t, Y, c, act=L.HM_ACT_PRELU, prelu=a2, epi=L.HM_CEPI_RES, res=Y,
                       res_ld=c)
            X, Y = Y, X
        if self.post is not None:
            lay, r, cp, a = self.post
            P.conv(lay, X, c, nband, t, t, Y, r * cp, act=L.HM_ACT_PRELU, prelu=a)
            t, c = t * r, cp
            X, Y = Y, X
        P.conv(self.final, X, c, nband, t, t, b["wave"], 1, y_f32=True)
        plan = dict(P=P, b=b, S=S)
        self._plans[key] = plan
        return plan

    # ------------------------------------------------------------------ API
    def scalar_decode(self, latent: torch.Tensor) -> torch.Tensor:
        """ScalarModel.decode of one window's latents [T, out_channels] (fp32 device tensor):
        the two bands -> [2, T * hop] fp32."""
        T = latent.shape[0]
        plan = self._decoder_plan(T)
        plan["b"]["xin"].copy_(latent)
        self._exec(plan)
        return plan["b"]["wave"]

    def estimator(self, x: torch.Tensor, t: float) -> torch.Tensor:
        """One estimator forward (test hook): x [nb, T, in_channels] (nb items, one timestep
        t for all) -> [nb, T, out_channels] fp32."""
        nb, T, _ = x.shape
        key = ("est", nb, T, float(t))
        if key not in self._plans:
            cfg, dev = self.cfg, self.dev
            D2, Cl = cfg.inner2, cfg.out_channels
            R, XW = nb * T, cfg.in_channels + cfg.inner
            f16, f32 = torch.float16, torch.float32
            b = dict(xin=torch.zeros(nb, T, XW, dtype=f16, device=dev), s16=torch.empty(R, D2, dtype=f16, device=dev),
                     h=torch.empty(R, D2, dtype=f32, device=dev), hn=torch.empty(R, D2, dtype=f16, device=dev),
                     qkv=torch.empty(R, 3 * D2, dtype=f16, device=dev), att=torch.empty(R, D2, dtype=f16, device=dev),
                     mlp=torch.empty(R, max(self.st1.f, self.st2.f), dtype=f16, device=dev),
                     p16=torch.empty(R, Cl, dtype=f16, device=dev), v=torch.empty(R, Cl, dtype=f32, device=dev),
                     rope1=_rope_table(T, self.st1.hd, dev), rope2=_rope_table(T, self.st2.hd, dev))
            mods = self._mod_tables((float(t),))
            P = _Plan()
            self._estimator_calls(P, b, mods, 0, nb, T)
            self._plans[key] = dict(P=P, b=b, mods=mods)
        plan = self._plans[key]
        plan["b"]["xin"][:, :, :self.cfg.in_channels].copy_(x)
        plan["P"].run(torch.cuda.current_stream(self.dev).cuda_stream)
        return plan["b"]["v"].view(nb, T, -1)

    def detokenize(self, codes: torch.Tensor, duration: float = 29.76, num_steps: int = 10,
                   disable_progress: bool = False, guidance_scale: float = 1.25, abort_signal=None, randn=None):
        """HeartCodec.detokenize (modeling_heartcodec.py:57-204): codes [nq, n] -> audio
        [2, n / 12.5 * sample_rate] (fp32, on the device), or None when ``abort_signal()``.

        ``randn(shape, where)`` draws the noise; by default ``torch.randn`` in the codec's
        dtype on the host (``where == "host"``) or on the device, in the reference's order and
        shapes, so a run after ``torch.manual_seed`` draws what the reference draws."""
        if abort_signal and abort_signal():
            return None
        cfg, dev = self.cfg, self.dev
        stream = torch.cuda.current_stream(dev).cuda_stream
        if randn is None:
            def randn(shape, where):
                return torch.randn(shape, dtype=self.dtype, device=dev if where == "device" else "cpu")
        codes = codes.to(dev).long().unsqueeze(0)
        randn((codes.shape[0], int(duration * 25), cfg.out_channels), "host")  # first_latent: masked out
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
        nb = 2 if guidance_scale > 1.0 else 1
        T = 2 * min_samples
        min_audio = int(duration * cfg.sample_rate)
        hop_audio = min_audio // 93 * 80
        ovlp_audio = min_audio - hop_audio
        starts = list(range(0, codes.shape[-1] - hop_samples + 1, hop_samples))
        total = min_audio + (len(starts) - 1) * hop_audio
        out = torch.empty(2, total, dtype=torch.float32, device=dev)
        prev = None
        for w, sinx in enumerate(starts):
            if abort_signal and abort_signal():
                return None
            first = sinx == 0 or ovlp_frames == 0
            L_in = 0 if first else ovlp_frames
            if not first:
                randn((1, latent_length - ovlp_frames, cfg.out_channels), "device")  # masked out
            plan = self._flow_plan(min_samples, nb, latent_length, L_in, num_steps, float(guidance_scale))
            b = plan["b"]
            b["codes"].copy_(codes[0, :, sinx:sinx + min_samples])
            b["noise"].copy_(randn((1, T, cfg.out_channels), "device")[0])
            if L_in:
                b["inc"].copy_(prev[-ovlp_frames:])
            self._exec(plan)
            lat = b["x"]
            wave = self.scalar_decode(lat)
            n = min(min_audio, wave.shape[1])
            L.check(L.lib().hm_codec_overlap_add(wave.data_ptr(), wave.shape[1], out.data_ptr(), total, 2,
                                                 0 if first else w * hop_audio, n, 0 if first else ovlp_audio,
                                                 stream), "hm_codec_overlap_add")
            prev = lat.clone() if len(starts) > 1 else lat
        return out[:, :target_len]

    def _exec(self, plan: dict) -> None:
        """Run a plan on the current stream: eagerly the first time (library set-up happens
        outside any capture), then as one CUDA graph captured from it."""
        stream = torch.cuda.current_stream(self.dev)
        g = plan.get("graph")
        if g is not None:
            g.replay()
            return
        plan["P"].run(stream.cuda_stream)
        if not self.use_graphs:
            return
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(stream)
        with L.capture_graph(g, side):
            plan["P"].run(side.cuda_stream)
        stream.wait_stream(side)
        plan["graph"] = g

    def n_launches(self, plan_key) -> int:
        """Kernels one run of a plan launches."""
        return len(self._plans[plan_key]["P"].calls)

    def release(self) -> None:
        """Free the per-shape buffers, call lists and graphs (weights stay)."""
        for plan in self._plans.values():
            plan.pop("graph", None)
        self._plans.clear()


def estimator_flops(cfg: CodecConfig, nb: int, T: int) -> int:
    """Multiply-add FLOPs of one estimator forward over nb items of T frames: every GEMM
    (ProjectLayer convs and linears, q|k|v, o, gate|up, down) plus attention (QK^T and PV)."""
    R = nb * T
    D1, D2, inc, out = cfg.inner, cfg.inner2, cfg.in_channels, cfg.out_channels

    def blocks(n, d, hd):
        f = CodecConfig.mlp_hidden(d)
        per = 2 * R * d * (3 * d + d + 2 * f) + 2 * R * f * d + 4 * nb * (d // hd) * T * T * hd
        return n * per

    fl = 2 * R * inc * D1 * 3 + 2 * R * D1 * D1
    fl += blocks(cfg.num_layers, D1, cfg.attention_head_dim)
    fl += 2 * R * (inc + D1) * D2 * 3 + 2 * R * D2 * D2
    fl += blocks(cfg.num_layers_2, D2, 2 * cfg.attention_head_dim)
    fl += 2 * R * D2 * out * 3 + 2 * R * out * out
    return fl


def decoder_flops(cfg: CodecConfig, T: int) -> int:
    """Multiply-add FLOPs of ScalarModel.decode on the two bands of T latent frames."""
    nb = cfg.out_channels // cfg.latent_hidden_dim
    ch = cfg.decoder_channels()
    fl = 2 * nb * T * cfg.latent_hidden_dim * ch[0] * cfg.delay_kernel_size
    t = T
    for i, s in enumerate(cfg.upsample_factors):
        fl += 2 * nb * t * ch[i] * s * ch[i + 1] * 2  # transposed conv: 2 taps per output
        t *= s
        fl += 5 * 2 * nb * t * ch[i + 1] * ch[i + 1] * (cfg.res_kernel_size + 1)
    if cfg.num_samples > 1:
        fl += 2 * nb * t * cfg.num_samples * cfg.init_channel * cfg.init_channel * cfg.default_kernel_size
        t *= cfg.num_samples
    return fl + 2 * nb * t * cfg.init_channel * cfg.num_bands * cfg.default_kernel_size


def load_codec(path, dtype=torch.float16, device="cuda", low_vram=None) -> HeartCodecB200:
    """codec_lite.load_codec (app/codec_lite.py:13-33): a codec checkpoint (directory or
    .safetensors + .json) on the GPU.  ``dtype`` and ``low_vram`` are accepted for the same
    call surface: activations are fp16 with fp32 accumulation, and the waveform decoder runs
    whole windows (the chunked low-VRAM decoder is unnecessary with 180 GB)."""
    tensors, cfg = load_codec_tensors(path)
    return HeartCodecB200(tensors, cfg, device=device)


def decode(codec: HeartCodecB200, frames: torch.Tensor, steps: int = 10, guidance: float = 1.25):
    """codec_lite.decode (app/codec_lite.py:63-75): frames [8, T] -> audio [2, samples]."""
    cb = codec.cfg.codebook_size
    return codec.detokenize(frames.clamp(0, cb - 1).to(codec.dev), num_steps=steps, guidance_scale=guidance,
                            disable_progress=True)
