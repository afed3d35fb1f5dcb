#!/usr/bin/env python
"""Benchmark of the HeartMuLa per-frame decode path on B200.

Workload: a 60 s song, 4 takes x 2 CFG rows = 8 rows, 750
frames after a 600-token prompt, BASELINE architecture (28-layer 3072-wide
backbone, 4-layer 1024-wide decoder, 8 codebooks of 8197) with random int8/fp16
weights.  One step = one whole song decode: 750 replays of the one-frame CUDA
graph (KV 600 -> 1350).  Weights (3.7 GB per frame) exceed L2, so no flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank decodes its own 4 takes (weak scaling) and the finished
token streams are gathered with NCCL; timing is the max over ranks.
``--impl reference`` times the reference engine's own CPU path (restated in
oracle/, bf16 with every host thread) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from estudiocanciones_b200._lib import capture_graph  # noqa: E402

METRIC = "audio s/s per GPU at 4 takes+CFG; µs per frame (3B + 7 decoder passes)"
UNIT = "audio-s/s"


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--takes", type=int, default=4)
    ap.add_argument("--frames", type=int, default=750)
    ap.add_argument("--prompt", type=int, default=600)
    ap.add_argument("--cpu-frames", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--case", default="frame",
                    choices=["frame", "gemv", "attn", "sampler", "prefill", "q8", "codec", "codec-est", "codec-dec",
                             "conv"],
                    help="frame: the benchmark; gemv/attn: a small single-kernel case for ncu captures; codec: "
                         "the detokenize timing alone; codec-est: estimator forwards of the full codec shape "
                         "(--reps of them, for launch lists and captures)")
    ap.add_argument("--layers", type=int, default=4, help="backbone layers of the small cases")
    ap.add_argument("--conv", default="2,744,1536,4608,1",
                    help="conv case: items,rows,cin,N,taps (default: the codec estimator's q|k|v GEMM)")
    ap.add_argument("--conv-bn", type=int, default=0, help="conv case: tile width (0 = automatic)")
    ap.add_argument("--prefill-layers", type=int, default=28, help="backbone layers of the prefill case")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--codec", default="auto", choices=["auto", "none"],
                    help="also time HeartCodec detokenize of a 60 s song (1 GPU runs)")
    ap.add_argument("--configs", default="auto", choices=["auto", "all", "none"],
                    help="also measure BASELINE configs 0/2/3 and the config-4 row sweep (auto: at N=1; config 4 "
                         "at 16 rows per GPU at every N)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- clocks
class Clocks(threading.Thread):
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    NAMES = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
             0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
             0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        super().__init__(daemon=True)
        self.index, self.samples, self.reasons, self.stop_ = index, [], 0, threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def run(self):
        while self.nv and not self.stop_.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.1)

    def result(self):
        self.stop_.set()
        self.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": [n for b, n in self.NAMES.items() if self.reasons & b and b != 0x1],
                "samples": len(self.samples)}


# ----------------------------------------------------------------------------- workload
def model_tensors(device, seed=0):
    from estudiocanciones_b200.checkpoint import BASELINE_SHAPE, synthetic_tensors
    return synthetic_tensors(BASELINE_SHAPE, seed=seed, device=device, gamma_one=True)


def frame_bytes(m, B, mean_len):
    """Algorithmic HBM bytes of one frame: every int8 weight byte and fp16 scale read
    once, the backbone K/V of every row over its attended length, the decoder K/V,
    the embedding rows and the logits/activations written once."""
    bb, dec = m.backbone, m.decoder
    w_bb = sum(l.nbytes for b in bb.blocks for l in (b.qkv, b.o, b.w13, b.w2))
    w_dec = sum(l.nbytes for b in dec.blocks for l in (b.qkv, b.o, b.w13, b.w2))
    w = w_bb + 7 * (w_dec + m.projection.nbytes) + m.c0_head.nbytes + sum(h.nbytes for h in m.audio_head)
    b0 = bb.blocks[0]
    kv = B * len(bb.blocks) * b0.kvh * b0.hd * 2 * 2 * mean_len
    d0 = dec.blocks[0]
    kv_dec = B * len(dec.blocks) * d0.kvh * d0.hd * 2 * 2 * (2 + sum(range(3, 9)))
    emb = B * (8 + 7) * bb.dim
    logits = 8 * B * m.vocab * 2
    return w + kv + kv_dec + emb + logits


def gemv_roofline(m, rt, peak, reps=10):
    """Dominant kernel (the fused int8 GEMV): the 112 backbone GEMV launches of one frame
    back to back (4 per layer, real prologues/epilogues), timed with CUDA events on the
    launching stream; algorithmic bytes = weights + scales + activations in/out."""
    from estudiocanciones_b200.engine import FramePlan
    from estudiocanciones_b200._lib import HM_EPI_ROPE_KV, HM_EPI_SILU
    bb = rt.bb
    B = rt.B
    p = FramePlan(rt.ctx)
    nbytes = 0
    for b in m.backbone.blocks:
        p._gemv(b.qkv, B, p.src_rms(bb.x, bb.ss, b.n1), epi=HM_EPI_ROPE_KV, rope=m.backbone.rope, pos=rt.pos, S=1,
                blk=b, q_out=bb.q)
        p._gemv(b.o, B, p.src_f16(bb.o), y=bb.x, res=bb.x, ss_out=bb.ss)
        p._gemv(b.w13, B, p.src_rms(bb.x, bb.ss, b.n2), epi=HM_EPI_SILU, y=bb.mm)
        p._gemv(b.w2, B, p.src_f16(bb.mm), y=bb.x, res=bb.x, ss_out=bb.ss)
        D = b.dim
        nbytes += b.qkv.nbytes + B * D * 2 + B * (b.qkv.N - b.kvh * b.hd) * 2 + b.kvh * b.hd * 2 * 2 * B
        nbytes += b.o.nbytes + B * b.o.K * 2 + 2 * B * D * 2
        nbytes += b.w13.nbytes + B * D * 2 + B * b.ffn * 2
        nbytes += b.w2.nbytes + B * b.ffn * 2 + 2 * B * D * 2
    p.run()
    torch.cuda.synchronize()
    # the launches are replayed from a CUDA graph so host launch cost does not enter
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with capture_graph(g, s):
        p.run()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    del g
    sec = t0.elapsed_time(t1) / 1000 / (reps * p.n_kernels)
    per_launch = nbytes / p.n_kernels
    achieved = per_launch / sec / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "kernel": "gemv_i8_kernel (112 backbone launches, R=8)",
            "bytes_per_launch": int(per_launch), "us_per_launch": round(sec * 1e6, 3)}


def traffic_profile():
    """DRAM bytes per GEMV launch from the committed ncu capture (profiles/gemv_traffic.json,
    `bench.py --case gemv` under ncu): a figure from that capture, not from this run."""
    f = ROOT / "profiles" / "gemv_traffic.json"
    if f.exists():
        try:
            d = json.loads(f.read_text())
            return {"file": "profiles/gemv_traffic.json", "dram_bytes_per_launch": d.get("dram_bytes_per_launch"),
                    "command": d.get("command")}
        except Exception:
            return None
    return None


def attn_roofline(m, rt, peak, reps=10):
    """Decode attention of the 28 backbone layers at the runtime's current positions, back to
    back in a CUDA graph, timed with CUDA events on the launching stream; algorithmic bytes =
    the K/V of every row over its attended length + q read + o written."""
    from estudiocanciones_b200.engine import FramePlan
    bb = rt.bb
    B = rt.B
    p = FramePlan(rt.ctx)
    nbytes = 0
    lens = (rt.pos + 1).tolist()
    for b in m.backbone.blocks:
        p.attn(b, bb.q, bb.o, rt.pos, 1, B, rt.nsplit)
        nbytes += sum(lens) * b.kvh * b.hd * 2 * 2 + 2 * B * b.h * b.hd * 2
    p.run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with capture_graph(g, s):
        p.run()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    del g
    sec = t0.elapsed_time(t1) / 1000 / (reps * p.n_kernels)
    per = nbytes / p.n_kernels
    gbs = per / sec / 1e9
    return {"bound": "hbm", "kernel": "decode_attn_tc_kernel (28 backbone layers)", "rows": B,
            "kv_len": int(max(lens)), "nsplit": int(rt.nsplit), "bytes_per_launch": int(per),
            "us_per_launch": round(sec * 1e6, 3), "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
            "frac": round(gbs / peak, 4)}


def frame_run(m, takes, cfg_on, prompt, frames, steps=1, warm_frames=50, warm=3):
    """A song of `frames` frames after a `prompt`-position cache (N(0,1) K/V) with `takes`
    takes (x 2 CFG rows when cfg_on): one CUDA-graph replay per frame, CUDA events around
    `steps` whole songs after `warm` shorter warm-up runs.  Returns (us per frame, rows, mean KV)."""
    dev = m.dev
    N = takes
    B = 2 * N if cfg_on else N
    L = prompt + frames + 2 + 256
    m.alloc(N, B, L)
    rt = m._rt
    g = torch.Generator(device=dev).manual_seed(0)
    for blk in m.backbone.blocks:
        blk.kc[:, :, :prompt].normal_(generator=g)
        blk.vc[:, :, :prompt].normal_(generator=g)
    rt.tok_in.copy_(torch.randint(0, 8192, (B, 8), generator=g, device=dev))
    cfg = 1.5 if cfg_on else 1.0
    rt.pos.fill_(prompt)
    graph = rt.graph_for(cfg, 50, 1.0)

    def song(nf):
        rt.pos.fill_(prompt)
        rt.frame.zero_()
        for _ in range(nf):
            graph.replay()
    for _ in range(warm):
        song(warm_frames)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        song(frames)
    e1.record()
    torch.cuda.synchronize()
    us = 1000 * e0.elapsed_time(e1) / (steps * frames)
    return us, B, prompt + (frames + 1) / 2


def config_entry(m, us, takes, B, mean_len, peak, **extra):
    fb = frame_bytes(m, B, mean_len)
    gbs = fb / (us * 1e-6) / 1e9
    return {"us_per_frame": round(us, 2), "audio_s_per_s_per_gpu": round(takes * 0.08 / (us * 1e-6), 3),
            "rows": B, "bytes_per_frame": int(fb), "frame_roofline_frac": round(gbs / peak, 4), **extra}


def measure_configs(a, m, peak, world, rank):
    """BASELINE configs besides the headline: 0 (1 row, CFG off, KV from 512), 2 (prefill of
    8 x 1024 tokens, tensor cores), 3 (8 rows, 3000 frames after a 1024-token prompt), and
    4 (16 rows per GPU; at N = 1 also the per-GPU sweep of 1/2/4/8/16 rows).  Each song is one
    timed step after short warm-up runs (timing: CUDA events)."""
    out = {}
    if world == 1:
        us, B, ml = frame_run(m, 1, False, 512, 100, steps=2)
        out["config0"] = config_entry(m, us, 1, B, ml, peak, workload="1 take, CFG off (1 row), KV 512 -> 612")
        us, B, ml = frame_run(m, 4, True, 1024, 3000, steps=1)
        out["config3"] = config_entry(m, us, 4, B, ml, peak,
                                      workload="4 takes x CFG = 8 rows, 3000 frames after a 1024-token prompt "
                                               "(KV 1024 -> 4024)")
        rt = m._rt
        rt.pos.fill_(4024)
        out["config3"]["attn_roofline_kv4024"] = attn_roofline(m, rt, peak)
        sweep = {}
        for R in (1, 2, 4, 8, 16):
            takes, cfg_on = (1, False) if R == 1 else (R // 2, True)
            us, B, ml = frame_run(m, takes, cfg_on, 600, 750, steps=1)
            sweep[str(R)] = config_entry(m, us, takes, B, ml, peak)
        out["config4_rows_per_gpu_sweep"] = sweep
        m.release()
        out["config2"] = prefill_entry(m, peak_tf=None)
    else:
        us, B, ml = frame_run(m, 8, True, 600, 750, steps=1)
        us = max_over_ranks(us, world)
        e = config_entry(m, us, 8, B, ml, peak, workload=f"8 takes x CFG = 16 rows per GPU, {world} GPUs, 750 "
                                                          f"frames after a 600-token prompt (max over ranks)")
        e["box_audio_s_per_s"] = round(world * 8 * 0.08 / (us * 1e-6), 3)
        out["config4"] = e
        m.release()
    return out


def prefill_entry(m, peak_tf=None):
    """Config 2 on the loaded model: 8 rows x 1024 tokens through the 28 backbone layers."""
    from estudiocanciones_b200.prefill import prefill_backbone
    B, P = 8, 1024
    m.alloc(4, B, P + 256)
    dev = m.dev
    h = (torch.randn(B, P, m.backbone.dim, generator=torch.Generator(device=dev).manual_seed(0), device=dev)
         * 0.05).half()
    for _ in range(2):
        prefill_backbone(m, h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        prefill_backbone(m, h)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    # the same prompt with the weights converted to fp16 inside the prompt (no kept copies)
    m.drop_prefill_weights()
    torch.cuda.synchronize()
    e0.record()
    prefill_backbone(m, h, keep_f16=False)
    e1.record()
    torch.cuda.synchronize()
    ms_conv = e0.elapsed_time(e1)
    fl = prefill_flops(m, B, P)
    tf = fl / (ms * 1e-3) / 1e12
    m.release()
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    burst, sus = pk.get("bf16_tflops", 1590.0), pk.get("bf16_tflops_sustained", 1400.0)
    return {"workload": "prefill 8 rows x 1024 tokens, 28 backbone layers (tcgen05 GEMMs + causal attention); "
                        "fp16 copies of the backbone weights kept resident (made by the first, untimed prefill)",
            "ms": round(ms, 3), "ms_converting_weights_per_prompt": round(ms_conv, 3),
            "flop": fl, "tflops": round(tf, 1), "frac_of_bf16_burst": round(tf / burst, 4),
            "frac_of_bf16_sustained": round(tf / sus, 4), "peak_kind": "measured" if pk else "fallback"}


def codec_entry(a, dev, cpu_sample=True):
    """HeartCodec detokenize of a 60 s song (750 frames x 8 codebooks: three 29.76 s windows,
    10 Euler steps each with CFG 1.25, then the waveform decoder) at the full codec shape with
    synthetic weights.  Timed with CUDA events: through the public call with host codes in and
    host audio out (e2e), and the dominant work alone (one window's solve graph: 10 estimator
    forwards, tensor-core bound) against the measured bf16 peak."""
    from estudiocanciones_b200.codec import HeartCodecB200, decoder_flops, estimator_flops
    from estudiocanciones_b200.codec_checkpoint import FULL_CODEC, synthetic_codec_tensors
    cfg, n_codes, steps, gs = FULL_CODEC, 750, 10, 1.25
    sd = synthetic_codec_tensors(cfg, 1)
    c = HeartCodecB200(sd, cfg, device=dev)
    codes = torch.randint(0, cfg.codebook_size, (cfg.num_quantizers, n_codes),
                          generator=torch.Generator().manual_seed(0)).pin_memory()

    def song():
        return c.detokenize(codes, num_steps=steps, guidance_scale=gs).cpu()

    for _ in range(2):
        wav = song()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        wav = song()
    e1.record()
    torch.cuda.synchronize()
    ms_song = e0.elapsed_time(e1) / reps
    # the solve of one later window (graph replay, inputs resident)
    key = next(k for k in c._plans if k[0] == "flow" and k[4] > 0)
    plan = c._plans[key]
    T = plan["T"]
    g = plan["graph"]
    g.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms_win = e0.elapsed_time(e1) / reps
    fl_win = steps * estimator_flops(cfg, 2, T)
    tf = fl_win / (ms_win * 1e-3) / 1e12
    dplan = c._plans[("dec", T)]
    dplan["graph"].replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        dplan["graph"].replay()
    e1.record()
    torch.cuda.synchronize()
    ms_dec = e0.elapsed_time(e1) / reps
    tf_dec = decoder_flops(cfg, T) / (ms_dec * 1e-3) / 1e12
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    burst = pk.get("bf16_tflops", 1590.0)
    nwin = sum(1 for k in c._plans if k[0] == "flow")
    n_windows = 3
    launches = n_windows * c.n_launches(key) + n_windows * len(dplan["P"].calls)
    out = {"workload": "HeartCodec detokenize, 60 s song (750 frames x 8 codebooks, 3 windows of 29.76 s), "
                       "10 Euler steps with CFG 1.25, full codec shape (24+6-layer estimator 1536/3072 wide, "
                       "decoder 2048->64 channels), synthetic weights",
           "ms_per_song": round(ms_song, 2), "audio_s_per_s": round(60.0 / (ms_song * 1e-3), 1),
           "e2e": {"h2d_bytes_per_step": codes.numel() * 8, "d2h_bytes_per_step": wav.numel() * 4},
           "window_solve_ms": round(ms_win, 3), "window_solve_tflops": round(tf, 1),
           "decoder_window_ms": round(ms_dec, 3), "decoder_tflops": round(tf_dec, 1),
           "roofline": {"bound": "tensor", "kernel": "one window's solve: 10 estimator forwards (conv_gemm_kernel, "
                                                     "prefill_attn_tc_kernel, norms)",
                        "achieved": round(tf, 1), "peak": burst, "unit": "TFLOP/s", "frac": round(tf / burst, 4),
                        "flop_per_launch_group": fl_win, "peak_kind": "measured bf16 burst" if pk else "fallback"},
           "gpu_launches_per_song": launches, "flow_plans": nwin}
    if cpu_sample:
        from oracle.heartcodec_oracle import OracleCodec
        orc = OracleCodec(sd, cfg)
        x = torch.randn(2, T, cfg.in_channels)
        with torch.inference_mode():
            t0 = time.perf_counter()
            orc.estimator(x, torch.tensor([0.5, 0.5]))
            t_est = time.perf_counter() - t0
            Td = T // 8
            t0 = time.perf_counter()
            orc.scalar_decode(torch.randn(2, cfg.latent_hidden_dim, Td))
            t_dec = (time.perf_counter() - t0) * T / Td
        sec = n_windows * (steps * t_est + t_dec)
        out["cpu_baseline"] = {"value": round(60.0 / sec, 4), "unit": "audio-s/s", "cores": torch.get_num_threads(),
                               "kind": "port",
                               "sample": f"one estimator forward (2 x {T} frames) and the waveform decoder on "
                                         f"{Td} frames, CPU oracle fp32, scaled to 3 windows x {steps} steps",
                               "s_per_song": round(sec, 2)}
    del c, sd
    torch.cuda.empty_cache()
    return out


def run_conv_case(a):
    """One implicit-GEMM conv (hm_conv1d_gemm) of the shape --conv = items,rows,cin,N,taps
    (centered taps, fp16 output), --reps timed launches after one warm-up."""
    from estudiocanciones_b200 import _lib as L
    B, T, cin, N, taps = (int(v) for v in a.conv.split(","))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, T, cin, generator=g, device=dev).half()
    w = (torch.randn(taps, N, cin, generator=g, device=dev) * (taps * cin) ** -0.5).half()
    y = torch.empty(B * T, N, dtype=torch.float16, device=dev)
    d = L.ConvDesc()
    d.x, d.x_ld, d.x_bstride, d.w, d.y, d.y_ld = x.data_ptr(), cin, T * cin, w.data_ptr(), y.data_ptr(), N
    d.B, d.T, d.tin, d.cin, d.N, d.npad, d.taps, d.off0, d.dil = B, T, T, cin, N, N, taps, -(taps // 2), 1
    d.scale, d.prelu, d.bn = 1.0, 1.0, a.conv_bn
    st = torch.cuda.current_stream().cuda_stream
    L.check(L.lib().hm_conv1d_gemm(d, st), "conv")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        L.lib().hm_conv1d_gemm(d, st)
    e1.record()
    torch.cuda.synchronize()
    us = 1000 * e0.elapsed_time(e1) / a.reps
    fl = 2 * B * T * cin * N * taps
    print(json.dumps({"case": "conv", "shape": a.conv, "bn": a.conv_bn, "us": round(us, 2),
                      "tflops": round(fl / us / 1e6, 1)}),
          flush=True)


def run_codec_dec_case(a):
    """--reps waveform-decoder runs of one full window (744 latent frames, two bands, full
    codec shape), eager, after one warm-up run: for launch lists and kernel captures."""
    from estudiocanciones_b200.codec import HeartCodecB200, decoder_flops
    from estudiocanciones_b200.codec_checkpoint import FULL_CODEC, synthetic_codec_tensors
    dev = torch.device("cuda", 0)
    c = HeartCodecB200(synthetic_codec_tensors(FULL_CODEC, 1), FULL_CODEC, device=dev, graphs=False)
    lat = torch.randn(744, FULL_CODEC.out_channels, device=dev) * 0.5
    c.scalar_decode(lat)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        c.scalar_decode(lat)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    fl = decoder_flops(FULL_CODEC, 744)
    print(json.dumps({"case": "codec-dec", "ms": round(ms, 3), "tflops": round(fl / ms / 1e9, 1)}), flush=True)


def run_codec_est_case(a):
    """--reps estimator forwards of the full codec shape (2 items x 744 frames), eager, after
    one warm-up forward: a short run for launch lists and kernel captures."""
    from estudiocanciones_b200.codec import HeartCodecB200, estimator_flops
    from estudiocanciones_b200.codec_checkpoint import FULL_CODEC, synthetic_codec_tensors
    dev = torch.device("cuda", 0)
    c = HeartCodecB200(synthetic_codec_tensors(FULL_CODEC, 1), FULL_CODEC, device=dev)
    x = torch.randn(2, 744, FULL_CODEC.in_channels, device=dev)
    c.estimator(x, 0.5)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        c.estimator(x, 0.5)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    fl = estimator_flops(FULL_CODEC, 2, 744)
    print(json.dumps({"case": "codec-est", "ms": round(ms, 3), "tflops": round(fl / ms / 1e9, 1)}), flush=True)


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ----------------------------------------------------------------------------- CPU path (reference arm / baseline)
def cpu_reference_timer(a, tensors_cpu):
    """The reference's own CPU path (app/engine.py CPU branch: bf16 weights dequantised at
    load, F.linear, masked SDPA, _frame_from_h) restated in oracle/, all host threads."""
    from oracle.heartmula_oracle import OracleModel
    torch.set_num_threads(os.cpu_count() or 1)
    B, N, P = 2 * a.takes, a.takes, a.prompt
    o = OracleModel(tensors_cpu, mode="cpu", dtype=torch.bfloat16)
    L = P + a.frames + 2 + 256
    o.alloc(B, L)
    g = torch.Generator().manual_seed(0)
    for ly in o.bb:
        ly.kc[:, :, :P] = torch.randn(ly.kc[:, :, :P].shape, generator=g).to(ly.kc.dtype)
        ly.vc[:, :, :P] = torch.randn(ly.vc[:, :, :P].shape, generator=g).to(ly.vc.dtype)
    tok = torch.randint(0, 8192, (B, 8), generator=g)
    state = {"pos": P, "tok": tok}

    def frames(n):
        t = time.perf_counter()
        for _ in range(n):
            pos = torch.full((B, 1), state["pos"])
            state["tok"] = o.step(state["tok"], pos, N, 1.5, 50, 1.0)
            state["pos"] += 1
        return time.perf_counter() - t
    return frames, torch.get_num_threads()


def run_reference(a, world, rank):
    if rank != 0:
        return
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t = {k: v.cpu() for k, v in model_tensors(dev).items()}
    frames, cores = cpu_reference_timer(a, t)
    del t
    for _ in range(a.warmup):
        frames(a.cpu_frames)
    times = [frames(a.cpu_frames) for _ in range(a.steps)]
    sec = sum(times)
    n = a.steps * a.cpu_frames
    value = a.takes * n * 0.08 / sec
    sample = f"{a.cpu_frames} frames per step of config 1 (8 rows, KV from {a.prompt}) on the CPU path, bf16"
    out = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(1000 * sec / a.steps, 2), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "impl": "reference", "us_per_frame": round(1e6 * sec / n, 1),
           "config": {"workload": "config1: 60 s song, 4 takes x CFG = 8 rows, KV 600->1350 (CPU sample)",
                      "model": "HeartMuLa BASELINE shape (28x3072 backbone, 4x1024 decoder), random int8"},
           "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                            "sample": sample,
                            "scope": "one host's CPU (rank 0 with every host thread) at every N: at N > 1 the "
                                     "GPU arm's whole-job value is set against this single-host figure"},
           "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------- our arm
def run_ours(a, world, rank, local):
    from estudiocanciones_b200 import kernels
    from estudiocanciones_b200.engine import HeartMuLaLite
    dev = torch.device("cuda", local)
    torch.manual_seed(1000 + rank)
    t = model_tensors(dev, seed=0)
    m = HeartMuLaLite(t, device=dev)
    del t
    N, B, P, F_ = a.takes, 2 * a.takes, a.prompt, a.frames
    L = P + F_ + 2 + 256
    m.alloc(N, B, L)
    rt = m._rt
    g = torch.Generator(device=dev).manual_seed(0)
    for blk in m.backbone.blocks:
        blk.kc[:, :, :P].normal_(generator=g)
        blk.vc[:, :, :P].normal_(generator=g)
    rt.tok_in.copy_(torch.randint(0, 8192, (B, 8), generator=g, device=dev))
    rt.pos.fill_(P)
    rt.pdl = not a.no_pdl
    graph = rt.graph_for(1.5, 50, 1.0)
    plan = rt.plan_for(1.5, 50, 1.0, with_backbone=True, commit=True)
    from estudiocanciones_b200.shard import gather_streams

    def step():
        rt.pos.fill_(P)
        rt.frame.zero_()
        for _ in range(F_):
            graph.replay()
        if world > 1:  # finished token streams of every rank's takes -> rank 0 (NCCL)
            gather_streams([rt.stream_out[:F_, i].t() for i in range(N)], N * world, world, rank, t_cap=F_, n_cb=8)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.result()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world)
    err = kernels.read_errors(dev)
    if err:
        raise RuntimeError(f"kernel error bits {err}")
    us_frame = 1000 * ms / F_
    value = world * a.takes * F_ * 0.08 / (ms / 1000)
    peak, peak_kind = peaks()
    mean_len = P + (F_ + 1) / 2
    fb = frame_bytes(m, B, mean_len)
    roof = gemv_roofline(m, rt, peak)
    roof["traffic"] = None  # no ncu in this run: the committed capture's figure is under traffic_profile
    roof["traffic_profile"] = traffic_profile()
    roof["peak_kind"] = f"{peak_kind} hbm_gbs (burst)"
    rt.pos.fill_(P + F_ // 2)
    attn_roof = attn_roofline(m, rt, peak)
    attn_roof["peak_kind"] = roof["peak_kind"]
    frame_gbs = fb / (us_frame * 1e-6) / 1e9
    out = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "fp16 activations x int8 weights (fp32 accumulate)", "data": "synthetic",
           "us_per_frame": round(us_frame, 2), "frames_per_s": round(1e6 / us_frame, 1),
           "audio_s_per_s_per_gpu": round(value / world, 3),
           "value_semantics": "whole job: audio seconds generated per second by all n_gpus GPUs (each GPU "
                              f"decodes its own {a.takes} takes); the metric's per-GPU figure is "
                              "audio_s_per_s_per_gpu",
           "config": {"workload": f"config1: 60 s song, {a.takes} takes x CFG = {B} rows per GPU, {F_} frames "
                                  f"after a {P}-token prompt (KV {P}->{P + F_}), one CUDA graph per frame",
                      "model": "HeartMuLa BASELINE shape (28x3072 backbone 24/8 heads, 4x1024 decoder 8/2 heads, "
                               "8x8197 codebooks), random int8 weights",
                      "parallelism": f"takes sharded, {world} GPU(s), NCCL gather of token streams",
                      "l2": "inputs larger than L2 (3.7 GB weights per frame)",
                      "pdl": not a.no_pdl},
           "roofline": roof,
           "attn_roofline": attn_roof,
           "frame_roofline": {"bytes_per_frame": int(fb), "achieved": round(frame_gbs, 1), "peak": peak,
                              "unit": "GB/s", "frac": round(frame_gbs / peak, 4)},
           "gpu_launches": int(plan.n_kernels * F_ * a.steps),
           "clocks": clk}
    # ---- end to end through the public API: host prompt ids -> generate -> host token streams
    if not a.no_e2e:
        text = torch.randint(0, 128256, (P,), generator=torch.Generator().manual_seed(0)).pin_memory()
        del graph
        rt = graph = None
        m.release()

        from estudiocanciones_b200.shard import generate_sharded

        def e2e_step():
            # this rank's takes of the whole job, streams gathered on rank 0 (NCCL) and read back
            res = generate_sharded(m, text, 10, a.takes * world, world=world, rank=rank, max_ms=F_ * 80,
                                   cfg_scale=1.5, stop_at_eos=False)
            return [r.cpu() for r in res] if res is not None else []
        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e2e_clocks = Clocks(local)
        e2e_clocks.start()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            res = e2e_step()
        torch.cuda.synchronize()
        sec = max_over_ranks((time.perf_counter() - t0) / a.e2e_steps, world)
        e2e_clk = e2e_clocks.result()
        d2h = sum(r.numel() * 8 for r in res) + math.ceil(F_ / 25) * 8 * a.takes  # streams + EOS reads
        out["e2e"] = {"value": round(world * a.takes * F_ * 0.08 / sec, 3), "unit": UNIT,
                      "h2d_bytes_per_step": P * 8, "d2h_bytes_per_step": int(d2h),
                      "ms_per_step": round(1000 * sec, 2),
                      "includes": f"prompt H2D, GPU text-embedding gather, tensor-core prefill, {F_} frames, "
                                  f"EOS checks every 25 frames, token streams gathered and read back",
                      "clocks": e2e_clk}
    # ---- the other BASELINE configs (sub-keys; the headline above is config 1)
    if a.configs == "all" or (a.configs == "auto"):
        graph = rt = None
        m.release()
        rt = None
        out["configs"] = measure_configs(a, m, peak, world, rank)
    # ---- the codec that turns the token streams into audio (the step after decoding), 1 GPU
    if world == 1 and a.codec != "none":
        out["codec"] = codec_entry(a, dev, cpu_sample=not a.no_cpu_baseline)
    # ---- CPU baseline: the reference CPU path on this host, rank 0 at N=1
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        tcpu = {k: v.cpu() for k, v in model_tensors(dev, seed=0).items()}
        torch.cuda.empty_cache()
        frames, cores = cpu_reference_timer(a, tcpu)
        del tcpu
        frames(1)
        sec = frames(a.cpu_frames)
        out["cpu_baseline"] = {"value": round(a.takes * a.cpu_frames * 0.08 / sec, 4), "unit": UNIT,
                               "cores": cores, "kind": "port",
                               "sample": f"{a.cpu_frames} frames of config 1 (8 rows, KV from {P}) through the "
                                         f"reference CPU path (bf16), after 1 warm-up frame",
                               "us_per_frame": round(1e6 * sec / a.cpu_frames, 1)}
    if rank == 0:
        print(json.dumps(out), flush=True)


def prefill_flops(m, B, P):
    """Multiply-add FLOPs of the prompt pass: every backbone GEMM over B*P rows plus
    causal attention (QK^T and PV over the lower triangle)."""
    Mrows = B * P
    f = 0
    for b in m.backbone.blocks:
        f += 2 * Mrows * (b.qkv.N * b.qkv.K + b.o.N * b.o.K + b.w13.N * b.w13.K + b.w2.N * b.w2.K)
        f += 2 * 2 * B * b.h * b.hd * (P * (P + 1) // 2)
    return f


def run_prefill_case(a, bb_layers=None):
    """Config 2: the prompt prefill of B rows x P tokens through the 28-layer backbone
    (tensor-core GEMMs and causal attention), timed with CUDA events."""
    from dataclasses import replace
    from estudiocanciones_b200.checkpoint import BASELINE_SHAPE, synthetic_tensors
    from estudiocanciones_b200.engine import HeartMuLaLite
    from estudiocanciones_b200.prefill import prefill_backbone
    dev = torch.device("cuda", 0)
    shape = replace(BASELINE_SHAPE, text_vocab=1024, **({"bb_layers": bb_layers} if bb_layers else {}))
    m = HeartMuLaLite(synthetic_tensors(shape, seed=0, device=dev, gamma_one=True), device=dev)
    B, P = 2 * a.takes, a.prompt
    m.alloc(a.takes, B, P + 256)
    h = (torch.randn(B, P, shape.bb_dim, generator=torch.Generator(device=dev).manual_seed(0), device=dev)
         * 0.05).half()
    for _ in range(2):
        prefill_backbone(m, h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        prefill_backbone(m, h)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    fl = prefill_flops(m, B, P)
    print(json.dumps({"case": "prefill", "rows": B, "prompt": P, "layers": len(m.backbone.blocks),
                      "ms": round(ms, 3), "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
                      "flop": fl}), flush=True)


def run_q8_case(a):
    """Checkpoint conversion: hm_q8_rows on the largest matrix of the converter (the
    fp32 text-embedding table, 128256 x 3072), timed with CUDA events; bytes = fp32
    read + int8 write + bf16 scales, against the measured HBM copy bandwidth."""
    from estudiocanciones_b200 import convert
    dev = torch.device("cuda", 0)
    N, K = 128256, 3072
    x = torch.randn(N, K, generator=torch.Generator(device=dev).manual_seed(0), device=dev) * 0.02
    for _ in range(3):
        convert.q8_rows(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        convert.q8_rows(x)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    nbytes = N * K * 4 + N * K + N * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    peak, kind = peaks()
    print(json.dumps({"case": "q8", "rows": N, "cols": K, "ms": round(ms, 3), "GBps": round(gbs, 1),
                      "frac": round(gbs / peak, 3), "peak_GBps": peak, "peak_kind": kind,
                      "note": "inputs (1.58 GB) exceed L2; each launch reads every row once from HBM"}),
          flush=True)


def run_case(a):
    """Small single-kernel cases for profiling: the GEMV launches of a few backbone
    layers (weights > L2 but well under a GB), one decode-attention launch at the
    benchmark's shapes, or the 8 samplers of a frame.  Graph replays; prints one JSON line."""
    from dataclasses import replace
    from estudiocanciones_b200.checkpoint import BASELINE_SHAPE, synthetic_tensors
    from estudiocanciones_b200.engine import FramePlan, HeartMuLaLite
    dev = torch.device("cuda", 0)
    shape = replace(BASELINE_SHAPE, bb_layers=a.layers, dec_layers=1, text_vocab=1024)
    t = synthetic_tensors(shape, seed=0, device=dev)
    m = HeartMuLaLite(t, device=dev)
    del t
    N, B, P = a.takes, 2 * a.takes, a.prompt
    L = P + a.frames + 2 + 256
    m.alloc(N, B, L)
    rt = m._rt
    rt.pos.fill_(P + a.frames // 2)
    g = torch.Generator(device=dev).manual_seed(0)
    for blk in m.backbone.blocks:
        blk.kc.normal_(generator=g)
        blk.vc.normal_(generator=g)
    p = FramePlan(rt.ctx, pdl=not a.no_pdl)
    if a.case == "sampler":
        for c in range(8):
            p.sample(rt.logits, N, 1.5, 50, 1.0, rt.noise[c], rt.tok_out, c)
    elif a.case == "gemv":
        from estudiocanciones_b200._lib import HM_EPI_ROPE_KV, HM_EPI_SILU
        bb = rt.bb
        for b in m.backbone.blocks:
            p._gemv(b.qkv, B, p.src_rms(bb.x, bb.ss, b.n1), epi=HM_EPI_ROPE_KV, rope=m.backbone.rope, pos=rt.pos,
                    S=1, blk=b, q_out=bb.q)
            p._gemv(b.o, B, p.src_f16(bb.o), y=bb.x, res=bb.x, ss_out=bb.ss)
            p._gemv(b.w13, B, p.src_rms(bb.x, bb.ss, b.n2), epi=HM_EPI_SILU, y=bb.mm)
            p._gemv(b.w2, B, p.src_f16(bb.mm), y=bb.x, res=bb.x, ss_out=bb.ss)
    else:
        b = m.backbone.blocks[0]
        p.attn(b, rt.bb.q, rt.bb.o, rt.pos, 1, B, rt.nsplit)
    p.run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with capture_graph(graph, st):
        p.run()
    torch.cuda.current_stream().wait_stream(st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph.replay()
    e0.record()
    for _ in range(a.reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = 1000 * e0.elapsed_time(e1) / (a.reps * p.n_kernels)
    out = {"case": a.case, "launches": p.n_kernels, "us_per_launch": round(us, 3), "rows": B,
           "pos": P + a.frames // 2, "nsplit": rt.nsplit,
           "env": {k: v for k, v in os.environ.items() if k.startswith("HM_")}}
    if a.case == "gemv":
        wb = sum(l.nbytes for b in m.backbone.blocks for l in (b.qkv, b.o, b.w13, b.w2))
        out["weight_GBps"] = round(wb / (us * 1e-6 * p.n_kernels) / 1e9, 1)
    print(json.dumps(out), flush=True)


def main():
    a = args_()
    if a.case == "prefill":
        run_prefill_case(a, bb_layers=a.prefill_layers)
        return
    if a.case == "q8":
        run_q8_case(a)
        return
    if a.case == "codec":
        print(json.dumps(codec_entry(a, torch.device("cuda", 0), cpu_sample=not a.no_cpu_baseline)), flush=True)
        return
    if a.case == "codec-est":
        run_codec_est_case(a)
        return
    if a.case == "conv":
        run_conv_case(a)
        return
    if a.case == "codec-dec":
        run_codec_dec_case(a)
        return
    if a.case != "frame":
        run_case(a)
        return
    world, rank, local = dist_setup()
    try:
        if a.impl == "reference":
            run_reference(a, world, rank)
        else:
            run_ours(a, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
