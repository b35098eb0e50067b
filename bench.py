#!/usr/bin/env python
"""Benchmark of the video-DiT denoising step (BASELINE.json metric:
"DiT denoising s/step (720p x 121f, 6-bit, 1/2/4/8 B200); qGEMM TFLOP/s % peak").

Workload (default ``--config c5``): one full-size
synthetic 720p x 121-frame step of the 48-block 6-bit H3-style DiT:
S = 512 text + 4 x 3600 reference-image rows + 111600 video rows (31x45x80) = 126512,
hidden 3072, 24 x 128 heads, FFN 12288 GELU, AdaLN modulation, attention policy
"mix" (dense anchors {0,1,24,25,46,47}, other layers block top-k 25 % over
128-row blocks, strip rows [0, 14912) exact), PAB over the 4-step window of
sigmaSchedule(4, shift 12) with maxStale 0.06 (refresh {0,1,3}, reuse {2}).
A bench "step" is one denoising step (patch embed, 48 blocks, final head,
Euler update); K timed steps follow W warm-up steps along the window.

Random-init weights quantized to 6 bits on the GPU, synthetic latents: no
checkpoint or dataset is used. Every kernel on the timed path is libwx
(sm_100a); torch only allocates buffers and copies host data.

``--impl reference`` times the reference algorithm's CPU restatement (the
oracle; the reference's own Swift/MLX/Metal path cannot run on this box) on
bounded samples of the same workload and reports the same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "DiT denoising s/step (720p x 121f, 6-bit); qGEMM TFLOP/s % peak"
PEAKS_FALLBACK = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)

CONFIGS = {
    # full-size 720p x 121f with reference-image conditioning
    "c5": dict(text=512, refs=4, ref_rows=3600, ref_hw=(120, 120), grid=(31, 45, 80), hidden=3072, heads=24,
               ffn=12288, layers=48, text_dim=4096),
    # half-size step
    "c4": dict(text=512, refs=0, ref_rows=0, ref_hw=(0, 0), grid=(31, 23, 40), hidden=3072, heads=24, ffn=12288,
               layers=48, text_dim=4096),
    # development geometry (seconds on one GPU)
    "tiny": dict(text=64, refs=1, ref_rows=192, ref_hw=(24, 32), grid=(3, 8, 16), hidden=512, heads=4, ffn=1024,
                 layers=4, text_dim=512),
}
PATCH_DIM = 96          # latent channels x 2 x 2 patch
TOPK_DENSITY = 0.25
SHIFT = 12.0
WINDOW = 4              # sampler steps in the PAB window
PAB_K = 2
PAB_MAX_STALE = 0.06    # lifts the reference default 0.04 so step 2 is reused (|dsigma| = 0.0499)
EPS = 1e-6
ROT = 96                # 3 axes x 16 inverse frequencies x 2
# DRAM bytes (read + write) of one attention call of the config-5 step, weighted over its
# 6 dense + 42 top-k layers, from one ncu capture of the attention kernels on a config-5 layer's
# attention call run standalone (bench.py --config c5attn / c5attn_dense)
ATTN_TRAFFIC_C5 = (6 * 1.1935e+10 + 42 * 1.0894e+10) / 48


def phase_summary(trace: list, steps: int) -> dict:
    """Per-layer phase trace of the timed region (this rank): milliseconds per step of each
    block phase summed over the layers, and the mean block time per attention mode."""
    phases = ("norm1", "qkv", "rope", "attn", "out", "mlp")
    out = dict(ms_per_step={p: sum(r[p + "_ms"] for r in trace) / steps for p in phases},
               blocks=len(trace), source="wx_ctx_trace (CUDA events at the block's phase boundaries)")
    for mode in ("dense", "sparse", "reuse"):
        sel = [r["total_ms"] for r in trace if r["mode"] == mode]
        if sel:
            out[f"{mode}_block_ms"] = dict(mean=sum(sel) / len(sel), count=len(sel))
    return out


def peer_store_summary(trace: list, phases: dict, c: dict, world: int, steps: int, att_bytes_per_launch: float) -> dict:
    """NVLink stores inside the compute kernels (the q|k|v projection's epilogue, the attention
    epilogue) under sequence parallelism: bytes this rank sends per step, and those bytes over
    the time of the phase that sends them, a lower bound on the store bandwidth (the phases
    also compute)."""
    blocks_refreshed = sum(1 for r in trace if r["mode"] != "reuse")
    rows = c["S"] // world
    qkv_b = rows * 3 * c["inner"] * 2 * (world - 1) / world * blocks_refreshed / steps
    att_b = att_bytes_per_launch * blocks_refreshed / steps
    ph = phases["ms_per_step"]
    return dict(peer_bytes_per_step=dict(qkv_from_projection_epilogue=qkv_b, attention_rows=att_b),
                peer_gbs_lower_bound=dict(
                    qkv_phase=qkv_b / (ph["qkv"] / 1e3) / 1e9 if ph["qkv"] > 0 else None,
                    attn_phase=att_b / (ph["attn"] / 1e3) / 1e9 if ph["attn"] > 0 else None,
                    what="bytes sent to the other ranks per step / the phase's time per step (the phase "
                         "also computes)"))


def geometry(name: str) -> dict:
    c = dict(CONFIGS[name])
    t, hh, ww = c["grid"]
    c["video"] = t * hh * ww
    c["g"] = c["text"] + c["refs"] * c["ref_rows"]
    c["S"] = c["g"] + c["video"]
    c["inner"] = c["heads"] * 128
    c["name"] = name
    return c


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# ------------------------------------------------------------------ work model
def step_flops(c: dict, refresh: bool) -> dict:
    """Algorithmic FLOPs of one step: GEMMs (2MNK) and attention (4*hd per query-key pair)."""
    S, hdn, inner, ffn, L = c["S"], c["hidden"], c["inner"], c["ffn"], c["layers"]
    mlp = 2 * S * (hdn * ffn + ffn * hdn)
    attn_proj = 2 * S * (hdn * 3 * inner + inner * hdn)
    gemm = L * (mlp + (attn_proj if refresh else 0))
    attn = 0.0
    if refresh:
        for layer in range(L):
            attn += attention_flops(c, dense=_is_dense(layer, L))
    return dict(gemm=gemm, attn=attn)


def _is_dense(layer: int, n: int) -> bool:
    mid = n // 2
    return layer < 2 or layer + 2 >= n or layer == mid or layer == mid + 1


def attention_flops(c: dict, dense: bool) -> float:
    S, g, H = c["S"], c["g"], c["heads"]
    if dense:
        pairs = S * S
    else:
        L = S - g
        nb = (L + 127) // 128
        keep = min(math.ceil(TOPK_DENSITY * nb), nb - 1) + 1
        # kept key rows per video row: strip + keep blocks (the ragged last block counted full: <0.1 %)
        pairs = g * S + L * (g + min(keep * 128, L))
    return 4.0 * 128 * H * pairs


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["no samples"])
        return dict(sm_mhz=float(np.median(sm)), sm_max_mhz=max(smax), samples=len(sm),
                    power_w_max=max(power) if power else None, reasons=sorted(reasons))


# ------------------------------------------------------------------ model
class Model:
    def __init__(self, c: dict, device, seed: int = 1234 + 5):
        import torch
        from wuxianhuabu_b200 import h3
        self.c = c
        self.dev = device
        g = torch.Generator(device=device).manual_seed(seed)
        hdn, inner, ffn, L = c["hidden"], c["inner"], c["ffn"], c["layers"]

        def qlin(n, k):
            w = torch.randn((n, k), device=device, generator=g) * 0.02
            b = (torch.randn((n,), device=device, generator=g) * 0.02).to(torch.bfloat16)
            m = h3.MfLinear.quantize(w, bits=6, group=64, bias=b)
            del w
            return m

        def norm(n):
            return (1.0 + 0.02 * torch.randn((n,), device=device, generator=g)).to(torch.bfloat16)

        blocks = []
        for _ in range(L):
            blocks.append(h3.H3BlockWeights(qlin(3 * inner, hdn), qlin(hdn, inner), qlin(ffn, hdn), qlin(hdn, ffn),
                                            norm(128), norm(128), norm(hdn), norm(hdn)))
        torch.cuda.synchronize()
        self.cfg = h3.H3DiTConfig(hidden=hdn, heads=c["heads"], head_dim=128, ffn=ffn, mlp_kind=h3.MLP_GELU, rot=ROT,
                                  eps=EPS, layers=L)
        self.dit = h3.H3DiTBlocks(self.cfg, blocks)
        # AdaLN tables (precomputeAdaln output): 6 x [12, hidden] per block, rows = t_row*3 + modality
        self.mods = [[(0.05 * torch.randn((12, hdn), device=device, generator=g)).to(torch.bfloat16)
                      for _ in range(6)] for _ in range(L)]
        self.final_norm = norm(hdn)
        self.final_mods = [(0.05 * torch.randn((4, hdn), device=device, generator=g)).to(torch.bfloat16)
                           for _ in range(2)]
        self.w_embed = torch.randn((PATCH_DIM, hdn), device=device, generator=g) * (1 / math.sqrt(PATCH_DIM))
        self.b_embed = torch.zeros((hdn,), device=device)
        self.w_out = torch.randn((hdn, PATCH_DIM), device=device, generator=g) * (1 / math.sqrt(hdn))
        self.b_out = torch.zeros((PATCH_DIM,), device=device)
        # refined text states (condition_proj output, computed once per generation)
        self.text = torch.randn((c["text"], hdn), device=device, generator=g).to(torch.bfloat16)
        self.gen = g
        self.h3dit = h3.H3DiT(self.dit, self.mods, self.w_embed, self.b_embed, self.final_norm, self.w_out,
                              self.b_out)


class Runner:
    """Device-resident sampler step over this rank's rows of the packed sequence
    (all rows on one GPU; S/P rows per rank under Ulysses sequence parallelism)."""

    def __init__(self, model: Model, rank: int = 0, world: int = 1):
        import torch
        from wuxianhuabu_b200 import h3
        self.m = model
        c = model.c
        dev = model.dev
        self.h3 = h3
        S, g, hdn, text = c["S"], c["g"], c["hidden"], c["text"]
        self.rows = S // world
        self.row0 = rank * self.rows
        r1 = self.row0 + self.rows
        # packed rows [text, S) come from the patch embed; the latent x_in covers them
        self.x_in = torch.randn((S - text, PATCH_DIM), device=dev, generator=model.gen)  # [cond ; videoX] fp32
        self.t0, self.t1 = self.row0, min(r1, text)            # local text rows
        self.e0, self.e1 = max(self.row0, text), r1            # local embedded rows
        self.v0, self.v1 = max(self.row0, g), r1               # local video rows
        self.n_embed = max(0, self.e1 - self.e0)
        nvl = max(0, self.v1 - self.v0)
        self.video_x = self.x_in[self.v0 - text:self.v1 - text]
        self.h = torch.empty((self.rows, hdn), dtype=torch.bfloat16, device=dev)
        self.emb32 = torch.empty((max(1, self.n_embed), hdn), dtype=torch.float32, device=dev)
        self.head32 = torch.empty((max(1, nvl), hdn), dtype=torch.float32, device=dev)
        self.head16 = torch.empty((max(1, nvl), hdn), dtype=torch.bfloat16, device=dev)
        self.vel = torch.empty((max(1, nvl), PATCH_DIM), dtype=torch.float32, device=dev)
        self.nvl = nvl
        cos, sin = self._rope(c, dev)
        self.cos, self.sin = cos[self.row0:r1].contiguous(), sin[self.row0:r1].contiguous()
        self.sigmas = h3.sigma_schedule(WINDOW, SHIFT)
        self.plan = h3.attn_broadcast_plan(self.sigmas, PAB_K, PAB_MAX_STALE)
        self.rowmaps = [self._rowmap(c, i, dev)[self.row0:r1].contiguous() for i in range(WINDOW)]
        self.pab = h3.H3AttnBroadcast(c["layers"])
        self.sparse = h3.H3SolAttnConfig(block=128, topk_ratio=TOPK_DENSITY, tail=False)
        self.ctx = h3.context(dev.index)
        self.S = S

    @staticmethod
    def _rope(c, dev):
        """Position ids of the packed layout (text, reference images, target video; H3Layout.swift
        PackedLayout) and buildRope (:725-740) through libwx, with the 16 inverse frequencies
        1/10000^(2j/32) standing in for the checkpoint's inv_freq."""
        import torch
        from wuxianhuabu_b200 import h3
        t, hh, ww = c["grid"]
        pos = h3.packed_positions(c["text"], [c["ref_hw"]] * c["refs"], t, 2 * hh, 2 * ww)
        assert pos.shape[0] == c["S"]
        inv = (1.0 / (10000.0 ** (np.arange(16, dtype=np.float64) * 2 / 32))).astype(np.float32)
        return h3.build_rope(pos, torch.from_numpy(inv).to(dev))

    @staticmethod
    def _rowmap(c, i, dev):
        """buildTimestepPlanGlobal + buildRowModMap: text/video rows use the step's t row, cond rows the aug t."""
        import torch
        from wuxianhuabu_b200 import h3
        t_row, cond_row = i % 4, 3
        g_text, g = c["text"], c["g"]
        runs = [h3.ModRun(0, g_text, t_row * 3 + 0)]
        if g > g_text:
            runs.append(h3.ModRun(g_text, g, cond_row * 3 + 1))
        runs.append(h3.ModRun(g, c["S"], t_row * 3 + 2))
        m = h3.H3FusedKernels.build_row_mod_map(c["S"], runs)
        return torch.from_numpy(m.view(np.int32)).to(dev)

    def step(self, i: int) -> None:
        """One sampler step (H3Pipeline.swift:1398-1445) at window position i: one native
        call (wx_dit_step) running patch embed, 48 blocks, final head and Euler update."""
        m, c = self.m, self.m.c
        pos = i % WINDOW
        m.h3dit.step(self.S, c["text"], c["g"], m.text, self.x_in, self.rowmaps[pos], self.cos, self.sin,
                     m.final_mods[0][pos], m.final_mods[1][pos], self.sparse, self.h3.SparsePolicy.MIX, self.pab,
                     self.plan[pos], self.sigmas[pos + 1] - self.sigmas[pos], sigma=self.sigmas[pos])


# ------------------------------------------------------------------ CPU baseline
class CpuSample:
    """Bounded sample of the step on the host cores with the oracle (the reference
    algorithm restated in C, OpenMP on every host thread): the four 6-bit linears on
    `rows` rows, the row kernels, and one head's routing and attention for `att_rows`
    strip rows (dense over all S keys) and `att_rows` video rows (strip + top-k kept
    blocks). Inputs and quantized weights are prepared once; run() times one sample and
    extrapolates it linearly in rows / heads / layers to s/step over the PAB window."""

    def __init__(self, c: dict, plan: list, rows: int = 1024, att_rows: int = 384, seed: int = 99):
        from oracle import oracle as O
        O.build()
        self.threads = O.set_num_threads(0)  # every host thread, whatever OMP_NUM_THREADS says
        self.O, self.c, self.plan, self.rows, self.att_rows = O, c, list(plan), rows, att_rows
        hdn, inner, ffn, S = c["hidden"], c["inner"], c["ffn"], c["S"]
        t0 = time.perf_counter()
        self.lin = {}
        for i, (name, n, k) in enumerate([("qkv", 3 * inner, hdn), ("out", hdn, inner), ("fc1", ffn, hdn),
                                          ("fc2", hdn, ffn)]):
            self.lin[name] = O.quantize(O.normal_f32((n, k), seed, i, std=0.02))
        self.x = O.normal_bf16((rows, hdn), seed, 10)
        self.xi = O.normal_bf16((rows, inner), seed, 11)
        self.xf = O.normal_bf16((rows, ffn), seed, 12)
        self.q = O.normal_bf16((S, 1, 128), seed, 13)
        self.k = O.normal_bf16((S, 1, 128), seed, 14)
        self.v = O.normal_bf16((S, 1, 128), seed, 15)
        self.w1 = O.normal_bf16((hdn,), seed, 16)
        self.mods = O.normal_bf16((4, hdn), seed, 17)
        self.prep_s = time.perf_counter() - t0
        self.sample = (f"oracle (C, OpenMP, {self.threads} threads) on {rows} rows through the 4 six-bit linears + "
                       f"row kernels and 1 of {c['heads']} heads' routing and attention for {att_rows} strip + "
                       f"{att_rows} video query rows at S={S}; extrapolated linearly in rows/heads/layers over the "
                       f"PAB window {self.plan}")

    def run(self) -> dict:
        O, c, rows, att_rows = self.O, self.c, self.rows, self.att_rows
        hdn, inner, ffn, S, g, H = c["hidden"], c["inner"], c["ffn"], c["S"], c["g"], c["heads"]
        lin = self.lin

        def tm(fn):
            a = time.perf_counter()
            fn()
            return time.perf_counter() - a

        # each oracle qlinear call expands its whole weight once (a per-layer cost) and then
        # does per-row work: split the two so the extrapolation scales only the row part
        t_dq = {n: tm(lambda n=n, k=k: O.dequantize(*lin[n], k)) for n, k in
                (("qkv", hdn), ("out", inner), ("fc1", hdn), ("fc2", ffn))}
        t_qkv = max(0.0, tm(lambda: O.qlinear(self.x, *lin["qkv"])) - t_dq["qkv"])
        t_out = max(0.0, tm(lambda: O.qlinear(self.xi, *lin["out"])) - t_dq["out"])
        t_fc1 = max(0.0, tm(lambda: O.qlinear(self.x, *lin["fc1"], epilogue=O.EPI_GELU)) - t_dq["fc1"])
        t_fc2 = max(0.0, tm(lambda: O.qlinear(self.xf, *lin["fc2"])) - t_dq["fc2"])
        rm = np.zeros(rows, np.uint32)
        t_norm = tm(lambda: O.norm_modscale(self.x, self.w1, self.mods, self.mods, rm, EPS))
        scale = float(1 / np.sqrt(128))
        route = {}
        t_route = tm(lambda: route.update(O.topk_route(self.q, self.k, self.v, g, scale, TOPK_DENSITY)))
        route.update(g=g, block=128)
        t_strip = tm(lambda: O.attention_rows(self.q, self.k, self.v, g, scale, 0, att_rows, route=route))
        t_video = tm(lambda: O.attention_rows(self.q, self.k, self.v, g, scale, g, g + att_rows, route=route))
        per_row = lambda t: t / rows
        gemm_attn_rows = per_row(t_qkv) + per_row(t_out)
        gemm_mlp_rows = per_row(t_fc1) + per_row(t_fc2)
        rowops = per_row(t_norm) * 4  # norm1, norm2, q/k rope (~norm cost), gate
        attn_sparse = H * (t_strip / att_rows * g + t_video / att_rows * (S - g)) + H * t_route
        attn_dense = H * (t_strip / att_rows * S)
        L = c["layers"]
        n_dense = sum(1 for lyr in range(L) if _is_dense(lyr, L))
        dq_attn = t_dq["qkv"] + t_dq["out"]
        dq_mlp = t_dq["fc1"] + t_dq["fc2"]
        refresh_step = (L * (S * (gemm_attn_rows + gemm_mlp_rows + rowops) + dq_attn + dq_mlp)
                        + n_dense * attn_dense + (L - n_dense) * attn_sparse)
        reuse_step = L * (S * (gemm_mlp_rows + rowops * 0.5) + dq_mlp)
        s_per_step = sum(refresh_step if r else reuse_step for r in self.plan) / len(self.plan)
        sampled = t_qkv + t_out + t_fc1 + t_fc2 + sum(t_dq.values()) * 2 + t_norm + t_route + t_strip + t_video
        return dict(value=s_per_step, sampled_s=sampled)


def window_plan() -> list:
    """The PAB refresh plan of the 4-step window (attnBroadcastPlan over sigmaSchedule(4, 12),
    k = 2, maxStale 0.06): host logic of libwx, no GPU needed."""
    from wuxianhuabu_b200 import h3
    return list(h3.attn_broadcast_plan(h3.sigma_schedule(WINDOW, SHIFT), PAB_K, PAB_MAX_STALE))


# ------------------------------------------------------------------ kernel-level configs
def run_c3(args, seq: int, dense: bool = False, g: int = 0) -> dict:
    """standalone block-sparse attention (24 x 128 heads,
    128-row blocks, diagonal + top-k 25 %, g = 0, no tail), routing included.
    dense=True: the dense attention of the dense layers and strip rows at the same size.
    g > 0: the attention call of the config-5 step's layers (strip rows [0, g) exact over all
    keys, video rows routed), standalone; used for the DRAM-traffic capture of the roofline.
    args.router == "sol": the reference's production router instead of top-k (H3SolAttnConfig
    defaults, SOL:79-98: tau 1.3 over 64-row blocks, pooled tail term); its selection depends on
    the data, so the FLOPs are counted from the selection the router made."""
    import torch
    from wuxianhuabu_b200 import h3
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1234 + 2)
    H = 24
    q, k, v = [torch.randn((seq, H, 128), device=dev, generator=gen).to(torch.bfloat16) for _ in range(3)]
    out = torch.empty_like(q)
    sol = args.router == "sol" and not dense
    cfg = (None if dense else h3.H3SolAttnConfig(tau=1.3, tail=True) if sol
           else h3.H3SolAttnConfig(block=128, topk_ratio=TOPK_DENSITY, tail=False))
    scale = float(1 / math.sqrt(128))
    ctx = h3.context(0)
    for _ in range(args.warmup):
        h3.H3SolAttn.forward(q, k, v, g, scale, cfg, out=out)
    torch.cuda.synchronize()
    import ctypes
    ctx.lib.wx_ctx_profile_enable(ctx.h, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        h3.H3SolAttn.forward(q, k, v, g, scale, cfg, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = (ctypes.c_double * 6)()
    cnt = (ctypes.c_int64 * 6)()
    ctx.lib.wx_ctx_profile_read(ctx.h, ms, cnt, 6)
    ctx.check_device()
    nb = (seq - g + 127) // 128
    keep = min(math.ceil(TOPK_DENSITY * nb), nb - 1) + 1
    flops = 4.0 * 128 * H * (seq * seq if dense else g * seq + (seq - g) * (g + min(keep * 128, seq - g)))
    density = None
    if sol:  # kept key rows of every (head, video query block) from the router's own selection
        r = h3.H3SolAttn.route(q, k, v, g, scale, cfg)
        lens = r["lens"].double()
        kept = (r["sel"].double() * lens[None, None, :]).sum(-1)  # [H, nb] video key rows kept
        flops = 4.0 * 128 * (H * g * seq + float((lens[None, :] * (g + kept)).sum()))
        density = float(r["sel"].double().mean())
        del r
    peaks, kind = load_peaks()
    per_call = e0.elapsed_time(e1) / args.steps
    flash_ms = ms[1] / max(1, cnt[1])
    ach = flops / (flash_ms / 1e3) / 1e12
    pk = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    kernel = ("flash_attn_pair_kernel<false, 128> (paired query tiles, shared K/V)" if dense else
              "flash_attn_pair_kernel<true, 128> (duo: two routed query tiles per CTA)")
    what = ("dense attention" if dense else "SOL tau 1.3 attention (64-row blocks, tail)" if sol
            else "SOL top-k 25% attention")
    name = "c3" if g == 0 else "c5 layer geometry"
    conf = dict(workload=f"{name}: {what}, S={seq}, strip rows {g}, 24x128 heads", S=seq, g=g,
                router="dense" if dense else "sol" if sol else "topk")
    if density is not None:
        conf.update(kept_block_fraction=density, data="q, k, v ~ N(0, 1) (no attention structure)")
    return dict(metric=f"{'dense' if dense else 'sparse'} attention ms/call ({name})", value=per_call, unit="ms/call",
                config=conf,
                higher_is_better=False,
                roofline=dict(kernel=kernel, bound="tensor", achieved=ach, peak=pk, unit="TFLOP/s",
                              frac=ach / pk, avg_launch_ms=flash_ms, flops_per_launch=flops,
                              peak_kind=f"{kind} burst bf16"),
                routing_ms=ms[2] / max(1, args.steps))


def _rope_grid16(O, S: int):
    """cos/sin [S, 32] of the config-1 latent grid (t, h, w each 0..15; 8/12/12 frequency
    pairs of theta 10000 per axis), formed as buildRope does (H3Layout.swift:725-740)."""
    t, hh, ww = np.meshgrid(np.arange(16), np.arange(16), np.arange(16), indexing="ij")
    pos = np.stack([t.ravel(), hh.ravel(), ww.ravel()], 1).astype(np.float32)[:S]
    ang = []
    for axis, nf in enumerate((8, 12, 12)):
        inv = (1.0 / 10000.0 ** (np.arange(nf, dtype=np.float64) * 2 / (2 * nf))).astype(np.float32)
        ang.append((pos[:, axis:axis + 1] * inv[None, :]).astype(np.float32))
    a = np.concatenate(ang, 1).astype(np.float64)
    return O.f32_to_bf16(np.cos(a).astype(np.float32)), O.f32_to_bf16(np.sin(a).astype(np.float32))


def run_c1(args) -> dict:
    """one DiT block (hidden 1024, 16 heads of 64, FFN 4096 GELU,
    S = 4096 = 16 x 16 x 16 latent grid, QK-RMSNorm eps 1e-6, 3-D RoPE over 8/12/12 frequency
    pairs, dense attention, 6-bit group-64 weights ~ N(0, 0.02), activations ~ N(0, 1)) on one
    GPU, beside the oracle's whole block on every host thread (timed whole, not extrapolated).
    The same quantized weights and inputs go to both sides; the line also carries the GPU
    block's max rel err and cosine against the oracle's output. `value` is the block replayed
    as one CUDA graph (wx_graph_launch: the same kernels, the launch gaps gone; its output is
    checked equal to the direct call's); `direct` is the plain wx_dit_block_forward call, and
    `e2e` the graph with the pinned H2D / D2H of h around it."""
    import ctypes
    import torch
    from oracle import oracle as O
    from wuxianhuabu_b200 import h3
    O.build()
    S, hdn, H, hd, ffn, rot, eps, seed = 4096, 1024, 16, 64, 4096, 64, 1e-6, 1234
    inner = H * hd
    w = {}
    for i, (name, n, k) in enumerate([("qkv", 3 * inner, hdn), ("out", hdn, inner), ("fc1", ffn, hdn),
                                      ("fc2", hdn, ffn)]):
        wq, sc, bi = O.quantize(O.normal_f32((n, k), seed, 10 + i, std=0.02))
        w[name] = (wq, sc, bi, O.normal_bf16((n,), seed, 20 + i, std=0.02))
    for j, name in enumerate(("q_norm", "k_norm")):
        w[name] = O.normal_bf16((hd,), seed, 30 + j, mean=1.0, std=0.02)
    for j, name in enumerate(("norm1", "norm2")):
        w[name] = O.normal_bf16((hdn,), seed, 32 + j, mean=1.0, std=0.02)
    mods = [O.normal_bf16((3, hdn), seed, 40 + j, std=0.05) for j in range(6)]
    h0 = O.normal_bf16((S, hdn), seed, 50)
    rowmap = np.zeros(S, np.uint32)  # one modulation row (a single video segment at one t)
    cos, sin = _rope_grid16(O, S)

    dev = torch.device("cuda", 0)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)

    def lin(t, k):
        wq, sc, bi, b = t
        return h3.MfLinear(torch.from_numpy(wq.view(np.int32)).to(dev), bf(sc), bf(bi), k, bf(b))
    bw = h3.H3BlockWeights(lin(w["qkv"], hdn), lin(w["out"], inner), lin(w["fc1"], hdn), lin(w["fc2"], ffn),
                           bf(w["q_norm"]), bf(w["k_norm"]), bf(w["norm1"]), bf(w["norm2"]))
    cfg = h3.H3DiTConfig(hidden=hdn, heads=H, head_dim=hd, ffn=ffn, mlp_kind=h3.MLP_GELU, rot=rot, eps=eps, layers=1)
    blk = h3.H3DiTBlocks(cfg, [bw])
    md = [bf(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).to(dev)
    ct, st = bf(cos), bf(sin)
    h_init = bf(h0)
    h = h_init.clone()
    blk.block_forward(0, h, md, rm, ct, st, None)  # parity run on the oracle's inputs
    got = h.cpu().view(torch.int16).numpy().view(np.uint16)
    ctx = h3.context(0)
    ctx.check_device()
    for _ in range(max(3, args.warmup)):
        h.copy_(h_init)
        blk.block_forward(0, h, md, rm, ct, st, None)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    clocks = ClockSampler(0)
    clocks.start()
    steps = max(1, args.steps)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # written between steps: L2 is 126 MB

    def timed(body) -> float:
        """mean ms of body() over `steps`, each step after an L2 flush that the events exclude"""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a_, b_ in evs:
            flush.fill_(1)
            a_.record(stream)
            body()
            b_.record(stream)
        torch.cuda.synchronize()
        return sum(a_.elapsed_time(b_) for a_, b_ in evs) / steps

    def direct():
        h.copy_(h_init)  # every step starts from the same input (an 8 MB device copy)
        blk.block_forward(0, h, md, rm, ct, st, None)

    ctx.lib.wx_ctx_profile_enable(ctx.h, 1)
    n0 = ctx.lib.wx_ctx_launch_count(ctx.h)
    ms_block = timed(direct)
    n1 = ctx.lib.wx_ctx_launch_count(ctx.h)
    ms = (ctypes.c_double * 10)()
    cnt = (ctypes.c_int64 * 10)()
    ctx.lib.wx_ctx_profile_read(ctx.h, ms, cnt, 10)
    ctx.lib.wx_ctx_profile_enable(ctx.h, 0)
    ctx.check_device()
    # the same block replayed as one CUDA graph (wx_dit_block_graph_create / wx_graph_launch)
    graph = blk.block_graph(0, h, md, rm, ct, st, None)
    for _ in range(max(3, args.warmup)):
        h.copy_(h_init)
        graph.launch()
    torch.cuda.synchronize()
    ng0 = ctx.lib.wx_ctx_launch_count(ctx.h)

    def replay():
        h.copy_(h_init)
        graph.launch()

    graph_ms = timed(replay)
    graph_launches = ctx.lib.wx_ctx_launch_count(ctx.h) - ng0
    clk = clocks.stop()  # sampled over the direct and the graph loops
    graph_kernels = graph.kernels()
    graph_ok = bool(torch.equal(h.cpu().view(torch.int16), torch.from_numpy(got.view(np.int16))))
    # end to end through the public API with host buffers: pinned H2D of h, the block's
    # graph, D2H of h
    host_in = torch.from_numpy(h0.view(np.int16).copy()).view(torch.bfloat16).pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    torch.cuda.synchronize()

    def end_to_end():
        h.copy_(host_in, non_blocking=True)
        graph.launch()
        host_out.copy_(h, non_blocking=True)

    e2e_ms = timed(end_to_end)
    graph.close()
    ctx.check_device()
    gemm_fl = 2.0 * S * (hdn * 3 * inner + inner * hdn + hdn * ffn + ffn * hdn)
    attn_fl = 4.0 * S * S * hd * H
    peaks, kind = load_peaks()
    pk = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    attn_ms, gemm_ms = ms[1] / steps, ms[0] / steps
    roof = dict(kernel="flash_attn_pair_kernel<false, 64> (dense, paired query tiles)", bound="tensor",
                achieved=attn_fl / (attn_ms / 1e3) / 1e12 if attn_ms > 0 else 0.0, peak=pk, unit="TFLOP/s",
                avg_launch_ms=attn_ms, flops_per_launch=attn_fl, traffic=None, peak_kind=f"{kind} burst bf16")
    roof["frac"] = roof["achieved"] / pk
    # the oracle's whole block on every host thread (best of 3)
    threads = O.set_num_threads(0)
    cfgd = dict(heads=H, head_dim=hd, eps=eps, rot=rot, mlp_kind=0)
    cpu_t, ref = [], None
    for _ in range(3):
        t0 = time.perf_counter()
        ref, _at = O.block_forward(h0, w, mods, rowmap, cos, sin, cfgd)
        cpu_t.append(time.perf_counter() - t0)
    gf, rf = O.bf16_to_f32(got).astype(np.float64), O.bf16_to_f32(ref).astype(np.float64)
    rel = float(np.abs(gf - rf).max() / np.abs(rf).max())
    cosv = float((gf.ravel() @ rf.ravel()) / (np.linalg.norm(gf) * np.linalg.norm(rf)))
    if not graph_ok:
        raise RuntimeError("the block's CUDA graph gave a different output from the direct call")
    return dict(metric="DiT block ms/block (c1)", value=graph_ms, unit="ms/block", n_gpus=1, steps=steps,
                warmup=max(3, args.warmup), ms_per_step=graph_ms, higher_is_better=False, scaling="weak",
                vs_baseline=None, dtype="bf16", data="synthetic",
                config=dict(workload="c1: one DiT block, S=4096 (16x16x16), hidden 1024, 16x64 heads, FFN 4096 GELU, "
                                     "dense attention, 6-bit g64", S=S, hidden=hdn, heads=H, head_dim=hd, ffn=ffn,
                            l2="inputs smaller than L2: a 256 MB buffer is written before each step, outside its "
                               "events; each step restarts from the same h (an 8 MB device copy inside them)"),
                roofline=roof,
                qgemm=dict(tflops=gemm_fl / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0, ms=gemm_ms,
                           flops=gemm_fl),
                kernel_ms_direct={k: dict(ms=float(ms[i]) / steps, launches=int(cnt[i]) // steps) for i, k in
                           enumerate(["qgemm", "attention", "routing", "row_kernels", "dequant", "other",
                                      "qk_norm_rope", "norm_modscale"])},
                gpu_launches=int(graph_launches), clocks=clk,
                e2e=dict(value=e2e_ms, unit="ms/block", h2d_bytes_per_step=S * hdn * 2, d2h_bytes_per_step=S * hdn * 2),
                graph=dict(kernels_per_replay=graph_kernels, same_output_as_direct=graph_ok,
                           what="value: the block replayed as one CUDA graph (wx_graph_launch), the same 8 MB "
                                "input copy per step"),
                direct=dict(ms_per_block=ms_block, graph_speedup=ms_block / graph_ms,
                            what="the plain wx_dit_block_forward call per step"),
                parity=dict(max_rel_err=rel, cosine=cosv, bound="max rel err <= 2e-2, cosine >= 0.999"),
                cpu_baseline=dict(value=min(cpu_t) * 1e3, unit="ms/block", cores=threads, kind="port",
                                  sample="the whole block (oracle, C, OpenMP), best of 3, same weights and inputs"))


def run_rowops(args) -> dict:
    """The HBM-bound row kernels standalone at the config-1 / config-4 / config-5 shapes:
    QK-RMSNorm + RoPE of q and k of a packed q|k|v buffer in place (K3, the separate path;
    in the step it runs in the q|k|v GEMM's epilogue where the geometry allows), RMSNorm +
    modulation (K4) and the gated residual (K5, the PAB reuse path; the step fuses it into
    GEMM epilogues otherwise). Kernel time = the CUDA events libwx records around each launch;
    a 256 MB buffer is written between launches to flush L2 (outside the events).
    Bytes: K3 2 x (read + write of S x H x hd bf16) + cos/sin rows; K4 read + write of S x hidden
    bf16 + the u32 row map; K5 two reads + one write of S x hidden bf16 + the row map."""
    import ctypes
    import torch
    from wuxianhuabu_b200 import h3
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1234 + 7)
    peaks, kind = load_peaks()
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    ctx = h3.context(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    shapes = [("c1", 4096, 16, 64, 64, 1024), ("c4", 29032, 24, 128, 96, 3072), ("c5", 126512, 24, 128, 96, 3072)]
    reps = max(1, args.steps)
    res = []
    for name, S, H, hd, rot, hidden in shapes:
        inner = H * hd
        qkv = torch.randn((S, 3 * inner), device=dev, generator=gen).to(torch.bfloat16)
        wq = (1 + 0.02 * torch.randn(hd, device=dev, generator=gen)).to(torch.bfloat16)
        wk = (1 + 0.02 * torch.randn(hd, device=dev, generator=gen)).to(torch.bfloat16)
        cos = torch.randn((S, rot // 2), device=dev, generator=gen).to(torch.bfloat16)
        sin = torch.randn((S, rot // 2), device=dev, generator=gen).to(torch.bfloat16)
        x = torch.randn((S, hidden), device=dev, generator=gen).to(torch.bfloat16)
        other = torch.randn((S, hidden), device=dev, generator=gen).to(torch.bfloat16)
        out = torch.empty_like(x)
        wn = (1 + 0.02 * torch.randn(hidden, device=dev, generator=gen)).to(torch.bfloat16)
        tabs = [(0.02 * torch.randn((6, hidden), device=dev, generator=gen)).to(torch.bfloat16) for _ in range(3)]
        rm = torch.from_numpy((np.arange(S) % 6).astype(np.int32)).to(dev)
        P = h3._p
        kernels = [
            ("qk_norm_rope", 6, 2 * (2 * S * inner * 2) + 2 * S * (rot // 2) * 2,
             lambda: ctx.call("wx_qk_norm_rope_qkv", P(qkv), S, H, hd, P(wq), P(wk), P(cos), P(sin), rot, 1e-6)),
            ("norm_modscale", 7, 2 * S * hidden * 2 + S * 4,
             lambda: ctx.call("wx_norm_modscale", P(x), S, hidden, P(wn), P(tabs[0]), P(tabs[1]), P(rm), 1e-6,
                              P(out))),
            ("mod_gate", 3, 3 * S * hidden * 2 + S * 4,
             lambda: ctx.call("wx_mod_gate", P(x), P(other), P(tabs[2]), P(rm), S, hidden, P(out))),
        ]
        for kname, kind_idx, nbytes, fn in kernels:
            for _ in range(max(1, args.warmup)):
                fn()
            torch.cuda.synchronize()
            ctx.lib.wx_ctx_profile_enable(ctx.h, 1)
            for _ in range(reps):
                flush.fill_(1)
                fn()
            torch.cuda.synchronize()
            ms = (ctypes.c_double * 10)()
            cnt = (ctypes.c_int64 * 10)()
            ctx.lib.wx_ctx_profile_read(ctx.h, ms, cnt, 10)
            ctx.lib.wx_ctx_profile_enable(ctx.h, 0)
            t = ms[kind_idx] / max(1, cnt[kind_idx]) / 1e3
            res.append(dict(config=name, kernel=kname, S=S, ms=t * 1e3, bytes=nbytes, gbs=nbytes / t / 1e9,
                            frac=nbytes / t / 1e9 / hbm, launches=int(cnt[kind_idx]), sm_mhz=_sm_clock_now(0)))
        ctx.check_device()
        del qkv, x, other, out
    return dict(metric="HBM-bound row kernels (K3 QK-norm+RoPE, K4 norm+modulation, K5 gated residual)",
                unit="GB/s", hbm_peak=hbm, peak_kind=f"{kind} HBM GB/s (copy)", kernels=res,
                l2="256 MB written between launches (outside the events)")


def _sm_clock_now(index: int = 0):
    """The SM clock (MHz) at this moment, from NVML (None where NVML is unavailable): small
    kernels are latency-bound and follow the clock, which the power cap lowers after heavy work."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(index)
        return int(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
    except Exception:
        return None


def _qkv_rope_point(args, lin, x, M, K, N, fl, pk, ctx, dev, g, flush) -> dict:
    """The same shape as a q|k|v projection (N = 3 * heads * 128) with QK-RMSNorm + RoPE
    (rot 96): one GEMM with the norm/RoPE epilogue (wx_qkv_norm_rope) against the projection
    followed by the separate row kernel, kernel CUDA-event time per call."""
    import ctypes
    import torch
    from wuxianhuabu_b200 import h3
    heads, hd, rot = N // 384, 128, 96
    qn = (1 + 0.02 * torch.randn(hd, device=dev, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.02 * torch.randn(hd, device=dev, generator=g)).to(torch.bfloat16)
    cos = torch.randn((M, rot // 2), device=dev, generator=g).to(torch.bfloat16)
    sin = torch.randn((M, rot // 2), device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    inner = N // 3
    reps = max(1, args.steps)

    def fused():
        lin.qkv_norm_rope(x, heads, hd, qn, kn, cos, sin, rot, 1e-6, out=y)

    def separate():
        lin(x, out=y)
        for part, w in ((0, qn), (1, kn)):
            v = y[:, part * inner:(part + 1) * inner].view(M, heads, hd)
            h3.H3FusedKernels.fused_rmsnorm_rope(v, w, cos, sin, rot, 1e-6, out=v)

    out = {}
    for name, fn in (("fused", fused), ("separate", separate)):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        ctx.lib.wx_ctx_profile_enable(ctx.h, 1)
        for _ in range(reps):
            flush.fill_(1)  # evicts L2 (outside the kernels' events)
            fn()
        torch.cuda.synchronize()
        ms = (ctypes.c_double * 10)()
        cnt = (ctypes.c_int64 * 10)()
        ctx.lib.wx_ctx_profile_read(ctx.h, ms, cnt, 10)
        ctx.lib.wx_ctx_profile_enable(ctx.h, 0)
        t = sum(ms[i] for i in (0, 4, 6)) / reps / 1e3  # GEMM + weight expansion + norm/RoPE kernel
        out[f"qkv_rope_{name}_ms"] = t * 1e3
        out[f"qkv_rope_{name}_frac"] = fl / t / 1e12 / pk
    return out


def c2_plan(shape: str, rows: str):
    """The config-2 points to time and the small-M CTA shapes to force at each.

    Points: the sweep (M 256 / 4096 / 28520 / 111600 at four K, N), or `shape` =
    "M,K,N[;M,K,N...]", consecutive points of one K, N sharing one weight. CTA shapes: `rows` =
    "R[/T],..." (WX_QGEMM_ROWS = R weight rows per CTA, WX_QGEMM_TPR = T expansion threads per
    row; 0 = the library's choice), or [None]: the environment left as it is."""
    ms_all = (256, 4096, 28520, 111600)
    plan = [((K, N), ms_all) for K, N in [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072)]]
    if shape:
        plan = []
        for pt in shape.split(";"):
            M0, K0, N0 = (int(v) for v in pt.split(","))
            if plan and plan[-1][0] == (K0, N0):
                plan[-1] = (plan[-1][0], plan[-1][1] + (M0,))
            else:
                plan.append(((K0, N0), (M0,)))
    rows_list = []
    for r in rows.split(",") if rows else []:
        parts = r.split("/")
        if len(parts) > 2 or not all(p.isdigit() for p in parts) or int(parts[0]) not in (0, 128, 256) or \
                (len(parts) == 2 and int(parts[1]) not in (0, 2, 4)):
            raise ValueError(f"--rows: {r!r} is not R or R/T with R in 0/128/256 and T in 0/2/4")
        rows_list.append(r)
    return plan, rows_list or [None]


def run_c2(args) -> dict:
    """the 6-bit quantized linear sweep."""
    import torch
    from wuxianhuabu_b200 import h3
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234 + 1)
    import ctypes
    peaks, kind = load_peaks()
    pk = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    res = []
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    plan, rows_list = c2_plan(args.shape, args.rows)
    for (K, N), ms_list in plan:
        bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16) if args.bias else None
        lin = h3.MfLinear.quantize(torch.randn((N, K), device=dev, generator=g) * 0.02, bias=bias)
        if args.lora > 0:  # one adapter of rank args.lora (the LoRA row: a K extension of the GEMM)
            a = (torch.randn((K, args.lora), device=dev, generator=g) * 0.02).to(torch.bfloat16)
            b = (torch.randn((args.lora, N), device=dev, generator=g) * 0.02).to(torch.bfloat16)
            lin.set_lora([h3.LoraRef(a, b, 1.0)])
        for M, rows in [(M, r) for M in ms_list for r in rows_list]:
            if rows is not None:  # "R" or "R/T": weight rows per CTA, expansion threads per row
                os.environ["WX_QGEMM_ROWS"] = rows.split("/")[0]
                os.environ["WX_QGEMM_TPR"] = rows.split("/")[1] if "/" in rows else "0"
            x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            for _ in range(max(1, args.warmup)):
                lin(x, out=y)
            torch.cuda.synchronize()
            ctx = h3.context(0)
            ctx.lib.wx_ctx_profile_enable(ctx.h, 1)
            reps = max(1, args.steps)
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            # each call after a 256 MB write that evicts L2 (the weights and activations of the
            # small points would stay L2-resident otherwise); the kernels' own events exclude it
            # and so do the events around each call. The write also gives the host time to
            # enqueue the next call, so no host launch time lands inside the events.
            for a_, b_ in evs:
                flush.fill_(1)
                a_.record()
                lin(x, out=y)
                b_.record()
            sm_mhz = _sm_clock_now(0)  # while the last calls still run
            torch.cuda.synchronize()
            ms = (ctypes.c_double * 10)()
            cnt = (ctypes.c_int64 * 10)()
            ctx.lib.wx_ctx_profile_read(ctx.h, ms, cnt, 10)
            ctx.lib.wx_ctx_profile_enable(ctx.h, 0)
            t_call = sum(a_.elapsed_time(b_) for a_, b_ in evs) / reps / 1e3
            # the kernels' own time: CUDA events libwx records around each launch (the GEMM,
            # plus the weight expansion of the two-pass path)
            t = (ms[0] + ms[4]) / reps / 1e3
            fl = 2.0 * M * N * K
            byts = 2 * M * K + 0.75 * N * K + 4 * N * (K // 64) + 2 * M * N
            row = dict(M=M, K=K, N=N, ms=t * 1e3, tflops=fl / t / 1e12, frac=fl / t / 1e12 / pk,
                       gbs=byts / t / 1e9, gbs_frac=byts / t / 1e9 / hbm, ms_per_call=t_call * 1e3,
                       path="fused" if (M <= 512 and N % 128 == 0 and args.lora == 0) else "two-pass",
                       lora_rank=args.lora, bias=bool(args.bias), sm_mhz=sm_mhz)
            if rows is not None:
                row["cta_rows"] = rows
            if args.qkv_rope and N % 384 == 0:
                row.update(_qkv_rope_point(args, lin, x, M, K, N, fl, pk, ctx, dev, g, flush))
            res.append(row)
            del x, y
    return dict(metric="6-bit qGEMM sweep (c2)", unit="TFLOP/s", peak=pk, peak_kind=f"{kind} burst bf16", hbm_peak=hbm,
                sweep=res, timing="ms = the kernels' CUDA-event time per call (libwx records events around each "
                                  "launch); ms_per_call = events around each call; L2 is evicted by a 256 MB write "
                                  "before every call, outside both")


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="wx", choices=["wx", "reference"])
    ap.add_argument("--config", default="c5",
                    choices=list(CONFIGS) + ["c1", "c3", "c3full", "c3dense", "c2", "c5attn", "c5attn_dense",
                                             "rowops"])
    ap.add_argument("--router", default="topk", choices=["topk", "sol"],
                    help="c3 / c3full / c5attn: top-k 25%% over 128-row blocks, or SOL tau 1.3 over 64-row blocks")
    ap.add_argument("--shape", default="", help="c2 only: points M,K,N[;M,K,N...] instead of the sweep")
    ap.add_argument("--rows", default="",
                    help="c2 only: small-M CTA shapes to time at each point, e.g. 128/2,128/4,256,0 (weight rows "
                         "per CTA [/ expansion threads per row]; 0 = the library's choice)")
    ap.add_argument("--lora", type=int, default=0, help="c2 only: attach one LoRA adapter of this rank")
    ap.add_argument("--bias", action="store_true", help="c2 only: the linears carry a bias (added in the epilogue)")
    ap.add_argument("--qkv-rope", action="store_true",
                    help="c2 only: also time N = 3*heads*128 shapes as q|k|v projections with QK-norm + RoPE, "
                         "fused epilogue against the separate kernel")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.config in ("c1", "c3", "c3full", "c3dense", "c2", "c5attn", "c5attn_dense", "rowops"):
        import torch
        torch.cuda.set_device(0)
        if args.config == "c1":
            r = run_c1(args)
        elif args.config == "rowops":
            r = run_rowops(args)
        elif args.config == "c2":
            r = run_c2(args)
        elif args.config.startswith("c5attn"):  # the config-5 step's attention call, standalone
            r = run_c3(args, 126512, dense=args.config == "c5attn_dense", g=14912)
        else:
            r = run_c3(args, 111600 if args.config == "c3full" else 28520, dense=args.config == "c3dense")
        print(json.dumps(r))
        return
    c = geometry(args.config)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    base_cfg = dict(workload=f"{args.config}: " + ("720p x 121f step, 4 ref images, PAB window" if args.config == "c5"
                                                   else "DiT step"),
                    S=c["S"], strip_rows=c["g"], video_rows=c["video"], layers=c["layers"], hidden=c["hidden"],
                    heads=c["heads"], ffn=c["ffn"], weights="6-bit affine g64", attention="mix: dense anchors + top-k 25% (128 blocks)",
                    pab=dict(k=PAB_K, max_stale=PAB_MAX_STALE, window=WINDOW), global_batch=1, seq_len=c["S"],
                    parallelism=f"ulysses{world}" if world > 1 else "single", l2="inputs larger than L2 (h 0.78 GB, weights 4.4 GB)")

    plan = window_plan()
    positions = [i % WINDOW for i in range(args.warmup, args.warmup + args.steps)]
    n_refresh = sum(1 for pos in positions if plan[pos])
    base_cfg.update(refresh_steps=n_refresh, reuse_steps=args.steps - n_refresh)

    if args.impl == "reference":
        if rank != 0:
            return
        cs = CpuSample(c, plan)
        vals, sampled = [], []
        for i in range(args.warmup + args.steps):
            r = cs.run()
            if i >= args.warmup:
                vals.append(r["value"])
                sampled.append(r["sampled_s"])
        v = float(np.mean(vals))
        line = dict(metric=METRIC, value=v, unit="s/step", n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                    ms_per_step=v * 1e3, higher_is_better=False, scaling="strong", vs_baseline=None, dtype="bf16",
                    data="synthetic", config=base_cfg, impl="reference",
                    cpu_baseline=dict(value=v, unit="s/step", cores=cs.threads, kind="port", sample=cs.sample,
                                      sampled_s_per_step=float(np.mean(sampled))),
                    e2e=dict(value=v, unit="s/step", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                    note="reference = the oracle's C restatement of the reference's MLX/Metal algorithm; "
                         "Swift/MLX/Metal cannot run on this box")
        print(json.dumps(line))
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from wuxianhuabu_b200 import h3
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

        def bcast(obj):
            box = [obj]
            dist.broadcast_object_list(box, src=0)
            return box[0]
        h3.init_sequence_parallel(world, rank, bcast)
    try:
        line = run_step_bench(args, c, base_cfg, dev, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def _max_over_ranks(x: float, dist) -> float:
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, dist) -> float:
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def memory_bound_kernels(c: dict, prof: dict, world: int, peaks: dict, peaks_kind: str) -> dict:
    """Achieved bandwidth of the HBM-bound kernels of the step (per launch, this rank's rows),
    from the CUDA-event times libwx recorded around each launch and the algorithmic bytes:
      QK-RMSNorm + RoPE of q and k: read + write of 2 x rows x inner bf16, + cos/sin rows;
      RMSNorm + modulation: read + write of rows x hidden bf16 (+ the u32 row map);
      the fused sequence-parallel exchange (QK-norm/RoPE + v copy stored into the owners'
      buffers): reads rows x 3 x inner bf16 and stores the same, (P-1)/P of it over NVLink.
    HBM peak: MEASURED_PEAKS hbm_gbs; NVLink: the pool's measured peer copy of 770 GB/s per
    direction per GPU (900 nominal)."""
    rows = c["S"] // world
    inner, hidden = c["inner"], c["hidden"]
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    nvlink = 770.0

    def rate(kind, nbytes, peak):
        ms_, n = prof[kind]["ms"], prof[kind]["launches"]
        if n == 0 or ms_ <= 0:
            return None
        t = ms_ / n / 1e3
        return dict(gbs=nbytes / t / 1e9, frac=nbytes / t / 1e9 / peak, avg_launch_ms=t * 1e3,
                    bytes_per_launch=nbytes, launches=n)
    rope_b = 2 * (2 * rows * inner * 2) + 2 * rows * (ROT // 2) * 2
    norm_b = 2 * rows * hidden * 2 + rows * 4
    out = dict(row_kernels=dict(qk_norm_rope=rate("qk_norm_rope", rope_b, hbm),
                                norm_modscale=rate("norm_modscale", norm_b, hbm),
                                peak=hbm, peak_kind=f"{peaks_kind} HBM GB/s (copy)"))
    if world > 1:
        xb = rows * 3 * inner * 2
        ex = rate("qkv_to_peers", xb * (world - 1) / world, nvlink)
        if ex is not None:
            ex["what"] = "bytes this rank stores into the other ranks' buffers per launch (q|k|v rows of their heads)"
        pw = prof["peer_wait"]
        out["exchange"] = dict(qkv_to_peers=ex, nvlink_peak_gbs=nvlink,
                               nvlink_peak_kind="measured peer copy per direction (pool figure)",
                               peer_wait_ms=pw["ms"], peer_wait_launches=pw["launches"],
                               attention_out_peer_bytes_per_launch=(c["S"] * (c["heads"] // world) * 128 * 2
                                                                    * (world - 1) / world))
    return out


def run_step_bench(args, c, base_cfg, dev, world, rank, local, dist) -> dict:
    import ctypes
    import torch
    peaks, peaks_kind = load_peaks()
    model = Model(c, dev)
    run = Runner(model, rank, world)
    ctx = run.ctx
    lib = ctx.lib

    def sync_all():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize()

    # warm-up along the window
    for i in range(args.warmup):
        run.step(i)
    sync_all()
    ctx.check_device()
    # timed region (device-resident inputs)
    clocks = ClockSampler(local)
    clocks.start()
    stream = torch.cuda.current_stream()
    lib.wx_ctx_profile_enable(ctx.h, 1)
    ctx.trace(True)
    n0 = lib.wx_ctx_launch_count(ctx.h)
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.warmup, args.warmup + args.steps):
        run.step(i)
    e1.record(stream)
    sync_all()
    n1 = lib.wx_ctx_launch_count(ctx.h)
    clk = clocks.stop()
    ms = (ctypes.c_double * 10)()
    cnt = (ctypes.c_int64 * 10)()
    lib.wx_ctx_profile_read(ctx.h, ms, cnt, 10)
    lib.wx_ctx_profile_enable(ctx.h, 0)
    trace = ctx.trace_read(max_records=64 * 48 * max(1, args.steps))
    ctx.trace(False)
    ctx.check_device()
    total_ms = _max_over_ranks(e0.elapsed_time(e1), dist)
    s_per_step = total_ms / 1e3 / args.steps
    positions = [i % WINDOW for i in range(args.warmup, args.warmup + args.steps)]
    n_refresh = sum(1 for p in positions if run.plan[p])
    fl = [step_flops(c, run.plan[p]) for p in positions]
    # work done by this rank: 1/world of every GEMM row and of every attention head
    gemm_flops = sum(f["gemm"] for f in fl) / world
    attn_flops = sum(f["attn"] for f in fl) / world
    kinds = ["qgemm", "attention", "routing", "row_kernels", "dequant", "collectives", "qk_norm_rope",
             "norm_modscale", "qkv_to_peers", "peer_wait"]
    prof = {k: dict(ms=float(ms[i]), launches=int(cnt[i])) for i, k in enumerate(kinds)}
    attn_ms = prof["attention"]["ms"]
    gemm_ms = prof["qgemm"]["ms"]
    attn_launches = max(1, prof["attention"]["launches"])
    peak_t = peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"])
    ach_attn = attn_flops / (attn_ms / 1e3) / 1e12 if attn_ms > 0 else 0.0
    ach_gemm = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    if attn_ms >= gemm_ms:
        # DRAM bytes per attention call from one ncu capture; a rank holds 1/world of the heads
        traffic = ATTN_TRAFFIC_C5 / world if c["name"] == "c5" else None
        roof = dict(kernel="flash_attn_pair_kernel <paired> + <duo> (tcgen05 sparse/dense flash attention)", bound="tensor",
                    achieved=ach_attn, peak=peak_t, unit="TFLOP/s", frac=ach_attn / peak_t,
                    flops_per_launch=attn_flops / attn_launches, avg_launch_ms=attn_ms / attn_launches,
                    traffic=traffic, traffic_unit="bytes per launch (ncu dram__bytes_read+write)",
                    peak_kind=f"{peaks_kind} sustained bf16", per_gpu=True)
    else:
        roof = dict(kernel="gemm_bf16_tc_kernel", bound="tensor", achieved=ach_gemm, peak=peak_t, unit="TFLOP/s",
                    frac=ach_gemm / peak_t, traffic=None, peak_kind=f"{peaks_kind} sustained bf16", per_gpu=True)
    line = dict(metric=METRIC, value=s_per_step, unit="s/step", n_gpus=world, steps=args.steps, warmup=args.warmup,
                ms_per_step=s_per_step * 1e3, higher_is_better=False, scaling="strong", vs_baseline=None,
                dtype="bf16", data="synthetic", config=dict(base_cfg),
                roofline=roof,
                qgemm=dict(tflops=ach_gemm, frac=ach_gemm / peak_t, ms=gemm_ms, launches=prof["qgemm"]["launches"],
                           flops=gemm_flops, peak_kind=f"{peaks_kind} sustained bf16", per_gpu=True),
                kernel_ms=prof, gpu_launches=int(_sum_over_ranks(n1 - n0, dist)), clocks=clk)
    line.update(memory_bound_kernels(c, prof, world, peaks, peaks_kind))
    line["phases"] = phase_summary(trace, args.steps)
    if world > 1 and "exchange" in line:
        line["exchange"].update(peer_store_summary(trace, line["phases"], c, world, args.steps,
                                                   line["exchange"]["attention_out_peer_bytes_per_launch"]))
    # e2e through the public API with host buffers (pinned H2D of each rank's latent rows,
    # D2H of the updated rows)
    if not args.no_e2e:
        host_in = torch.empty(run.video_x.shape, dtype=torch.float32, pin_memory=True)
        host_in.copy_(run.video_x)
        host_out = torch.empty_like(host_in, pin_memory=True)
        sync_all()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            run.video_x.copy_(host_in, non_blocking=True)
            run.step(i)
            host_out.copy_(run.video_x, non_blocking=True)
        f1.record(stream)
        sync_all()
        e2e = _max_over_ranks(f0.elapsed_time(f1), dist) / 1e3 / args.steps
        nbytes = int(_sum_over_ranks(run.video_x.numel() * 4, dist))
        finite = _sum_over_ranks(float(not bool(torch.isfinite(host_out).all().item())), dist) == 0
        line["e2e"] = dict(value=e2e, unit="s/step", h2d_bytes_per_step=nbytes, d2h_bytes_per_step=nbytes,
                           finite=finite)
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        cs = CpuSample(c, run.plan)
        r = cs.run()
        line["cpu_baseline"] = dict(value=r["value"], unit="s/step", cores=cs.threads, kind="port",
                                    sample=cs.sample, sampled_s=r["sampled_s"])
    return line


if __name__ == "__main__":
    main()
