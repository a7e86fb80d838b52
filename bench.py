"""Benchmark: dynamic block-shape block-sparse attention, forward + backward of
one video self-attention layer (benchmark config 1, 720p: B=1, 40 heads,
head_dim 128, grid 21x45x80 = 75,600 tokens + 125 audio tokens, zone-structured
q/k/v, top-k 8% + cumulative mass 0.9) on 1..N B200s of one node.

A step = audio token norms + zone statistics + shape choice + permutation +
pooled selection + sparse attention forward + scatter, then the backward
(gather dO, sparse attention backward, scatter dQ/dK/dV).  With N > 1 GPUs the
layer runs under Ulysses sequence parallelism (each rank holds S/N tokens of
all 40 heads; all-to-all to 40/N heads of the full sequence and back), so the
total work is fixed: "scaling": "strong".

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 720p|1080p|2k]
    torchrun --nproc-per-node N bench.py --gpus N ...

--config picks benchmark config 1 (720p, default: the metric's workload), 2 (1080p,
21x68x120) or 3 (2K, 31x90x160, top-k 5%); every config has 40 heads of 128.

value = whole-job effective TFLOPS = FLOPs of the selected 64x64 tile pairs
(4*D*64*64 per pair for the forward, 2.5x that for the backward) / time.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = dict(workload="720p dynamic BSA layer fwd+bwd (benchmark config 1)", model="prism-video-self-attn",
              grid=(21, 45, 80), heads=40, head_dim=128, audio_tokens=125, hidden=5120,
              sparsity=0.92, cdf_threshold=0.9, method="ivpq")
# benchmark configs 2 and 3 (same value generator and selection rule; 2K uses top-k 5%)
CONFIGS = {
    "720p": dict(CONFIG),
    "1080p": dict(CONFIG, workload="1080p dynamic BSA layer fwd+bwd (benchmark config 2)",
                  grid=(21, 68, 120)),
    # config 3's zone-statistics inputs: V ~ N(0, 1) (the video hidden states) and the a2v
    # residual N(0, 1) scaled per zone by U(0.2, 2)
    "2k": dict(CONFIG, workload="2K dynamic BSA layer fwd+bwd (benchmark config 3)",
               grid=(31, 90, 160), audio_tokens=189, sparsity=0.95, v_values="normal",
               a2v_zone_scale=(0.2, 2.0)),
}
# DRAM bytes (read + write) per head of one launch of each attention kernel on the 720p
# layer: ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-head capture / 4.  Heads
# are independent (one head's K/V tiles stay in L2), so a launch over h heads moves h times
# this; roofline.traffic reports it for the dominant kernel.
TRAFFIC_PER_HEAD_720P = {"bsa_fwd": (545.0e6 + 170.6e6) / 4,
                         "bsa_bwd_dkdv": (584.3e6 + 174.3e6) / 4,
                         "bsa_bwd_dq": (555.9e6 + 88.9e6) / 4}
FWD_BWD_FACTOR = 3.5  # 1 (forward) + 2.5 (backward): the canonical FLOP count of one fwd+bwd
# --path uniform: the uniform fixed-shape path (flash_attn_bsa_3d) with the training
# configs' block-sparse settings (4x4x4 chunks, sparsity 0.75, cdf threshold 0.2)
UNIFORM = dict(chunk=(4, 4, 4), sparsity=0.75, cdf_threshold=0.2)


def uniform_grid():
    c = CONFIG["chunk"]
    return tuple(math.ceil(x / ci) * ci for x, ci in zip(CONFIG["grid"], c))


def padded_grid():
    if CONFIG.get("path") == "uniform":
        return uniform_grid()
    return tuple(math.ceil(x / 8) * 8 for x in CONFIG["grid"])


# ------------------------------------------------------------------ inputs
def make_layer_inputs(device, rank=0, world=1, seed=0):
    """Synthetic layer inputs, generated on the device from a seeded generator: q, k (and
    v, except for config 3) per zone = zone mean + 0.3 noise, both N(0, 0.5^2); config 3's
    v is N(0, 1) and its a2v residual N(0, 1) scaled per zone by U(0.2, 2)."""
    import torch
    T, H, W = CONFIG["grid"]
    h, D = CONFIG["heads"], CONFIG["head_dim"]
    Tp, Hp, Wp = (math.ceil(x / 8) * 8 for x in (T, H, W))
    g = torch.Generator(device=device).manual_seed(seed)

    def zoned():
        mean = torch.randn(h, Tp // 8, Hp // 8, Wp // 8, D, generator=g, device=device) * 0.5
        m = mean.repeat_interleave(8, 1).repeat_interleave(8, 2).repeat_interleave(8, 3)
        x = m + 0.3 * 0.5 * torch.randn(h, Tp, Hp, Wp, D, generator=g, device=device)
        return x[:, :T, :H, :W].reshape(h, T * H * W, D).transpose(0, 1).to(torch.bfloat16)

    S = T * H * W
    q, k = zoned(), zoned()                      # [S, h, D]  (sequence-major, like the projections)
    if CONFIG.get("v_values") == "normal":
        v = torch.randn(S, h, D, generator=g, device=device).to(torch.bfloat16)
    else:
        v = zoned()
    do = torch.randn(S, h, D, generator=g, device=device).to(torch.bfloat16)
    a2v = torch.randn(S, CONFIG["hidden"], generator=g, device=device)
    if CONFIG.get("a2v_zone_scale"):
        lo, hi = CONFIG["a2v_zone_scale"]
        zs = lo + (hi - lo) * torch.rand(Tp // 8, Hp // 8, Wp // 8, generator=g, device=device)
        zs = zs.repeat_interleave(8, 0).repeat_interleave(8, 1).repeat_interleave(8, 2)
        a2v = a2v * zs[:T, :H, :W].reshape(S, 1)
    a2v = a2v.to(torch.bfloat16)
    C = -(-S // world)  # ceil(S / P) rows per shard, the last one shorter
    sl = slice(min(rank * C, S), min(rank * C + C, S))
    sizes = [sl.stop - sl.start if r == rank else 0 for r in range(world)]
    out = {}
    for name, t in (("q", q), ("k", k), ("v", v), ("do", do)):
        out[name] = t[sl].reshape(1, sizes[rank], h * D).contiguous()
    out["a2v"] = a2v[sl].unsqueeze(0).contiguous()
    return out, S


# ------------------------------------------------------------------ clocks
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        def run():
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            while not self._stop.is_set():
                try:
                    r = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                        "--format=csv,noheader,nounits"], capture_output=True,
                                       text=True, timeout=5)
                    self.samples.append([x.strip() for x in r.stdout.strip().split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        sm = [float(s[0]) for s in self.samples if len(s) >= 7 and s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if len(s) >= 7 and s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples if len(s) >= 7 for i in range(4)
                          if s[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ------------------------------------------------------------------ step
def attend(q, k, v, a2v, S):
    """The layer's attention core through the package's public API (either path)."""
    from prism_b200.attention import dynamic_self_attention, uniform_self_attention
    if CONFIG.get("path") == "uniform":
        g = CONFIG.get("guidance", "none")
        gkw = {}
        if g in ("variance", "audio_variance"):
            gkw["variance_boost_gamma"] = 1.0
        if g in ("audio", "audio_variance"):
            gkw.update(a2v_bridge_residual=a2v, audio_boost_gamma=1.0, audio_weighted_lambda=1.0)
        corr = CONFIG.get("correction", "none")
        if corr != "none":
            gkw.update(correction=corr, taylor_alpha_f=0.5)
        return uniform_self_attention(q, k, v, CONFIG["grid"], CONFIG["heads"], full_seq_len=S,
                                      sparsity=CONFIG["sparsity"],
                                      cdf_threshold=CONFIG["cdf_threshold"],
                                      chunk_3d_shape_q=CONFIG["chunk"],
                                      chunk_3d_shape_k=CONFIG["chunk"], **gkw)
    return dynamic_self_attention(q, k, v, CONFIG["grid"], CONFIG["heads"], a2v_bridge_residual=a2v,
                                  full_seq_len=S, method=CONFIG["method"],
                                  sparsity=CONFIG["sparsity"],
                                  cdf_threshold=CONFIG["cdf_threshold"])


def inference_only():
    """The bias-rectified path runs forward only (inference)."""
    return CONFIG.get("correction", "none") != "none"


def make_step(inp, S, world, capture=None):
    import torch

    def step(q, k, v, do, a2v):
        if inference_only():
            with torch.no_grad():
                return attend(q, k, v, a2v, S)
        x = attend(q, k, v, a2v, S)
        x.backward(do)
        return x
    return step


def selected_pairs(q, k, v, a2v, S, world):
    """Count selected (q tile, k tile) pairs over all heads of this rank."""
    import torch
    from prism_b200.attention import audio_token_norms
    from prism_b200.communications import all_to_all_4D
    from prism_b200.bsa_interface import run_bsa_uniform
    from prism_b200.dynamic_block_attention import run_bsa_dynamic
    from prism_b200.parallel_states import get_sequence_parallel_state, nccl_info
    h, D = CONFIG["heads"], CONFIG["head_dim"]
    with torch.no_grad():
        norms = audio_token_norms(a2v, S)
        q4, k4, v4 = (t.view(1, t.shape[1], h, D) for t in (q, k, v))
        if get_sequence_parallel_state():
            g = nccl_info.sp_group
            q4, k4, v4 = (all_to_all_4D(t, g, 2, 1, S) for t in (q4, k4, v4))
        if CONFIG.get("path") == "uniform":
            _, plan = run_bsa_uniform(q4, k4, v4, CONFIG["grid"], layout="bshd",
                                      sparsity=CONFIG["sparsity"],
                                      cdf_threshold=CONFIG["cdf_threshold"],
                                      chunk_3d_shape_q=CONFIG["chunk"],
                                      chunk_3d_shape_k=CONFIG["chunk"], return_plan=True)
        else:
            _, plan = run_bsa_dynamic(q4, k4, v4, CONFIG["grid"], layout="bshd",
                                      method=CONFIG["method"], sparsity=CONFIG["sparsity"],
                                      cdf_threshold=CONFIG["cdf_threshold"],
                                      audio_token_norms=norms, return_plan=True)
        def popcount(words):
            x = words.to(torch.int64) & 0xFFFFFFFF
            cnt = torch.zeros_like(x)
            for _ in range(32):
                cnt += x & 1
                x = x >> 1
            return int(cnt.sum().item())
        bq = plan.bits_q.view(torch.int32)
        pairs = popcount(bq)
        # 64x64 products the kernels execute: a CTA walks the union of its query tiles' rows
        hq, nt, wq = bq.shape
        union2 = bq.view(hq, nt // 2, 2, wq)
        executed = 2 * popcount(union2[:, :, 0] | union2[:, :, 1])
    return pairs, plan, (q4, k4, v4, norms), executed


def kernel_times(plan, q4, k4, v4, reps=3):
    """CUDA-event timing of each attention kernel launch on its own stream."""
    import torch
    from prism_b200 import ops, _lib
    from prism_b200.dynamic_block_attention import _hsd
    qh, kh, vh = (_hsd(t, "bshd") for t in (q4, k4, v4))
    q_re = ops.gather_rows(qh, plan.grid, plan.grid_padded, plan.src_idx)
    k_re = ops.gather_rows(kh, plan.grid, plan.grid_padded, plan.src_idx_k)
    v_re = ops.gather_rows(vh, plan.grid, plan.grid_padded, plan.src_idx_k)
    heads, Sp, D = q_re.shape
    stream = torch.cuda.current_stream()
    ev = lambda: torch.cuda.Event(enable_timing=True)
    res = {}
    o, lse, o_lo = ops.bsa_fwd(q_re, k_re, v_re, plan.bits_q, plan.tile_bits, plan.sm_scale, want_lo=True)
    do = torch.randn_like(o)
    delta = torch.empty(heads, Sp, dtype=torch.float32, device=o.device)
    dq, dk, dv = torch.empty_like(o), torch.empty_like(o), torch.empty_like(o)
    P = ops._p
    st = ops._stream(o)
    calls = {
        "bsa_fwd": lambda: ops.bsa_fwd(q_re, k_re, v_re, plan.bits_q, plan.tile_bits, plan.sm_scale, want_lo=True),
        "bsa_bwd_delta": lambda: _lib.call("prism_bsa_bwd_delta", P(o), P(o_lo), P(do), heads, Sp, D, P(delta), st),
        "bsa_bwd_dkdv": lambda: _lib.call("prism_bsa_bwd_dkdv", P(q_re), P(k_re), P(v_re), P(do), P(lse),
                                          P(delta), heads, Sp, D, float(plan.sm_scale), P(plan.bits_k),
                                          P(plan.tile_bits), P(dk), P(dv), st),
        "bsa_bwd_dq": lambda: _lib.call("prism_bsa_bwd_dq", P(q_re), P(k_re), P(v_re), P(do), P(lse),
                                        P(delta), heads, Sp, D, float(plan.sm_scale), P(plan.bits_q),
                                        P(plan.tile_bits), P(dq), st),
    }
    for name, fn in calls.items():
        fn()
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / reps
    return res


# ------------------------------------------------------------------ CPU leg
class CpuLayerSample:
    """The CPU restatement of the layer (oracle/: the C selection side and numpy
    float32 block-gather attention), timed on the host cores on the GPU arm's own
    inputs: the same seeded tensors (generated on the device by torch's generator,
    copied to the host once) and the same selection rule, so its shape ids and
    head-0 selection are the GPU arm's (checked when the GPU bitmap is given).

    One sample = audio token norms + zone statistics over all heads + shape choice
    + permutation + the selection of head 0 (full, measured) + forward and backward
    of as many of head 0's query tiles as fit the time budget (measured).  value =
    FLOPs of the sampled tiles / their attention time; the layer time is
    extrapolated separately (statistics once, selection and attention per head)."""

    def __init__(self, inp, S, head0_bits=None):
        import numpy as np
        import torch
        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        from oracle import oracle as O  # CPU checker / baseline only
        self.O, self.np = O, np
        T, H, W = CONFIG["grid"]
        h, D = CONFIG["heads"], CONFIG["head_dim"]
        self.gp = padded_grid()
        Tp, Hp, Wp = self.gp
        to_bits = lambda t: t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
        x = {n: to_bits(inp[n][0]) for n in ("q", "k", "v", "do", "a2v")}  # [S, h*D] / [S, hidden]
        self.a2v = x["a2v"]

        def pad(a):  # [S, c] THW order -> [Sp, c] on the padded grid
            out = np.zeros((Tp, Hp, Wp, a.shape[-1]), np.uint16)
            out[:T, :H, :W] = a.reshape(T, H, W, -1)
            return out.reshape(Tp * Hp * Wp, -1)

        self.v_all = np.ascontiguousarray(pad(x["v"]).reshape(-1, h, D).transpose(1, 0, 2))
        self.q0 = pad(x["q"][:, :D])[None]
        self.k0 = pad(x["k"][:, :D])[None]
        self.v0 = pad(x["v"][:, :D])
        self.do0 = pad(x["do"][:, :D])
        valid = np.zeros((Tp, Hp, Wp), np.uint8)
        valid[:T, :H, :W] = 1
        self.valid = valid.reshape(-1)
        self.head0_bits = head0_bits
        self.pad = pad
        self.S = S

    def run(self, seconds):
        np, O = self.np, self.O
        D = CONFIG["head_dim"]
        uniform = CONFIG.get("path") == "uniform"
        t0 = time.perf_counter()
        if uniform:
            # the uniform path: 3D-chunk order, no zone statistics or shape choice
            # (unguided chunk selection; --guidance / --correction are not restated here)
            t_stats = 0.0
            t1 = time.perf_counter()
            src, inv = O.uniform_layout(self.gp, CONFIG["chunk"])
            q_re, k_re = self.q0[:, src], self.k0[:, src]
            valid_re = self.valid[src]
            vol = int(np.prod(CONFIG["chunk"]))
            bq, _, _ = O.block_select_uniform(q_re, k_re, src.size, src.size, vol, vol, valid_re,
                                              valid_re, CONFIG["sparsity"], CONFIG["cdf_threshold"])
        else:
            norms = self.pad(O.token_norms(self.a2v)[:, None])[:, 0]
            packed, av, audio = O.zone_stats(self.v_all, self.gp, self.valid, norms)
            ids, _, _ = O.shape_select(packed, av, audio, True, CONFIG["method"])
            t_stats = time.perf_counter() - t0
            t1 = time.perf_counter()
            src, inv, bot, bt, nb = O.layout(ids, self.gp)
            q_re, k_re = self.q0[:, src], self.k0[:, src]
            valid_re = self.valid[src]
            bq, _, _ = O.block_select(q_re, k_re, valid_re, bt, nb, CONFIG["sparsity"],
                                      CONFIG["cdf_threshold"])
        t_sel = time.perf_counter() - t1
        nt = src.size // 64
        dense = O.bits_to_dense(bq, nt)[0]
        same = None if self.head0_bits is None else bool(np.array_equal(bq[0], self.head0_bits))
        f = O.bf16_bits_to_f32
        q, k = f(q_re[0]), f(k_re[0])
        v, do = f(self.v0[src]), f(self.do0[src])
        kvalid = valid_re.astype(bool)
        sc = 1.0 / math.sqrt(D)
        rng = np.random.default_rng(0)
        flops, n_done, pairs = 0.0, 0, 0
        t2 = time.perf_counter()
        for qt in rng.permutation(nt):
            cols = np.nonzero(dense[qt])[0]
            keys = (cols[:, None] * 64 + np.arange(64)).reshape(-1)
            kv = kvalid[keys]
            rows = slice(qt * 64, qt * 64 + 64)
            Q, K, V, dO = q[rows], k[keys], v[keys], do[rows]
            s_ = Q @ K.T * sc
            s_[:, ~kv] = -np.inf
            mx = s_.max(1, keepdims=True)
            mx[~np.isfinite(mx)] = 0.0
            p = np.exp(s_ - mx)
            p /= np.maximum(p.sum(1, keepdims=True), 1e-30)
            o = p @ V
            dv_ = p.T @ dO
            dp = dO @ V.T
            ds = p * (dp - (o * dO).sum(1, keepdims=True))
            dq_ = ds @ K * sc
            dk_ = ds.T @ Q * sc
            flops += FWD_BWD_FACTOR * 4 * D * 64 * 64 * cols.size
            pairs += cols.size
            n_done += 1
            if time.perf_counter() - t2 > seconds:
                break
        t_attn = time.perf_counter() - t2
        wall = time.perf_counter() - t0
        heads = CONFIG["heads"]
        layer_ms = (t_stats + heads * (t_sel + t_attn / max(n_done, 1) * nt)) * 1e3
        return {"value": flops / t_attn / 1e12, "unit": "TFLOPS", "cores": os.cpu_count() or 1,
                "kind": "port", "wall_ms": wall * 1e3,
                "sample": ("the GPU arm's inputs: uniform 3D-chunk order, " if uniform else
                           f"the GPU arm's inputs: audio norms + zone statistics over {heads} heads + "
                           f"shape choice ({t_stats:.1f} s, C oracle), ")
                          + f"head 0's full selection "
                          f"({t_sel:.1f} s, C oracle, {int(dense.sum())} tile pairs, density "
                          f"{dense.sum() / nt / nt:.3f}"
                          + ("" if same is None else f", identical to the GPU arm's: {same}")
                          + f"), then {n_done} of head 0's {nt} q tiles fwd+bwd in numpy float32 "
                          f"block-gather form ({t_attn:.1f} s)",
                "same_selection_as_gpu": same, "sample_pair_density": float(dense.sum() / nt / nt),
                "stats_ms": t_stats * 1e3, "selection_ms_per_head": t_sel * 1e3,
                "ms_per_layer_extrapolated": layer_ms}


# ------------------------------------------------------------------ main
def run_producer(args):
    """--path producer: the producer side of the 720p layer (RMSNorm + 3D RoPE of q, k
    and the all-to-all pack of q, k, v, forward + backward) fused
    (prism_b200.producer.norm_rope_pack) against the reference's eager op sequence
    (wan_video_dit.py:699-705: torch.nn.RMSNorm, rope_apply_head_dim in float64 complex,
    the b s (n d) -> b n s d copy that feeds the attention), restated with torch ops."""
    import torch
    import torch.nn.functional as F
    from prism_b200 import _lib
    from prism_b200.producer import norm_rope_pack, rope_table, rope_table_ff
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load(build_if_missing=False)
    grid, H, D = CONFIG["grid"], CONFIG["heads"], CONFIG["head_dim"]
    S, C = grid[0] * grid[1] * grid[2], H * D
    gen = torch.Generator(device=dev).manual_seed(0)
    lin = [torch.randn(S, C, generator=gen, device=dev).to(torch.bfloat16).requires_grad_(True)
           for _ in range(3)]
    gam = [(1 + 0.1 * torch.randn(C, generator=gen, device=dev)).requires_grad_(True) for _ in range(2)]
    grads = [torch.randn(S, H, D, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    cs = rope_table(grid, D, device=dev)
    ff = rope_table_ff(cs)
    freqs = torch.view_as_complex(cs.view(S, 1, D // 2, 2))

    def fused():
        q, k, v = norm_rope_pack(lin[0], lin[1], lin[2], gam[0], gam[1], 1e-6, ff, H)
        torch.autograd.backward([q.view(S, H, D), k.view(S, H, D), v.view(S, H, D)], grads)

    def eager():
        outs = []
        for i in range(3):
            x = lin[i]
            if i < 2:
                x = F.rms_norm(x, (C,), gam[i].to(torch.bfloat16), 1e-6)
                xc = torch.view_as_complex(x.view(S, H, D // 2, 2).to(torch.float64))
                x = torch.view_as_real(xc * freqs).flatten(1).to(torch.bfloat16)
            outs.append(x.view(1, S, H, D).permute(0, 2, 1, 3).contiguous())
        torch.autograd.backward(outs, [g.view(1, S, H, D).permute(0, 2, 1, 3) for g in grads])

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    clk = ClockSampler(0)
    clk.start()
    l0 = _lib.launch_count
    ms_f = timed(fused, args.steps, args.warmup)
    launches = (_lib.launch_count - l0) // (args.steps + args.warmup)
    clocks = clk.stop()
    ms_e = timed(eager, args.steps, args.warmup)
    # algorithmic bytes: forward reads q, k, v rows and writes the packed q, k, v (+ rstd);
    # backward reads the packed gradients and the q, k rows, writes dq, dk, dv
    row = S * C * 2
    fwd_bytes, bwd_bytes = 6 * row + 8 * S, 8 * row + 8 * S
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    achieved = (fwd_bytes + bwd_bytes) / (ms_f * 1e-3) / 1e9
    line = {"metric": "producer_fwd_bwd_ms", "value": ms_f, "unit": "ms", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_f, "higher_is_better": False,
            "scaling": "none", "vs_baseline": None, "dtype": "bf16 (RoPE in f64)", "data": "synthetic",
            "config": {"workload": "720p layer producer side: RMSNorm + 3D RoPE of q, k and the "
                                   "all-to-all pack of q, k, v, forward + backward",
                       "tokens": S, "heads": H, "head_dim": D, "grid": list(grid)},
            "eager_torch_ms": ms_e, "speedup_vs_eager": ms_e / ms_f,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback"},
            "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_gemm(args):
    """--path gemm: the self-attention layer's projection GEMMs on the repository's
    tensor-core GEMM (prism_gemm_bf16) at the 720p shape -- x [75,600, 5,120] times
    W [5,120, 5,120]: forward y = x W^T + b, dgrad dx = dy W, wgrad dW = dy^T x --
    against torch.matmul (cuBLAS) on the same operands; effective TFLOPS =
    2 M N K per GEMM / CUDA-event time, fraction of the measured burst bf16 peak."""
    import torch
    from prism_b200 import _lib, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load(build_if_missing=False)
    grid, H, D = CONFIG["grid"], CONFIG["heads"], CONFIG["head_dim"]
    M, C = grid[0] * grid[1] * grid[2], H * D
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, C, generator=gen, device=dev).to(torch.bfloat16)
    W = (torch.randn(C, C, generator=gen, device=dev) / C ** 0.5).to(torch.bfloat16)
    b = torch.randn(C, generator=gen, device=dev)
    dy = torch.randn(M, C, generator=gen, device=dev).to(torch.bfloat16)
    y, dx, dW = (torch.empty(M, C, dtype=torch.bfloat16, device=dev),
                 torch.empty(M, C, dtype=torch.bfloat16, device=dev),
                 torch.empty(C, C, dtype=torch.bfloat16, device=dev))
    ours = {"forward": lambda: ops.gemm(x, W, bias=b, out=y),
            "dgrad": lambda: ops.gemm(dy, W, b_mn=True, out=dx),
            "wgrad": lambda: ops.gemm(dy, x, a_mn=True, b_mn=True, out=dW)}
    bf = b.to(torch.bfloat16)
    cublas = {"forward": lambda: torch.addmm(bf, x, W.t(), out=y),
              "dgrad": lambda: torch.mm(dy, W, out=dx),
              "wgrad": lambda: torch.mm(dy.t(), x, out=dW)}

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    burst = peaks.get("bf16_tflops") or 1590.0
    flops = 2.0 * M * C * C
    clk = ClockSampler(0)
    clk.start()
    l0 = _lib.launch_count
    res = {n: timed(fn) for n, fn in ours.items()}
    launches = (_lib.launch_count - l0) // (len(ours) * (args.steps + args.warmup))
    clocks = clk.stop()
    ref = {n: timed(fn) for n, fn in cublas.items()}
    ms = sum(res.values())
    tf = {n: flops / (t * 1e-3) / 1e12 for n, t in res.items()}
    line = {"metric": "projection_gemm_tflops", "value": 3 * flops / (ms * 1e-3) / 1e12, "unit": "TFLOPS",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1)",
            "config": {"workload": "720p layer projection GEMMs (x W^T, dy W, dy^T x), one of q/k/v/o",
                       "M": M, "N": C, "K": C},
            "ms": res, "tflops": tf, "frac_of_burst": {n: v / burst for n, v in tf.items()},
            "cublas_ms": ref, "cublas_tflops": {n: flops / (t * 1e-3) / 1e12 for n, t in ref.items()},
            "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel", "achieved": max(tf.values()),
                         "peak": burst, "unit": "TFLOP/s", "frac": max(tf.values()) / burst, "traffic": None,
                         "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst)" if peaks else "fallback"},
            "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_cross(args):
    """--path cross: the v2a / a2v bridge's cross-modal BSA at 720p (flash_attn_bsa_cross,
    bsa_interface.py:1276-1392): audio queries (1D, the config's audio tokens) over the
    video keys (3D grid, 4x4x4 chunks) and video queries over the audio keys, forward +
    backward, 40 heads x 128; sparsity 0.75 over the video chunks, 0.5 over the two audio
    chunks (int((1 - 0.75) * 2) = 0 would keep none)."""
    import torch
    from prism_b200 import _lib, flash_attn_bsa_cross
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load(build_if_missing=False)
    grid, H, D, A = CONFIG["grid"], CONFIG["heads"], CONFIG["head_dim"], CONFIG["audio_tokens"]
    Sv = grid[0] * grid[1] * grid[2]
    gen = torch.Generator(device=dev).manual_seed(0)
    mk = lambda S: torch.randn(1, H, S, D, generator=gen, device=dev).to(torch.bfloat16)
    lines = {}
    for name, (qs, ks, Sq, Sk, sp) in {"a2v": ("1d", "3d", A, Sv, 0.75),
                                        "v2a": ("3d", "1d", Sv, A, 0.5)}.items():
        q, k, v, do = mk(Sq).requires_grad_(True), mk(Sk).requires_grad_(True), mk(Sk).requires_grad_(True), mk(Sq)
        kw = dict(q_grid_size=grid if qs == "3d" else None, k_grid_size=grid if ks == "3d" else None,
                  sparsity=sp, cdf_threshold=None, chunk_3d_shape_q=(4, 4, 4), chunk_3d_shape_k=(4, 4, 4))

        def step():
            q.grad = k.grad = v.grad = None
            out = flash_attn_bsa_cross(q, k, v, qs, ks, **kw)
            out.backward(do)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        lines[name] = {"ms_per_step": e0.elapsed_time(e1) / args.steps, "queries": Sq, "keys": Sk,
                       "sparsity": sp}
    line = {"metric": "cross_bsa_fwd_bwd_ms", "value": lines["v2a"]["ms_per_step"], "unit": "ms",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "none", "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1)",
            "config": {"workload": "720p MOVA bridge cross-modal BSA (flash_attn_bsa_cross), fwd+bwd",
                       "heads": H, "head_dim": D, "grid": list(grid), "audio_tokens": A},
            "directions": lines}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="prism", choices=["prism", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--config", default="720p", choices=sorted(CONFIGS),
                    help="benchmark config: 720p (config 1, default), 1080p (config 2), 2k (config 3)")
    ap.add_argument("--path", default="dynamic", choices=["dynamic", "uniform", "producer", "cross", "gemm"],
                    help="dynamic block shapes (flash_attn_bsa_3d_dynamic, the metric's path) or "
                         "the uniform fixed-shape path (flash_attn_bsa_3d, 4x4x4 chunks, "
                         "sparsity 0.75, cdf 0.2)")
    ap.add_argument("--guidance", default="none",
                    choices=["none", "variance", "audio", "audio_variance"],
                    help="--path uniform: guided selection (variance density gain 1; audio "
                         "saliency gain 1 with Path B pooling weight 1)")
    ap.add_argument("--correction", default="none", choices=["none", "rectified", "taylor"],
                    help="--path uniform: bias-rectified forward (inference: the step is the "
                         "forward alone, the metric its effective TFLOPS)")
    ap.add_argument("--heads", type=int, default=CONFIG["heads"],
                    help="attention heads of the layer (40 in every benchmark config; smaller only "
                         "for profiler captures)")
    args = ap.parse_args()
    CONFIG.update(CONFIGS[args.config])
    if args.path in ("producer", "cross", "gemm"):
        CONFIG["heads"] = args.heads
        {"producer": run_producer, "cross": run_cross, "gemm": run_gemm}[args.path](args)
        return
    CONFIG["heads"] = args.heads
    CONFIG["path"] = args.path
    if args.path == "uniform":
        CONFIG.update(UNIFORM, method=None, guidance=args.guidance, correction=args.correction)
        CONFIG["workload"] = CONFIG["workload"].replace(
            "dynamic BSA", "uniform BSA (4x4x4 chunks, sparsity 0.75, cdf 0.2)")
        if args.guidance != "none":
            CONFIG["workload"] += f", {args.guidance}-guided selection"
        if args.correction != "none":
            CONFIG["workload"] = CONFIG["workload"].replace(
                "fwd+bwd", f"forward with {args.correction} bias rectification (inference)")
    elif args.guidance != "none" or args.correction != "none":
        ap.error("--guidance / --correction need --path uniform")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        import torch
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        # the GPU arm's inputs (torch's seeded generator on the device; data generation
        # only, nothing of prism_b200 runs in this arm), copied to the host once
        inp, S = make_layer_inputs(dev)
        sample = CpuLayerSample(inp, S)
        del inp
        steps = []
        for i in range(args.warmup + args.steps):
            r = sample.run(seconds=6.0)
            if i >= args.warmup:
                steps.append(r)
        val = statistics.mean(x["value"] for x in steps)
        last = steps[-1]
        line = {"impl": "reference", "metric": "bsa_fwd_bwd_effective_tflops", "value": val,
                "unit": "TFLOPS", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": statistics.mean(x["wall_ms"] for x in steps),
                "step": "one bounded CPU sample of the layer (see cpu_baseline.sample); "
                        "ms_per_step is its measured wall time",
                "ms_per_layer_extrapolated": statistics.mean(x["ms_per_layer_extrapolated"] for x in steps),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (the GPU arm's seeded inputs"
                + ("" if dev.type == "cuda" else "; generated on the CPU here, other values") + ")",
                "config": dict(CONFIG, grid=list(CONFIG["grid"])),
                "cpu_baseline": {k: last[k] for k in ("kind", "cores", "sample")} | {"value": val, "unit": "TFLOPS"},
                "e2e": {"value": val, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    from prism_b200 import _lib
    from prism_b200.parallel_states import initialize_sequence_parallel
    _lib.load(build_if_missing=False)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        initialize_sequence_parallel()

    inp, S = make_layer_inputs(dev, rank, world)
    q = inp["q"].requires_grad_(True)
    k = inp["k"].requires_grad_(True)
    v = inp["v"].requires_grad_(True)
    do, a2v = inp["do"], inp["a2v"]
    step = make_step(inp, S, world)

    infer = inference_only()

    def run_step():
        q.grad = k.grad = v.grad = None
        step(q, k, v, do, a2v)

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    from prism_b200 import ops as _ops
    clk = ClockSampler(local_rank)
    clk.start()
    l0 = _lib.launch_count
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    timer = _ops.KernelTimer() if args.path == "dynamic" else None
    _ops.set_kernel_timer(timer)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(args.steps):
        run_step()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    _ops.set_kernel_timer(None)
    clocks = clk.stop()
    launches = (_lib.launch_count - l0) // args.steps
    ms_local = e0.elapsed_time(e1) / args.steps
    kt_step = timer.totals_ms() if timer is not None else None
    t = torch.tensor([ms_local], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # FLOPs actually computed (selected tile pairs, all ranks)
    pairs, plan, (q4, k4, v4, norms), executed = selected_pairs(q.detach(), k.detach(), v.detach(),
                                                                a2v, S, world)
    # per-rank exchange time inside the timed steps (NCCL all-to-alls and the layout
    # copies around them, CUDA events on the step's stream)
    a2a_ms = (kt_step or {}).get("sp_all_to_all", 0.0) / args.steps
    copy_ms = (kt_step or {}).get("sp_layout_copy", 0.0) / args.steps
    mine = torch.tensor([pairs, executed, ms_local, a2a_ms, copy_ms], device=dev, dtype=torch.float64)
    every = torch.empty(world, 5, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_gather_into_tensor(every, mine)
    else:
        every.copy_(mine[None])
    per_rank = {"selected_tile_pairs": [int(x) for x in every[:, 0].tolist()],
                "ms_per_step": [round(float(x), 3) for x in every[:, 2].tolist()]}
    if world > 1:
        per_rank["all_to_all_ms_per_step"] = [round(float(x), 3) for x in every[:, 3].tolist()]
        per_rank["layout_copy_ms_per_step"] = [round(float(x), 3) for x in every[:, 4].tolist()]
    total_pairs = float(every[:, 0].sum().item())
    total_executed = float(every[:, 1].sum().item())
    D = CONFIG["head_dim"]
    flops = (1.0 if infer else FWD_BWD_FACTOR) * 4 * D * 64 * 64 * total_pairs
    tflops = flops / (ms * 1e-3) / 1e12
    Tp, Hp, Wp = padded_grid()
    n_tiles = Tp * Hp * Wp // 64
    density = total_pairs / (CONFIG["heads"] * n_tiles * n_tiles)

    # per-kernel times of this rank's launches: inside the timed steps (CUDA events
    # around each attention kernel, ops.KernelTimer) and each kernel timed alone
    kt_iso = kernel_times(plan, q4, k4, v4)
    kt = {n: kt_step[n] / args.steps for n in kt_step} if kt_step else kt_iso
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    burst = peaks.get("bf16_tflops") or 1590.0
    sustained = peaks.get("bf16_tflops_sustained") or 1400.0
    local_pairs = pairs
    # per (q tile, k tile) pair one 64x64xD product is 2*64*64*D FLOPs; the forward
    # computes 2 of them (QK^T, PV), dK/dV 4 (S^T, dP^T, dV, dK), dQ 3 (S, dP, dQ)
    mm = 2 * 64 * 64 * D * local_pairs
    algo = {"bsa_fwd": 2 * mm, "bsa_bwd_dkdv": 4 * mm, "bsa_bwd_dq": 3 * mm}
    dom = "bsa_fwd" if infer else max(("bsa_fwd", "bsa_bwd_dkdv", "bsa_bwd_dq"), key=lambda n: kt[n])
    achieved = algo[dom] / (kt[dom] * 1e-3) / 1e12
    traffic = None
    if args.config == "720p" and D == 128 and args.path == "dynamic":
        traffic = TRAFFIC_PER_HEAD_720P[dom] * (CONFIG["heads"] // world)
    roofline = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": burst,
                "unit": "TFLOP/s", "frac": achieved / burst, "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 720p layer "
                                  "at 4 heads, scaled by heads per launch" if traffic else None,
                "peak_source": ("MEASURED_PEAKS.json bf16_tflops (burst)" if peaks else "fallback"),
                "frac_of_sustained": achieved / sustained,
                "timing": "CUDA events around the kernel inside the timed steps" if kt_step
                          else "the kernel timed alone",
                "kernel_ms": kt, "kernel_ms_isolated": kt_iso,
                "kernel_frac_of_burst": {n: algo[n] / (kt[n] * 1e-3) / 1e12 / burst for n in algo}}

    # end-to-end through host buffers (pinned), H2D inputs + D2H output and grads
    e2e = None
    if not args.no_e2e:
        # End to end through pinned host buffers: every step uploads its inputs and
        # downloads its result (output and, for training, the three gradients).  The
        # transfers are pipelined as a serving / training loop runs them: step i+1's
        # inputs upload on a copy-in stream into the second of two device buffer sets
        # while step i computes, and step i's results download on a copy-out stream
        # while step i+1 computes.  The timed region runs from before the first upload
        # to the end of the last download.
        names_in = ("q", "k", "v", "a2v") if infer else ("q", "k", "v", "do", "a2v")
        out_names = ("o",) if infer else ("o", "dq", "dk", "dv")
        host = {n: inp[n].detach().cpu().pin_memory() for n in names_in}
        outs = [{n: torch.empty(inp["q"].shape, dtype=torch.bfloat16).pin_memory() for n in out_names}
                for _ in range(2)]
        h2d = sum(x.numel() * x.element_size() for x in host.values())
        d2h = sum(x.numel() * x.element_size() for x in outs[0].values())
        dbuf = [{n: torch.empty_like(inp[n].detach()) for n in names_in} for _ in range(2)]
        comp = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        buf_free = [torch.cuda.Event() for _ in range(2)]

        def upload(i):
            b = i % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(buf_free[b])  # step i - 2 no longer reads this set
                for n in names_in:
                    dbuf[b][n].copy_(host[n], non_blocking=True)
                in_ready[b].record(s_in)

        def run(n_steps):
            s_in.wait_stream(comp)
            upload(0)
            for i in range(n_steps):
                b = i % 2
                comp.wait_event(in_ready[b])
                if i + 1 < n_steps:
                    upload(i + 1)
                d = dbuf[b]
                if infer:
                    with torch.no_grad():
                        res = {"o": attend(d["q"], d["k"], d["v"], d["a2v"], S)}
                else:
                    qq, kk, vv = (d[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
                    x = attend(qq, kk, vv, d["a2v"], S)
                    x.backward(d["do"])
                    res = {"o": x.detach(), "dq": qq.grad, "dk": kk.grad, "dv": vv.grad}
                buf_free[b].record(comp)
                s_out.wait_stream(comp)
                with torch.cuda.stream(s_out):
                    for n, t in res.items():
                        outs[b][n].copy_(t, non_blocking=True)
                        t.record_stream(s_out)
            comp.wait_stream(s_out)

        run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record(comp)
        run(args.steps)
        f1.record(comp)
        torch.cuda.synchronize()
        ms_e = f0.elapsed_time(f1) / args.steps
        te = torch.tensor([ms_e], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        ms_e = float(te.item())
        e2e = {"value": flops / (ms_e * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": ms_e,
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "transfers": "pinned host buffers; uploads and downloads overlap the neighbouring "
                            "steps' compute (two device buffer sets, copy-in / copy-out streams)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        head0 = plan.bits_q[0].cpu().numpy().view("uint32")
        cpu = CpuLayerSample(inp, S, head0_bits=head0).run(seconds=12.0)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "same_selection_as_gpu",
                                   "sample_pair_density", "ms_per_layer_extrapolated")}

    if rank == 0:
        line = {"metric": "bsa_fwd_effective_tflops" if infer else "bsa_fwd_bwd_effective_tflops",
                "value": tflops, "unit": "TFLOPS",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded zone-structured q/k/v, N(0,1) a2v residual)",
                "config": dict(CONFIG, grid=list(CONFIG["grid"]), parallelism=f"ulysses_sp{world}",
                               global_batch=1, seq_len=S, selected_tile_pairs=int(total_pairs),
                               executed_tile_pairs_dq=int(total_executed), pair_density=density,
                               l2="inputs larger than L2 (q/k/v >= 774 MB each)"),
                "per_rank": per_rank,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
