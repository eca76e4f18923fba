"""Benchmark of the GDN prefill hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5|cfg3] [--tokens T]

Default workload (cfg5): one 65536-token sequence through causal_conv1d
(8192 channels, width 4, SiLU) -> chunked gated delta rule (Hk 16 -> Hv 32,
dk = dv = 128; the q/k L2 norm fused into the conv kernel) -> gated RMSNorm (group 128,
SiLU(z) gate; fused into the chunked rule's chain kernel, which writes the
normalised output instead of o).  The 32 value heads, their key heads and conv channels are
split over the N ranks (one process per GPU, no collective on the data path);
the sequence is the unit of work, so `value` = 65536 tokens / max-over-ranks
step time ("scaling": "strong").  cfg3 is the varlen 8-sequence 16384-token
GDN prefill alone.

Inputs are seeded synthetic tensors (torch_npu_ops_b200.workloads), resident
in HBM for `value`; each step touches > 1 GB, far above the 126 MB L2, so no
flush is needed between steps.  `e2e` repeats the step through the public
API with the step's inputs copied from pinned host memory and the output
copied back inside the timed region.  `--impl reference` times the
reference algorithm (the CPU oracle restating the reference's torch
implementation) on the host cores instead.
"""

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GDN prefill tokens/s/GPU; norm/RoPE/conv1d HBM GB/s vs B200 peak"
# 1,444.3 MB of DRAM traffic for 16,384 tokens x 32 value heads (prep, both
# chain phases with the fused output norm, combine), measured by ncu
# (dram__bytes_read.sum + write.sum)
GDN_DRAM_BYTES_PER_TOKEN_HEAD = 1.4443e9 / (16384 * 32)


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------- workloads --
def build_cfg5(rank, world, T, dev):
    from torch_npu_ops_b200 import workloads
    w = workloads.long_config5_shard(rank, world, T=T)
    (v0, v1), (k0, k1) = w["heads"], w["k_heads"]
    hv, hk = v1 - v0, k1 - k0
    host = {"x": w["x"], "g": w["g"], "beta": w["beta"], "initial_state": w["initial_state"],
            "z": w["z"]}
    dev_t = {n: t.to(dev) for n, t in host.items()}
    consts = {"weight": w["weight"].to(dev), "bias": w["bias"].to(dev),
              "norm_w": w["norm_w"].to(dev)}
    C = w["x"].shape[1]
    return {"T": T, "hv": hv, "hk": hk, "C": C, "host": host, "dev": dev_t, "consts": consts,
            "lengths": [T]}


def build_cfg3(dev):
    from torch_npu_ops_b200 import workloads
    w = workloads.chunk_config3()
    host = {n: w[n] for n in ("q", "k", "v", "g", "beta", "initial_state")}
    return {"T": int(w["cu_seqlens"][-1]), "hv": 32, "hk": 16, "host": host,
            "dev": {n: t.to(dev) for n, t in host.items()},
            "consts": {"cu": w["cu_seqlens"].to(dev)}, "lengths": w["lengths"]}


def make_step(cfg, kind, dev):
    """Returns step(inputs) -> tuple of output tensors, plus the stage names
    its optional event list brackets."""
    import torch_npu_ops_b200 as ops
    c = cfg["consts"]
    if kind == "cfg3":
        def step(inp, ev=None):
            if ev: ev[0].record()
            o, ht = ops.npu_chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"],
                                                   inp["beta"], None, inp["initial_state"], True,
                                                   c["cu"])
            if ev: ev[1].record()
            return o, ht
        return step, ["gdn"]
    from torch_npu_ops_b200.pipeline import gdn_prefill
    T, hv, hk = cfg["T"], cfg["hv"], cfg["hk"]
    state = torch.zeros(1, cfg["C"], 3, dtype=torch.bfloat16, device=dev)
    qsl = torch.tensor([0, T], dtype=torch.int32, device=dev)

    def step(inp, ev=None):
        state.zero_()  # fresh prefill: zero conv history
        _, _, ht, out = gdn_prefill(inp["x"], state, c["weight"], c["bias"], inp["g"], inp["beta"],
                                    inp["initial_state"], inp["z"], c["norm_w"], hk, hv,
                                    query_start_loc=qsl, events=ev)
        return out, ht
    # the gated RMSNorm runs inside the chunked rule's chain kernel: the
    # "gdn" stage is the rule and the norm together
    return step, ["conv", "gdn"]


def rule_only_ms(cfg, dev, reps=5):
    """cfg5: the chunked rule alone (npu_chunk_gated_delta_rule, the same
    preparation / chain / combine kernels without the fused norm) on the
    step's own conv output, median of `reps` CUDA-event timings; run after
    the timed steps, outside them."""
    import torch_npu_ops_b200 as ops
    c, inp = cfg["consts"], cfg["dev"]
    T, hv, hk, d = cfg["T"], cfg["hv"], cfg["hk"], 128
    state = torch.zeros(1, cfg["C"], 3, dtype=torch.bfloat16, device=dev)
    qsl = torch.tensor([0, T], dtype=torch.int32, device=dev)
    y = ops.causal_conv1d_varlen_qk_l2norm(inp["x"], state, c["weight"], c["bias"], qsl,
                                           2 * hk * d)
    q = y[:, : hk * d].view(1, T, hk, d)
    k = y[:, hk * d: 2 * hk * d].view(1, T, hk, d)
    v = y[:, 2 * hk * d:].view(1, T, hv, d)

    def rule():
        return ops.npu_chunk_gated_delta_rule(q, k, v, inp["g"], inp["beta"], None,
                                              inp["initial_state"], True, None, False, False)
    for _ in range(2):
        rule()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rule()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def stage_bytes(cfg, kind):
    """Algorithmic HBM bytes per launch of the bandwidth-bound stages."""
    if kind == "cfg3":
        return {}
    T, C = cfg["T"], cfg["C"]
    return {"conv": 2 * 2 * T * C + 2 * C * 5}


# ------------------------------------------------------------- reference ----
def cpu_reference(kind, T_sample, reps=3, warmup=1):
    """Times the CPU oracle (the reference's torch algorithm) on a bounded
    sample of the workload with every host thread; returns tokens/s info."""
    import oracle
    from torch_npu_ops_b200 import workloads
    torch.set_num_threads(os.cpu_count() or 1)
    if kind == "cfg3":
        w = workloads.chunk_config3(lengths=[T_sample // 2, T_sample - T_sample // 2])
        fn = lambda: oracle.chunk_gated_delta_rule(w["q"], w["k"], w["v"], w["g"], w["beta"], None,
                                                   w["initial_state"], True, w["cu_seqlens"])
        sample = f"chunked GDN oracle, {T_sample} tokens (2 seqs), Hv 32"
    else:
        w = workloads.long_config5_shard(0, 1, T=T_sample)
        d, hk, hv = 128, 16, 32
        st = torch.zeros(1, w["x"].shape[1], 3, dtype=torch.bfloat16)
        qsl = torch.tensor([0, T_sample], dtype=torch.int32)

        def fn():
            y = oracle.causal_conv1d_varlen(w["x"], st.clone(), w["weight"], w["bias"], True, qsl)
            q = y[:, : hk * d].reshape(1, T_sample, hk, d)
            k = y[:, hk * d: 2 * hk * d].reshape(1, T_sample, hk, d)
            v = y[:, 2 * hk * d:].reshape(1, T_sample, hv, d)
            o, _ = oracle.chunk_gated_delta_rule(q, k, v, w["g"], w["beta"], None,
                                                 w["initial_state"], True, None, True)
            return oracle.layer_norm_fwd(o.reshape(-1, d), w["norm_w"], None, 1e-6,
                                         w["z"].reshape(-1, d), d, True, True)[0]
        sample = (f"conv->chunk GDN->gated RMSNorm oracle on the first {T_sample} tokens of the "
                  "65536-token sequence, all 32 heads")
    for _ in range(max(1, warmup)):
        fn()
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t)
    med = statistics.median(ts)
    return {"value": T_sample / med, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": sample, "seconds_per_sample": med,
            "extrapolated": True,
            "extrapolation": f"tokens/s = {T_sample} sample tokens / sample seconds; the oracle's "
                             "cost is linear in tokens (chunk-serial over the sequence)"}


# ------------------------------------------------------------------ main ----
def kernel_sweep(dev, peaks, profile=False):
    """Achieved HBM bandwidth of every bandwidth-bound operator at its
    configuration size and at a size well above L2.  Each operator call is
    captured once in a CUDA graph; every timed replay follows a 1 GB buffer
    write (which flushes L2 and keeps the GPU busy while the host enqueues
    the events and the replay, so the events see device time only, not the
    host's launch path).  Median of 10.  Bytes are the algorithmic bytes
    (every input read once, every output written once)."""
    import statistics
    import torch_npu_ops_b200 as ops
    from torch_npu_ops_b200 import workloads
    flush = torch.empty(1 << 30, dtype=torch.uint8, device=dev)

    def timed(fn, reps=10):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            graph.replay()
            e.record()
            e.synchronize()
            ts.append(s.elapsed_time(e))
        # steady state: 20 replays between one pair of events, no flush (a
        # working set under 126 MB then stays in L2, as in a decode loop)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(20):
            graph.replay()
        e.record()
        e.synchronize()
        del graph
        return statistics.median(ts), s.elapsed_time(e) / 20

    out = {}

    def add(name, fn, nbytes):
        if profile:
            # for profiler runs: the large shape of each operator, launched
            # twice (a warm-up and the one to capture), nothing timed
            fn()
            fn()
            torch.cuda.synchronize()
            out[name] = {"bytes": int(nbytes)}
            return
        ms, ms_b2b = timed(fn)
        gbs = nbytes / (ms / 1000.0) / 1e9
        out[name] = {"bytes": int(nbytes), "ms": ms, "GB/s": gbs, "frac_hbm": gbs / peaks["hbm_gbs"],
                     "ms_back_to_back": ms_b2b}

    for T in ((16384,) if profile else (128, 16384)):  # a1: cfg1 shape, and a token sweep point
        r = workloads.rope_config1(T=T)
        t = [x.to(dev) for x in r["tensors"]]
        add(f"split_rmsnorm_rope fp32 T={T}", lambda: ops.npu_split_rmsnorm_rope(*t, **r["kwargs"]),
            4 * T * (5120 + 5120) + 2 * 4 * T * 64 + 2 * 4 * 256)
    for Bd in ((4096,) if profile else (256, 4096)):  # a3: cfg2 decode, and a larger batch
        d = workloads.conv_decode_config2(batch=Bd)
        cx, cs, cw, cb = (d[k].to(dev) for k in ("x", "conv_state", "weight", "bias"))
        add(f"causal_conv1d_update B={Bd}",
            lambda: ops.npu_causal_conv1d_update(cx, cs, cw, True, cb),
            2 * 2 * Bd * 8192 + 2 * 2 * Bd * 8192 * 3 + 2 * 8192 * 5)
    dec = workloads.decode_config4()
    a = {n: (t.to(dev) if torch.is_tensor(t) else t) for n, t in dec.items()}
    st = a["state"].clone()
    add("fused_recurrent_gated_delta_rule cfg4 B=256",  # a10
        lambda: ops.npu_fused_recurrent_gated_delta_rule(
            a["q"], a["k"], a["v"], a["g"], a["beta"], None, st, True, a["cu_seqlens"],
            a["ssm_state_indices"], None, True),
        2 * st.numel() * 4 + 2 * a["q"].numel() * 2 + 2 * a["v"].numel() * 2 + 2 * a["g"].numel() * 4)
    for M in ((2097152,) if profile else (8192, 2097152)):  # a11: cfg4 (256 x 32 heads) and the cfg5 size
        x = torch.randn(M, 128, device=dev).to(torch.bfloat16)
        z = torch.randn(M, 128, device=dev).to(torch.bfloat16)
        w = torch.ones(128, device=dev, dtype=torch.bfloat16)
        add(f"gated RMSNorm g128 rows={M}",
            lambda: ops.layer_norm_fwd(x, w, None, 1e-6, z, 128, True, True), 3 * 2 * M * 128 + 4 * M)
    for M in ((65536,) if profile else (256, 65536)):  # a12 / a13: cfg4 hidden [256, 2048], and a large batch
        x = torch.randn(M, 2048, device=dev).to(torch.bfloat16)
        w = torch.ones(2048, device=dev, dtype=torch.bfloat16)
        b = torch.zeros(2048, device=dev, dtype=torch.bfloat16)
        add(f"layer_norm_fwd [{M},2048]",
            lambda: ops.layer_norm_fwd(x, w, b, 1e-6, None, 2048, True, False),
            2 * 2 * M * 2048 + 8 * M + 4 * 2048)
        add(f"gemma_rms_norm [{M},2048]", lambda: ops.npu_gemma_rms_norm(x, w, 1e-6),
            2 * 2 * M * 2048 + 4 * M + 2 * 2048)
    x = torch.randn(65536 * 16, 128, device=dev).to(torch.bfloat16)  # a14: q/k heads of cfg5
    add("l2norm_last_dim [1048576,128]", lambda: ops.npu_l2norm_last_dim(x, 1e-6), 2 * 2 * x.numel())
    # next rows: the gate projections of a decode batch and of the cfg5 prefill
    # (a, b bf16 in; g fp32 and beta bf16 out)
    A_log = torch.rand(32, device=dev) * 2.7
    dtb = torch.rand(32, device=dev)
    for rows in ((65536,) if profile else (256, 65536)):
        ga = torch.randn(rows, 32, device=dev).to(torch.bfloat16)
        gb = torch.randn(rows, 32, device=dev).to(torch.bfloat16)
        add(f"fused_gdn_gating [{rows},32]",
            lambda: ops.npu_fused_gdn_gating(A_log, ga, gb, dtb), (2 + 2 + 4 + 2) * rows * 32)
    # de-interleave of the input projections (16 -> 32 heads of 128): a decode
    # batch and a 16,384-token prefill chunk
    for rows in ((16384,) if profile else (256, 16384)):
        mq = torch.randn(rows, 16 * (256 + 512), device=dev).to(torch.bfloat16)
        mb = torch.randn(rows, 16 * 4, device=dev).to(torch.bfloat16)
        add(f"fused_qkvzba_split_reshape_cat [{rows}, 16->32]",
            lambda: ops.npu_fused_qkvzba_split_reshape_cat(mq, mb, 16, 32, 128, 128),
            2 * (mq.numel() + mb.numel()) * 2)
    # the recurrent step with in-step gates, cfg4 decode shape
    sa = torch.randn(1, 256, 32, device=dev).to(torch.bfloat16)
    sb = torch.randn(1, 256, 32, device=dev).to(torch.bfloat16)
    sidx = torch.arange(256, dtype=torch.int32, device=dev)
    scu = torch.arange(257, dtype=torch.int32, device=dev)
    st2 = a["state"].clone()
    add("fused_sigmoid_gating_delta_rule_update cfg4 B=256",
        lambda: ops.npu_fused_sigmoid_gating_delta_rule_update(
            A_log, sa, dtb, a["q"], a["k"], a["v"], sb, st2, sidx, scu, None, True),
        2 * st2.numel() * 4 + 2 * a["q"].numel() * 2 + 2 * a["v"].numel() * 2 + 2 * sa.numel() * 2)
    return out


def layer_compare(dev, T, steps, warmup):
    """cfg5-shaped GDN layer prefill (Hk 16 -> Hv 32) from the projection
    outputs mixed_qkvz / mixed_ba: the fused path (no split, gates and z read
    in place) against the reference's sequence of five operators on the same
    kernels.  Times are CUDA events around each step, median of `steps`."""
    import torch_npu_ops_b200 as ops
    from torch_npu_ops_b200.pipeline import gdn_layer_prefill, gdn_prefill
    hk, hv, d = 16, 32, 128
    r = hv // hk
    C = (2 * hk + hv) * d
    g = torch.Generator(device=dev).manual_seed(6)
    mixed_qkvz = torch.randn(T, hk * (2 + 2 * r) * d, generator=g, device=dev).to(torch.bfloat16)
    mixed_ba = torch.randn(T, hk * 2 * r, generator=g, device=dev).to(torch.bfloat16)
    w = (0.5 * torch.randn(C, 4, generator=g, device=dev)).to(torch.bfloat16)
    cb = (0.5 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    A_log = torch.rand(hv, generator=g, device=dev) * 2.7
    dt_bias = torch.rand(hv, generator=g, device=dev)
    nw = (1 + 0.1 * torch.randn(d, generator=g, device=dev)).to(torch.bfloat16)
    h0 = 0.02 * torch.randn(1, hv, d, d, generator=g, device=dev)
    qsl = torch.tensor([0, T], dtype=torch.int32, device=dev)
    st = torch.zeros(1, C, 3, dtype=torch.bfloat16, device=dev)

    def fused():
        st.zero_()
        return gdn_layer_prefill(mixed_qkvz, mixed_ba, st, w, cb, A_log, dt_bias, h0, nw, hk, hv,
                                 query_start_loc=qsl)

    def unfused():
        st.zero_()
        mixed_qkv, z, b, a = ops.npu_fused_qkvzba_split_reshape_cat(mixed_qkvz, mixed_ba, hk, hv,
                                                                    d, d)
        gt, beta = ops.npu_fused_gdn_gating(A_log, a, b, dt_bias)
        return gdn_prefill(mixed_qkv, st, w, cb, gt, beta.float(), h0, z, nw, hk, hv,
                           query_start_loc=qsl, fuse_norm=False)

    res = {}
    for name, fn in (("fused", fused), ("five_operators", unfused)):
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = sorted(ts)[len(ts) // 2]
        res[name] = {"ms_per_step": ms, "tokens_per_s": T / (ms / 1000.0)}
    res["speedup"] = res["five_operators"]["ms_per_step"] / res["fused"]["ms_per_step"]
    return {"metric": "GDN layer prefill from the input projections, tokens/s", "workload": "layer",
            "config": {"tokens": T, "k_heads": hk, "v_heads": hv, "head_dim": d,
                       "inputs": "mixed_qkvz [T, 12288], mixed_ba [T, 64] bf16 ~N(0,1), resident",
                       "l2_flush": "inputs > L2 (1.6 GB per step)"}, **res}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg5", choices=["cfg5", "cfg3", "kernels", "layer"],
                    help="kernels: HBM bandwidth of every bandwidth-bound operator; layer: the "
                         "GDN layer prefill from its un-split projections, fused against the "
                         "split -> conv -> gating -> rule -> norm sequence")
    ap.add_argument("--tokens", type=int, default=65536)
    ap.add_argument("--shard", type=int, default=0,
                    help="cfg5 only, for profiling on one GPU: run rank 0's head shard of an "
                         "N-GPU job in this single process (N in 2, 4, 8)")
    ap.add_argument("--cpu-sample", type=int, default=8192)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="for profiler runs: no clock soak, no e2e, no CPU baseline, no "
                         "rule-only timing")
    a = ap.parse_args()
    if a.profile:
        a.no_e2e = a.no_cpu_baseline = True

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    shard_world = world
    if a.shard:
        if world != 1 or a.workload != "cfg5" or a.shard not in (2, 4, 8):
            raise SystemExit("--shard N: one process, cfg5, N in 2, 4, 8")
        shard_world = a.shard
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kind = a.workload
    T = a.tokens if kind == "cfg5" else 16384
    config = ({"workload": "cfg5: 1 x 65536-token prefill, conv1d(8192ch,w4,SiLU; q/k blocks "
                           "L2-normalised in the conv kernel) -> chunked GDN (Hk16->Hv32, "
                           "dk=dv=128, initial state ~N(0,0.02), final state returned) -> gated "
                           "RMSNorm(g128)",
               "tokens": T, "heads_per_gpu": 32 // max(1, world, a.shard),
               "parallelism": f"head-shard x{world}" if not a.shard else
                              f"rank 0 of a head-shard x{a.shard} job, run alone",
               "value_is": "whole-job tokens/s (all ranks; the sequence's 32 heads are split over "
                           "them); value_per_gpu = value / n_gpus",
               "l2_flush": "inputs > L2 (>1 GB per step)"}
              if kind == "cfg5" else
              {"workload": "cfg3: 8 seqs / 16384 tokens varlen chunked GDN (Hk16->Hv32)",
               "tokens": T, "parallelism": "replica", "l2_flush": "inputs > L2 (~0.45 GB per step)"})

    if a.shard:
        config["value_is"] = (f"tokens/s of rank 0's shard run alone on one GPU (profiling mode); "
                              f"the {a.shard}-GPU job runs {a.shard} such shards at once")
    if a.impl == "reference":
        if rank != 0:
            return
        ref = cpu_reference(kind, a.cpu_sample, reps=a.steps, warmup=a.warmup)
        line = {"impl": "reference", "metric": METRIC, "value": ref["value"], "unit": "tokens/s",
                "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": 1000.0 * ref["seconds_per_sample"], "higher_is_better": True,
                "scaling": "strong" if kind == "cfg5" else "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": config,
                "cpu_baseline": ref,
                "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    from torch_npu_ops_b200 import _lib, workloads
    _lib.load()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if kind == "kernels":
        if rank == 0:
            peaks = _peaks()
            print(json.dumps({"metric": "HBM GB/s of the bandwidth-bound operators",
                              "workload": "kernels", "l2_flush": "1 GB written before each graph replay",
                              "back_to_back": "ms_back_to_back: 20 replays between one event pair, no flush",
                              "hbm_peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"],
                              "kernels": kernel_sweep(dev, peaks, a.profile)}))
        return
    if kind == "layer":
        if rank == 0:
            print(json.dumps(layer_compare(dev, a.tokens, a.steps, a.warmup)))
        return
    if world > 1:
        import torch.distributed as dist
        # gloo, not NCCL: nothing on the data path is a collective, and the
        # barrier and the max over ranks of the CUDA-event times are host work
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    cfg = build_cfg5(rank, shard_world, T, dev) if kind == "cfg5" else build_cfg3(dev)
    step, stages = make_step(cfg, kind, dev)
    inp = cfg["dev"]

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(a.warmup):
        step(inp)
    barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)]
           for _ in range(a.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = _lib.launch_count()
    barrier()
    start.record()
    for i in range(a.steps):
        step(inp, evs[i])
    stop.record()
    barrier()
    launches = _lib.launch_count() - l0
    elapsed = start.elapsed_time(stop)
    # short timed regions: keep the same load running ~1 s so the sampler
    # (100 ms period) sees the clocks under this workload
    t_end = time.time() + (0.0 if a.profile else max(0.0, 1.0 - elapsed / 1000.0))
    while time.time() < t_end:
        step(inp)
        torch.cuda.synchronize()
    clk = clocks.stop()
    stage_ms = {s: statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs)
                for j, s in enumerate(stages)}
    t_local = torch.tensor([elapsed])
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
    ms_step = t_local.item() / a.steps
    value = T / (ms_step / 1000.0)

    peaks = _peaks()
    flops = workloads.chunk_flops(cfg["lengths"], cfg["hv"])
    gdn_ms = stage_ms["gdn"]
    achieved = flops / (gdn_ms / 1000.0) / 1e12
    # DRAM bytes (read + write) of the GDN stage's kernels (prep, both chain
    # phases, combine) from one ncu capture of the cfg5 shape at 16,384
    # tokens, per (token, value head), scaled by this run's tokens and heads.
    traffic = GDN_DRAM_BYTES_PER_TOKEN_HEAD * cfg["T"] * cfg["hv"]
    roofline = {"kernel": "chunked GDN stage (prep + chain with the gated RMSNorm fused into "
                          "its output + combine)", "bound": "tensor",
                "achieved": achieved,
                "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops_sustained"],
                "peak_source": f"{peaks['source']} sustained bf16",
                "flops_per_launch": flops, "launch_ms": gdn_ms, "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, cfg5 shape "
                                  "at 16384 tokens, scaled by tokens x heads"}
    if kind == "cfg5" and not a.profile:
        r_ms = rule_only_ms(cfg, dev)
        r_tf = flops / (r_ms / 1000.0) / 1e12
        roofline["rule_only"] = {
            "ms": r_ms, "achieved": r_tf, "frac": r_tf / peaks["bf16_tflops_sustained"],
            "what": "the same rule kernels without the fused norm (npu_chunk_gated_delta_rule), "
                    "timed after the steps"}
    kernels = {}
    for s, byt in stage_bytes(cfg, kind).items():
        gbs = byt / (stage_ms[s] / 1000.0) / 1e9
        kernels[s] = {"ms": stage_ms[s], "bytes": byt, "GB/s": gbs,
                      "frac_hbm": gbs / peaks["hbm_gbs"]}
    kernels["gdn"] = {"ms": gdn_ms, "TFLOP/s": achieved}

    e2e = None
    if not a.no_e2e:
        host = {n: t.pin_memory() for n, t in cfg["host"].items()}
        dbuf = {n: torch.empty_like(t) for n, t in cfg["dev"].items()}
        outs0 = step(inp)
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        d2h = sum(t.numel() * t.element_size() for t in outs0)

        # Every step uploads its own inputs and reads back its own results
        # (the normed output and the final state).  The copies run on their own
        # streams (PCIe is full duplex) into two alternating device buffer
        # sets, so step i+1's upload overlaps step i's compute and readback;
        # compute itself stays on one stream.  The upload is split over two
        # streams by bytes, so two copy engines share it.
        comp = torch.cuda.current_stream(dev)
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        h2d_s2 = torch.cuda.Stream(device=dev)
        order = sorted(host, key=lambda n: -host[n].numel() * host[n].element_size())
        lanes = ([], [])
        loads = [0, 0]
        for n in order:
            j = 0 if loads[0] <= loads[1] else 1
            lanes[j].append(n)
            loads[j] += host[n].numel() * host[n].element_size()
        dbufs = [dbuf, {n: torch.empty_like(t) for n, t in cfg["dev"].items()}]
        houts = [[torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs0]
                 for _ in range(2)]
        in_free = [torch.cuda.Event(), torch.cuda.Event()]

        def e2e_step(i):
            b = i & 1
            for cs, names in zip((h2d_s, h2d_s2), lanes):
                with torch.cuda.stream(cs):
                    cs.wait_event(in_free[b])  # the compute that read this buffer set is done
                    for n in names:
                        dbufs[b][n].copy_(host[n], non_blocking=True)
                    loaded = torch.cuda.Event()
                    loaded.record(cs)
                comp.wait_event(loaded)
            outs = step(dbufs[b])
            in_free[b].record(comp)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(done)
                for h, t in zip(houts[b], outs):
                    h.copy_(t, non_blocking=True)
                    t.record_stream(d2h_s)

        for i in range(2):
            e2e_step(i)
        comp.wait_stream(d2h_s)
        torch.cuda.synchronize(dev)
        barrier()
        s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(comp)
        for i in range(a.steps):
            e2e_step(i)
        comp.wait_stream(h2d_s)
        comp.wait_stream(h2d_s2)
        comp.wait_stream(d2h_s)
        t2.record(comp)
        torch.cuda.synchronize(dev)
        barrier()
        te = torch.tensor([s2.elapsed_time(t2)])
        if world > 1:
            torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        e2e = {"value": T / (te.item() / a.steps / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "torch_npu_ops_b200 public API, pinned host <-> HBM copies inside the "
                       "timed region"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_reference(kind, a.cpu_sample)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "value_per_gpu": value / world,
                "unit": "tokens/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong" if kind == "cfg5" else "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
                "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches, "clocks": clk}
        print(json.dumps(line))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
