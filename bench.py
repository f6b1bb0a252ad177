#!/usr/bin/env python
"""Benchmark of the B200 MHA forward path — metric "MHA prefill tok/s + decode tok/s
at 1/2/4/8 B200; % of roofline".

Default workload (cfg5, the metric's 1/2/4/8-GPU configuration): batch 32 x seq
8192, d_model 4096, 32 heads x 128, causal, RoPE, BF16 activations and weights,
FP32 accumulation. Heads are sharded 32/N per GPU. At N > 1 the device-timed
prefill runs in 4 chunks of 8 sequences and rank r keeps the r-th row slice of each
chunk (--output exchange, the default: each chunk's attention output goes to the
rank owning its rows over NVLink peer memory, which runs the output projection over
every head; --output reducescatter: the row-sharded output projection's partial
sums are reduce-scattered; --output allreduce: NCCL all-reduce, every rank holds
every row). A step = one prefill forward over all 262144 tokens; value = whole-job
prefill tok/s. After the timed prefill, 256
autoregressive decode steps run against the resulting KV cache and are reported
under "decode". The line's "parity" compares rows of the timed forward's output
with the FP64 oracle (oracle/, test infrastructure: the checker, never the thing
measured).

On one GPU the default line also carries "configs": the other configurations of
the metric, each with its own roofline and parity — cfg2 (FP32 prefill B=8
T=2048 d=1024 16x64), cfg3 (decode of 64 sequences over a 4096-token KV cache,
GQA 32/8 x 64), cfg4-fp8 / cfg4-nf4 (prefill B=4 T=4096 d=4096 32x128 with FP8
row-scale / NF4 block-64 weights) — and "dequant" (FP8 / NF4 -> BF16 GB/s).
Each is also selectable on its own with --workload.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Data is synthetic (no dataset is named by the baseline): the counter-based
SplitMix64 stream of welvet_b200_fill_synthetic — Xavier-uniform weights (seed 0,
order Wq, Wk, Wv, Wo; N(0, 0.02) for the quantised configs), N(0,1) inputs (seed 1),
KV cache N(0,1)*0.5 (seed 2). Inputs (cfg5 x: 2.1 GB; cfg3 KV cache: 1.1 GB) exceed
L2 (126 MB), so no explicit flush is needed between steps.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

# nominal dense FP64 of one B200 (HGX B200 datasheet: 296 TFLOP/s for 8 GPUs); the pool
# measures no FP64 peak, so the NormalBP backward's fraction is quoted against this
FP64_NOMINAL_TFLOPS = 37.0
# DRAM bytes per unit measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum) for
# the cfg5 head shape (32 x 128, BF16) at B=2, T=4096: prefill attention per token,
# decode attention per cached (sequence, position); scaled to the bench's launches
TRAFFIC_PREFILL_PER_TOKEN = 247.8e6 / 8192
TRAFFIC_DECODE_PER_ROW = 135.12e6 / (2 * 4097)
TRAFFIC_SOURCE = "ncu dram__bytes_read.sum+dram__bytes_write.sum at B=2 T=4096, scaled by units"

# output collective of a device-buffer prefill at N > 1 (welvet_b200_mha_set_output_mode)
OUTPUT_MODES = {"allreduce": 0, "reducescatter": 1, "exchange": 2}
OUTPUT_NAMES = {"allreduce": "all-reduce", "reducescatter": "reduce-scatter",
                "exchange": "attention-output exchange before the output projection"}

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "welvet.metal_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# B, T (sequence or cached context), d_model, heads, kv heads, weight format
# (0 BF16/FP32, 1 FP8-E4M3 row scale, 2 NF4 block-64), precision (1 BF16, 0 FP32), kind
WORKLOADS = {
    "cfg5": dict(B=32, T=8192, d=4096, H=32, NK=32, wf=0, prec=1, kind="prefill+decode"),
    "cfg4-fp8": dict(B=4, T=4096, d=4096, H=32, NK=32, wf=1, prec=1, kind="prefill"),
    "cfg4-nf4": dict(B=4, T=4096, d=4096, H=32, NK=32, wf=2, prec=1, kind="prefill"),
    # the reference's own FormatNone Int4 codes (per-tensor scale) kept resident and
    # dequantised inside the GEMM mainloop (weight_format 3, dtype 14)
    "cfg4-int4": dict(B=4, T=4096, d=4096, H=32, NK=32, wf=3, dt=14, prec=1, kind="prefill"),
    "cfg3": dict(B=64, T=4096, d=2048, H=32, NK=8, wf=0, prec=1, kind="decode"),
    # diagnostic: one GPU's share of cfg5 at 8 GPUs (4 of the 32 heads: q/k/v
    # projection N = 1536, output projection K = 512), without the collective
    "cfg5-shard8": dict(B=32, T=8192, d=4096, H=4, NK=4, hd=128, wf=0, prec=1, kind="prefill+decode"),
    "cfg2": dict(B=8, T=2048, d=1024, H=16, NK=16, wf=0, prec=0, kind="prefill"),
    # FormatNone weight round trip (mount-time encode -> decode), all dtypes 0-33
    "codec": dict(n=1 << 28, kind="codec"),
    # transformer-block forwards around the MHA, at the config-5 model width:
    # SwiGLU d=4096 with the reference's default_ffn width (swiglu.cpp:59-65), BF16;
    # RMSNorm / LayerNorm over 4096-wide rows, FP32 as the reference's entries;
    # Embedding of a 128256 x 4096 FP32 table
    "swiglu": dict(B=8, T=8192, d=4096, inter=10928, prec=1, kind="swiglu"),
    "rmsnorm": dict(B=16, T=4096, d=4096, kind="rmsnorm"),
    "layernorm": dict(B=16, T=4096, d=4096, kind="layernorm"),
    "embedding": dict(B=16, T=4096, d=4096, vocab=128256, kind="embedding"),
    # FP8 row-scale / NF4 block-64 -> BF16 dequantisation (the extension weight formats)
    "dequant": dict(n=1 << 30, kind="dequant"),
    # MHA NormalBP leaf (welvet_mha_normalbp_f32): forward + MSE + backward + SGD, FP32,
    # the reference's stream semantics, one call per step from host buffers
    "mha-nbp": dict(B=4, T=512, d=1024, H=16, kind="nbp"),
}
BLOCK_KINDS = ("swiglu", "rmsnorm", "layernorm", "embedding")
CODEC_DTYPES = range(34)
CODEC_STATS_FREE = (0, 1, 2, 3, 4, 5, 16, 24, 25)  # dtypes without a per-tensor statistics pass

METRIC = "MHA prefill tok/s (decode tok/s under 'decode'); % of roofline"
METRIC_DECODE = "MHA decode tok/s; % of HBM roofline"
SUB_WORKLOADS = ("cfg2", "cfg3", "cfg4-fp8", "cfg4-nf4", "cfg4-int4")
# FP32 kernels (cfg2) run as 3xTF32 on the tensor cores: kind::tf32 issues at half
# the kind::f16 rate (1.1 against 2.25 PFLOP/s dense, nominal) and every FP32 product
# is three TF32 products, so their ceiling is the measured sustained BF16 rate / 6.
# FP32 attention with a head_dim other than 64 runs on the CUDA cores
# (attn_f32_kernel): its roofline is the FFMA peak.
TF32X3_PER_BF16 = 1.0 / 6.0
METRIC_CODEC = "FormatNone weight round trip GB/s (decode(encode(w)), dtypes 0-33)"
METRIC_NBP = "MHA NormalBP tok/s (forward + backward + SGD)"
METRIC_BLOCK = {"swiglu": "SwiGLU forward tok/s", "rmsnorm": "RMSNorm forward tok/s",
                "layernorm": "LayerNorm forward tok/s", "embedding": "Embedding forward tok/s"}


def workload_of(wname, args):
    """Shape of workload `wname`; --batch / --seq override the selected workload only."""
    w = dict(WORKLOADS[wname])
    own = wname == args.workload
    if w["kind"] in ("codec", "dequant"):
        w["n"] = (args.batch if own else 0) or w["n"]
        return w
    w["B"] = (args.batch if own else 0) or w["B"]
    w["T"] = (args.seq if own else 0) or w["T"]
    if w["kind"] in BLOCK_KINDS or w["kind"] == "nbp":
        return w
    w["hd"] = w.get("hd") or w["d"] // w["H"]
    return w


def workload(args):
    return workload_of(args.workload, args)


def workload_config_of(wname, args, world):
    """The `config` object of a JSON line, the same for both arms."""
    w = workload_of(wname, args)
    if w["kind"] == "dequant":
        return {"workload": f"dequant: FP8 row-scale and NF4 block-64 -> BF16 of {w['n']} weights each",
                "global_batch": w["n"], "seq_len": 1, "parallelism": f"replicas x{world}",
                "l2": "codes and outputs larger than L2"}
    if w["kind"] == "codec":
        return {"workload": f"codec: decode(encode(w)) of {w['n']} FP32 weights, FormatNone dtypes 0-33",
                "global_batch": w["n"], "seq_len": 1, "parallelism": f"replicas x{world}",
                "l2": "tensor larger than L2 (%.2f GB)" % (w["n"] * 4 / 1e9)}
    if w["kind"] == "nbp":
        return {"workload": f"mha-nbp: NormalBP leaf (forward, MSE, backward, SGD) B={w['B']} T={w['T']} "
                            f"d={w['d']} H={w['H']}x{w['d'] // w['H']} causal RoPE FP32, stream semantics",
                "global_batch": w["B"], "seq_len": w["T"], "parallelism": f"replicas x{world}",
                "l2": "one call per step from host buffers (the reference entry's contract)"}
    if w["kind"] in BLOCK_KINDS:
        B, T, d = w["B"], w["T"], w["d"]
        desc = {"swiglu": f"SwiGLU d={d} inter={w.get('inter')} BF16",
                "rmsnorm": f"RMSNorm dim={d} FP32", "layernorm": f"LayerNorm dim={d} FP32",
                "embedding": f"Embedding vocab={w.get('vocab')} emb={d} FP32 table, Linear"}[w["kind"]]
        return {"workload": f"{wname}: {desc}, B={B} T={T}", "global_batch": B, "seq_len": T,
                "parallelism": f"replicas x{world}", "l2": "activations larger than L2 (x is %.2f GB)"
                % (B * T * d * (2 if w["kind"] == "swiglu" else 4) / 1e9)}
    B, T, d, H, NK, hd, wf = w["B"], w["T"], w["d"], w["H"], w["NK"], w["hd"], w["wf"]
    fmt = {1: " fp8 weights", 2: " nf4 weights", 3: f" FormatNone dtype {w.get('dt')} code weights"}.get(wf, "")
    es = 2 if w["prec"] == 1 else 4
    prec = " BF16" if w["prec"] == 1 else " FP32"
    if w["kind"] == "decode":
        return {"workload": f"{wname}: decode B={B} context {T} d={d} H={H}x{hd} NK={NK} RoPE{prec}{fmt}",
                "global_batch": B, "seq_len": 1, "context": T, "parallelism": f"tp{world} (heads {H // world}/GPU)",
                "l2": "KV cache larger than L2 (%.1f GB)" % (2 * B * T * NK * hd * es / 1e9)}
    out = "" if world == 1 else {
        "reducescatter": ", reduce-scatter output (rank r keeps its row slice of each chunk)",
        "exchange": ", attention-output exchange before the output projection (rank r keeps its row slice of "
                    "each chunk)",
        "allreduce": ", all-reduce output"}[args.output]
    return {"workload": f"{wname}: B={B} T={T} d={d} H={H}x{hd} NK={NK} causal RoPE{prec}{fmt}",
            "global_batch": B, "seq_len": T, "parallelism": f"tp{world} (heads {H // world}/GPU){out}",
            "l2": "inputs larger than L2 (x is %.1f GB)" % (B * T * d * es / 1e9)}


def workload_config(args, world):
    return workload_config_of(args.workload, args, world)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return dict(hbm=j["hbm_gbs"], bf16=j["bf16_tflops"], bf16_sus=j.get("bf16_tflops_sustained", j["bf16_tflops"]),
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: through NVML
    (pynvml) every 10 ms in a thread, so that a timed region of a few hundred ms
    (8 GPUs) still gets its own record; nvidia-smi (200 ms) when NVML is missing."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): sw power cap, hw slowdown, sw thermal,
    # hw thermal
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None
        self.nvml = None
        self.samples = []  # (sm_mhz, reason bits)
        self.max_mhz = None
        self.stop_evt = threading.Event()

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nvml = pynvml

            def loop():
                while not self.stop_evt.is_set():
                    try:
                        self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                             int(reasons(h))))
                    except pynvml.NVMLError:
                        pass
                    self.stop_evt.wait(0.01)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            sm = [c for c, _ in self.samples]
            reasons = sorted({n for _, bits in self.samples for n, b in self.BITS.items() if bits & b})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "samples": len(sm), "reasons": reasons, "source": "nvml 10 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons), "source": "nvidia-smi 200 ms"}


def flops_prefill(B, T, d, H, NK, hd):
    qd, kd = H * hd, NK * hd
    proj = 2.0 * B * T * d * (qd + 2 * kd) + 2.0 * B * T * qd * d
    attn = 4.0 * hd * H * B * T * (T + 1) / 2
    return proj, attn


def cpu_sample_decode(w, B_s, threads=0):
    """Times the FP64 oracle's decode step for B_s sequences over the workload's
    context; returns seconds."""
    import oracle_py as O
    import welvet_b200 as W
    d, H, NK, hd, T = w["d"], w["H"], w["NK"], w["hd"], w["T"]
    Ws = W.xavier_weights(d, H * hd, NK * hd, seed=0)
    kc = W.synthetic(B_s * T * NK * hd, 2, 1, 0.5).reshape(B_s, T, NK * hd)
    vc = W.synthetic(B_s * T * NK * hd, 2, 1, 0.5, offset=B_s * T * NK * hd).reshape(B_s, T, NK * hd)
    x = W.synthetic(B_s * d, 1, 1, 1.0).reshape(B_s, d)
    cfg = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, max_seq_len=T + 1, per_sequence=1)
    t0 = time.perf_counter()
    O.mha_decode(cfg, [T] * B_s, kc, vc, *Ws, x, threads=threads)
    return time.perf_counter() - t0


def codec_bytes(n, dtype):
    """Algorithmic HBM bytes of one round trip: the statistics pass reads w once,
    the element pass reads w and writes the result."""
    return n * 4 * (2 if dtype in CODEC_STATS_FREE else 3)


def codec_cpu_sample(n_s, use_ref):
    """Times decode(encode(w)) of every dtype on n_s weights on one host core:
    the reference's own WeightStore round trip (oracle/_ref) or the C port.
    Returns (seconds, bytes in the GPU arm's accounting)."""
    import oracle_py as O
    import welvet_b200 as W
    w = W.synthetic(n_s, 0, 1, 0.02)
    wm = w.reshape(-1, 1024)
    t0 = time.perf_counter()
    for dt in CODEC_DTYPES:
        if use_ref:
            code, msg, _, _, _ = O.ref_weight_roundtrip(dt, wm)
            if code:
                raise RuntimeError(msg)
        else:
            O.roundtrip(dt, w)
    dt_s = time.perf_counter() - t0
    return dt_s, sum(codec_bytes(n_s, d) for d in CODEC_DTYPES)


def run_reference(args):
    """Reference arm: the reference's own MHA code (mha.cpp + dense.cpp + soft-double
    shaders, oracle/_ref) on the host cores through its one-shot entry
    (welvet_mha_forward_f32 semantics: encode + mount + forward per call). Falls back
    to the FP64 port when oracle/_ref was not built. Prefill workloads: see
    reference_prefill_sample for how each step's samples become the workload's tok/s."""
    import oracle_py as O
    import welvet_b200 as W
    w = workload(args)
    if w["kind"] == "decode":
        print(json.dumps({"impl": "reference", "unavailable": "the reference MHA has no KV cache or decode step"}),
              flush=True)
        return
    if w["kind"] in BLOCK_KINDS:
        return run_block_reference(args, w)
    if w["kind"] == "nbp":
        return run_nbp_reference(args, w)
    if w["kind"] == "codec":
        use_ref = O.ref_available()
        n_s = 1 << 20
        for _ in range(args.warmup):
            codec_cpu_sample(1 << 16, use_ref)
        tot_s = tot_b = 0.0
        for _ in range(args.steps):
            dt_s, b = codec_cpu_sample(n_s, use_ref)
            tot_s += dt_s
            tot_b += b
        value = tot_b / tot_s / 1e9
        kind = "reference" if use_ref else "port"
        sample = f"{n_s} weights (1024-wide rows) x 34 dtypes per step, one core, WeightStore round trip"
        print(json.dumps({"impl": "reference", "metric": METRIC_CODEC, "value": value, "unit": "GB/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": tot_s / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": workload_config(args, args.gpus),
                          "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": kind,
                                           "sample": sample},
                          "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    return run_reference_prefill(args, w)


def reference_prefill_sample(O, W, w, kind):
    """One step of the prefill reference arm: four bounded calls of the reference's
    one-shot forward (stream semantics, one sequence), timed separately:
      A1, A16: the workload's layer (d, H x hd) on 1 and 16 tokens. Their difference is
               15 tokens of projections (soft-double matvec, spread over all host
               threads by the CPU executor) -> seconds per token p; A1 - p is the
               per-call mount (encode + decode of the four weight matrices) c.
      B256, B512: a one-head layer with the workload's head_dim (d = hd) on 256 and
               512 tokens: time = a T + b T^2, so b = (B512 - 2 B256) / (512^2 - 2 256^2)
               and one (query, key) pair of one head costs r = 2 b seconds (the
               reference's attention runs on one thread, shaders/ops_mha.metal:32-33).
    The workload's time is modelled as c + M p + r H B T (T + 1) / 2: the mount once,
    projections per token, attention per causal pair and head."""
    d, H, NK, hd = w["d"], w["H"], w["NK"], w["hd"]
    Ws = W.xavier_weights(d, H * hd, NK * hd, seed=0)
    W1 = W.xavier_weights(hd, hd, hd, seed=0)

    def call(cfg, T, Wt, dd):
        x = W.synthetic(T * dd, 1, 1, 1.0).reshape(T, dd)
        t0 = time.perf_counter()
        if kind == "reference":
            code, msg, _, _ = O.ref_mha_forward(cfg, 1, T, *Wt, x, 1)
            if code:
                raise RuntimeError(msg)
        else:
            O.mha_forward(cfg, 1, T, *Wt, x)
        return time.perf_counter() - t0

    big = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, max_seq_len=512)
    one = O.MhaCfg(d_model=hd, num_heads=1, num_kv_heads=1, max_seq_len=512)
    tA1 = call(big, 1, Ws, d)
    tA16 = call(big, 16, Ws, d)
    tB256 = call(one, 256, W1, hd)
    tB512 = call(one, 512, W1, hd)
    p = max((tA16 - tA1) / 15.0, 1e-9)
    c = max(tA1 - p, 0.0)
    b = (tB512 - 2.0 * tB256) / (512.0 ** 2 - 2.0 * 256.0 ** 2)
    if b <= 0:  # timing noise: bound the pair cost by the whole 512-token call
        b = tB512 / 512.0 ** 2
    return {"mount_s": c, "proj_s_per_token": p, "attn_s_per_pair_head": 2.0 * b,
            "sample_s": tA1 + tA16 + tB256 + tB512}


def run_reference_prefill(args, w):
    import oracle_py as O
    import welvet_b200 as W
    B, T, d, H, NK, hd = w["B"], w["T"], w["d"], w["H"], w["NK"], w["hd"]
    M = B * T
    kind = "reference" if O.ref_available() else "port"
    small = dict(w, d=hd, H=1, NK=1)
    for _ in range(args.warmup):
        reference_prefill_sample(O, W, small, kind)
    samples = [reference_prefill_sample(O, W, w, kind) for _ in range(args.steps)]
    med = {k: statistics.median(s_[k] for s_ in samples) for k in samples[0]}
    pairs = H * B * T * (T + 1) / 2.0
    est_s = med["mount_s"] + M * med["proj_s_per_token"] + pairs * med["attn_s_per_pair_head"]
    value = M / est_s
    step_s = sum(s_["sample_s"] for s_ in samples) / len(samples)
    cores = os.cpu_count()
    sample = (f"per step: the reference's one-shot forward on 1 and 16 tokens of the {args.workload} layer "
              f"(d={d}, {H}x{hd}) and on 256 and 512 tokens of a one-head layer with head_dim {hd}; the workload "
              f"time is modelled as mount + M x projection s/token + H B T(T+1)/2 x attention s/pair (medians "
              f"over the steps): mount {med['mount_s']:.2f} s, {med['proj_s_per_token'] * 1e3:.1f} ms/token, "
              f"{med['attn_s_per_pair_head'] * 1e6:.2f} us/pair/head -> {est_s / 3600:.1f} h per step "
              f"(attention {pairs * med['attn_s_per_pair_head'] / est_s * 100:.0f} %)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64 (soft-double)",
            "data": "synthetic", "config": workload_config(args, args.gpus),
            "method": "projection and attention timed separately on the reference's own code, each scaled by "
                      "its own unit count (tokens, causal pairs x heads)",
            "model_s_per_workload_step": est_s,
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def block_sample(w, use_ref, tokens):
    """One bounded CPU sample of a block workload: `tokens` tokens of the same layer
    through the reference's own entry (oracle/_ref, when use_ref: weights encoded and
    mounted per call, as its one-shot entry does) or the FP64 port on decoded weights.
    Returns seconds."""
    import oracle_py as O
    import welvet_b200 as W
    k, d = w["kind"], w["d"]
    x = W.synthetic(tokens * d, 1, 1, 1.0)
    if k == "swiglu":
        h = w["inter"]
        a = (6.0 / (d + h)) ** 0.5
        G = W.synthetic(h * d, 0, 0, a).reshape(h, d)
        U = W.synthetic(h * d, 0, 0, a, offset=h * d).reshape(h, d)
        D = W.synthetic(d * h, 0, 0, a, offset=2 * h * d).reshape(d, h)
        t0 = time.perf_counter()
        if use_ref:
            code, msg, _, _ = O.ref_swiglu_forward(1, tokens, G, U, D, x)
            if code:
                raise RuntimeError(msg)
        else:
            O.swiglu_forward(x.reshape(tokens, d), G, U, D)
        return time.perf_counter() - t0
    if k in ("rmsnorm", "layernorm"):
        g = W.synthetic(d, 5, 1, 0.1) + np.float32(1)
        b = W.synthetic(d, 6, 1, 0.1)
        t0 = time.perf_counter()
        if use_ref:
            code, msg, _, _ = O.ref_norm_forward(k == "layernorm", 1, tokens, d, 0.0, g, x, beta=b)
            if code:
                raise RuntimeError(msg)
        else:
            O.norm_forward(k == "layernorm", x.reshape(tokens, d), g, b, 0.0)
        return time.perf_counter() - t0
    vocab = min(w["vocab"], 8192)  # the table is decoded per call: bounded here
    Wt = W.synthetic(vocab * d, 7, 1, 1.0).reshape(vocab, d)
    ids = np.floor(W.synthetic(tokens, 8, 0, float(vocab))).astype(np.float32)
    t0 = time.perf_counter()
    if use_ref:
        code, msg, _, _ = O.ref_embedding_forward(1, vocab, d, tokens, 2, 1, -1, Wt, ids)
        if code:
            raise RuntimeError(msg)
    else:
        O.embedding_forward(ids, Wt, 1, -1)
    return time.perf_counter() - t0


BLOCK_CPU_TOKENS = {"swiglu": 8, "rmsnorm": 8192, "layernorm": 8192, "embedding": 8192}
BLOCK_REF_TOKENS = {"swiglu": 2, "rmsnorm": 1024, "layernorm": 1024, "embedding": 1024}


def run_block_reference(args, w):
    """Reference arm of the block workloads: the reference's own layer code
    (oracle/_ref; its one-shot entries encode and mount the weights on every call,
    as timed here) on a bounded token sample per step, reported as tok/s; the FP64
    port when oracle/_ref is absent."""
    import oracle_py as O
    use_ref = O.ref_available()
    n = BLOCK_REF_TOKENS[w["kind"]]
    for _ in range(args.warmup):
        block_sample(w, use_ref, max(1, n // 4))
    tot = sum(block_sample(w, use_ref, n) for _ in range(args.steps))
    value = n * args.steps / tot
    kind = "reference" if use_ref else "port"
    sample = (f"{n} tokens of the {args.workload} layer per step through the reference's one-shot entry "
              f"(weights encoded per call){', vocab bounded to 8192' if w['kind'] == 'embedding' else ''}")
    print(json.dumps({"impl": "reference", "metric": METRIC_BLOCK[w["kind"]], "value": value, "unit": "tok/s",
                      "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": tot / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f64 (soft-double)", "data": "synthetic",
                      "config": workload_config(args, args.gpus),
                      "cpu_baseline": {"value": value, "unit": "tok/s", "cores": os.cpu_count(), "kind": kind,
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def run_block(args, rank, world, local):
    """Transformer-block forwards (SwiGLU, RMSNorm, LayerNorm, Embedding) on one
    GPU per rank; replicas only (each rank runs its own batch, no collective). A step
    = one forward over B*T tokens with activations resident in HBM."""
    import torch
    import torch.distributed as dist
    import welvet_b200 as W
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    w = workload(args)
    k, B, T, d = w["kind"], w["B"], w["T"], w["d"]
    M = B * T
    pk = peaks()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    host_args = None
    if k == "swiglu":
        h = w["inter"]
        a = (6.0 / (d + h)) ** 0.5
        ws = []
        for i, (r, c) in enumerate(((h, d), (h, d), (d, h))):
            t = torch.empty(r, c, device="cuda")
            W.fill_synthetic(t, 0, 0, a, offset=i * h * d)
            ws.append(t)
        layer = W.SwigluLayer(*ws, dtype=1, precision=1)
        del ws
        x = torch.empty(M, d, device="cuda", dtype=torch.bfloat16)
        W.fill_synthetic(x, 1, 1, 1.0, offset=rank * M * d)
        pre = torch.empty(M, h, device="cuda", dtype=torch.bfloat16)
        post = torch.empty(M, d, device="cuda", dtype=torch.bfloat16)
        step = lambda: layer.forward(M, x, pre, post, stream=stream)  # noqa: E731
        slots = ("gemm_gate_up", "gemm_down")
        work = {"gemm_gate_up": 2.0 * M * d * 2 * h, "gemm_down": 2.0 * M * h * d}
        unit, bound = "TFLOP/s", "tensor"
        dtype = "bf16"
    elif k in ("rmsnorm", "layernorm"):
        x = torch.empty(M, d, device="cuda")
        W.fill_synthetic(x, 1, 1, 1.0, offset=rank * M * d)
        g = torch.empty(d, device="cuda")
        b = torch.empty(d, device="cuda")
        W.fill_synthetic(g, 5, 1, 0.1)
        W.fill_synthetic(b, 6, 1, 0.1)
        g += 1.0
        pre = torch.empty_like(x)
        post = torch.empty_like(x)
        ln = k == "layernorm"
        step = lambda: W.norm_forward(ln, M, d, 0.0, g, x, pre, post, beta=b, stream=stream)  # noqa: E731
        slots = ("norm",)
        work = {"norm": 3.0 * M * d * 4 + (2 if ln else 1) * d * 4}
        unit, bound = "GB/s", "hbm"
        dtype = "f32 (FP64 statistics)"
    else:
        vocab = w["vocab"]
        Wt = torch.empty(vocab, d, device="cuda")
        W.fill_synthetic(Wt, 7, 1, 1.0)
        ids = torch.empty(M, device="cuda")
        W.fill_synthetic(ids, 8, 0, float(vocab), offset=rank * M)
        ids = ids.abs().floor()
        out = torch.empty(M, d, device="cuda")
        step = lambda: W.embedding_forward(M, vocab, d, 1, -1, Wt, ids, out, stream=stream)  # noqa: E731
        slots = ("embedding",)
        work = {"embedding": 2.0 * M * d * 4 + M * 4}
        unit, bound = "GB/s", "hbm"
        dtype = "f32"
    for _ in range(args.warmup):
        step()
    barrier()
    W.device_check()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    clocks.start()
    W.profile_read(reset=True)
    W.profile_enable(True)
    W.launch_count(reset=True)
    barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    barrier()
    launches = W.launch_count(reset=True)
    W.profile_enable(False)
    prof = W.profile_read(reset=True)
    clk = clocks.stop()
    W.device_check()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    tokps = world * M / (ms / 1e3)
    dom = max(slots, key=lambda s_: prof[s_][0])
    tot, cnt = prof[dom]
    avg_ms = tot / max(cnt, 1)
    per_launch = work[dom] * args.steps / max(cnt, 1)
    if bound == "tensor":
        achieved = per_launch / (avg_ms / 1e3) / 1e12
        peak, pkind = pk["bf16_sus"], f"{pk['src']} sustained bf16 (of {pk['src']})"
    else:
        achieved = per_launch / (avg_ms / 1e3) / 1e9
        peak, pkind = pk["hbm"], f"{pk['src']} HBM copy (of {pk['src']})"
    roof = {"bound": bound, "kernel": dom, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "peak_kind": pkind, "traffic": None,
            ("flops_per_launch" if bound == "tensor" else "bytes_per_launch"): per_launch,
            "avg_launch_ms": avg_ms, "kernel_ms_per_step": {s_: prof[s_][0] / args.steps for s_ in slots}}
    e2e = None
    if not args.no_e2e:
        # the reference's one-shot entry over host buffers: weights encoded and
        # mounted, x uploaded, outputs downloaded, per call (as the reference does)
        n_e = min(M, 8192)
        xh = W.synthetic(n_e * d, 1, 1, 1.0)
        if k == "swiglu":
            hh = w["inter"]
            a = (6.0 / (d + hh)) ** 0.5
            Wh = [W.synthetic(r * c, 0, 0, a, offset=i * hh * d).reshape(r, c)
                  for i, (r, c) in enumerate(((hh, d), (hh, d), (d, hh)))]
            call = lambda: W.swiglu_forward_f32(1, n_e, *Wh, xh)  # noqa: E731
            hb, db = n_e * d * 4 + 3 * hh * d * 4, n_e * (d + hh) * 4
        elif k in ("rmsnorm", "layernorm"):
            gh = W.synthetic(d, 5, 1, 0.1) + np.float32(1)
            bh = W.synthetic(d, 6, 1, 0.1)
            call = lambda: W.norm_forward_f32(k == "layernorm", 1, n_e, d, 0.0, gh, xh, beta=bh)  # noqa: E731
            hb, db = n_e * d * 4 + 2 * d * 4, 2 * n_e * d * 4
        else:
            vocab_e = min(w["vocab"], 32768)  # host table bounded to 0.5 GB
            Wh = W.synthetic(vocab_e * d, 7, 1, 1.0).reshape(vocab_e, d)
            idh = np.floor(W.synthetic(n_e, 8, 0, float(vocab_e))).astype(np.float32)
            idh = np.abs(idh)
            call = lambda: W.embedding_forward_f32(1, vocab_e, d, n_e, 2, 1, -1, Wh, idh)  # noqa: E731
            hb, db = vocab_e * d * 4 + n_e * 4, 2 * n_e * d * 4
        call()
        barrier()
        n_rep = 2
        t0 = time.perf_counter()
        for _ in range(n_rep):
            call()
        e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / n_rep)
        e2e = {"value": world * n_e / (e_ms / 1e3), "unit": "tok/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": hb, "d2h_bytes_per_step": db,
               "api": f"welvet_{k}_forward_f32 (host buffers, weights encoded per call), {n_e} tokens"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_c = BLOCK_CPU_TOKENS[k]
        dt_c = block_sample(w, False, n_c)
        cpu = {"value": n_c / dt_c, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"FP64 oracle, {n_c} tokens of the layer, {dt_c:.2f} s"
                         f"{' (vocab bounded to 8192)' if k == 'embedding' else ''}"}
    if rank == 0:
        print(json.dumps({"metric": METRIC_BLOCK[k], "value": tokps, "unit": "tok/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": dtype,
                          "data": "synthetic (SplitMix64 counter stream)", "config": workload_config(args, world),
                          "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                          "clocks": clk,
                          "profile_ms": {s_: prof[s_][0] / args.steps for s_ in slots}}), flush=True)
    if k == "swiglu":
        layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def nbp_inputs(d, H, M, seed=0):
    import welvet_b200 as W
    Ws = W.xavier_weights(d, d, d, seed=seed)
    x = W.synthetic(M * d, 1, 1, 1.0)
    tgt = W.synthetic(M * d, 2, 1, 1.0)
    return Ws, x, tgt


def nbp_sample(w, use_ref, B, T):
    """One NormalBP call of B x T tokens of the workload's layer on the host: the
    reference's own entry (oracle/_ref) or the FP64 port. Returns seconds."""
    import oracle_py as O
    d, H = w["d"], w["H"]
    Ws, x, tgt = nbp_inputs(d, H, B * T)
    cfg = O.MhaCfg(d_model=d, num_heads=H, max_seq_len=max(512, T))
    t0 = time.perf_counter()
    if use_ref:
        code, msg, *_ = O.ref_mha_normalbp(cfg, B, T, *Ws, x, tgt, 1, 0.01)
        if code:
            raise RuntimeError(msg)
    else:
        code, *_ = O.mha_normalbp(cfg, B, T, *Ws, x, tgt, 1, 0.01)
        if code:
            raise RuntimeError(f"oracle {code}")
    return time.perf_counter() - t0


def run_nbp_reference(args, w):
    import oracle_py as O
    use_ref = O.ref_available()
    T_s = 16
    for _ in range(args.warmup):
        nbp_sample(w, use_ref, 1, 4)
    tot = sum(nbp_sample(w, use_ref, 1, T_s) for _ in range(args.steps))
    value = T_s * args.steps / tot
    kind = "reference" if use_ref else "port"
    sample = f"1 x {T_s} tokens of the mha-nbp layer per step through the reference's welvet_mha_normalbp_f32 body"
    print(json.dumps({"impl": "reference", "metric": METRIC_NBP, "value": value, "unit": "tok/s",
                      "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": tot / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f64 (soft-double)", "data": "synthetic",
                      "config": workload_config(args, args.gpus),
                      "cpu_baseline": {"value": value, "unit": "tok/s", "cores": os.cpu_count(), "kind": kind,
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def run_nbp(args, rank, world, local):
    """The NormalBP leaf: a step is one welvet_mha_normalbp_f32 call (host buffers in
    and out, weights encoded per call, as the reference entry), so `value` and `e2e`
    are the same measurement; the live per-kernel event profile splits it."""
    import torch
    import torch.distributed as dist
    import welvet_b200 as W
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    w = workload(args)
    B, T, d, H = w["B"], w["T"], w["d"], w["H"]
    M = B * T
    Ws, x, tgt = nbp_inputs(d, H, M, seed=rank)

    # the caller's host output buffers, allocated once (as a training loop would)
    outs = tuple(np.zeros(n, np.float32) for n in (M * d, M * d, M * d, 4 * d * d, 4 * d * d))

    def step():
        return W.mha_normalbp_f32(B, T, d, H, 0, 0, max(512, T), 1, 0, 1, *Ws, x, tgt, 1, 0.01, out=outs)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    W.profile_read(reset=True)
    W.profile_enable(True)
    W.launch_count(reset=True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = (time.perf_counter() - t0) / args.steps * 1e3
    launches = W.launch_count(reset=True)
    W.profile_enable(False)
    prof = W.profile_read(reset=True)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([el], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    value = world * M / (el / 1e3)
    hd = d // H
    # algorithmic FP64 work of the attention backward: per (head, query, allowed key)
    # the score dot, dw dot, gv / gk / gq updates ~ 5 x 2 hd FLOPs; keys = all earlier
    # positions of the stream (causal)
    keys = sum(T * b * T + T * (T + 1) / 2 for b in range(B))
    attn_flops = H * keys * 10.0 * hd
    gemm_flops = 2.0 * M * d * d * (4 + 4)  # QKV recompute, dX, dWqkv (3 d x d each) + O grads
    a_ms = prof["attn_bwd"][0] / args.steps
    g_ms = prof["gemm_grad"][0] / args.steps
    achieved = attn_flops / (a_ms / 1e3) / 1e12
    roof = {"bound": "fp64", "kernel": "attention backward (per batch: dgemm_kernel x3, attn_bwd_row_kernel, "
            "kv_grad_kernel, ring_fill_kernel, batch_end_kernel)", "achieved": achieved,
            "peak": FP64_NOMINAL_TFLOPS, "unit": "TFLOP/s", "frac": achieved / FP64_NOMINAL_TFLOPS,
            "peak_kind": "nominal FP64 of a B200 (no measured FP64 peak on this pool)",
            "traffic": None, "kernel_ms_per_step": {"attn_bwd": a_ms, "gemm_grad": g_ms},
            "gemm_grad_tflops": gemm_flops / (g_ms / 1e3) / 1e12 if g_ms > 0 else None}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        T_c = 64
        dt = nbp_sample(w, False, 1, T_c)
        cpu = {"value": T_c / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"FP64 oracle, 1 x {T_c} tokens of the layer, {dt:.2f} s"}
    if rank == 0:
        print(json.dumps({"metric": METRIC_NBP, "value": value, "unit": "tok/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": el, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32 (FP64 attention backward)",
                          "data": "synthetic", "config": workload_config(args, world), "roofline": roof,
                          "cpu_baseline": cpu,
                          "e2e": {"value": value, "unit": "tok/s", "ms_per_step": el,
                                  "h2d_bytes_per_step": 4 * (4 * d * d + 2 * M * d),
                                  "d2h_bytes_per_step": 4 * (M * d * 3 + 8 * d * d),
                                  "api": "welvet_mha_normalbp_f32 (host buffers)"},
                          "gpu_launches": launches, "clocks": clk,
                          "profile_ms": {k: v[0] / args.steps for k, v in prof.items() if v[1]}}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_codec(args, rank, world, local):
    """FormatNone round trips (the mount-time weight codec) of one 1 GiB FP32 tensor
    per GPU, every dtype in turn; a step = all 34 dtypes. Replicas only: each rank
    converts its own tensor, no collective."""
    import torch
    import torch.distributed as dist
    import welvet_b200 as W
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    n = workload(args)["n"]
    w = torch.empty(n, device="cuda", dtype=torch.float32)
    W.fill_synthetic(w, 0, 1, 0.02, offset=rank * n)
    out = torch.empty_like(w)
    stream = torch.cuda.current_stream()
    pk = peaks()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        for dt in CODEC_DTYPES:
            W.codec_roundtrip(dt, w, out, stream=stream)
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(CODEC_DTYPES) + 1)]
    clocks = Clocks(local)
    clocks.start()
    W.launch_count(reset=True)
    barrier()
    per = {dt: 0.0 for dt in CODEC_DTYPES}
    t_all = 0.0
    for _ in range(args.steps):
        evs[0].record(stream)
        for i, dt in enumerate(CODEC_DTYPES):
            W.codec_roundtrip(dt, w, out, stream=stream)
            evs[i + 1].record(stream)
        stream.synchronize()
        for i, dt in enumerate(CODEC_DTYPES):
            per[dt] += evs[i].elapsed_time(evs[i + 1])
        t_all += evs[0].elapsed_time(evs[-1])
    barrier()
    launches = W.launch_count(reset=True)
    clk = clocks.stop()
    W.device_check()
    ms = max_over_ranks(t_all / args.steps)
    step_bytes = sum(codec_bytes(n, dt) for dt in CODEC_DTYPES)
    value = world * step_bytes / (ms / 1e3) / 1e9
    per_dtype = {str(dt): {"ms": per[dt] / args.steps,
                           "gbs": codec_bytes(n, dt) / (per[dt] / args.steps / 1e3) / 1e9} for dt in CODEC_DTYPES}
    slow = min(per_dtype, key=lambda k: per_dtype[k]["gbs"])
    achieved = step_bytes / (ms / 1e3) / 1e9
    roof = {"bound": "hbm", "kernel": "roundtrip_kernel + stats_first (all dtypes)", "achieved": achieved,
            "peak": pk["hbm"], "unit": "GB/s", "frac": achieved / pk["hbm"],
            "peak_kind": f"{pk['src']} HBM copy (of {pk['src']})", "traffic": None,
            "bytes_per_step": step_bytes, "slowest_dtype": {slow: per_dtype[slow]}}
    # end to end: pinned host weights -> device, round trip, result back to the host
    e2e = None
    if not args.no_e2e:
        n_e = min(n, 1 << 26)
        wh = w[:n_e].cpu().pin_memory()
        oh = torch.empty(n_e, dtype=torch.float32).pin_memory()
        wd = torch.empty(n_e, device="cuda", dtype=torch.float32)
        od = torch.empty_like(wd)
        barrier()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        ea.record(stream)
        for dt in CODEC_DTYPES:
            wd.copy_(wh, non_blocking=True)
            W.codec_roundtrip(dt, wd, od, stream=stream)
            oh.copy_(od, non_blocking=True)
        eb.record(stream)
        barrier()
        e_ms = max_over_ranks(max(ea.elapsed_time(eb), (time.perf_counter() - t0) * 1e3))
        e_bytes = sum(codec_bytes(n_e, dt) for dt in CODEC_DTYPES)
        e2e = {"value": world * e_bytes / (e_ms / 1e3) / 1e9, "unit": "GB/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": 34 * n_e * 4, "d2h_bytes_per_step": 34 * n_e * 4,
               "api": "welvet_b200_codec_roundtrip between pinned host copies (%d weights)" % n_e}
        del wh, oh, wd, od
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        dt_s, b = codec_cpu_sample(1 << 20, False)
        cpu = {"value": b / dt_s / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"C port of the round trip, 1048576 weights x 34 dtypes, {dt_s:.2f} s"}
    if rank == 0:
        print(json.dumps({"metric": METRIC_CODEC, "value": value, "unit": "GB/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic (SplitMix64 normal(0, 0.02) weights)",
                          "config": workload_config(args, world), "roofline": roof, "cpu_baseline": cpu,
                          "e2e": e2e, "gpu_launches": launches, "clocks": clk, "per_dtype": per_dtype}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bf16_round(a):
    """float32 -> the nearest bfloat16 (round to nearest even) as float32: the value a
    BF16 device buffer holds after __float2bfloat16_rn of the same float."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)) << np.uint64(16)
    return r.astype(np.uint32).view(np.float32).reshape(a.shape)


def oracle_weights(O, host_ws, wf, prec, dt=1):
    """The dequantised weights the device layer computes with (the parity checker's
    inputs): FP32 as given (3xTF32 splits are exact), BF16 rounded, FP8 row-scale or
    NF4 block-64 decoded by the oracle's codecs, or the FormatNone decode(encode)
    of dtype dt (weight_format 3)."""
    if wf == 3:
        return [O.roundtrip(dt, w).reshape(w.shape) for w in host_ws]
    if wf == 1:
        return [O.fp8_rowscale(w)[2] for w in host_ws]
    if wf == 2:
        return [O.nf4_block(w, 64)[2] for w in host_ws]
    return [bf16_round(w) for w in host_ws] if prec == 1 else list(host_ws)


def parity_record(got, want, tol, rows):
    """max|y - ŷ| / max|ŷ| of each output tensor against the FP64 oracle."""
    out = {"metric": "max|y-yhat|/max|yhat| vs the FP64 oracle on the same (dequantised) weights and inputs",
           "rows": rows, "tol": tol}
    ok = True
    for name, (g, r) in {k: (got[k], want[k]) for k in got}.items():
        g = np.asarray(g, np.float64)
        r = np.asarray(r, np.float64)
        e = float(np.abs(g - r).max() / max(np.abs(r).max(), 1e-30))
        out[name] = e
        ok = ok and bool(np.isfinite(g).all()) and e <= tol
    out["ok"] = ok
    return out


def run_mha(args, wname, rank, world, local, primary=True):
    """One MHA workload on this rank's head shard; returns the JSON record (rank 0)
    or None. A step = one prefill forward over B x T tokens (prefill workloads) or
    one decode step of B sequences (decode workloads), device-resident inputs.
    primary: the headline line (clocks, e2e through the host-buffer API, CPU
    baseline); sub-records carry their own roofline, parity and clocks."""
    import torch
    import torch.distributed as dist
    import welvet_b200 as W
    wall0 = time.perf_counter()
    w = workload_of(wname, args)
    B, T, d, H, NK, hd, wf, prec = w["B"], w["T"], w["d"], w["H"], w["NK"], w["hd"], w["wf"], w["prec"]
    decode_only = w["kind"] == "decode"
    act = torch.bfloat16 if prec == 1 else torch.float32
    es = 2 if prec == 1 else 4
    steps, warmup = args.steps, args.warmup
    hb, hc = W.head_shard(H, NK, world, rank)
    kd_l = (hc // (H // NK)) * hd  # this rank's KV columns
    cfg = W.MhaConfig.make(d, H, NK, precision=prec, weight_format=wf, head_begin=hb, head_count=hc,
                           device=local, head_dim=hd)
    check_parity = not args.no_parity and rank == 0
    # Full FP32 weights generated on the device (same stream on every rank), then mounted.
    shapes = [(H * hd, d), (NK * hd, d), (NK * hd, d), (d, H * hd)]
    ws, off = [], 0
    for r, c in shapes:
        t = torch.empty(r, c, device="cuda", dtype=torch.float32)
        a = (6.0 / (r + c)) ** 0.5 if wf == 0 else 0.02
        W.fill_synthetic(t, 0, 0 if wf == 0 else 1, a, offset=off)
        off += r * c
        ws.append(t)
    torch.cuda.synchronize()
    host_ws = [t.cpu().numpy() for t in ws] if (check_parity or (primary and not args.no_cpu)) else None
    layer = W.MhaLayer(cfg, *ws, dtype=w.get("dt", 1))
    del ws
    torch.cuda.empty_cache()
    if world > 1:
        uid = [W.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        layer.attach_comm(uid[0], world, rank)
        # output collective of the device-timed prefill: reduce-scatter (rank r keeps
        # the r-th row slice of each chunk summed; half the NVLink bytes), the
        # attention-output exchange (the same rows, the exchange before the output
        # projection) or all-reduce (--output); decode and the host-buffer e2e path
        # all-reduce
        layer.set_output_mode(OUTPUT_MODES[args.output])
    stream = torch.cuda.current_stream()
    pk = peaks()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    M = B * T
    x = None
    tokps = ms = None
    roof = e2e = cpu = parity = None
    launches = 0
    clk = {}
    prof = {}
    dparity = None
    n_oracle = min(args.parity_tokens, T)

    # ------------------------------------------------------------ timed prefill
    if not decode_only:
        x = torch.empty(M, d, device="cuda", dtype=act)
        W.fill_synthetic(x, 1, 1, 1.0)
        post = torch.empty(M, d, device="cuda", dtype=act)
        for _ in range(warmup):
            layer.forward(B, T, x, None, post, stream=stream)
        barrier()
        layer.check_device()

        clocks = Clocks(local)
        clocks.start()
        W.profile_read(reset=True)
        W.profile_enable(True)
        W.launch_count(reset=True)
        barrier()
        ev0.record(stream)
        for _ in range(steps):
            layer.forward(B, T, x, None, post, stream=stream)
        ev1.record(stream)
        barrier()
        launches = W.launch_count(reset=True)
        W.profile_enable(False)
        prof = W.profile_read(reset=True)
        clk = clocks.stop()
        layer.check_device()
        ms = max_over_ranks(ev0.elapsed_time(ev1) / steps)
        tokps = M / (ms / 1e3)

        pf, af = flops_prefill(B, T, d, H, NK, hd)
        per_step = {"gemm_qkv": 2.0 * M * d * (hc * hd + 2 * kd_l),
                    "attn_prefill": 4.0 * hd * hc * B * T * (T + 1) / 2,
                    "gemm_o": 2.0 * M * hc * hd * d}
        shares = {k: prof[k][0] for k in per_step}
        dom = max(shares, key=shares.get)
        tot, cnt = prof[dom]
        avg_ms = tot / max(cnt, 1)
        # with a communicator the batch runs in chunks: several launches per step
        flops_launch = per_step[dom] * steps / max(cnt, 1)
        achieved = flops_launch / (avg_ms / 1e3) / 1e12
        if prec == 0 and dom == "attn_prefill" and hd != 64:
            # FP32 attention on the CUDA cores (FFMA): 148 SMs x 128 lanes x 2 x 1.965 GHz
            peak, pkind, bound = 148 * 128 * 2 * 1.965e9 / 1e12, "nominal FP32 FFMA peak (CUDA cores)", "fp32-fma"
        elif prec == 0:
            peak = pk["bf16_sus"] * TF32X3_PER_BF16
            pkind = (f"3xTF32 ceiling: {pk['src']} sustained bf16 / 2 (kind::tf32 rate) / 3 (TF32 products "
                     f"per FP32 product) (derived from {pk['src']})")
            bound = "tensor"
        else:
            peak, pkind, bound = pk["bf16_sus"], f"{pk['src']} sustained bf16 (of {pk['src']})", "tensor"
        cfg5_heads = prec == 1 and hd == 128 and hc == 32 and kd_l == 4096
        traffic = TRAFFIC_PREFILL_PER_TOKEN * M * steps / max(cnt, 1) \
            if dom == "attn_prefill" and cfg5_heads else None
        roof = {"bound": bound, "kernel": dom, "achieved": achieved,
                "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "peak_kind": pkind,
                "traffic": traffic, "traffic_source": TRAFFIC_SOURCE if traffic else None,
                "flops_per_launch": flops_launch, "avg_launch_ms": avg_ms,
                "launches_per_step": cnt / steps,
                "kernel_ms_per_step": {k: prof[k][0] / steps for k in per_step},
                "collective_ms_per_step": prof["allreduce"][0] / steps if world > 1 else 0.0,
                "collective": OUTPUT_NAMES[args.output] if world > 1 else None,
                "step_tflops": (pf + af) / world / (ms / 1e3) / 1e12}
        if world > 1 and args.output != "allreduce":
            # the same step with the all-reduce output, for comparison (3 steps)
            layer.set_output_mode(0)
            layer.forward(B, T, x, None, post, stream=stream)
            barrier()
            ev0.record(stream)
            for _ in range(3):
                layer.forward(B, T, x, None, post, stream=stream)
            ev1.record(stream)
            barrier()
            roof["allreduce_output_ms_per_step"] = max_over_ranks(ev0.elapsed_time(ev1) / 3)
            layer.set_output_mode(OUTPUT_MODES[args.output])

        if primary and not args.no_e2e:
            # With N ranks each holds its B/N sequences in host memory and receives the
            # summed output of those rows (welvet_b200_mha_forward_rows: all-gather in,
            # reduce-scatter out over NVLink); one rank uses the host-buffer forward.
            rows_io = world > 1 and B % world == 0
            bl = B // world if rows_io else B
            xh = x[rank * bl * T:(rank + 1) * bl * T].cpu().pin_memory() if rows_io else x.cpu().pin_memory()
            ph = torch.empty(bl * T, d, dtype=act).pin_memory()

            def e2e_step():  # H2D x, forward, D2H post, synchronise
                if rows_io:
                    layer.forward_rows(bl, T, xh, ph)
                else:
                    layer.forward(B, T, xh, None, ph)
            e2e_step()  # warm the staging buffers
            barrier()
            t0 = time.perf_counter()
            ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ea.record(stream)
            for _ in range(steps):
                e2e_step()
            eb.record(stream)
            barrier()
            e_ms = max_over_ranks(max(ea.elapsed_time(eb), (time.perf_counter() - t0) * 1e3) / steps)
            e2e = {"value": M / (e_ms / 1e3), "unit": "tok/s", "ms_per_step": e_ms, "steps": steps,
                   "h2d_bytes_per_step": M * d * es, "d2h_bytes_per_step": M * d * es,
                   "bytes_scope": "whole job (each rank copies its B/N sequences)" if rows_io else "one GPU",
                   "api": ("welvet_b200_mha_forward_rows (host buffers, pinned, row-sharded)" if rows_io
                           else "welvet_b200_mha_forward (host buffers, pinned)")}
            del xh, ph

        # parity of the timed configuration: one more forward of the same inputs, then
        # rows [0, n_oracle) of sequence 0 against the FP64 oracle (causal: they depend
        # on those tokens only); with a communicator post is the sum over ranks
        pre = torch.empty(M, hc * hd, device="cuda", dtype=act) if world == 1 else None
        layer.forward(B, T, x, pre, post, stream=stream)
        barrier()
        got = {"post": post[:n_oracle].float().cpu().numpy()}
        if pre is not None:
            got["pre"] = pre[:n_oracle].float().cpu().numpy()
            del pre
        x_rows = x[:n_oracle].float().cpu().numpy()
        del post
        torch.cuda.empty_cache()
        if check_parity or (primary and rank == 0 and world == 1 and not args.no_cpu):
            import oracle_py as O
            oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, head_dim=hd, max_seq_len=n_oracle, per_sequence=1)
            t0 = time.perf_counter()
            rpre, rpost = O.mha_forward(oc, 1, n_oracle, *oracle_weights(O, host_ws, wf, prec, w.get("dt", 1)), x_rows)
            dt = time.perf_counter() - t0
            if check_parity:
                want = {"post": rpost}
                if "pre" in got:
                    want["pre"] = rpre
                parity = parity_record(got, want, 1e-4 if prec == 0 else 2e-2,
                                       f"sequence 0, tokens 0..{n_oracle - 1} of the timed B={B} T={T} forward")
            if primary and world == 1 and not args.no_cpu:
                # the same oracle run is the CPU baseline (FP64, all host threads)
                fl_s = sum(flops_prefill(1, n_oracle, d, H, NK, hd))
                cpu = {"value": fl_s / dt / ((pf + af) / M), "unit": "tok/s",
                       "cores": os.cpu_count(), "kind": "port",
                       "sample": f"FP64 oracle, 1 sequence x {n_oracle} tokens of the layer (d={d}, {H}x{hd}), "
                                 f"{dt:.1f} s; tok/s scaled by algorithmic FLOPs/token of the full workload"}
        barrier()
        print(f"[bench] {wname} prefill {ms:.3f} ms/step, {tokps:.0f} tok/s; parity {parity}", file=sys.stderr,
              flush=True)

    # --------------------------------------------------------------- decode
    decode = None
    n_dec = steps if decode_only else (args.decode_steps if primary else 0)
    if n_dec > 0 and w["kind"] != "prefill":
        n_prof = min(n_dec, 32)  # the instrumented pass (per-kernel times) after the timed one
        extra = n_dec + n_prof + warmup + 1 + (steps if decode_only and primary and not args.no_e2e else 0)
        kv = W.KvCache(layer, B, T + extra + 16)
        xd = torch.empty(B, d, device="cuda", dtype=act)
        W.fill_synthetic(xd, 1, 1, 1.0, offset=M * d)
        pd = torch.empty(B, d, device="cuda", dtype=act)
        if decode_only:
            # context: N(0,1)*0.5 keys/values (seed 2), as cached (after RoPE)
            kc = torch.empty(B, T, kd_l, device="cuda", dtype=act)
            vc = torch.empty(B, T, kd_l, device="cuda", dtype=act)
            n = kc.numel()
            W.fill_synthetic(kc, 2, 1, 0.5, offset=2 * rank * n)
            W.fill_synthetic(vc, 2, 1, 0.5, offset=(2 * rank + 1) * n)
            kv.fill(B, T, kc, vc, stream=stream)
            torch.cuda.synchronize()
            if world == 1:
                # parity: one decode step at context T against the oracle's decode for
                # a few sequences; then the cached lengths go back to T
                layer.decode(kv, B, xd, None, pd, stream=stream)
                torch.cuda.synchronize()
                if check_parity:
                    import oracle_py as O
                    sel = [0, B // 2, B - 1]
                    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, head_dim=hd, max_seq_len=T + 1, per_sequence=1)
                    _, rpost, _, _ = O.mha_decode(oc, [T] * len(sel), kc[sel].float().cpu().numpy(),
                                                  vc[sel].float().cpu().numpy(),
                                                  *oracle_weights(O, host_ws, wf, prec, w.get("dt", 1)),
                                                  xd[sel].float().cpu().numpy())
                    dparity = parity_record({"post": pd[sel].float().cpu().numpy()}, {"post": rpost},
                                            1e-4 if prec == 0 else 2e-2,
                                            f"sequences {sel}: one decode step over {T} cached tokens")
                kv.fill(B, T, None, None, stream=stream)
            del kc, vc
        else:
            post = torch.empty(M, d, device="cuda", dtype=act)
            layer.prefill(kv, B, T, x, None, post, stream=stream)
            del post
        for _ in range(warmup):  # first launches load the decode kernels' module
            layer.decode(kv, B, xd, None, pd, stream=stream)
        if decode_only:
            clocks = Clocks(local)
            clocks.start()
            W.launch_count(reset=True)
        barrier()
        ctx0 = T + warmup
        # The timed pass runs uninstrumented: per-kernel events between the step's
        # kernels would break the programmatic-dependent-launch overlap of its short
        # kernels. A second pass of n_prof steps records the per-kernel times.
        ev0.record(stream)
        for _ in range(n_dec):
            layer.decode(kv, B, xd, None, pd, stream=stream)
        ev1.record(stream)
        barrier()
        if decode_only:
            launches = W.launch_count(reset=True)
            clk = clocks.stop()
        dms = max_over_ranks(ev0.elapsed_time(ev1) / n_dec)
        W.profile_read(reset=True)
        W.profile_enable(True)
        for _ in range(n_prof):
            layer.decode(kv, B, xd, None, pd, stream=stream)
        barrier()
        W.profile_enable(False)
        dprof = W.profile_read(reset=True)
        layer.check_device()
        # algorithmic bytes of one decode-attention launch: the K and V rows of every
        # cached position (average context over the instrumented steps) + q and the output
        avg_ctx = ctx0 + n_dec + (n_prof + 1) / 2.0
        attn_bytes = B * avg_ctx * kd_l * es * 2 + 2 * B * hc * hd * es
        at, ac = dprof["attn_decode"]
        a_ms = at / max(ac, 1)
        gbs = attn_bytes / (a_ms / 1e3) / 1e9
        wbytes = (d * (hc * hd + 2 * kd_l) + hc * hd * d) * es
        step_bytes = attn_bytes + wbytes
        droof = {"bound": "hbm", "kernel": "attn_decode", "achieved": gbs, "peak": pk["hbm"],
                 "unit": "GB/s", "frac": gbs / pk["hbm"], "peak_kind": f"{pk['src']} HBM copy (of {pk['src']})",
                 "traffic": (TRAFFIC_DECODE_PER_ROW * B * avg_ctx if es == 2 and hd == 128 and kd_l == 4096
                             else None),
                 "bytes_per_launch": attn_bytes, "avg_launch_ms": a_ms,
                 "step_bytes": step_bytes, "step_gbs": step_bytes / (dms / 1e3) / 1e9,
                 "kernel_ms_per_step": {k: dprof[k][0] / n_prof for k in
                                        ("gemm_qkv_decode", "attn_decode", "gemm_o_decode", "allreduce")},
                 "kernel_times": f"CUDA events around each kernel over {n_prof} further steps (instrumented pass)"}
        decode = {"value": B / (dms / 1e3), "unit": "tok/s", "ms_per_step": dms, "steps": n_dec,
                  "context": f"{ctx0}..{ctx0 + n_dec}", "roofline": droof}
        if decode_only:
            ms, tokps, roof, prof, parity = dms, B / (dms / 1e3), droof, dprof, dparity
            if primary and not args.no_e2e:
                xh = xd.cpu().pin_memory()
                ph = torch.empty(B, d, dtype=act).pin_memory()
                barrier()
                t0 = time.perf_counter()
                for _ in range(steps):
                    layer.decode(kv, B, xh, None, ph)  # H2D x, decode step, D2H post, synchronise
                barrier()
                e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / steps)
                e2e = {"value": B / (e_ms / 1e3), "unit": "tok/s", "ms_per_step": e_ms, "steps": steps,
                       "h2d_bytes_per_step": B * d * es, "d2h_bytes_per_step": B * d * es,
                       "api": "welvet_b200_mha_decode (host buffers, pinned)"}
            if primary and rank == 0 and world == 1 and not args.no_cpu:
                B_s = 4
                dt = cpu_sample_decode(w, B_s)
                cpu = {"value": B_s / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                       "sample": f"FP64 oracle decode step, {B_s} sequences over {T} cached tokens "
                                 f"(d={d}, {H}x{hd}, {NK} KV heads), {dt:.2f} s"}
        kv.close()
    layer.close()
    del x
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"metric": METRIC_DECODE if decode_only else METRIC,
            "value": tokps, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if prec == 1 else "f32 (3xTF32 tensor cores)",
            "data": "synthetic (SplitMix64 counter stream: weights seed 0, x seed 1, KV seed 2)",
            "config": workload_config_of(wname, args, world),
            "roofline": roof, "parity": parity, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk, "decode": None if decode_only else decode,
            "profile_ms": {k: v[0] / steps for k, v in prof.items() if v[1]},
            "wall_s": time.perf_counter() - wall0}


def run_dequant(args, rank, world, local):
    """Standalone dequantisation of the extension weight formats to BF16 (the
    in-mainloop dequant's data path as a kernel of its own): FP8-E4M3 codes with one
    FP32 scale per row, and NF4 codes (two per byte) with one FP32 absmax per 64
    weights, over 2^30 weights each by default (inputs and outputs larger than L2).
    HBM-bound: bytes = codes + scales read + BF16 written. Parity: the FP32 decode
    of the first 2^20 weights equals the oracle's decode bit for bit."""
    import torch
    import welvet_b200 as W
    wall0 = time.perf_counter()
    n = workload_of("dequant", args)["n"]
    cols = 4096
    rows = n // cols
    pk = peaks()
    stream = torch.cuda.current_stream()
    w = torch.empty(n, device="cuda", dtype=torch.float32)
    W.fill_synthetic(w, 0, 1, 0.02, offset=rank * n)
    codes = torch.empty(n, device="cuda", dtype=torch.uint8)
    # (the encoders below are set-up, outside the timed region)
    scales = torch.empty(rows, device="cuda", dtype=torch.float32)
    W.fp8_rowscale_encode(w.view(rows, cols), codes, scales, stream=stream)
    packed = torch.empty(n // 2, device="cuda", dtype=torch.uint8)
    absmax = torch.empty(n // 64, device="cuda", dtype=torch.float32)
    W.nf4_block_encode(w, packed, absmax, stream=stream)
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    kinds = {
        "fp8_rowscale": (lambda: W.fp8_rowscale_decode(codes.view(rows, cols), scales, out, out_bf16=1,
                                                       stream=stream),
                         n + rows * 4 + 2 * n),
        "nf4_block64": (lambda: W.nf4_block_decode(packed, absmax, out, out_bf16=1, stream=stream),
                        n // 2 + (n // 64) * 4 + 2 * n),
    }
    res = {}
    for name, (fn, nbytes) in kinds.items():
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = Clocks(local)
        clocks.start()
        ea.record(stream)
        for _ in range(args.steps):
            fn()
        eb.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        ms = ea.elapsed_time(eb) / args.steps
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"value": gbs, "unit": "GB/s", "ms_per_launch": ms, "bytes_per_launch": nbytes,
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm"], "unit": "GB/s",
                                  "frac": gbs / pk["hbm"], "peak_kind": f"{pk['src']} HBM copy (of {pk['src']})",
                                  "traffic": None},
                     "clocks": clk}
    # parity (checker): FP32 decode of the first 2^20 weights vs the oracle, bit for bit
    parity = None
    if not args.no_parity and rank == 0:
        import oracle_py as O
        ns = 1 << 20
        wh = w[:ns].cpu().numpy()
        of = torch.empty(ns, device="cuda", dtype=torch.float32)
        W.fp8_rowscale_decode(codes[:ns].view(ns // cols, cols), scales[:ns // cols], of, out_bf16=0, stream=stream)
        got8 = of.cpu().numpy()
        W.nf4_block_decode(packed[:ns // 2], absmax[:ns // 64], of, out_bf16=0, stream=stream)
        torch.cuda.synchronize()
        got4 = of.cpu().numpy()
        want8 = O.fp8_rowscale(wh.reshape(-1, cols))[2].reshape(-1)
        want4 = O.nf4_block(wh, 64)[2].reshape(-1)
        mis8 = int((got8.view(np.uint32) != want8.view(np.uint32)).sum())
        mis4 = int((got4.view(np.uint32) != want4.view(np.uint32)).sum())
        parity = {"metric": "bit-exact FP32 decode vs the oracle's decode", "weights": ns,
                  "fp8_rowscale_mismatches": mis8, "nf4_block64_mismatches": mis4, "ok": mis8 == 0 and mis4 == 0}
    del w, codes, scales, packed, absmax, out
    torch.cuda.empty_cache()
    return {"metric": "FP8 row-scale / NF4 block-64 -> BF16 dequant GB/s", "weights": n,
            "kernels": res, "parity": parity, "wall_s": time.perf_counter() - wall0}


def bind_local_cpus(index: int):
    """Pins this rank's process to the CPUs NVML names as local to its GPU, so that its
    pinned host buffers (first touched here) sit on the GPU's own NUMA node: with 8
    ranks the host-buffer end-to-end copies are otherwise limited by cross-socket
    memory traffic. Nothing changes when NVML or the affinity call is unavailable."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(index)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:
        pass


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg5", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="override batch (small ncu cases)")
    ap.add_argument("--seq", type=int, default=0, help="override seq (decode workloads: context)")
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the cfg2/cfg3/cfg4/dequant sub-records of the default one-GPU line")
    ap.add_argument("--parity-tokens", type=int, default=1024)
    ap.add_argument("--output", default="exchange", choices=sorted(OUTPUT_MODES),
                    help="output collective of the device-timed prefill at N > 1")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        bind_local_cpus(local)
    torch.cuda.set_device(local)
    if workload(args)["kind"] == "codec":
        return run_codec(args, rank, world, local)
    if workload(args)["kind"] in BLOCK_KINDS:
        return run_block(args, rank, world, local)
    if workload(args)["kind"] == "nbp":
        return run_nbp(args, rank, world, local)
    if workload(args)["kind"] == "dequant":
        rec = run_dequant(args, rank, world, local)
        if rank == 0:
            k8 = rec["kernels"]["fp8_rowscale"]
            print(json.dumps(dict(rec, value=k8["value"], unit="GB/s", n_gpus=world, steps=args.steps,
                                  warmup=args.warmup, ms_per_step=k8["ms_per_launch"], higher_is_better=True,
                                  scaling="weak", vs_baseline=None, dtype="u8 codes -> bf16", data="synthetic",
                                  config=workload_config(args, world), roofline=k8["roofline"],
                                  gpu_launches=2 * args.steps, cpu_baseline=None, e2e=None)), flush=True)
        return
    if world > 1:
        # NVLS (in-switch reduction) is off unless the caller sets it: on this pool's
        # 8-GPU boxes the 256 KB decode all-reduce took 31 ms with NVLS and 0.05 ms
        # without, while the 0.5 GB prefill chunks lost only 4 %. NCCL reads the
        # variable once, at the first communicator, so it is set before any.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    import welvet_b200 as W
    w = workload(args)
    try:
        W.head_shard(w["H"], w["NK"], world, rank)
    except ValueError as e:
        raise SystemExit(str(e))
    t_all = time.perf_counter()
    line = run_mha(args, args.workload, rank, world, local, primary=True)
    if world == 1 and args.workload == "cfg5" and not args.no_configs and not (args.batch or args.seq):
        # the other configurations of the metric, each with its roofline and parity
        subs = {}
        for wname in SUB_WORKLOADS:
            subs[wname] = run_mha(args, wname, rank, world, local, primary=False)
        subs["dequant"] = run_dequant(args, rank, world, local)
        total = time.perf_counter() - t_all
        for r in subs.values():
            r["share_of_run"] = r["wall_s"] / total
        line["configs"] = subs
        line["wall_s_total"] = total
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
