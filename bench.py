"""Benchmark of the B200 EXL3 backend (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Workloads (synthetic, seeded):
* ``decode`` (default): greedy decode of the Llama-70B-shaped model (config 4:
  80 layers, hidden 8192, 64/8 heads x 128, SwiGLU 28672, vocab 128256, all
  linears EXL3 4 bpw 3INST on this backend; bf16 embeddings, lm_head and KV
  cache) at ``--batch`` sequences with a 2048-token context (KV cache filled with
  random values instead of running the random prompt) - one CUDA graph per step.
  Under torchrun the model is tensor-parallel over the N GPUs (NCCL all-reduce
  after o and down, vocab-sharded lm_head).  ``value`` is generated tokens/s.
* ``linears``: the EXL3 linear layers of one decode step of the
  Llama-70B-shaped model (config 4: 80 layers, hidden 8192, 64/8 heads x 128,
  SwiGLU 28672, all linears 4 bpw 3INST) at batch 1: q/k/v/o/gate/up/down = 560
  matmuls over 34.23 GB of trellis codes per step.  Inputs exceed L2, so no flush
  is needed.  Under torchrun the step is tensor-parallel over N GPUs:
  q/k/v/gate/up column-sharded, o/down row-sharded with an NCCL all-reduce.
* ``linear``: one ``--k`` x ``--n`` ``--bits``-bpw 3INST linear at ``--batch`` rows
  (default 4096x4096 4 bpw M=1: config 1), rotating weight copies (> 2x L2)
  between calls; value in GB/s of trellis + activations.
* ``mlp``: config 2, the dense SwiGLU MLP block (hidden 5120, intermediate 25600;
  fused gate+up one 3-bpw 3INST trellis of N = 2 x 25600, SiLU*mul, down 4 bpw MCG;
  seed 1) at ``--batch`` = M rows, one ``exl3b200_mlp`` call (SiLU*mul fused into the
  gate+up epilogue); small-M kernels up to 16 rows, the tensor-core GEMMs from 17.  Under torchrun: tensor parallel (gate/up column shards, down row
  shards, NCCL all-reduce).  Value in tokens (rows)/s; roofline in TFLOP/s.
* ``moe``: config 3, a routed MoE layer (288 experts top-8, hidden 2048, expert
  intermediate 1024, 3 bpw 3INST; one 4-bpw shared expert; router logits fp32
  N(0,1) -> softmax -> renormalised top-8; seed 2) at ``--batch`` = T tokens.  Under
  torchrun: expert parallel (288/N experts per rank, all-to-all dispatch and
  combine, ``exl3_b200.ep``); value in tokens/s.

``--impl reference`` times the reference's own CPU path for the same workload on
the host cores: its compiled ``dequant_trellis`` + ``at::mm``
(``csrc/bindings.cpp:15-147``, built into ``oracle/_ref`` by
``oracle/build_ref.py``) on a bounded sample (one 4096x4096 linear per step),
scaled to the workload's unit.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sglang-exl3_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode tok/s (70B-shape 4bpw); EXL3 GEMV HBM GB/s vs roofline"
# DRAM bytes per launch of the fused gate+up matmul kernel (8192 x 2 x 28672, 4 bpw, M = 1):
# ncu dram__bytes_read.sum + dram__bytes_write.sum, mean of three launches on a B200
GATEUP_TRAFFIC_BYTES = 237_192_363

# Llama-70B shape (config 4)
L70 = dict(layers=80, hidden=8192, heads=64, kv_heads=8, head_dim=128, inter=28672, vocab=128256, K=4, cb=0)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        sm = sorted(r[0] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v.lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": rows[0][1], "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, v: float) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def make_linear(gen, k_in, n_out, K, device):
    tr = torch.randint(-32768, 32768, (k_in // 16, n_out // 16, 16 * K), dtype=torch.int16, device=device,
                       generator=gen)
    su = ((torch.randint(0, 2, (k_in,), device=device, generator=gen) * 2 - 1).half()
          * (torch.rand(k_in, device=device, generator=gen) + 0.5).half())
    sv = ((torch.randint(0, 2, (n_out,), device=device, generator=gen) * 2 - 1).half()
          * (torch.rand(n_out, device=device, generator=gen) + 0.5).half())
    return tr, su, sv


def linear_bytes(k_in, n_out, K, m):
    return k_in * n_out * K // 8 + 2 * (m * k_in + m * n_out) + 2 * (k_in + n_out)


def build_linear_stack(world, rank, device, batch):
    """Per-rank shards of the 80-layer EXL3 linear stack (TP = world)."""
    from exl3_b200 import ops  # noqa: F401

    c = L70
    H, I, K = c["hidden"], c["inter"], c["K"]
    q_out = c["heads"] * c["head_dim"] // world
    kv_out = c["kv_heads"] * c["head_dim"] // world
    i_loc = I // world
    h_in_loc = H // world  # row-parallel o input
    gen = torch.Generator(device=device)
    gen.manual_seed(3 + 1000 * rank)
    layers = []
    for _ in range(c["layers"]):
        layers.append({
            "q": make_linear(gen, H, q_out, K, device),
            "k": make_linear(gen, H, kv_out, K, device),
            "v": make_linear(gen, H, kv_out, K, device),
            "o": make_linear(gen, h_in_loc, H, K, device),
            "gate": make_linear(gen, H, i_loc, K, device),
            "up": make_linear(gen, H, i_loc, K, device),
            "down": make_linear(gen, i_loc, H, K, device),
        })
    shapes = [(H, q_out), (H, kv_out), (H, kv_out), (h_in_loc, H), (H, i_loc), (H, i_loc), (i_loc, H)]
    step_bytes = c["layers"] * sum(linear_bytes(a, b, K, batch) for a, b in shapes)
    bufs = {
        "x": torch.randn(batch, H, dtype=torch.float16, device=device),
        "qkv": torch.empty(batch, q_out + 2 * kv_out, dtype=torch.float16, device=device),
        "attn": torch.randn(batch, h_in_loc, dtype=torch.float16, device=device),
        "o": torch.empty(batch, H, dtype=torch.float16, device=device),
        "gu": torch.empty(batch, 2 * i_loc, dtype=torch.float16, device=device),
        "act": torch.empty(batch, i_loc, dtype=torch.float16, device=device),
        "down": torch.empty(batch, H, dtype=torch.float16, device=device),
    }
    return layers, bufs, step_bytes, (q_out, kv_out, i_loc)


def linear_stack_step(layers, bufs, dims, world, K, cb, group=None):
    """One decode step's EXL3 matmuls (+ the TP all-reduces)."""
    from exl3_b200 import ops

    q_out, kv_out, i_loc = dims
    x = bufs["x"]
    for L in layers:
        ops.matmul(x, *L["q"], K, cb, out=bufs["qkv"][:, :q_out])
        ops.matmul(x, *L["k"], K, cb, out=bufs["qkv"][:, q_out:q_out + kv_out])
        ops.matmul(x, *L["v"], K, cb, out=bufs["qkv"][:, q_out + kv_out:])
        ops.matmul(bufs["attn"], *L["o"], K, cb, out=bufs["o"])
        if world > 1:
            torch.distributed.all_reduce(bufs["o"], group=group)
        ops.matmul(x, *L["gate"], K, cb, out=bufs["gu"][:, :i_loc])
        ops.matmul(x, *L["up"], K, cb, out=bufs["gu"][:, i_loc:])
        g, u = bufs["gu"][:, :i_loc], bufs["gu"][:, i_loc:]
        torch.mul(torch.nn.functional.silu(g), u, out=bufs["act"])
        ops.matmul(bufs["act"], *L["down"], K, cb, out=bufs["down"])
        if world > 1:
            torch.distributed.all_reduce(bufs["down"], group=group)


def time_graph(graph, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps


def isolated_kernel_time(tr_list, su_list, sv_list, K, cb, m, reps, device):
    """Average device time of one small-M matmul launch pair (input + gemv) over
    rotating weights, captured in a graph; returns ms per call."""
    from exl3_b200 import ops

    k_in = tr_list[0].size(0) * 16
    n_out = tr_list[0].size(1) * 16
    x = torch.randn(m, k_in, dtype=torch.float16, device=device)
    out = torch.empty(m, n_out, dtype=torch.float16, device=device)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for i in range(3):
            ops.matmul(x, tr_list[i % len(tr_list)], su_list[i % len(su_list)], sv_list[i % len(sv_list)], K, cb, out=out)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(len(tr_list)):
                ops.matmul(x, tr_list[i], su_list[i], sv_list[i], K, cb, out=out)
        g.replay()
        t = time_graph(g, reps, s)
    torch.cuda.current_stream(device).wait_stream(s)
    return t / len(tr_list)


# Reference CPU sample: the reference's dequant_trellis + at::mm on REF_SAMPLE_ROWS x 4096
# weights (4 bpw MCG: its binding cannot select 3INST) - about a second per step on the
# single-threaded reference dequant, so a default --steps/--warmup run ends in well under
# a minute.
REF_SAMPLE_ROWS, REF_SAMPLE_COLS = 256, 4096


def ref_module():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from build_ref import load_ref_module

    return load_ref_module()


def ref_sample_inputs():
    rng = np.random.default_rng(0)
    k, n = REF_SAMPLE_ROWS, REF_SAMPLE_COLS
    tr = torch.from_numpy(rng.integers(-32768, 32768, size=(k // 16, n // 16, 64)).astype(np.int16))
    su = torch.from_numpy((np.where(rng.integers(0, 2, k) == 0, -1.0, 1.0) * rng.uniform(0.5, 1.5, k)).astype(np.float16))
    sv = torch.from_numpy((np.where(rng.integers(0, 2, n) == 0, -1.0, 1.0) * rng.uniform(0.5, 1.5, n)).astype(np.float16))
    x = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float16))
    return x, tr, su, sv


def ref_cpu_times(ref, steps: int, warmup: int):
    """Seconds of each of ``steps`` timed calls of the reference's CPU ``exl3_gemv``
    (``csrc/bindings.cpp:134-147``: dequant_trellis + at::mm) on the sample, after
    ``warmup`` untimed ones."""
    x, tr, su, sv = ref_sample_inputs()
    for _ in range(warmup):
        ref.exl3_gemv(x, tr, su, sv, 4, True, 1)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ref.exl3_gemv(x, tr, su, sv, 4, True, 1)
        ts.append(time.perf_counter() - t0)
    return ts


def port_sample_shape(args):
    """(k, n, K, cb, rows, name) of the full projection the CPU port is timed on."""
    if args.workload == "linear":
        return args.k, args.n, args.bits, 0, args.batch, f"{args.k}x{args.n} {args.bits}-bpw 3INST linear"
    if args.workload == "mlp":
        return 25600, 5120, 4, 1, args.batch, "config-2 down projection 25600x5120 4-bpw MCG"
    if args.workload in ("moe", "verify"):
        if args.workload == "verify" or getattr(args, "moe", "c3") == "c5":
            return 4096, 1536, 3, 0, 5, "config-5 expert gate projection 4096x1536 3-bpw 3INST"
        return 2048, 1024, 3, 0, 1, "config-3 expert gate projection 2048x1024 3-bpw 3INST"
    return 8192, 8192, 4, 0, args.batch, "config-4 o projection 8192x8192 4-bpw 3INST"


def port_cpu_time(args):
    """CPU baseline (ii): the pure-torch table decode + torch.mm (oracle/torch_lut.py) on
    all host cores, one full projection of the workload; returns (seconds, weights, threads, name)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from torch_lut import TorchLutLinear

    k, n, K, cb, rows, name = port_sample_shape(args)
    g = torch.Generator()
    g.manual_seed(0)
    tr = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), dtype=torch.int16, generator=g)
    su = ((torch.randint(0, 2, (k,), generator=g) * 2 - 1) * (torch.rand(k, generator=g) + 0.5)).half()
    sv = ((torch.randint(0, 2, (n,), generator=g) * 2 - 1) * (torch.rand(n, generator=g) + 0.5)).half()
    x = torch.randn(rows, k, generator=g).half()
    lin = TorchLutLinear(tr, su, sv, K, cb)
    lin(x[:, :])  # warm the allocator and thread pool
    t0 = time.perf_counter()
    lin(x)
    return time.perf_counter() - t0, k * n, torch.get_num_threads(), name


def workload_scale(args):
    """(weights decoded per step, units per step, unit) of a workload, to scale the
    reference CPU sample (its cost is the per-weight dequant; at::mm is minor)."""
    c = L70
    if args.workload == "linear":
        return args.k * args.n, args.k * args.n * args.bits / 8 / 1e9, "GB/s"
    if args.workload == "mlp":
        H, I = 5120, 25600
        return H * 2 * I + I * H, args.batch, "rows/s"
    if args.workload == "verify":
        E, topk, H, I, R = 128, 8, 4096, 1536, 5 * args.batch
        touched = E * (1.0 - (1.0 - topk / E) ** R)
        return 48 * (touched * 3 * H * I + 2 * H * H + 2 * H * 512), R, "tok/s"
    if args.workload == "moe":
        if getattr(args, "moe", "c3") == "c5":
            E, topk, H, I, T = 128, 8, 4096, 1536, 5 * args.batch
            touched = E * (1.0 - (1.0 - topk / E) ** T)
            return touched * 3 * H * I, T, "tok/s"
        E, topk, H, I = 288, 8, 2048, 1024
        touched = E * (1.0 - (1.0 - topk / E) ** args.batch)  # expected distinct experts under uniform routing
        return touched * 3 * H * I + 3 * H * I, args.batch, "tok/s"
    model_weights = c["layers"] * (2 * c["hidden"] ** 2 + 2 * c["hidden"] * c["kv_heads"] * c["head_dim"]
                                   + 3 * c["hidden"] * c["inter"])
    return model_weights, args.batch, "tok/s"


def workload_metric(args):
    if args.workload == "mlp":
        return "C2 SwiGLU MLP block rows/s"
    if args.workload == "moe":
        return ("C5" if args.moe == "c5" else "C3") + " routed MoE layer tokens/s"
    if args.workload == "verify":
        return "C5 speculative verify tok/s (48-layer MoE, 5 tokens per sequence)"
    return METRIC


def decode_steps(args):
    return min(args.steps, 512 - args.warmup - 8)


def decode_config(args, world, fused=None):
    """The ``config`` of the decode workload (both arms print the same one)."""
    from exl3_b200.harness import LLAMA_70B, exl3_weight_bytes

    import dataclasses

    cfg = LLAMA_70B if args.layers == LLAMA_70B.layers else dataclasses.replace(LLAMA_70B, layers=args.layers)
    if fused is None:
        fused = args.batch <= 16
    fold = fused and getattr(args, "fold", True)
    return {"workload": "llama70b-shape decode (config 4), greedy, one CUDA graph per step"
                        + ((", fused decode layers, RMSNorm folded into the residual epilogues" if fold
                            else ", fused decode layers") if fused else ", unfused torch glue"),
            "model": "llama-70b-shape (random init)", "layers": cfg.layers, "global_batch": args.batch,
            "seq_len": args.ctx, "new_tokens_timed": decode_steps(args), "parallelism": f"tp{world}", "bpw": cfg.K,
            "codebook": "3INST", "kv_cache": "bf16, random contents for the 2048-token prompt",
            "l2": "no flush needed: 34.2 GB / tp of codes per step >> 126 MB L2",
            "exl3_bytes_per_step_per_rank": exl3_weight_bytes(cfg, world)}


def workload_config(args, world):
    if args.workload == "decode":
        return decode_config(args, world)
    return {"workload": args.workload, "batch": args.batch,
            **({"moe": args.moe} if args.workload == "moe" else {}),
            **({"k": args.k, "n": args.n, "bits": args.bits} if args.workload == "linear" else {}),
            "parallelism": f"tp{world}" if args.workload in ("mlp", "linears") else
            (f"ep{world}" if world > 1 else "single GPU")}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def run_reference(args, world, rank):
    """The reference's own CPU path on the host cores (rank 0 only): each step is one
    bounded sample, scaled to the workload's unit by the weights a step decodes."""
    if rank != 0:
        return
    ref = ref_module()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (python oracle/build_ref.py)"}))
        return
    ts = ref_cpu_times(ref, args.steps, args.warmup)
    sec = float(np.mean(ts))
    weights = REF_SAMPLE_ROWS * REF_SAMPLE_COLS
    step_weights, units, unit = workload_scale(args)
    step_s = sec * step_weights / weights
    value = units / step_s
    sample = (f"reference dequant_trellis + at::mm (csrc/bindings.cpp:134-147) on a {REF_SAMPLE_ROWS}x{REF_SAMPLE_COLS} "
              f"4-bpw MCG linear per step (its binding cannot select 3INST), scaled by the {step_weights:.4g} "
              "weights one workload step decodes")
    line = {
        "impl": "reference", "metric": workload_metric(args), "value": value, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "ms_per_step_extrapolated": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32 (reference CPU dequant + at::mm)", "data": "synthetic (seeded)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": torch.get_num_threads(), "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def run_ours(args, world, rank, local):
    device = torch.device("cuda", local)
    from exl3_b200 import ops  # noqa: F401

    hbm_peak, tc_peak, peak_kind = peaks()
    c = L70
    K, cb = c["K"], c["cb"]
    batch = args.batch
    group = None
    if args.workload == "linear":
        if world > 1:
            raise SystemExit("linear is a single-GPU workload (replicas only)")
        gen = torch.Generator(device=device)
        gen.manual_seed(0)
        k_in, n_out, bits = args.k, args.n, args.bits
        wbytes = k_in * n_out * bits // 8
        copies = max(1, min(40, (336 << 20) // wbytes + 1))  # rotate > 2x L2 worth of codes
        lins = [make_linear(gen, k_in, n_out, bits, device) for _ in range(copies)]
        trs, sus, svs = zip(*lins)
        for _ in range(args.warmup):
            isolated_kernel_time(trs, sus, svs, bits, 0, batch, 1, device)
        with ClockSampler(local) as clk:
            ms = isolated_kernel_time(trs, sus, svs, bits, 0, batch, args.steps, device)
        byts = linear_bytes(k_in, n_out, bits, batch)
        gbs = byts / (ms * 1e-3) / 1e9
        line = {"metric": METRIC, "value": gbs, "unit": "GB/s", "ms_per_step": ms,
                "config": {"workload": f"linear {k_in}x{n_out} {bits}bpw 3INST m={batch}"
                                       + (" (config 1)" if (k_in, n_out, bits) == (4096, 4096, 4) else ""),
                           "m": batch, "copies": copies,
                           "l2": f"{copies} rotating weight copies ({copies * wbytes >> 20} MB) between calls"},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                             "frac": gbs / hbm_peak, "traffic": None, "peak_kind": peak_kind,
                             "kernel": "exl3_gv_matmul_kernel (+ input and epilogue kernels)"},
                "gpu_launches": 3 * copies * args.steps,
                "clocks": clk.summary()}
        return finish(line, args, world)

    if args.workload == "decode":
        return run_decode(args, world, rank, local, device)
    if args.workload == "mlp":
        return run_mlp(args, world, rank, local, device)
    if args.workload == "moe":
        return run_moe(args, world, rank, local, device)
    if args.workload == "verify":
        return run_verify(args, world, rank, local, device)

    layers, bufs, step_bytes, dims = build_linear_stack(world, rank, device, batch)
    torch.cuda.synchronize()
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        linear_stack_step(layers, bufs, dims, world, K, cb, group)  # warm workspaces
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            linear_stack_step(layers, bufs, dims, world, K, cb, group)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        barrier(world)
        with ClockSampler(local) as clk:
            ms = time_graph(g, args.steps, s)
        ms = max_over_ranks(world, ms)
    torch.cuda.current_stream(device).wait_stream(s)
    tok_s = batch / (ms * 1e-3)

    # dominant kernel in isolation: the gate/up shape over the 80 layers' distinct copies
    q_out, kv_out, i_loc = dims
    trs = [L["gate"][0] for L in layers]
    sus = [L["gate"][1] for L in layers]
    svs = [L["gate"][2] for L in layers]
    ms_k = isolated_kernel_time(trs, sus, svs, K, cb, batch, 5, device)
    kb = linear_bytes(c["hidden"], i_loc, K, batch)
    k_gbs = kb / (ms_k * 1e-3) / 1e9

    # end to end through the public API: host x -> device, the 560 op calls, result -> host
    pinned_x = torch.randn(batch, c["hidden"], dtype=torch.float16).pin_memory()
    pinned_y = torch.empty(batch, c["hidden"], dtype=torch.float16).pin_memory()
    e2e_steps = max(1, min(args.steps, 3))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        bufs["x"].copy_(pinned_x, non_blocking=True)
        linear_stack_step(layers, bufs, dims, world, K, cb, group)
        pinned_y.copy_(bufs["down"], non_blocking=True)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(world, (time.perf_counter() - t0) / e2e_steps * 1e3)

    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "ms_per_step": ms,
        "config": {"workload": "llama70b-shape decode step, EXL3 linears only (attention, norms, lm_head not included)",
                   "model": "llama-70b-shape", "layers": c["layers"], "global_batch": batch, "seq_len": 1,
                   "parallelism": f"tp{world}", "bpw": K, "codebook": "3INST",
                   "l2": "no flush needed: 34.2 GB of codes per step >> 126 MB L2",
                   "step_weight_bytes_per_rank": step_bytes},
        "step_gbs_per_rank": step_bytes / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": k_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": k_gbs / hbm_peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": f"exl3_gemv_kernel 8192x{i_loc} 4bpw M={batch} (input stage included)"},
        "e2e": {"value": batch / (e2e_ms * 1e-3), "unit": "tok/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": pinned_x.numel() * 2, "d2h_bytes_per_step": pinned_y.numel() * 2,
                "path": "exl3_b200.ops.matmul eager calls (no graph), host pinned x in, y out"},
        "gpu_launches": 2 * 7 * c["layers"] * ((batch + 15) // 16),
        "clocks": clk.summary(),
    }
    del g
    return finish(line, args, world)


def run_mlp(args, world, rank, local, device):
    """Config 2: dense SwiGLU MLP block at M = --batch rows (TP over the ranks)."""
    from exl3_b200 import ops

    hbm_peak, tc_peak, peak_kind = peaks()
    H, I = 5120, 25600
    if I % (128 * world):
        raise SystemExit("intermediate size does not shard over this many ranks")
    i_loc = I // world
    m = args.batch
    gen = torch.Generator(device=device)
    gen.manual_seed(1 + 1000 * rank)
    gu = make_linear(gen, H, 2 * i_loc, 3, device)       # [gate_r | up_r], 3 bpw 3INST
    down = make_linear(gen, i_loc, H, 4, device)         # 4 bpw MCG
    x = torch.randn(m, H, dtype=torch.float16, device=device, generator=gen)
    out = torch.empty(m, H, dtype=torch.float16, device=device)
    group = torch.distributed.group.WORLD if world > 1 else None

    def step():
        # one library call: gate|up matmul with the SwiGLU and the down projection's input
        # transform in its epilogue, then the down matmul (no torch ops in between)
        ops.mlp(x, gu, down, 3, 0, 4, 1, out=out)
        if world > 1:
            torch.distributed.all_reduce(out, group=group)

    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        barrier(world)
        with ClockSampler(local) as clk:
            ms = time_graph(g, args.steps, s)
        ms = max_over_ranks(world, ms)
    torch.cuda.current_stream(device).wait_stream(s)
    flops = 2.0 * m * (H * 2 * I + I * H)
    wbytes = (H * 2 * I * 3 + I * H * 4) // 8
    tflops = flops / (ms * 1e-3) / 1e12
    gbs = wbytes / world / (ms * 1e-3) / 1e9
    tensor_bound = m >= 64
    roof = ({"bound": "tensor", "achieved": tflops / world, "peak": tc_peak, "unit": "TFLOP/s",
             "frac": tflops / world / tc_peak} if tensor_bound else
            {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak})
    roof.update({"traffic": None, "peak_kind": peak_kind, "per": "rank",
                 "kernel": "whole MLP block per rank (exl3b200_mlp: gate+up with SiLU*mul in its epilogue, down)"})

    # end to end: host x in, host y out, eager calls
    px = torch.randn(m, H, dtype=torch.float16).pin_memory()
    py = torch.empty(m, H, dtype=torch.float16).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    n_e2e = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        x.copy_(px, non_blocking=True)
        step()
        py.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(world, (time.perf_counter() - t0) / n_e2e * 1e3)
    del g
    line = {"metric": "C2 SwiGLU MLP block rows/s", "value": m / (ms * 1e-3), "unit": "rows/s", "ms_per_step": ms,
            "config": {"workload": f"config 2 SwiGLU MLP block, M={m}", "hidden": H, "intermediate": I,
                       "gate_up": "3 bpw 3INST fused N=2x25600", "down": "4 bpw MCG", "parallelism": f"tp{world}",
                       "l2": f"{wbytes >> 20} MB of codes per step (> 126 MB L2), no flush",
                       "path": "tensor-core GEMMs" if m >= 17 else "small-M kernels",
                       "swiglu": "fused into the gate+up epilogue"},
            "tflops": tflops, "exl3_gbs_per_rank": gbs,
            "roofline": roof,
            "e2e": {"value": m / (e2e_ms * 1e-3), "unit": "rows/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": px.numel() * 2, "d2h_bytes_per_step": py.numel() * 2},
            # input stage, gate|up matmul (+ its split-tile finish), down matmul (+ finish) on the
            # tensor cores; input, matmul, epilogue, matmul, epilogue on the small-M path
            "gpu_launches": args.steps * 5,
            "clocks": clk.summary()}
    return finish(line, args, world)


def run_moe(args, world, rank, local, device):
    """Config 3: routed MoE layer (288 experts top-8) + shared expert at T = --batch tokens."""
    from exl3_b200 import moe as M
    from exl3_b200 import ops
    from exl3_b200.ep import PeerExpertParallelMoE, exl3_local_experts

    hbm_peak, tc_peak, peak_kind = peaks()
    c5 = args.moe == "c5"
    E, topk, H, I, K = (128, 8, 4096, 1536, 3) if c5 else (288, 8, 2048, 1024, 3)
    if E % world:
        raise SystemExit(f"{E} experts do not split over this many ranks")
    el = E // world
    T = 5 * args.batch if c5 else args.batch  # config 5 verifies 4 draft tokens + 1 per sequence
    seed = 4 if c5 else 2
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 1000 * rank)
    w13 = torch.randint(-32768, 32768, (el, 2, H // 16, I // 16, 16 * K), dtype=torch.int16, device=device, generator=gen)
    w2 = torch.randint(-32768, 32768, (el, I // 16, H // 16, 16 * K), dtype=torch.int16, device=device, generator=gen)

    def signs(*shape):
        return ((torch.randint(0, 2, shape, device=device, generator=gen) * 2 - 1).half()
                * (torch.rand(shape, device=device, generator=gen) + 0.5).half())

    w13_suh, w13_svh, w2_suh, w2_svh = signs(el, 2, H), signs(el, 2, I), signs(el, I), signs(el, H)

    def ptrs(t):
        return torch.tensor([int(t[e].data_ptr()) for e in range(el)], dtype=torch.int64, device=device)

    tables = {"gate_trellis": ptrs(w13[:, 0]), "gate_suh": ptrs(w13_suh[:, 0]), "gate_svh": ptrs(w13_svh[:, 0]),
              "up_trellis": ptrs(w13[:, 1]), "up_suh": ptrs(w13_suh[:, 1]), "up_svh": ptrs(w13_svh[:, 1]),
              "down_trellis": ptrs(w2), "down_suh": ptrs(w2_suh), "down_svh": ptrs(w2_svh)}
    shared_gen = torch.Generator(device=device)
    shared_gen.manual_seed(2)  # the shared expert is replicated
    sh_gate_up = make_linear(shared_gen, H, 2 * I, 4, device)  # merged gate|up, as the dense MLP's
    sh_down = make_linear(shared_gen, I, H, 4, device)
    rgen = torch.Generator(device=device)
    rgen.manual_seed(seed + 1000 * rank)  # every rank holds its own T tokens
    x = torch.randn(T, H, dtype=torch.float16, device=device, generator=rgen)
    logits = torch.randn(T, E, dtype=torch.float32, device=device, generator=rgen)
    local_fn = exl3_local_experts(tables, K, K, K, 0, I)
    # expert parallelism: dispatch and combine over NVLink peer memory by the library
    ep = PeerExpertParallelMoE(E, T, topk, H, group=torch.distributed.group.WORLD) if world > 1 else None
    sh_out = torch.empty(T, H, dtype=torch.float16, device=device)

    def step():
        p = torch.softmax(logits, dim=-1)
        w, ids = torch.topk(p, topk, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        if ep is None:
            out = local_fn(x, ids.to(torch.int32), w)
        else:
            out = ep(x, ids, w, tables, K, K, K, 0, I)
        if not c5:  # config 3's shared expert (config 5 has none): the fused SwiGLU MLP block
            ops.mlp(x, sh_gate_up, sh_down, 4, 0, 4, 0, out=sh_out)
            out += sh_out.float()
        return out

    # the layer step as one CUDA graph (as a serving step runs it), replayed
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out_g = step()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        with ClockSampler(local) as clk:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(args.steps):
                graph.replay()
            e1.record(s)
            e1.synchronize()
    torch.cuda.current_stream(device).wait_stream(s)
    ms = max_over_ranks(world, e0.elapsed_time(e1) / args.steps)
    # distinct experts touched by the job's tokens (every rank's) and their code bytes:
    # the HBM roofline of the step; a rank streams its own share of them
    with torch.no_grad():
        ids_all = torch.topk(torch.softmax(logits, -1), topk, dim=-1)[1].to(torch.int32)
        if world > 1:
            parts = [torch.empty_like(ids_all) for _ in range(world)]
            torch.distributed.all_gather(parts, ids_all)
            ids_all = torch.cat(parts)
        touched = int(torch.unique(ids_all).numel())
    expert_bytes = (2 * H * I + I * H) * K // 8
    step_bytes = touched * expert_bytes / world + (0 if c5 else 3 * H * I * 4 // 8)
    gbs = step_bytes / (ms * 1e-3) / 1e9

    px = torch.randn(T, H, dtype=torch.float16).pin_memory()
    py = torch.empty(T, H, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    n_e2e = max(1, min(args.steps, 5))
    for i in range(n_e2e + 1):  # the first (untimed) call warms the eager path's workspaces
        if i == 1:
            torch.cuda.synchronize()
            barrier(world)
            t0 = time.perf_counter()
        x.copy_(px, non_blocking=True)
        y = step()
        py.copy_(y, non_blocking=True)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(world, (time.perf_counter() - t0) / n_e2e * 1e3)
    name = (f"config 5 MoE layer, speculative verify of {args.batch} sequences x 5 tokens (T={T})" if c5
            else f"config 3 MoE layer, T={T}")
    del graph
    if ep is not None:
        ep.close()
    # every rank holds its own T tokens: the job processes world x T tokens per step
    line = {"metric": ("C5" if c5 else "C3") + " routed MoE layer tokens/s", "value": world * T / (ms * 1e-3),
            "unit": "tok/s", "ms_per_step": ms, "scaling": "weak",
            "config": {"workload": name, "experts": E, "topk": topk, "hidden": H,
                       "intermediate": I, "bpw": K, "codebook": "3INST", "shared_expert": "none" if c5 else "4 bpw",
                       "parallelism": f"ep{world}" if world > 1 else "single GPU",
                       "tokens_per_rank": T, "experts_touched": touched, "moe_path": M.moe_path(T, topk, el),
                       "ep_exchange": ("NVLink peer stores: each token row once to every rank owning one of its "
                                       "experts, weighted results back (exl3b200_ep_moe)") if world > 1 else "none",
                       "l2": (f"expert codes {expert_bytes / 1e6:.2f} MB each, {touched * expert_bytes / 1e6:.0f} MB "
                              "touched per step (> 126 MB L2), no flush; one CUDA graph per step, time includes "
                              "routing (softmax/top-k)" + ("" if c5 else " and the shared expert (fused MLP block)"))},
            "exl3_gbs_per_rank": gbs,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole MoE layer per rank (touched experts' codes / step time)"},
            "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": "tok/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": px.numel() * 2, "d2h_bytes_per_step": py.numel() * 4},
            # routed layer: 6 launches (small-M pipeline) or 4 (tensor-core pipeline, SwiGLU in
            # the gate|up epilogue); under EP + plan, dispatch, receive, return, combine;
            # config 3's shared expert: the fused MLP block, 5
            "gpu_launches": args.steps * ((4 if M.moe_path(T, topk, el) == "tc" else 6) + (5 if world > 1 else 0)
                                          + (0 if c5 else 5)),
            "clocks": clk.summary()}
    return finish(line, args, world)


def run_verify(args, world, rank, local, device):
    """Config 5: speculative verify of --batch sequences x 5 tokens through the whole
    48-layer MoE model (experts split over the ranks under torchrun)."""
    import dataclasses

    from exl3_b200.verify import CONFIG5, VerifyModel

    hbm_peak, tc_peak, peak_kind = peaks()
    cfg = CONFIG5 if args.layers == 80 else dataclasses.replace(CONFIG5, layers=args.layers)
    ctx = args.ctx
    group = torch.distributed.group.WORLD if world > 1 else None
    model = VerifyModel(cfg, args.batch, ctx + cfg.rows_per_seq, device, world, rank, group)
    model.fill_random_kv(ctx)
    model.tokens.random_(0, cfg.vocab, generator=torch.Generator(device=device).manual_seed(9))
    # one eager step records how many experts the routing touches per layer (HBM roofline)
    model.record = []
    with torch.cuda.stream(model.stream):
        finite = bool(torch.isfinite(model.step()).all())
    torch.cuda.synchronize()
    touched = model.record
    model.record = None
    model.pos.fill_(ctx)
    model.capture()
    for _ in range(args.warmup):
        model.replay()
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(model.stream)
        model.replay(args.steps)
        e1.record(model.stream)
        e1.synchronize()
    ms = max_over_ranks(world, e0.elapsed_time(e1) / args.steps)
    R = model.rows
    tok_s = R / (ms * 1e-3)
    H, hd = cfg.hidden, cfg.head_dim
    per_expert = 3 * H * cfg.inter * cfg.K_expert // 8
    attn_codes = cfg.layers * (2 * H * cfg.heads * hd + 2 * H * cfg.kv_heads * hd) * cfg.K_attn // 8
    kv = cfg.layers * args.batch * (ctx + cfg.rows_per_seq) * cfg.kv_heads * hd * 2 * 2
    lm = cfg.vocab * H * 2
    step_bytes = sum(touched) * per_expert / world + attn_codes + kv + lm
    gbs = step_bytes / (ms * 1e-3) / 1e9

    # end to end: the rows' tokens in from pinned host memory, the argmax of every row out
    ptok = torch.randint(0, cfg.vocab, (args.batch, cfg.rows_per_seq), dtype=torch.long).pin_memory()
    pout = torch.empty(R, dtype=torch.long).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    n_e2e = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        with torch.cuda.stream(model.stream):
            model.tokens.copy_(ptok, non_blocking=True)
            model.graph.replay()
            pout.copy_(model.logits.argmax(-1), non_blocking=True)
        model.stream.synchronize()
    e2e_ms = max_over_ranks(world, (time.perf_counter() - t0) / n_e2e * 1e3)
    model.close()
    line = {
        "metric": "C5 speculative verify tok/s (48-layer MoE, 5 tokens per sequence)", "value": tok_s,
        "unit": "tok/s", "ms_per_step": ms,
        "config": {"workload": f"config 5 verify: {args.batch} sequences x {cfg.rows_per_seq} tokens, "
                               f"context {ctx}, one CUDA graph per step",
                   "layers": cfg.layers, "experts": cfg.experts, "topk": cfg.topk, "hidden": H,
                   "intermediate": cfg.inter, "expert_bpw": cfg.K_expert, "attention_bpw": cfg.K_attn,
                   "codebook": "3INST", "global_batch": args.batch, "seq_len": ctx,
                   "parallelism": f"ep{world}" if world > 1 else "single GPU",
                   "experts_touched_per_layer": round(sum(touched) / len(touched), 1), "logits_finite": finite,
                   "moe_path": _moe_path_name(world * R, cfg.topk, cfg.experts // world),
                   "kv_cache": "bf16, random contents for the context",
                   "attention": ("fused decode sub-layer, 5 rows per sequence (exl3b200_decode_attention_rows)"
                                 if model.fused else "EXL3 projections + torch RoPE / SDPA glue"),
                   "l2": "no flush needed: expert codes per step >> 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": "whole verify step per rank (touched expert codes + attention codes + KV + lm_head)"},
        "e2e": {"value": R / (e2e_ms * 1e-3), "unit": "tok/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": ptok.numel() * 8, "d2h_bytes_per_step": pout.numel() * 8,
                "path": "VerifyModel graph replay: draft tokens H2D from pinned memory, argmax of every row D2H"},
        # per layer: q/k/v and o EXL3 launches (3 each) + the routed MoE pipeline (5 or 6)
        "gpu_launches": args.steps * cfg.layers * (6 + (5 if _moe_path_name(world * R, cfg.topk,
                                                                            cfg.experts // world) == "tc" else 6)),
        "clocks": clk.summary(),
    }
    return finish(line, args, world)


def _moe_path_name(rows, topk, experts):
    from exl3_b200 import moe as M
    return M.moe_path(rows, topk, experts)


def run_decode(args, world, rank, local, device):
    from exl3_b200 import ops
    from exl3_b200.harness import LLAMA_70B, DecodeModel, exl3_weight_bytes

    import dataclasses

    hbm_peak, tc_peak, peak_kind = peaks()
    cfg = LLAMA_70B if args.layers == LLAMA_70B.layers else dataclasses.replace(LLAMA_70B, layers=args.layers)
    batch = args.batch
    new_tokens = 512
    group = torch.distributed.group.WORLD if world > 1 else None
    model = DecodeModel(cfg, batch, args.ctx + new_tokens, device, world, rank, group, fold=args.fold)
    model.fill_random_kv(args.ctx)
    model.capture()
    steps = decode_steps(args)
    model.pos.fill_(args.ctx)
    model.decode(args.warmup)
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        e0.record(model.stream)
        model.decode(steps)
        e1.record(model.stream)
        e1.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = max_over_ranks(world, e0.elapsed_time(e1) / steps)
    tok_s = batch / (ms * 1e-3)
    step_bytes = exl3_weight_bytes(cfg, world)

    # end to end through the public API: each step's tokens in from pinned host memory,
    # its output tokens back to the host
    e2e_n = 32
    model.pos.fill_(args.ctx)
    model.generate(torch.zeros(batch, dtype=torch.long), 2)  # allocates the pinned buffers
    model.pos.fill_(args.ctx)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    model.generate(torch.zeros(batch, dtype=torch.long), e2e_n)
    e2e_ms = max_over_ranks(world, (time.perf_counter() - t0) / e2e_n * 1e3)

    # dominant kernel in isolation: the fused gate/up launch of each layer
    gu = [L["gu"] for L in model.layers]
    x = torch.randn(batch, cfg.hidden, dtype=torch.float16, device=device)
    outs = [torch.empty(batch, model.i_loc, dtype=torch.float16, device=device) for _ in range(2)]
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    torch.cuda.nvtx.range_push("roofline")  # ncu --nvtx-include "roofline/" selects these launches
    with torch.cuda.stream(s):
        for pair in gu[:3]:
            ops.matmul_multi(x, pair, cfg.K, cfg.cb, outs=outs)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for pair in gu:
                ops.matmul_multi(x, pair, cfg.K, cfg.cb, outs=outs)
        g.replay()
        kt = time_graph(g, 3, s) / len(gu)
    torch.cuda.nvtx.range_pop()
    torch.cuda.current_stream(device).wait_stream(s)
    peer_exchange = model.peers is not None
    rope_kernel = 0 if batch * model.hkv <= 8 else 1  # a separate RoPE/KV epilogue per layer
    kbytes = 2 * (cfg.hidden * model.i_loc * cfg.K // 8) + 2 * batch * (cfg.hidden + 2 * model.i_loc)
    k_gbs = kbytes / (kt * 1e-3) / 1e9
    del g
    model.close()

    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "ms_per_step": ms,
        "config": decode_config(args, world, model.fused),
        "exl3_gbs_per_rank": step_bytes / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": k_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": k_gbs / hbm_peak,
                     "traffic": GATEUP_TRAFFIC_BYTES * model.i_loc / 28672, "peak_kind": peak_kind,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the matmul kernel, "
                                       "mean of 3 launches at 8192x2x28672 M=1, scaled by the shard's columns",
                     "kernel": f"fused gate+up EXL3 matmul 8192x2x{model.i_loc} 4bpw M={batch} (3 kernels)"},
        "e2e": {"value": batch / (e2e_ms * 1e-3), "unit": "tok/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 8 * batch, "d2h_bytes_per_step": 8 * batch + 4,
                "path": "DecodeModel.generate: per step, tokens H2D from pinned host memory, graph replay, tokens "
                        "and the device status word D2H, stream sync"},
        # fused: per layer 5 (attention, whose kernel also finishes q/k/v when all its clusters are
        # resident at once - batch 1 - else + the RoPE/KV epilogue) + 5 (MLP) launches (the NVLink
        # exchange runs inside the o/down epilogues); + 2 residual-add kernels per layer when TP goes
        # through NCCL instead; with the norm fold 8 per layer and the first layer's input stage
        "gpu_launches": steps * (((8 + rope_kernel) * cfg.layers + 1) if model.fold else
                                 cfg.layers * ((10 + rope_kernel + (2 if world > 1 and not peer_exchange else 0))
                                               if model.fused else 12)),
        "clocks": clk.summary(),
    }
    return finish(line, args, world)


def finish(line, args, world):
    base = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 x 4-bit trellis -> fp32 acc",
            "data": "synthetic (seeded random trellis codes, random-init)"}
    base.update(line)
    if int(os.environ.get("RANK", "0")) == 0:
        if args.cpu_baseline and world == 1:
            step_weights, units, u = workload_scale(args)
            sec, weights, threads, name = port_cpu_time(args)
            base["cpu_baseline"] = {
                "value": units / (sec * step_weights / weights), "unit": u, "cores": threads, "kind": "port",
                "sample": f"pure-torch 3INST/MCG table decode + torch.mm (oracle/torch_lut.py) on all host threads, "
                          f"one full {name} ({sec:.3f} s), scaled by the {step_weights:.4g} weights of a step"}
            ref = ref_module()
            if ref is not None:
                rsec = float(np.median(ref_cpu_times(ref, 2, 1)))
                base["cpu_baseline_reference"] = {
                    "value": units / (rsec * step_weights / (REF_SAMPLE_ROWS * REF_SAMPLE_COLS)), "unit": u,
                    "cores": torch.get_num_threads(), "kind": "reference",
                    "sample": f"reference dequant_trellis + at::mm on a {REF_SAMPLE_ROWS}x{REF_SAMPLE_COLS} 4-bpw MCG "
                              f"linear ({rsec:.3f} s; single-threaded dequant), scaled the same way"}
        if not getattr(args, "quiet", False):
            print(json.dumps(base))
    return base


# The other benchmark configurations, measured after the default decode line in the same
# process and reported in its "workloads" object (one summary each), so that one run
# records every config: (name, argument overrides, runs under torchrun too - the MoE
# layers then run expert-parallel over the ranks, every rank with its own tokens).
EXTRA_WORKLOADS = [
    ("config 1 linear 4096x4096 4bpw M=1", dict(workload="linear", k=4096, n=4096, bits=4, batch=1), False),
    ("config 2 MLP block M=1", dict(workload="mlp", batch=1), False),
    ("config 2 MLP block M=2048", dict(workload="mlp", batch=2048), False),
    ("config 3 MoE layer T=64", dict(workload="moe", moe="c3", batch=64), False),
    ("config 3 MoE layer T=512", dict(workload="moe", moe="c3", batch=512), True),
    ("config 5 MoE layer, verify batch 64", dict(workload="moe", moe="c5", batch=64), True),
    # config 4 at its other batch sizes (one GPU: the default line carries the TP scaling)
    ("config 4 decode batch 8", dict(workload="decode", batch=8), False),
    ("config 4 decode batch 64", dict(workload="decode", batch=64), False),
]


def run_extras(args, world, rank, local):
    """Each extra workload with 10 timed steps; a summary of its line, or the error."""
    import copy

    out = {}
    for name, over, multi in EXTRA_WORKLOADS:
        if world > 1 and not multi:
            continue
        sub = copy.copy(args)
        for k, v in over.items():
            setattr(sub, k, v)
        sub.steps, sub.warmup, sub.cpu_baseline, sub.quiet = min(args.steps, 10), 3, False, True
        try:
            ln = run_ours(sub, world, rank, local)
            roof = ln.get("roofline", {})
            out[name] = {"value": ln["value"], "unit": ln["unit"], "ms_per_step": ln["ms_per_step"],
                         "steps": sub.steps, "workload": ln["config"].get("workload"),
                         "path": ln["config"].get("path") or ln["config"].get("moe_path"),
                         "parallelism": ln["config"].get("parallelism"),
                         "roofline": {k: roof.get(k) for k in ("bound", "achieved", "unit", "peak", "frac")},
                         "e2e": (ln.get("e2e") or {}).get("value"),
                         "gpu_launches": ln.get("gpu_launches"), "clocks": ln.get("clocks")}
        except Exception as e:  # reported, not fatal: the default line stands on its own
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "linears", "linear", "mlp", "moe", "verify"])
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--ctx", type=int, default=None, help="context length (decode: 2048, verify: 8192)")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=80, help="decode: decoder layers (80 = config 4; fewer for profiling)")
    ap.add_argument("--moe", default="c3", choices=["c3", "c5"],
                    help="moe workload: c3 = 288 experts, hidden 2048 (+ shared expert); c5 = the MoE layer of "
                         "config 5's speculative verify: 128 experts, hidden 4096, 5 rows per sequence")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-fold", dest="fold", action="store_false",
                    help="decode: keep the RMSNorm input stages as kernels (two sub-layer calls per layer)")
    ap.add_argument("--no-extra", dest="extra", action="store_false",
                    help="default decode run: skip the other configs' summaries")
    args = ap.parse_args()
    if args.ctx is None:
        args.ctx = 8192 if args.workload == "verify" else 2048
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "decode" and args.extra:
            args.quiet = True
            line = run_ours(args, world, rank, local)
            line["workloads"] = run_extras(args, world, rank, local)
            if rank == 0:
                print(json.dumps(line))
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
