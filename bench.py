"""Benchmark: talker decode seq-steps/s, B=64 ragged, on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = the whole talker decode step of 64 ragged sequences (contexts
U[64, 2048], seeded), 28-layer random-init bf16 decoder (hidden 2048, 16/8
heads, head_dim 128, FFN 6144, RoPE theta 1e6, codec vocab 3072), bf16 KV in
16-token pages scattered over a 512k-token pool, GPU planner, fused sampler,
commit - replayed from one CUDA graph.  Under torchrun each rank owns its own
64 requests and page pool (request-sharded data parallelism, no collective on
the data path); timing is the max over ranks (gloo for the scalar reduce).

Reported on the JSON line besides the throughput:
  e2e          the same metric through TalkerDecodeStep.step() with host
               buffers: pinned H2D of the step inputs, replay, D2H of tokens;
  roofline     the decode-attention launch (one decode kernel, fused fix-up) timed
               alone with CUDA events over the same metadata: algorithmic
               KV + q + out bytes / duration vs the measured HBM copy peak;
  sampler_roofline  the fused sampler on 256 stacked talker steps (16384 x
               3072 rows) timed in the same process: algorithmic logits +
               seen-mask bytes / duration vs the measured HBM copy peak;
  cpu_baseline whole steps of the CPU port (oracle/talker_step.py: every
               layer, every row) for about --cpu-seconds (rank 0, N = 1);
  clocks       nvidia-smi samples taken during the timed region;
  config4_mixed, config3_code_predictor
               at N = 1, the mixed continuous batch and
               the code-predictor frame (config 3) measured in the same run
               (the --workload mixed / cp lines, summarised).
``--impl reference`` times whole steps of the CPU port alone (the reference
arm), on rank 0 only at every N.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "talker decode seq-steps/s (B=64 ragged) at 1/2/4/8 B200; attn HBM GB/s vs peak"
UNIT = "seq-steps/s"
BATCH = 64
CTX_LO, CTX_HI = 64, 2048
POOL_TOKENS = 512 * 1024


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("decode", "mixed", "cp", "sampler", "serve", "gate_up"), default="decode",
                   help="decode = BASELINE config 2 (the headline); mixed = config 4 (prefill chunks + decode rows); "
                        "cp = config 3; serve = config 5 (box serving simulation); sampler = the sampler roofline; "
                        "gate_up = the FP8 gate/up GEMM against cuBLAS bf16")
    p.add_argument("--serve-seconds", type=float, default=10.0, help="config 5: arrival window per GPU (s)")
    p.add_argument("--serve-rps", type=float, default=20.0, help="config 5: Poisson arrival rate per GPU")
    p.add_argument("--layers", type=int, default=28, help="decoder layers (28 = BASELINE config 2)")
    p.add_argument("--gate-up", choices=("fp8", "bf16"), default=None,
                   help="talker gate/up: fp8 = the reference's production path (128x128 e4m3 weight blocks, "
                        "per-token 1x128 activation blocks); bf16 = unquantised.  Default: fp8 for the decode "
                        "step, bf16 for the mixed batch (prefill-scale M)")
    p.add_argument("--pool-tokens", type=int, default=POOL_TOKENS)
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-other-configs", action="store_true",
                   help="headline run only: skip the config-3 / config-4 measurements carried on its line")
    p.add_argument("--grow", action="store_true",
                   help="publish each step (contexts grow by one token per step) instead of holding them fixed")
    return p.parse_args()


def peaks() -> tuple[float, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def contexts_for(rank: int) -> list[int]:
    g = torch.Generator().manual_seed(1000 + rank)
    return torch.randint(CTX_LO, CTX_HI + 1, (BATCH,), generator=g).tolist()


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device) -> None:
        self.proc = None
        self.target = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.target = str(device.index or 0)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in getattr(self, "lines", []):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7], strict=True):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _cpu_port(layers: int):
    from oracle.talker_step import CpuTalkerStep

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step = CpuTalkerStep(contexts=contexts_for(0), num_layers=layers)
    step.time_step(layers=2)  # warm-up: first-touch of the weights, caches and the allocator
    return step, threads


def cpu_baseline(budget_s: float, layers: int) -> dict:
    """Whole steps of the CPU port (every row, every layer) until ``budget_s`` is spent (at least one)."""

    step, threads = _cpu_port(layers)
    runs = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or not runs:
        runs.append(step.time_step()["step_s"])
    per_step = statistics.mean(runs)
    return {
        "value": BATCH / per_step,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": (f"{len(runs)} whole steps of the CPU port (oracle/talker_step.py): host planner, all {layers} "
                   f"decoder layers for all {BATCH} rows (fp32 math, bf16-rounded activations), head and the "
                   f"reference CPU sampler; {per_step:.2f} s per step"),
    }


# Wall-clock budget of the reference arm's timed steps.  Each step is a whole CPU step (seconds); a request for
# more steps than fit is cut to the number that fits and the line says so.
REFERENCE_BUDGET_S = 180.0


def run_reference(args, world, rank):
    """The reference arm: the CPU port of the whole step on the host cores, rank 0 only."""

    if rank != 0:
        return
    step, threads = _cpu_port(args.layers)
    for _ in range(args.warmup):
        step.time_step(layers=2)  # untimed warm-up steps run 2 of the layers to bound the run
    first = step.time_step()["step_s"]
    steps = max(1, min(args.steps, int(REFERENCE_BUDGET_S / first)))
    times = [first] + [step.time_step()["step_s"] for _ in range(steps - 1)]
    per_step = statistics.mean(times)
    value = BATCH / per_step
    sample = (f"each step: the whole CPU step - host planner, all {args.layers} decoder layers for all {BATCH} rows "
              f"(fp32 math, bf16-rounded activations), head and the reference CPU sampler; {threads} threads")
    if steps < args.steps:
        sample += f"; {steps} of the {args.steps} requested steps timed ({REFERENCE_BUDGET_S:.0f} s budget)"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": per_step * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (random-init weights, N(0,1) KV, seeded ragged contexts)",
        "config": {"workload": "BASELINE config 2: talker decode step, B=64, ctx U[64,2048], 28 layers, "
                               "P=16, 512k-token pool", "global_batch": BATCH, "seq_len": CTX_HI,
                   "parallelism": "cpu (one host process at every N)",
                   "gate_up": "bf16: the reference quantises gate/up to FP8 only on a CUDA device "
                              "(model/layers.py:225-237), so its CPU path keeps bf16"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def peak_tflops() -> float:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return float(json.loads(f.read_text())["bf16_tflops"])
    return 1590.0


def time_graph(fn, reps: int, stream) -> float:
    """ms per replay of a graph of fn() (after warm replays)."""

    fn()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(reps):
        graph.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    return a0.elapsed_time(a1) / reps


def run_mixed(args, world, rank, local, emit: bool = True) -> dict:
    """8 chunked prefills U[128, 1024] + 240 decode rows ctx U[32, 4096], GPU planner each
    step, 10 % of the sequences finish and are replaced each step (on the device)."""

    from importlib import import_module

    nqt = import_module("nari-qwen3-tts_b200")
    talker_step = import_module("nari-qwen3-tts_b200.talker_step")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(2000 + rank)
    chunks = torch.randint(128, 1025, (8,), generator=g).tolist()
    decode_ctx = torch.randint(32, 4097, (240,), generator=g).tolist()
    shape = talker_step.TalkerShape(num_layers=args.layers)
    pool_tokens = max(args.pool_tokens, sum(decode_ctx) + sum(chunks) + 64 * 1024)
    step = talker_step.TalkerMixedStep(shape=shape, chunks=chunks, decode_contexts=decode_ctx, churn_rows=24,
                                       total_pages=pool_tokens // 16, page_size=16, device=dev, seed=rank,
                                       gate_up=args.gate_up or "bf16")
    step.admit(scatter_seed=rank)
    step.capture(warmup=2)
    for _ in range(args.warmup):
        step.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step.replay()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / args.steps
    tokens = step.tokens
    # prefill attention (tcgen05) alone over the step's metadata, all layers
    q = torch.randn(tokens, shape.num_heads, shape.head_dim, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    pb, db = step.pre_b, step.dec_b

    def prefill_pass():
        for layer in range(shape.num_layers):
            nqt.batch_prefill_paged(q[: step.t_pre], step.storage[layer], pb.qo_indptr, pb.paged_kv_indptr,
                                    pb.paged_kv_indices, pb.paged_kv_last_page_len, batch=step.n_pre,
                                    out=out[: step.t_pre])

    def decode_pass():
        for layer in range(shape.num_layers):
            nqt.batch_decode_paged(q[step.t_pre:], step.storage[layer], db.paged_kv_indptr, db.paged_kv_indices,
                                   db.paged_kv_last_page_len, db.decode_workspace, batch_capacity=step.n_dec,
                                   out=out[step.t_pre:], plan=False)

    reps = 10
    pre_ms = time_graph(prefill_pass, reps, stream) / shape.num_layers
    dec_ms = time_graph(decode_pass, reps, stream) / shape.num_layers
    tflops = step.prefill_flops_per_layer() / (pre_ms / 1e3) / 1e12
    dec_gbs = step.decode_bytes_per_layer() / (dec_ms / 1e3) / 1e9
    hbm, _ = peaks()
    status = nqt.kernels.read_status(dev) | int(step.dec.status.item())
    line = {
        "metric": "mixed continuous batch tokens/s (8 prefill chunks + 240 decode rows)",
        "value": world * tokens / (ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights, N(0,1) KV, seeded chunk and context lengths)",
        "config": {
            "workload": f"BASELINE config 4: {shape.num_layers}-layer talker, prefill chunks {chunks} "
                        f"(sum {step.t_pre}), 240 decode rows ctx U[32,4096] (sum {sum(decode_ctx)}), "
                        "24 requests replaced per step on the device, GPU planner, CUDA graph",
            "global_batch": world * step.rows,
            "seq_len": 4096,
            "parallelism": f"dp{world} (request-sharded, no collective)",
            "l2": "inputs larger than L2: ~57 GB of decode KV read per step",
            "gate_up": GATE_UP_NOTE[args.gate_up or "bf16"],
        },
        "decode_seq_steps_per_s": world * step.n_dec / (ms / 1e3),
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak_tflops(), "unit": "TFLOP/s",
                     "frac": tflops / peak_tflops(), "traffic": None,
                     "kernel": "prefill_tc_kernel (tcgen05 causal prefill)", "flop_per_launch":
                     step.prefill_flops_per_layer(), "us_per_launch": pre_ms * 1e3,
                     "peak_source": "measured cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops)"},
        "decode_roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": hbm, "unit": "GB/s", "frac": dec_gbs / hbm,
                            "us_per_launch": dec_ms * 1e3, "bytes_per_launch": step.decode_bytes_per_layer()},
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if emit and rank == 0:
        print(json.dumps(line), flush=True)
    if emit and world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return line


def run_cp(args, world, rank, local, emit: bool = True) -> dict:
    """one code-predictor frame (15 residual codebooks, each with its own 2048-way head and
    sampler call) for B=256 rows, 5-layer decoder, hidden 1024, 16/8 heads, D 64, FFN 3072, top-k 50, T 0.9."""

    from importlib import import_module

    nqt = import_module("nari-qwen3-tts_b200")
    cp = import_module("nari-qwen3-tts_b200.code_predictor")
    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    rows = 256
    frame = cp.CodePredictorFrame(rows=rows, device=dev, seed=rank)
    s = frame.shape
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    frame.past_hidden.copy_(torch.randn(rows, s.talker_hidden, generator=g, device=dev))
    frame.layer0_token.copy_(torch.randint(0, s.vocab, (rows,), generator=g, device=dev))
    frame.set_frame(0)
    lib_mod.reset_launch_count()
    frame.capture(warmup=2)
    launches_per_frame = lib_mod.launch_count() // 3
    for _ in range(args.warmup):
        frame.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            frame.replay()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / args.steps

    # e2e through CodePredictorFrame.step(): pinned H2D of the talker hidden + layer-0 token, D2H of the codes
    host_hidden = frame.past_hidden.cpu()
    host_token = frame.layer0_token.cpu()
    frame.step(host_hidden, host_token)
    e2e_steps = max(10, args.steps // 2)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        frame.step(host_hidden, host_token)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / e2e_steps

    # the fused CP attention launches of one frame (5 layers x 16 positions), timed alone
    hq, hkv, d = s.num_heads, s.num_kv_heads, s.head_dim
    q = torch.randn(rows, hq, d, device=dev).to(torch.bfloat16)
    k = torch.randn(rows, hkv, d, device=dev).to(torch.bfloat16)
    v = torch.randn(rows, hkv, d, device=dev).to(torch.bfloat16)
    cache = torch.randn(s.num_layers, rows, 2, s.groups, hkv, d, device=dev).to(torch.bfloat16)

    def cp_attention_pass():
        for pos in range(s.groups):
            for layer in range(s.num_layers):
                nqt.cp_decode_attention_(q, k, v, frame.q_norm[layer], frame.k_norm[layer], frame.positions[:, pos],
                                         s.eps, s.rope_theta, cache[layer, :, 0], cache[layer, :, 1], pos)

    launches = s.groups * s.num_layers
    attn_ms = time_graph(cp_attention_pass, 10, stream) / launches
    # algorithmic bytes: q, k, v read, out written, K/V row written, cache prefix read (positions 0..pos)
    row_bytes = hkv * d * 2
    per_pos = [rows * (2 * hq * d * 2 + 2 * row_bytes + 2 * row_bytes + 2 * (pos + 1) * row_bytes)
               for pos in range(s.groups)]
    attn_bytes = sum(per_pos) / s.groups
    logits = frame.logits[0]

    def sampler_pass():
        for group in range(s.groups - 1):
            nqt.sample_rows(logits, frame.temperature, frame.top_k, frame.top_p, frame.seed, frame.offsets[:, group],
                            round_scaled_to_input=False, out=frame._token)

    sampler_us = time_graph(sampler_pass, 10, stream) / (s.groups - 1) * 1e3
    peak, peak_kind = peaks()
    achieved = attn_bytes / (attn_ms / 1e3) / 1e9
    status = nqt.kernels.read_status(dev)
    line = {
        "metric": "code-predictor frames/s (B=256, 15 residual codebooks per frame)",
        "value": world * rows / (ms / 1e3),
        "unit": "frames/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights, seeded talker hidden states and layer-0 codes)",
        "config": {
            "workload": "BASELINE config 3: code-predictor whole frame, B=256 rows, 5 layers, hidden 1024, "
                        "16/8 heads, D 64, FFN 3072, 15 x (2048-way head + fused sampler, top-k 50, T 0.9), "
                        "dense 16-position frame cache, one CUDA graph per frame",
            "global_batch": world * rows,
            "seq_len": s.groups,
            "parallelism": f"dp{world} (request-sharded, no collective)",
            "l2": "inputs larger than L2: 147 MB of layer weights streamed per depth step, 16 depth steps",
        },
        "e2e": {"value": world * rows / (e2e_ms / 1e3), "unit": "frames/s",
                "h2d_bytes_per_step": frame.h2d_bytes(), "d2h_bytes_per_step": frame.d2h_bytes()},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "cp_decode_kernel (fused QK norm + RoPE + cache write + attention)",
                     "bytes_per_launch": attn_bytes, "us_per_launch": attn_ms * 1e3,
                     "peak_source": f"{peak_kind} HBM copy (MEASURED_PEAKS.json hbm_gbs)"},
        "sampler_us_per_launch": sampler_us,
        "gpu_launches": launches_per_frame * args.steps,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if emit and rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.code_predictor import CpuCodePredictorFrame

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        port = CpuCodePredictorFrame.random()
        sample_rows_cpu = 64
        port.time_frame(8)
        times = []
        t_end = time.perf_counter() + args.cpu_seconds
        while time.perf_counter() < t_end or not times:
            times.append(port.time_frame(sample_rows_cpu))
        per_frame = statistics.mean(times) / sample_rows_cpu
        line["cpu_baseline"] = {
            "value": 1.0 / per_frame, "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} whole frames of {sample_rows_cpu} rows through the CPU port "
                      "(oracle/code_predictor.py: bf16-rounded activations, fp32 math, reference CPU sampler)",
        }
    if emit and rank == 0:
        print(json.dumps(line), flush=True)
    if emit and world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return line


class SamplerWorkload:
    """The fused sampler's HBM roofline case: the talker sampling of 256 decode steps of B=64 stacked into one
    16384-row launch (V 3072, bf16 logits, seen mask with 64 ids per row, penalty 1.05, T 0.9, top-k 50,
    top-p 0.95).  Two logits/seen buffer sets alternate so consecutive launches miss L2."""

    ROWS, VOCAB = 256 * BATCH, 3072

    def __init__(self, nqt, dev, seed: int) -> None:
        self.nqt = nqt
        rows, vocab = self.ROWS, self.VOCAB
        g = torch.Generator(device=dev).manual_seed(seed)
        self.sets = []
        for _ in range(2):
            logits = (torch.randn(rows, vocab, generator=g, device=dev) * 2.0).to(torch.bfloat16)
            seen = torch.zeros(rows, vocab, dtype=torch.bool, device=dev)
            seen.scatter_(1, torch.randint(0, vocab, (rows, 64), generator=g, device=dev), True)
            self.sets.append((logits, seen))
        self.temp = torch.full((rows,), 0.9, device=dev)
        self.top_k = torch.full((rows,), 50, dtype=torch.int32, device=dev)
        self.top_p = torch.full((rows,), 0.95, device=dev)
        self.pen = torch.full((rows,), 1.05, device=dev)
        self.seed = torch.arange(rows, device=dev)
        self.offset = torch.zeros(rows, dtype=torch.long, device=dev)
        self.out = torch.empty(rows, dtype=torch.long, device=dev)
        # algorithmic bytes: logits + seen mask read, tokens written
        self.bytes_per_launch = rows * vocab * (2 + 1) + rows * 8

    def launch(self, i: int) -> None:
        logits, seen = self.sets[i & 1]
        self.nqt.sample_rows(logits, self.temp, self.top_k, self.top_p, self.seed, self.offset,
                             repetition_penalty=self.pen, seen_token_mask=seen, out=self.out)

    def time_ms(self, steps: int, warmup: int, stream) -> float:
        """Device ms per launch, launches replayed from a CUDA graph (alternating the two input sets) so
        the host's per-call cost does not enter the measurement."""

        for i in range(max(warmup, 2)):
            self.launch(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(steps):
                self.launch(i)
        graph.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / steps

    def roofline(self, ms: float) -> dict:
        peak, peak_kind = peaks()
        achieved = self.bytes_per_launch / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": None, "kernel": "sample_kernel", "bytes_per_launch": self.bytes_per_launch,
                "us_per_launch": ms * 1e3, "rows_per_launch": self.ROWS,
                "peak_source": f"{peak_kind} HBM copy (MEASURED_PEAKS.json hbm_gbs)"}


def run_gate_up(args, world, rank, local, emit: bool = True) -> dict:
    """The talker's FP8 gate/up GEMM (the reference's production path) on its own: 28 layers of gate/up
    weights (larger than L2) called in turn from one CUDA graph, B = 64 rows quantised by the activation rule,
    SwiGLU fused; cuBLAS bf16 gate_up + silu_and_mul on the same weights timed beside it."""

    from importlib import import_module

    nqt = import_module("nari-qwen3-tts_b200")
    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layers, rows, hidden, ffn = args.layers, BATCH, 2048, 6144
    g = torch.Generator(device=dev).manual_seed(6000 + rank)
    w16 = [(torch.randn(2 * ffn, hidden, generator=g, device=dev) * hidden ** -0.5).to(torch.bfloat16)
           for _ in range(layers)]
    w8 = [nqt.kernels.Fp8BlockWeight(w, gate_up=True) for w in w16]
    x = torch.randn(rows, hidden, generator=g, device=dev).to(torch.bfloat16)
    xq, xs = nqt.kernels.fp8_quantize_rows(x)
    act = torch.empty(rows, ffn, dtype=torch.bfloat16, device=dev)
    ws = nqt.kernels.fp8_gemm_workspace(dev, rows, 2 * ffn, hidden)

    def fp8_pass():
        for w in w8:
            nqt.kernels.linear_fp8(xq, xs, w, out=act, workspace=ws)

    def bf16_pass():
        for w in w16:
            nqt.kernels.silu_and_mul(torch.nn.functional.linear(x, w), out=act)

    def graph_ms(fn) -> float:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(args.warmup, 1)):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        for _ in range(args.warmup):
            gr.replay()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), world) / args.steps

    lib_mod.reset_launch_count()
    with ClockSampler(dev) as clocks:
        fp8_ms = graph_ms(fp8_pass)
    launches = lib_mod.launch_count()
    bf16_ms = graph_ms(bf16_pass)
    us = fp8_ms * 1e3 / layers
    # algorithmic bytes of one call: e4m3 weights + block scales, e4m3 X + its scales, bf16 Y
    nbytes = 2 * ffn * hidden + (2 * ffn // 128) * (hidden // 128) * 4 + rows * hidden + (hidden // 128) * rows * 4 \
        + rows * ffn * 2
    peak, peak_kind = peaks()
    achieved = nbytes / (us * 1e-6) / 1e9
    line = {
        "metric": "talker FP8 gate/up GEMM time per call (M=64, N=12288, K=2048, SwiGLU fused)",
        "value": us,
        "unit": "us",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": fp8_ms,
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8 e4m3 (block-scaled, fp32 accumulate)",
        "data": "synthetic (random-init bf16 weights quantised at load, N(0,1) rows)",
        "config": {"workload": f"{layers} layers of talker gate/up weights called in turn from one CUDA graph "
                               "(weights larger than L2)", "global_batch": rows * world, "seq_len": hidden,
                   "parallelism": f"dp{world}", "gate_up": GATE_UP_NOTE["fp8"]},
        "bf16_cublas_us_per_call": bf16_ms * 1e3 / layers,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "gemm_fp8_kernel", "bytes_per_launch": nbytes, "us_per_launch": us,
                     "peak_source": f"{peak_kind} HBM copy (MEASURED_PEAKS.json hbm_gbs)"},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "device_status": nqt.kernels.read_status(dev),
    }
    if emit and rank == 0:
        print(json.dumps(line), flush=True)
    return line


def run_sampler(args, world, rank, local) -> None:
    """The fused sampler's HBM roofline (SamplerWorkload) as its own bench line."""

    from importlib import import_module

    nqt = import_module("nari-qwen3-tts_b200")
    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    work = SamplerWorkload(nqt, dev, 4000 + rank)
    rows = work.ROWS
    for i in range(args.warmup):
        work.launch(i)
    torch.cuda.synchronize()
    lib_mod.reset_launch_count()
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(dev) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        ms = work.time_ms(args.steps, 0, stream)
        barrier(world)
    launches = lib_mod.launch_count()
    ms = max_over_ranks(ms, world)
    # e2e: the same launch from pinned host logits (H2D inside the timed region) and tokens read back
    host_logits = work.sets[0][0].cpu().pin_memory()
    host_tokens = torch.empty(rows, dtype=torch.long).pin_memory()
    e_steps = max(5, args.steps // 4)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        work.sets[0][0].copy_(host_logits, non_blocking=True)
        work.launch(0)
        host_tokens.copy_(work.out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1), world) / e_steps
    line = {
        "metric": "fused sampler rows/s (talker sampling, 16384 stacked rows x V 3072)",
        "value": world * rows / (ms / 1e3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (N(0,2) logits, 64 seen ids per row)",
        "config": {"workload": "sampler roofline: 256 talker steps x B=64 stacked, V 3072, penalty 1.05, T 0.9, "
                               "top-k 50, top-p 0.95, Philox draw", "global_batch": world * rows,
                   "seq_len": work.VOCAB, "parallelism": f"dp{world}", "l2": "two 151 MB input sets alternate (> L2)"},
        "e2e": {"value": world * rows / (e_ms / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": host_logits.numel() * 2, "d2h_bytes_per_step": rows * 8},
        "roofline": work.roofline(ms),
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "device_status": nqt.kernels.read_status(dev),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def _summary(line: dict) -> dict:
    """The parts of another workload's bench line carried on the headline line."""

    keys = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "e2e", "roofline", "decode_roofline",
            "decode_seq_steps_per_s", "sampler_us_per_launch", "gpu_launches", "clocks", "device_status")
    out = {k: line[k] for k in keys if k in line}
    out["workload"] = line["config"]["workload"]
    return out


def run_serve(args, world, rank, local) -> None:
    """box-level request-sharded serving simulation.  Poisson arrivals (args.serve_rps per
    GPU, seeded) are routed round-robin to the ranks; each rank is one ServingWorker (64 request slots, its own
    page pool, GPU planner, device request table, talker decode step and code-predictor frame, all captured);
    text 20-200 tokens of prefill, 2-20 s of audio at 12 frames/s.  Reported: frames/s per box (sum over
    ranks / the slowest rank's wall time) and time-to-first-frame percentiles over every request."""

    from importlib import import_module

    serving = import_module("nari-qwen3-tts_b200.serving")
    talker_step = import_module("nari-qwen3-tts_b200.talker_step")
    nqt = import_module("nari-qwen3-tts_b200")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = talker_step.TalkerShape(num_layers=args.layers)
    worker = serving.ServingWorker(shape=shape, slots=BATCH, pool_tokens=128 * 1024, device=dev, seed=rank)
    worker.capture()
    requests = serving.poisson_requests(rate=args.serve_rps, horizon=args.serve_seconds, seed=5000, rank=rank,
                                        world=world)
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(dev) as clocks:
        rep = worker.run(requests, horizon=args.serve_seconds)
    barrier(world)
    elapsed = max_over_ranks(rep.elapsed, world)
    local_stats = torch.tensor([rep.frames, rep.steps, rep.finished, rep.admitted, len(requests)], dtype=torch.float64)
    ttff = torch.tensor(rep.ttff, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(local_stats)
        sizes = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([ttff.numel()]))
        width = int(max(x.item() for x in sizes))
        padded = torch.full((width,), float("nan"), dtype=torch.float64)
        padded[: ttff.numel()] = ttff
        gathered = [torch.empty(width, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, padded)
        ttff = torch.cat(gathered)
        ttff = ttff[~torch.isnan(ttff)]
    frames, steps, finished, admitted, offered = (float(x) for x in local_stats)
    q = (lambda p: float(torch.quantile(ttff, p)) * 1e3) if ttff.numel() else (lambda p: None)
    status = nqt.kernels.read_status(dev) | int(worker.step.planner.status.item())
    line = {
        "metric": "box serving frames/s (talker + code predictor, Poisson arrivals per GPU)",
        "value": frames / elapsed,
        "unit": "frames/s",
        "n_gpus": world,
        "steps": int(rep.steps),
        "warmup": 1,
        "ms_per_step": rep.elapsed / max(rep.steps, 1) * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights; seeded Poisson arrivals, text and audio lengths)",
        "config": {
            "workload": f"BASELINE config 5: {args.serve_rps:g} RPS per GPU for {args.serve_seconds:g} s, text 20-200 "
                        f"tokens, audio 2-20 s at 12 frames/s; per GPU 64 request slots, {shape.num_layers}-layer talker "
                        "+ 5-layer code predictor, one page pool, GPU planner and device request table",
            "global_batch": world * BATCH,
            "seq_len": 256 + 240,
            "parallelism": f"dp{world} (request-sharded: round-robin router, no collective)",
            "timing": "host wall clock over the arrival window plus the drain, each step synchronised",
        },
        "p50_ttff_ms": q(0.5),
        "p95_ttff_ms": q(0.95),
        "requests": {"offered": int(offered), "admitted": int(admitted), "finished": int(finished)},
        "frames": int(frames),
        "mean_busy_rows_rank0": sum(rep.busy_rows) / max(len(rep.busy_rows), 1),
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


GATE_UP_NOTE = {
    "fp8": "fp8 e4m3: 128x128 weight blocks with power-of-two scales, per-token 1x128 activation blocks, "
           "fp32 accumulation (the reference's production talker path, executor/build.py:73)",
    "bf16": "bf16 (unquantised)",
}


def main() -> None:
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.workload == "mixed":
        run_mixed(args, world, rank, local)
        return
    if args.workload == "cp":
        run_cp(args, world, rank, local)
        return
    if args.workload == "sampler":
        run_sampler(args, world, rank, local)
        return
    if args.workload == "serve":
        run_serve(args, world, rank, local)
        return
    if args.workload == "gate_up":
        run_gate_up(args, world, rank, local)
        return
    nqt = importlib.import_module("nari-qwen3-tts_b200")
    from importlib import import_module

    talker_step = import_module("nari-qwen3-tts_b200.talker_step")
    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = talker_step.TalkerShape(num_layers=args.layers)
    pages = args.pool_tokens // 16
    step = talker_step.TalkerDecodeStep(shape=shape, batch=BATCH, total_pages=pages, page_size=16,
                                        max_pages_per_seq=(CTX_HI + 1024) // 16, device=dev, seed=rank,
                                        publish=args.grow, gate_up=args.gate_up or "fp8")
    contexts = contexts_for(rank)
    step.admit(contexts, scatter_seed=rank)
    lib_mod.reset_launch_count()
    step.capture(warmup=2)
    launches_per_step = lib_mod.launch_count() // 3  # two eager warm-ups + the captured pass
    executed = 2
    for _ in range(args.warmup):
        step.replay()
    executed += args.warmup
    torch.cuda.synchronize()

    # ---------------------------------------------------------------- timed region
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step.replay()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    executed += args.steps
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    value = world * BATCH * args.steps / (elapsed_ms / 1e3)

    # ---------------------------------------------------------------- e2e through step()
    g = torch.Generator().manual_seed(rank)
    host_in = torch.randn(BATCH, shape.hidden, generator=g).to(torch.bfloat16)
    step.step(host_in)
    executed += 1
    e2e_steps = max(20, args.steps // 2)
    torch.cuda.synchronize()
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(e2e_steps):
        step.step(host_in)
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    executed += e2e_steps
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
    e2e_value = world * BATCH * e2e_steps / (e2e_ms / 1e3)

    # ---------------------------------------------------------------- attention roofline
    # the binding holds the metadata of the last executed step
    lengths = [n + (executed if args.grow else 1) for n in contexts]
    attn_bytes = sum(lengths) * 2 * shape.num_kv_heads * shape.head_dim * 2 + 2 * BATCH * shape.num_heads * shape.head_dim * 2
    q = torch.randn(BATCH, shape.num_heads, shape.head_dim, device=dev).to(torch.bfloat16)
    b = step.binding
    outs = torch.empty(BATCH, shape.num_heads, shape.head_dim, dtype=torch.bfloat16, device=dev)

    def attention_pass():
        for layer in range(shape.num_layers):
            nqt.batch_decode_paged(q, step.storage[layer], b.paged_kv_indptr, b.paged_kv_indices,
                                   b.paged_kv_last_page_len, b.decode_workspace, batch_capacity=BATCH, out=outs,
                                   plan=False)

    attention_pass()
    ag = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ag):
        attention_pass()
    for _ in range(3):
        ag.replay()
    reps = max(10, args.steps // 4)
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(reps):
        ag.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    attn_ms = max_over_ranks(a0.elapsed_time(a1), world) / (reps * shape.num_layers)
    peak, peak_kind = peaks()
    achieved = attn_bytes / (attn_ms / 1e3) / 1e9
    # DRAM traffic of one decode launch from an ncu capture of this kernel on the same contexts
    # (2-layer model, Sum(ctx + 2) = 74466 tokens): 307.88 MB read + 4.19 MB written, scaled by tokens
    traffic = (307.876352e6 + 4.194816e6) * (sum(lengths) / 74466.0) if args.layers == 28 else None

    # ---------------------------------------------------------------- sampler roofline (same process)
    sampler = SamplerWorkload(nqt, dev, 4000 + rank)
    sampler_ms = max_over_ranks(sampler.time_ms(20, 3, stream), world)
    sampler_line = sampler.roofline(sampler_ms)
    del sampler
    status = nqt.kernels.read_status(dev) | int(step.planner.status.item())

    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights, N(0,1) KV, seeded ragged contexts)",
        "config": {
            "workload": f"BASELINE config 2: talker decode step, B={BATCH} ragged ctx U[{CTX_LO},{CTX_HI}], "
                        f"{shape.num_layers} layers, hidden 2048, 16/8 heads, D 128, FFN 6144, vocab 3072, P=16, "
                        f"{args.pool_tokens // 1024}k-token pool, GPU planner + fused sampler, CUDA graph",
            "global_batch": BATCH * world,
            "seq_len": CTX_HI,
            "parallelism": f"dp{world} (request-sharded, no collective)",
            "l2": "inputs larger than L2: ~8.5 GB of KV read per step",
            "gate_up": GATE_UP_NOTE[args.gate_up or "fp8"],
            "contexts": "held at the sampled lengths (each step's reservation is discarded)" if not args.grow
            else "growing by one token per step (published)",
        },
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                "d2h_bytes_per_step": step.d2h_bytes()},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "traffic_source": "scaled_from_profile: ncu DRAM bytes of one launch "
                     "on the same contexts (2-layer capture), scaled by the tokens read",
                     "kernel": "decode attention (decode_kernel, fused split fix-up)",
                     "bytes_per_launch": attn_bytes, "us_per_launch": attn_ms * 1e3,
                     "peak_source": f"{peak_kind} HBM copy (MEASURED_PEAKS.json hbm_gbs)"},
        "sampler_roofline": sampler_line,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    del ag, attention_pass, b, step, q, outs
    if world == 1 and args.layers == 28 and not args.no_other_configs:
        # BASELINE configs 3 and 4 on the same GPU, after the config-2 step's memory is released
        torch.cuda.empty_cache()
        sub = argparse.Namespace(**{**vars(args), "steps": min(args.steps, 20), "warmup": min(args.warmup, 3)})
        line["config4_mixed"] = _summary(run_mixed(sub, world, rank, local, emit=False))
        torch.cuda.empty_cache()
        line["config3_code_predictor"] = _summary(run_cp(sub, world, rank, local, emit=False))
        torch.cuda.empty_cache()
        gu = run_gate_up(sub, world, rank, local, emit=False)
        line["gate_up_fp8_gemm"] = {"us_per_call": gu["value"], "bf16_cublas_us_per_call": gu["bf16_cublas_us_per_call"],
                                    "roofline": gu["roofline"]}
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds, shape.num_layers)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
