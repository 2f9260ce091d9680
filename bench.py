#!/usr/bin/env python
"""Aggregate decode throughput of the native Qwen2 Q4_K_M stage engine on B200.

Workload (configs[2] of the benchmark definition, the metric's "Qwen2 Q4_K
pipeline at 1/2/4/8 B200"): Qwen2-architecture 7B Q4_K_M (28 layers, hidden
3584, 28/4 heads, FFN 18944, vocabulary 152,064), seeded N(0, 0.02) weights
quantized with this repository's K-quant encoders, 64 concurrent sequences of
1024 uniform-random prompt tokens, 256 greedy output tokens each. One "step"
serves the whole batch: one batched prefill of all prompts, then 255 batched
decode steps. The weights (4.68 GB) and the KV caches (up to 4.7 GB) are far
larger than L2 (126 MB), so every decode step streams them from HBM.
`--preset` selects the other configurations (1.5b, 3b, 14b, 32b) with their
own default batch shapes.

    value      aggregate output tok/s, device-timed (CUDA events on the
               engine stream), prompts already resident in HBM
    e2e        the same workload through the engine's C ABI with host
               buffers: prompts copied in, every step's tokens copied in and
               the sampled tokens read back (wall clock)
    roofline   the decode matmuls (weight-streaming K-quant x Q8_K dot
               products, the dominant kernel family) of one decode step at
               the workload's batch, bytes / CUDA-event time vs measured HBM
    parity     a bounded sample through the same engine (sequence 0's first
               32 prompt tokens, 8 greedy tokens) against the CPU oracle
    cpu_baseline  the CPU oracle (this repository's restatement of the
               reference's GGML-CPU path) on that sample, with its prefill
               and decode token rates; for --preset 1.5b (the configuration
               the reference times end to end on its CPU backend) the whole
               workload once instead

--impl reference runs the CPU oracle on the host cores instead (the
reference's own native engine needs GGML, which cannot be built here): each
step the bounded sample, or with --cpu-full (the default for --preset 1.5b)
the whole workload.

With torchrun (N > 1) the same workload runs as an N-stage pipeline (one
process and GPU per contiguous layer range, jetsonfabric_b200/pipeline.py):
F16 activations cross each stage boundary over NCCL point-to-point (NVLink)
as Stagewire v2 frames (jetsonfabric_b200/stagewire.py: payload CRC-32
computed and stamped on the device, every received frame checked against its
checksum on the device and against the decoder's rules on the host at the
end of each run; --frames raw sends bare payloads), the last stage returns
each micro-batch's greedy tokens to the first in the same frames, and N
micro-batches of sequences keep every stage busy. The workload is fixed as N
grows (strong scaling); the value is its output tokens over the slowest
rank's device time. TTFT and ITL are measured on the last stage. e2e runs
the same pipeline with the prompts copied in from pinned host memory every
step and every sampled token copied back to host memory (wall clock, slowest
rank). --replicas instead gives every rank its own full-model replica (weak
scaling, a comparison only).
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from jetsonfabric_b200.jfm import QWEN2_PRESETS as PRESETS  # noqa: E402

# default batch shape of each preset: (concurrency, prompt tokens, output
# tokens, session capacity or 0 for prompt + output - 1), from the benchmark
# configurations: cfg 1 1.5B C2 p128 o128; cfg 2 3B C32 p512 o256; cfg 3 7B
# C64 p1024 o256; cfg 4 14B 128 streams of 4096-token prompts with the KV
# cache reserved for 8192 positions; cfg 5 32B Q2_K 256 sequences p2048 o512
WORKLOADS = {"1.5b": (2, 128, 128, 0), "3b": (32, 512, 256, 0), "7b": (64, 1024, 256, 0),
             "14b": (128, 4096, 256, 8192), "32b": (256, 2048, 512, 0)}
METRIC = "aggregate decode tok/s + p50 ITL, Qwen2 Q4_K pipeline at 1/2/4/8 B200"


def matmul_shapes(preset: str) -> dict:
    """Weight shapes (type, rows, cols) of one layer and the head, for --matmul-shape."""
    m = PRESETS[preset]
    h, f, v = m["embedding_length"], m["feed_forward_length"], m["vocabulary_size"]
    kvd = h // m["head_count"] * m["kv_head_count"]
    lt = m.get("layer_type", 11)
    return {"ffn_gate": (lt, f, h), "ffn_down_q6": (13, h, f), "attn_q": (lt, h, h), "attn_k": (lt, kvd, h),
            "output_q6": (13, v, h)}


MATMUL_SHAPE_NAMES = ["attn_k", "attn_q", "ffn_down_q6", "ffn_gate", "output_q6"]
UNIT = "tok/s"
DTYPE = "q4_k/q6_k/q2_k x q8_k int8 dot, f32 block terms, f64 sums; f16 KV with f64 attention sums"


def workload_name(args) -> str:
    return f"{model_label(args.preset)} c{args.concurrency} p{args.prompt_tokens} o{args.output_tokens}"


def model_name(args) -> str:
    kind = "Q2_K (Q6_K output)" if PRESETS[args.preset].get("layer_type") == 9 else "Q4_K_M"
    return f"Qwen2-arch {args.preset} {kind}"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--preset", default="7b", choices=sorted(PRESETS))
    p.add_argument("--concurrency", type=int, default=None)
    p.add_argument("--prompt-tokens", type=int, default=None)
    p.add_argument("--output-tokens", type=int, default=None)
    p.add_argument("--capacity", type=int, default=None, help="KV positions reserved per session")
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--package-dir", default=os.environ.get("JFB_BENCH_DIR",
                                                           os.path.join(tempfile.gettempdir(), "jfb_bench")))
    p.add_argument("--skip-parity", action="store_true")
    p.add_argument("--skip-e2e", action="store_true")
    p.add_argument("--skip-cpu", action="store_true")
    p.add_argument("--micro-batches", type=int, default=0, help="pipeline micro-batches (default: one per stage)")
    p.add_argument("--replicas", action="store_true", help="N > 1: full-model replicas instead of a pipeline")
    p.add_argument("--cpu-full", action="store_true", default=None,
                   help="--impl reference: serve the whole workload on the CPU oracle instead of the bounded sample "
                        "(default for --preset 1.5b, the configuration the reference times end to end on CPU)")
    p.add_argument("--frames", choices=["stagewire", "raw"], default="stagewire",
                   help="N > 1 pipeline: stage traffic as Stagewire v2 frames (default) or bare payloads")
    p.add_argument("--matmul-shape", choices=MATMUL_SHAPE_NAMES, default=None,
                   help="time only the tcgen05 K-quant matmul on one weight shape of the workload (profiling target)")
    p.add_argument("--matmul-rows", type=int, default=32, help="activation rows for --matmul-shape")
    p.add_argument("--matmul-path", choices=["tensor-core", "cuda-core"], default="tensor-core",
                   help="kernel for --matmul-shape: jfb_matmul_tc or the CUDA-core jfb_matmul (1-7 rows in the engine)")
    p.add_argument("--attention-shape", choices=["decode", "prefill"], default=None,
                   help="time only jfb_attention on the workload's decode (32 rows x 768 keys) or prefill "
                        "(32 x 512 causal rows) shape (profiling target)")
    a = p.parse_args()
    c, pt, ot, cap = WORKLOADS[a.preset]
    a.concurrency = c if a.concurrency is None else a.concurrency
    a.prompt_tokens = pt if a.prompt_tokens is None else a.prompt_tokens
    a.output_tokens = ot if a.output_tokens is None else a.output_tokens
    need = a.prompt_tokens + a.output_tokens - 1
    a.capacity = max(need, cap) if a.capacity is None else max(need, a.capacity)
    if a.cpu_full is None:
        a.cpu_full = a.preset == "1.5b"
    return a


def model_label(preset: str) -> str:
    return f"qwen2-{preset}-" + ("q2k" if PRESETS[preset].get("layer_type") == 9 else "q4km")


def package_path(args) -> Path:
    return Path(args.package_dir) / f"{model_label(args.preset)}-seed{args.seed}.jfm"


def ensure_package(args, rank: int) -> Path:
    from jetsonfabric_b200 import jfm
    path = package_path(args)
    done = path / ".complete"
    if rank == 0 and not done.exists():
        path.mkdir(parents=True, exist_ok=True)
        ctx = max(4096, args.capacity)
        jfm.write_synthetic_package(path, **PRESETS[args.preset], context_length=ctx, seed=args.seed,
                                    draw_norms=False, draw_biases=True)
        done.write_text("ok")
    while not done.exists():
        time.sleep(0.5)
    return path


def prompts_for(args, vocab: int):
    import numpy as np
    rng = np.random.default_rng(args.seed)
    return rng.integers(0, vocab, (args.concurrency, args.prompt_tokens), dtype=np.int32)


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([v.strip() for v in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i, v in enumerate(s[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import numpy as np
    import torch
    from jetsonfabric_b200 import engine as E

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    pkg = ensure_package(args, rank if world == 1 else int(os.environ.get("LOCAL_RANK", rank)))
    if dist is not None:
        dist.barrier()
    eng = E.NativeEngine(pkg, "cuda", device=local_rank)
    info = eng.model_info()
    C, P, O = args.concurrency, args.prompt_tokens, args.output_tokens
    capacity = args.capacity
    prompts = prompts_for(args, info.vocabulary_size)
    sessions = [eng.create_session(capacity) for _ in range(C)]
    handles = eng._handles(sessions)
    stream = torch.cuda.ExternalStream(eng.stream())
    d_prompts = torch.from_numpy(prompts.ravel().copy()).cuda()
    tok_a = torch.zeros(C, dtype=torch.int32, device="cuda")
    tok_b = torch.zeros(C, dtype=torch.int32, device="cuda")
    counts = [P] * C
    launches = {"prefill": 0, "decode": 0}

    def device_step(record=None, timing_at: int | None = None):
        for s in sessions:
            s.reset()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(O + 1)]
        ev[0].record(stream)
        eng.prefill_batch_device(sessions, d_prompts.data_ptr(), counts, tok_a.data_ptr())
        launches["prefill"] = eng.last_launch_count()
        ev[1].record(stream)
        src, dst = tok_a, tok_b
        for i in range(O - 1):
            if timing_at is not None and i == timing_at:
                eng.set_kernel_timing(True)
            eng.decode_batch_device(sessions, src.data_ptr(), dst.data_ptr(), handles)
            if timing_at is not None and i == timing_at:
                eng.set_kernel_timing(False)
                if record is not None:
                    record.update(eng.kernel_timing())
            ev[i + 2].record(stream)
            src, dst = dst, src
        launches["decode"] = eng.last_launch_count()
        eng.synchronize()
        total = ev[0].elapsed_time(ev[O])
        prefill = ev[0].elapsed_time(ev[1])
        gaps = [ev[i].elapsed_time(ev[i + 1]) for i in range(1, O)]
        return total, prefill, gaps

    for _ in range(max(args.warmup, 0)):
        device_step()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    totals, prefills, gaps = [], [], []
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.steps):
            t, p, g = device_step()
            totals.append(t)
            prefills.append(p)
            gaps.extend(g)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    # roofline of the decode matmuls: one extra step with per-launch CUDA events
    timing: dict = {}
    device_step(record=timing, timing_at=O // 2)
    ms_per_step = statistics.mean(totals)
    if dist is not None:
        t = torch.tensor([ms_per_step], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_per_step = float(t.item())
    tokens_per_step = C * O * world
    value = tokens_per_step / (ms_per_step / 1000.0)

    # end to end through the C ABI with host buffers
    e2e = None
    if not args.skip_e2e:
        e2e_times = []
        for _ in range(max(1, args.steps)):
            for s in sessions:
                s.reset()
            t0 = time.perf_counter()
            res = eng.prefill_stage_batch(sessions, [p.tolist() for p in prompts])
            cur = [r.sampled_token for r in res]
            for _ in range(O - 1):
                cur = [r.sampled_token for r in eng.decode_stage_batch(sessions, cur)]
            e2e_times.append(time.perf_counter() - t0)
        e2e_s = statistics.mean(e2e_times)
        if dist is not None:
            t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = {"value": tokens_per_step / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": C * P * 4 + (O - 1) * C * 4, "d2h_bytes_per_step": O * C * 4}

    peaks = measured_peaks()
    roof = None
    if timing.get("matmul_ms"):
        achieved = timing["matmul_bytes"] / (timing["matmul_ms"] / 1000.0) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic_from_profiles(),
                "kernel": "decode matmuls (K-quant x Q8_K on tcgen05 for 8+ rows), one decode step",
                "launches": timing["matmul_launches"],
                "bytes_per_launch": timing["matmul_bytes"] / max(1, timing["matmul_launches"]),
                "ms_per_launch": timing["matmul_ms"] / max(1, timing["matmul_launches"]),
                "peak_source": peaks["source"],
                "attention": {"achieved": round(timing["attention_bytes"] / (timing["attention_ms"] / 1000.0) / 1e9, 1),
                              "launches": timing["attention_launches"]}}

    result = None
    if rank == 0:
        cpu = parity = None
        if not (args.skip_cpu and args.skip_parity):
            prompt = sample_prompt(args, info.vocabulary_size)
            gpu_tokens = gpu_sample_tokens(eng, prompt)
            threads = os.cpu_count() or 1
            runner = OracleRunner(pkg, threads)
            res = runner.sample(prompt)
            full = None
            if args.cpu_full and not args.skip_cpu and world == 1:
                full = reference_full_workload(args, runner)
            runner.close()
            parity = None if args.skip_parity else parity_line(gpu_tokens, res["tokens"])
            cpu = None if (args.skip_cpu or world > 1) else cpu_line(args, res, threads)
            if full is not None:
                cpu = {"value": round(C * O / full["seconds"], 4), "unit": UNIT, "cores": threads, "kind": "port",
                       "ttft_ms": round(full["ttft_s"] * 1000, 1),
                       "itl_p50_ms": round(statistics.median(full["gaps_s"]) * 1000, 2) if full["gaps_s"] else None,
                       "sample": f"the whole {workload_name(args)} workload once (CPU oracle, OpenMP over "
                                 f"{threads} threads); value = output tokens / wall time"}
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "weak" if world > 1 else "strong", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": workload_name(args), "model": model_name(args),
                       "layers": info.layer_count, "hidden": info.embedding_length, "concurrency": C,
                       "prompt_tokens": P, "output_tokens": O, "session_capacity": capacity,
                       "weight_bytes": info.weight_bytes,
                       "global_batch": C * world, "seq_len": P + O,
                       "parallelism": "replicas" if world > 1 else "single stage",
                       "l2": f"weights ({info.weight_bytes / 1e9:.2f} GB) exceed L2 (126 MB) every decode step"},
            "parity": parity,
            "ttft_p50_ms": round(statistics.median(prefills), 3),
            "itl_p50_ms": round(statistics.median(gaps), 4),
            "decode_tok_s": round(C * world / (statistics.mean(gaps) / 1000.0), 1),
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks.summary(),
            "gpu_launches": int((launches["prefill"] + (O - 1) * launches["decode"]) * args.steps),
        }
    for s in sessions:
        s.close()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


def progress(rank: int, phase: str) -> None:
    """One line per phase on stderr, so that a stalled run shows where it stopped."""
    print(f"[bench rank {rank}] {phase} {time.strftime('%H:%M:%S')}", file=sys.stderr, flush=True)


def run_pipeline(args, rank: int, world: int, local_rank: int) -> dict | None:
    """N-stage pipeline over contiguous layer ranges (see the module docstring)."""
    import datetime

    import torch
    import torch.distributed as dist
    from jetsonfabric_b200 import engine as E
    from jetsonfabric_b200 import pipeline as PL

    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    pkg = ensure_package(args, local_rank)
    dist.barrier()
    preset = PRESETS[args.preset]
    L = preset["layer_count"]
    ranges = PL.stage_ranges(L, world)
    start, end = ranges[rank]
    eng = E.NativeEngine(pkg, "cuda", layer_start=start, layer_end=end, device=local_rank)
    groups = PL.make_groups(world)
    PL.warm_groups(rank, world, groups, device=torch.device("cuda", local_rank))
    torch_link = PL.TorchLink(rank, world, groups)
    C, P, O = args.concurrency, args.prompt_tokens, args.output_tokens
    micro = args.micro_batches or world
    batches = PL.split_batches(C, micro)
    prompts = prompts_for(args, preset["vocabulary_size"]).tolist()
    stage = PL.EngineStage(eng, prompts, batches, capacity=args.capacity)

    def framed(plan_batches, lengths, steps):
        if args.frames == "raw":
            return torch_link
        from jetsonfabric_b200 import stagewire as SW
        plan = SW.FramePlan(model_id=model_name(args), stage_layers=ranges, batches=plan_batches,
                            prompt_lengths=lengths, steps=steps, hidden=preset["embedding_length"])
        return SW.StagewireLink(torch_link, rank, plan, device=torch.device("cuda", local_rank), stream=stage.stream)

    link = framed(batches, [P] * C, O)
    last = rank == world - 1
    launches = {"n": 0}

    def one_run():
        stage.reset()
        torch.cuda.synchronize()
        dist.barrier()
        marks = {}
        with torch.cuda.stream(stage.stream):
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(stage.stream)

            def on_output(step, m, _out):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stage.stream)
                marks[(step, m)] = ev

            orig_forward = stage.forward

            def counted(m, prefill, inputs):
                out = orig_forward(m, prefill, inputs)
                launches["n"] += eng.last_launch_count()
                return out

            stage.forward = counted
            try:
                PL.run_schedule(rank, world, batches, [P] * C, O, stage, link, on_output if last else None)
            finally:
                stage.forward = orig_forward
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record(stage.stream)
        torch.cuda.synchronize()
        total = t0.elapsed_time(t1)
        ttft, gaps = [], []
        if last:
            for m in range(len(batches)):
                ttft.append(t0.elapsed_time(marks[(0, m)]))
                for t in range(1, O):
                    gaps.append(marks[(t - 1, m)].elapsed_time(marks[(t, m)]))
        return total, ttft, gaps

    progress(rank, "warm-up")
    for _ in range(max(args.warmup, 0)):
        one_run()
    progress(rank, "timed")
    totals, ttfts, gaps = [], [], []
    launches["n"] = 0
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.steps):
            t, tt, g = one_run()
            totals.append(t)
            ttfts.extend(tt)
            gaps.extend(g)
    ms = torch.tensor([statistics.mean(totals)], device="cuda", dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    launch_total = torch.tensor([launches["n"]], device="cuda", dtype=torch.float64)
    dist.all_reduce(launch_total, op=dist.ReduceOp.SUM)
    lat = torch.zeros(3, device="cuda", dtype=torch.float64)
    if last:
        lat[0] = statistics.median(ttfts)
        lat[1] = statistics.median(gaps)
        lat[2] = statistics.mean(gaps)
    dist.broadcast(lat, src=world - 1)
    ms_per_step = float(ms.item())
    value = C * O / (ms_per_step / 1000.0)

    # roofline of the first stage's decode matmuls: one timed decode pass of micro-batch 0
    progress(rank, "roofline pass")
    timing: dict = {}
    if rank == 0:
        stage.reset()
        with torch.cuda.stream(stage.stream):
            mb = batches[0]
            acts = stage.forward(0, True, stage.prompt_tokens(0))
            toks = torch.zeros(len(mb), dtype=torch.int32, device="cuda")
            eng.set_kernel_timing(True)
            stage.forward(0, False, toks)
            eng.set_kernel_timing(False)
            timing = eng.kernel_timing()
        del acts
    torch.cuda.synchronize()
    dist.barrier()

    # end to end: the same pipeline through the stage API, fed from and read
    # back to host memory. Each step the first stage copies every micro-batch's
    # prompts from pinned host memory, and the last stage copies every sampled
    # token to pinned host memory as it is produced; wall clock, slowest rank.
    e2e = None
    pinned: dict = {}
    if not args.skip_e2e:
        progress(rank, "e2e (pinned host prompts in, host tokens out)")
        pinned["prompts"] = [stage.prompt_dev[m].cpu().pin_memory() for m in range(len(batches))] if rank == 0 else []
        pinned["tokens"] = torch.empty((O, C), dtype=torch.int32).pin_memory() if last else None
        offsets = [mb[0] for mb in batches]

        def to_host(step, m, out):
            pinned["tokens"][step, offsets[m]:offsets[m] + len(batches[m])].copy_(out, non_blocking=True)

        times = []
        for _ in range(max(1, args.steps)):
            stage.reset()
            torch.cuda.synchronize()
            dist.barrier()
            a = time.perf_counter()
            with torch.cuda.stream(stage.stream):
                # indexing, not a loop variable: no name outlives the loop
                # holding a pinned buffer (see the engine close below)
                for m in range(len(pinned["prompts"])):
                    stage.prompt_dev[m].copy_(pinned["prompts"][m], non_blocking=True)
                PL.run_schedule(rank, world, batches, [P] * C, O, stage, link, to_host if last else None)
            torch.cuda.synchronize()
            times.append(time.perf_counter() - a)
        sec = torch.tensor([statistics.mean(times)], device="cuda", dtype=torch.float64)
        dist.all_reduce(sec, op=dist.ReduceOp.MAX)
        e2e = {"value": C * O / float(sec.item()), "unit": UNIT,
               "h2d_bytes_per_step": C * P * 4, "d2h_bytes_per_step": O * C * 4,
               "path": "stage API over the NCCL pipeline; prompts from pinned host memory, tokens to host memory"}

    # parity: the bounded sample through the same pipeline (one micro-batch of
    # one sequence); the first stage receives every greedy token from the last
    parity = None
    if not args.skip_parity:
        progress(rank, "parity sample")
        prompt = sample_prompt(args, preset["vocabulary_size"])
        n_out = CPU_SAMPLE["output_tokens"]
        pstage = PL.EngineStage(eng, [prompt], [[0]], capacity=len(prompt) + n_out + 1)
        plink = framed([[0]], [len(prompt)], n_out + 1)
        received = []
        if rank == 0:
            plain = pstage.forward

            def recording(m, prefill, inputs):
                if not prefill:
                    received.append(inputs)
                return plain(m, prefill, inputs)

            pstage.forward = recording
        with torch.cuda.stream(pstage.stream):
            PL.run_schedule(rank, world, [[0]], [len(prompt)], n_out + 1, pstage, plink)
        torch.cuda.synchronize()
        pstage.close()
        if rank == 0:
            gpu_tokens = [int(t.cpu().item()) for t in received]
            runner = OracleRunner(pkg, os.cpu_count() or 1)
            res = runner.sample(prompt)
            runner.close()
            parity = parity_line(gpu_tokens, res["tokens"])
            parity["path"] = f"pp{world} pipeline, NCCL boundary"
        dist.barrier()

    result = None
    if rank == 0:
        peaks = measured_peaks()
        roof = None
        if timing.get("matmul_ms"):
            achieved = timing["matmul_bytes"] / (timing["matmul_ms"] / 1000.0) / 1e9
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic_from_profiles(),
                    "kernel": f"decode matmuls of stage 0 (layers {ranges[0][0]}-{ranges[0][1]}), one micro-batch "
                              f"of {len(batches[0])} rows",
                    "launches": timing["matmul_launches"], "peak_source": peaks["source"]}
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": workload_name(args), "model": model_name(args),
                       "concurrency": C, "prompt_tokens": P, "output_tokens": O, "global_batch": C, "seq_len": P + O,
                       "parallelism": f"pp{world}", "stages": ranges, "micro_batches": [len(b) for b in batches],
                       "boundary": ("F16 codec in Stagewire v2 frames (device CRC-32) over NCCL send/recv (NVLink)"
                                    if args.frames == "stagewire" else "F16 codec over NCCL send/recv (NVLink)"),
                       "l2": "weights exceed L2 every decode step"},
            "ttft_p50_ms": round(float(lat[0].item()), 3), "itl_p50_ms": round(float(lat[1].item()), 4),
            "decode_tok_s": round(C / (float(lat[2].item()) / 1000.0), 1),
            "parity": parity,
            "e2e": e2e, "roofline": roof, "cpu_baseline": None, "clocks": clocks.summary(),
            "gpu_launches": int(float(launch_total.item()) / max(1, args.steps) * args.steps),
        }
    # A pinned host buffer that took part in a copy on the engine's stream
    # records an event on that stream when it is freed: free them all while
    # the stream still exists, before the engine closes it.
    torch.cuda.synchronize()
    pinned.clear()
    gc.collect()
    stage.close()
    eng.close()
    dist.barrier()
    dist.destroy_process_group()
    return result


def run_matmul_shape(args) -> dict:
    """The tcgen05 matmul alone on one weight shape: enough weight copies to
    exceed L2, `warmup` untimed then `steps` timed launches (CUDA events on
    the launching stream)."""
    import numpy as np
    import torch
    from jetsonfabric_b200 import jfm
    from jetsonfabric_b200 import kernels as K

    t, rows, cols = matmul_shapes(args.preset)[args.matmul_shape]
    n = args.matmul_rows
    raw = jfm.quantize_blocks(t, np.random.default_rng(args.seed).normal(0, 0.02, rows * cols).astype(np.float32))
    copies = max(1, int(np.ceil(256e6 / len(raw))))
    weights = [K.DeviceWeight(t, rows, cols, raw) for _ in range(copies)]
    q8 = K.Q8Buffer(n, cols)
    K.quantize_q8k(torch.randn(n, cols, device="cuda"), q8)
    out = torch.empty(n, rows, device="cuda")
    ws = torch.zeros(K.matmul_tc_workspace_bytes(rows, cols, n), dtype=torch.uint8, device="cuda")
    cuda_core = args.matmul_path == "cuda-core"

    def launch(wt):
        if cuda_core:
            K.matmul(wt, n, out, x_q8=q8)
        else:
            K.matmul_tc(wt, n, out, q8, ws)

    for i in range(max(args.warmup, 0)):
        launch(weights[i % copies])
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    for i in range(args.steps):
        ev[2 * i].record()
        launch(weights[i % copies])
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    us = sorted(ev[2 * i].elapsed_time(ev[2 * i + 1]) * 1000 for i in range(args.steps))
    med = us[len(us) // 2]
    return {"kernel": "jfb_matmul" if cuda_core else "jfb_matmul_tc", "shape": args.matmul_shape, "type": t, "rows": rows, "cols": cols, "n": n,
            "weight_bytes": len(raw), "launches": args.steps, "median_us": round(med, 2),
            "gbs": round(len(raw) / (med * 1e-6) / 1e9, 1), "l2": f"{copies} weight copies rotated"}


def run_attention_shape(args) -> dict:
    """jfb_attention alone on the preset's attention shape: random F16 KV
    caches for `concurrency` sequences with the preset's heads (head_dim
    128), Q8_K output fused. decode: one row per sequence at position
    prompt + output/2; prefill: every causal row of the prompt. `warmup`
    untimed then `steps` timed launches (CUDA events on the launching
    stream)."""
    import torch
    from jetsonfabric_b200 import kernels as K

    m = PRESETS[args.preset]
    heads, kvh, n_seq = m["head_count"], m["kv_head_count"], args.concurrency
    hd = m["embedding_length"] // heads
    ctx = args.prompt_tokens + args.output_tokens // 2 if args.attention_shape == "decode" else args.prompt_tokens
    rows_per_seq = 1 if args.attention_shape == "decode" else ctx
    kvd = kvh * hd
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    kb = torch.randn(n_seq, 1, ctx, kvd, device="cuda", generator=gen).half()
    vb = torch.randn(n_seq, 1, ctx, kvd, device="cuda", generator=gen).half()
    slots = (K.KvSlot * n_seq)()
    for i in range(n_seq):
        slots[i] = K.KvSlot(kb[i].data_ptr(), vb[i].data_ptr(), ctx, 0)
    slots_dev = torch.frombuffer(bytearray(bytes(slots)), dtype=torch.uint8).cuda()
    rows = [(s, p) for s in range(n_seq) for p in range(ctx - rows_per_seq, ctx)]
    n = len(rows)
    seq = torch.tensor([s for s, _ in rows], dtype=torch.int32, device="cuda")
    pos = torch.tensor([p for _, p in rows], dtype=torch.int32, device="cuda")
    q = torch.randn(n, heads * hd, device="cuda", generator=gen)
    scratch = torch.empty(K.attention_scratch_bytes(n, heads, hd, ctx), dtype=torch.uint8, device="cuda")
    out = torch.empty(n, heads * hd, device="cuda")
    q8 = K.Q8Buffer(n, heads * hd)
    for _ in range(max(args.warmup, 0)):
        K.attention(q, seq, pos, heads, kvh, hd, ctx, slots_dev, 0, scratch, out, out_q8=q8)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    for i in range(args.steps):
        ev[2 * i].record()
        K.attention(q, seq, pos, heads, kvh, hd, ctx, slots_dev, 0, scratch, out, out_q8=q8)
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    us = sorted(ev[2 * i].elapsed_time(ev[2 * i + 1]) * 1000 for i in range(args.steps))
    med = us[len(us) // 2]
    kv_bytes = sum(p + 1 for _, p in rows) * kvd * 2 * 2
    return {"kernel": "jfb_attention", "shape": args.attention_shape, "rows": n, "keys_max": ctx, "heads": heads,
            "kv_heads": kvh, "head_dim": hd, "launches": args.steps, "median_us": round(med, 2),
            "kv_bytes": kv_bytes, "kv_gbs": round(kv_bytes / (med * 1e-6) / 1e9, 1)}


def traffic_from_profiles():
    path = REPO / "profiles" / "decode_matmul_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------------
# CPU oracle (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------------

CPU_SAMPLE = {"sequences": 1, "prompt_tokens": 32, "output_tokens": 8}


def sample_prompt(args, vocab: int) -> list[int]:
    """The bounded sample: the first CPU_SAMPLE prompt tokens of sequence 0."""
    return prompts_for(args, vocab)[0, :CPU_SAMPLE["prompt_tokens"]].tolist()


class OracleRunner:
    """The CPU oracle over the whole model, loaded once, serving CPU_SAMPLE."""

    def __init__(self, pkg: Path, threads: int):
        from oracle import binding as ob
        ob.set_threads(threads)
        self.threads = threads
        self.stage = ob.OracleStage(pkg)

    def sample(self, prompt: list[int]) -> dict:
        O = CPU_SAMPLE["output_tokens"]
        s = self.stage.session(len(prompt) + O)
        t0 = time.perf_counter()
        tokens = [s.forward(True, tokens=prompt)["token"]]
        t1 = time.perf_counter()
        gaps = []
        for _ in range(O - 1):
            b = time.perf_counter()
            tokens.append(s.forward(False, tokens=[tokens[-1]])["token"])
            gaps.append(time.perf_counter() - b)
        seconds = time.perf_counter() - t0
        del s
        return {"seconds": seconds, "prefill_s": t1 - t0, "gaps_s": gaps, "tokens": tokens}

    def close(self):
        self.stage.close()


def cpu_line(args, res: dict, threads: int) -> dict:
    O, P = CPU_SAMPLE["output_tokens"], CPU_SAMPLE["prompt_tokens"]
    return {"value": round(O / res["seconds"], 4), "unit": UNIT, "cores": threads, "kind": "port",
            "prefill_tok_s": round(P / res["prefill_s"], 2),
            "decode_tok_s": round(1.0 / statistics.mean(res["gaps_s"]), 3) if res["gaps_s"] else None,
            "sample": f"sequence 0 of the {model_label(args.preset)} workload: its first {P} prompt tokens, "
                      f"{O} greedy output tokens, one sequence (CPU oracle, OpenMP over {threads} threads); "
                      "value = output tokens / wall time of the sample"}


def parity_line(gpu_tokens: list[int], cpu_tokens: list[int]) -> dict:
    return {"status": "ok" if gpu_tokens == cpu_tokens else "fail", "gpu_tokens": gpu_tokens,
            "oracle_tokens": cpu_tokens,
            "sample": f"sequence 0's first {CPU_SAMPLE['prompt_tokens']} prompt tokens, "
                      f"{CPU_SAMPLE['output_tokens']} greedy tokens through the benched engine vs the CPU oracle"}


def gpu_sample_tokens(eng, prompt: list[int]) -> list[int]:
    """CPU_SAMPLE through the benched single-stage engine (a fresh session)."""
    O = CPU_SAMPLE["output_tokens"]
    s = eng.create_session(len(prompt) + O)
    tokens = [s.prefill_greedy(prompt)]
    for _ in range(O - 1):
        tokens.append(s.decode_greedy(tokens[-1]))
    s.close()
    return tokens


def reference_full_workload(args, runner: "OracleRunner") -> dict:
    """One pass of the whole configured workload on the CPU oracle: every
    sequence's prompt, then output_tokens - 1 decode rounds over all
    sequences (the reference's CPU backend serving C concurrent requests on
    the host cores). Returns total seconds, time to the last first token, and
    the per-round gaps."""
    prompts = prompts_for(args, PRESETS[args.preset]["vocabulary_size"]).tolist()
    P, O = args.prompt_tokens, args.output_tokens
    sessions = [runner.stage.session(P + O) for _ in prompts]
    t0 = time.perf_counter()
    tokens = [[s.forward(True, tokens=p)["token"]] for s, p in zip(sessions, prompts)]
    ttft = time.perf_counter() - t0
    gaps = []
    for _ in range(O - 1):
        b = time.perf_counter()
        for s, tk in zip(sessions, tokens):
            tk.append(s.forward(False, tokens=[tk[-1]])["token"])
        gaps.append(time.perf_counter() - b)
    total = time.perf_counter() - t0
    del sessions
    return {"seconds": total, "ttft_s": ttft, "gaps_s": gaps}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    pkg = ensure_package(args, 0)
    threads = os.cpu_count() or 1
    runner = OracleRunner(pkg, threads)
    if args.cpu_full:
        for _ in range(max(args.warmup, 0)):
            reference_full_workload(args, runner)
        results = [reference_full_workload(args, runner) for _ in range(args.steps)]
        runner.close()
        seconds = statistics.mean(r["seconds"] for r in results)
        value = args.concurrency * args.output_tokens / seconds
        gaps = [g for r in results for g in r["gaps_s"]]
        return {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(seconds * 1000, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "impl": "reference",
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": workload_name(args), "model": model_name(args), "mode": "whole workload",
                       "note": "the reference's GGML CPU backend cannot be built offline, so its C restatement "
                               "(oracle/) serves every sequence end to end on the host cores"},
            "ttft_p50_ms": round(statistics.median(r["ttft_s"] for r in results) * 1000, 1),
            "itl_p50_ms": round(statistics.median(gaps) * 1000, 2) if gaps else None,
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"the whole {workload_name(args)} workload, every step"},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    prompt = sample_prompt(args, PRESETS[args.preset]["vocabulary_size"])
    for _ in range(max(args.warmup, 0)):
        runner.sample(prompt)
    results = [runner.sample(prompt) for _ in range(args.steps)]
    runner.close()
    seconds = statistics.mean(r["seconds"] for r in results)
    value = CPU_SAMPLE["output_tokens"] / seconds
    merged = {"seconds": seconds, "prefill_s": statistics.mean(r["prefill_s"] for r in results),
              "gaps_s": [g for r in results for g in r["gaps_s"]]}
    cpu = cpu_line(args, merged, threads)
    cpu["value"] = round(value, 4)
    return {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(seconds * 1000, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "impl": "reference",
        "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
        "config": {"workload": workload_name(args), "model": model_name(args), "sample": CPU_SAMPLE,
                   "note": "each step serves the bounded sample; the reference's GGML CPU backend cannot be built "
                           "offline, so its C restatement (oracle/) runs on the host cores"},
        "ttft_p50_ms": round(statistics.median(r["prefill_s"] for r in results) * 1000, 1),
        "itl_p50_ms": round(statistics.median(merged["gaps_s"]) * 1000, 1) if merged["gaps_s"] else None,
        "cpu_baseline": cpu,
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.attention_shape is not None:
        print(json.dumps(run_attention_shape(args)), flush=True)
        return
    if args.matmul_shape is not None:
        result = run_matmul_shape(args)
    elif args.impl == "reference":
        result = run_reference(args, rank)
    elif world > 1 and not args.replicas:
        result = run_pipeline(args, rank, world, local_rank)
    else:
        result = run_ours(args, rank, world, local_rank)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
