#!/usr/bin/env python
"""Aggregate decode throughput of the native Qwen2 Q4_K_M stage engine on B200.

Workload (configs[1] of the benchmark definition): Qwen2-architecture 3B
Q4_K_M (36 layers, hidden 2048, 16/2 heads, FFN 11008, vocabulary 151,936),
seeded N(0, 0.02) weights quantized with this repository's K-quant encoders,
32 concurrent requests of 512 uniform-random prompt tokens, 256 greedy output
tokens each. One "step" serves the whole batch: one batched prefill of all
prompts, then 255 batched decode steps. The weights (2.1 GB) are larger than
L2 (126 MB), so every decode step streams them from HBM.

    value      aggregate output tok/s, device-timed (CUDA events on the
               engine stream), prompts already resident in HBM
    e2e        the same workload through the engine's C ABI with host
               buffers: prompts copied in, every step's tokens copied in and
               the sampled tokens read back (wall clock)
    roofline   the decode matmuls (weight-streaming K-quant x Q8_K dot
               products, the dominant kernel family) of one decode step at
               the workload's batch, bytes / CUDA-event time vs measured HBM
    cpu_baseline  the CPU oracle (this repository's restatement of the
               reference's GGML-CPU path) on a bounded sample

--impl reference runs the CPU oracle on the host cores instead (the
reference's own native engine needs GGML, which cannot be built here).
With torchrun (N > 1) every rank serves its own full-model replica of the
workload on its GPU (weak scaling, no data-path collective); the value is
the tokens of all ranks over the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PRESETS = {
    "3b": dict(layer_count=36, embedding_length=2048, head_count=16, kv_head_count=2, feed_forward_length=11008,
               vocabulary_size=151936),
    "1.5b": dict(layer_count=28, embedding_length=1536, head_count=12, kv_head_count=2, feed_forward_length=8960,
                 vocabulary_size=151936),
    "7b": dict(layer_count=28, embedding_length=3584, head_count=28, kv_head_count=4, feed_forward_length=18944,
               vocabulary_size=152064),
}
METRIC = "aggregate decode tok/s + p50 ITL, Qwen2 Q4_K pipeline at 1/2/4/8 B200"
UNIT = "tok/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--preset", default="3b", choices=sorted(PRESETS))
    p.add_argument("--concurrency", type=int, default=32)
    p.add_argument("--prompt-tokens", type=int, default=512)
    p.add_argument("--output-tokens", type=int, default=256)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--package-dir", default=os.environ.get("JFB_BENCH_DIR", "/tmp/jfb_bench"))
    p.add_argument("--skip-e2e", action="store_true")
    p.add_argument("--skip-cpu", action="store_true")
    return p.parse_args()


def package_path(args) -> Path:
    return Path(args.package_dir) / f"qwen2-{args.preset}-q4km-seed{args.seed}.jfm"


def ensure_package(args, rank: int) -> Path:
    from jetsonfabric_b200 import jfm
    path = package_path(args)
    done = path / ".complete"
    if rank == 0 and not done.exists():
        path.mkdir(parents=True, exist_ok=True)
        ctx = max(4096, args.prompt_tokens + args.output_tokens)
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
    capacity = P + O - 1
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
        cpu = None if (args.skip_cpu or world > 1) else cpu_baseline(args, pkg)
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_k/q6_k x q8_k int8 dot, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": f"qwen2-{args.preset}-q4km c{C} p{P} o{O}", "model": f"Qwen2-arch {args.preset} Q4_K_M",
                       "layers": info.layer_count, "hidden": info.embedding_length, "concurrency": C,
                       "prompt_tokens": P, "output_tokens": O, "weight_bytes": info.weight_bytes,
                       "global_batch": C * world, "seq_len": P + O,
                       "parallelism": "replicas" if world > 1 else "single stage",
                       "l2": "weights (2.1 GB) exceed L2 every decode step"},
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

CPU_SAMPLE = {"sequences": 2, "prompt_tokens": 16, "output_tokens": 4}


def oracle_sample(pkg: Path, args, threads: int) -> tuple[float, float, list[float], float]:
    """Serves CPU_SAMPLE with the oracle; returns (seconds, ttft_ms, itl_ms list, tokens)."""
    import numpy as np
    from oracle import binding as ob
    ob.set_threads(threads)
    stage = ob.OracleStage(pkg)
    rng = np.random.default_rng(args.seed)
    n, P, O = CPU_SAMPLE["sequences"], CPU_SAMPLE["prompt_tokens"], CPU_SAMPLE["output_tokens"]
    t0 = time.perf_counter()
    ttft, gaps = [], []
    for _ in range(n):
        prompt = rng.integers(0, stage.vocab, P).tolist()
        s = stage.session(P + O)
        a = time.perf_counter()
        tok = s.forward(True, tokens=prompt)["token"]
        ttft.append((time.perf_counter() - a) * 1000)
        for _ in range(O - 1):
            b = time.perf_counter()
            tok = s.forward(False, tokens=[tok])["token"]
            gaps.append((time.perf_counter() - b) * 1000)
    seconds = time.perf_counter() - t0
    stage.close()
    return seconds, statistics.median(ttft), gaps, float(n * O)


def cpu_baseline(args, pkg: Path) -> dict:
    threads = os.cpu_count() or 1
    seconds, _, _, tokens = oracle_sample(pkg, args, threads)
    return {"value": round(tokens / seconds, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{CPU_SAMPLE['sequences']} sequences x {CPU_SAMPLE['prompt_tokens']} prompt tokens x "
                      f"{CPU_SAMPLE['output_tokens']} output tokens of the {args.preset} workload (oracle, OpenMP)"}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    pkg = ensure_package(args, 0)
    threads = os.cpu_count() or 1
    for _ in range(max(args.warmup, 0)):
        oracle_sample(pkg, args, threads)
    times, ttfts, gaps, toks = [], [], [], 0.0
    for _ in range(args.steps):
        s, t, g, n = oracle_sample(pkg, args, threads)
        times.append(s)
        ttfts.append(t)
        gaps.extend(g)
        toks = n
    seconds = statistics.mean(times)
    value = toks / seconds
    return {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(seconds * 1000, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_k/q6_k x q8_k int8 dot, f32 accumulate", "impl": "reference",
        "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
        "config": {"workload": f"qwen2-{args.preset}-q4km c{args.concurrency} p{args.prompt_tokens} o{args.output_tokens}",
                   "model": f"Qwen2-arch {args.preset} Q4_K_M", "sample": CPU_SAMPLE},
        "ttft_p50_ms": round(statistics.median(ttfts), 1), "itl_p50_ms": round(statistics.median(gaps), 1),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{CPU_SAMPLE} per step; the reference's GGML CPU backend cannot be built "
                                   "offline, so its C restatement (oracle/) runs"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        result = run_reference(args, rank)
    else:
        result = run_ours(args, rank, world, local_rank)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
