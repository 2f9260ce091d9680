"""Pipeline-parallel schedule on CPU: gloo ranks, each running the CPU oracle
over its contiguous layer range, must produce exactly the tokens of one
process that chains the same stages with the F16 activation codec at every
boundary (the reference pipeline's Stagewire hop).

This covers the host side of the multi-GPU path, which the benchmark drives
with the engine over NCCL:
- the even layer split;
- micro-batching;
- message order on the activation and token links (world sizes 2, 3 and 4,
  more and fewer micro-batches than stages).
"""
from __future__ import annotations

import json
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from jetsonfabric_b200 import pipeline  # noqa: E402


def test_stage_ranges_and_batches():
    assert pipeline.stage_ranges(36, 2) == [(0, 18), (18, 36)]
    assert pipeline.stage_ranges(36, 8) == [(0, 5), (5, 10), (10, 15), (15, 20), (20, 24), (24, 28), (28, 32),
                                            (32, 36)]
    assert pipeline.stage_ranges(4, 3) == [(0, 2), (2, 3), (3, 4)]
    assert pipeline.split_batches(32, 3) == [list(range(0, 11)), list(range(11, 22)), list(range(22, 32))]
    with pytest.raises(ValueError):
        pipeline.stage_ranges(4, 5)
    with pytest.raises(ValueError):
        pipeline.split_batches(2, 3)


class OracleScheduleStage:
    """The CPU oracle as a `pipeline.Stage`: host arrays, one oracle session
    per sequence, boundary payloads as CPU float16 tensors."""

    def __init__(self, stage, prompts, batches, capacity):
        self.stage, self.prompts, self.batches = stage, prompts, batches
        self.sessions = [stage.session(capacity) for _ in prompts]
        self.first, self.last, self.hidden = stage.first, stage.last, stage.hidden

    def prompt_tokens(self, m):
        return [self.prompts[s] for s in self.batches[m]]

    def empty_tokens(self, count):
        return torch.empty(count, dtype=torch.int32)

    def empty_payload(self, rows):
        return torch.empty((rows, self.hidden), dtype=torch.float16)

    def encode(self, activations, out=None):
        payload = torch.from_numpy(np.ascontiguousarray(activations, dtype=np.float32).astype(np.float16))
        if out is None:
            return payload
        out.copy_(payload)
        return out

    def decode(self, payload):
        return payload.numpy().astype(np.float32)

    def forward(self, m, prefill, inputs):
        mb = self.batches[m]
        outs, row = [], 0
        for i, s in enumerate(mb):
            sess = self.sessions[s]
            if self.first:
                tokens = list(inputs[i]) if prefill else [int(np.asarray(inputs)[i])]
                r = sess.forward(prefill, tokens=tokens)
            else:
                n = len(self.prompts[s]) if prefill else 1
                r = sess.forward(prefill, activations=np.asarray(inputs)[row:row + n])
                row += n
            outs.append(r)
        if self.last:
            return torch.tensor([r["token"] for r in outs], dtype=torch.int32)
        return np.concatenate([r["activations"] for r in outs], axis=0)


class _CorruptingLink(pipeline.TorchLink):
    """Flips one payload byte of the `nth` activation message it sends (a
    wire fault planted on the host)."""

    def __init__(self, rank, world, groups, nth, offset):
        super().__init__(rank, world, groups)
        self.nth, self.offset, self.count = nth, offset, 0

    def send_next(self, payload) -> None:
        if self.count == self.nth:
            payload[self.offset] ^= 0x5A
        self.count += 1
        super().send_next(payload)


def _rank_main(rank, world, port, package, prompts, micro, steps, out_path, framed=False, corrupt=-1):
    import torch.distributed as dist
    from oracle import binding as ob

    from jetsonfabric_b200 import stagewire

    ob.set_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        groups = pipeline.make_groups(world)
        pipeline.warm_groups(rank, world, groups)
        meta = ob.OracleStage(package)
        layers = meta.model.layer_count
        hidden = meta.hidden
        meta.close()
        ranges = pipeline.stage_ranges(layers, world)
        start, end = ranges[rank]
        batches = pipeline.split_batches(len(prompts), micro)
        if corrupt >= 0:
            link = _CorruptingLink(rank, world, groups, corrupt, 1024 + 3)
        else:
            link = pipeline.TorchLink(rank, world, groups)
        if framed:
            plan = stagewire.FramePlan(model_id="small-q4k", stage_layers=ranges, batches=batches,
                                       prompt_lengths=[len(p) for p in prompts], steps=steps, hidden=hidden)
            link = stagewire.StagewireLink(link, rank, plan)
        stage = ob.OracleStage(package, start, end)
        capacity = max(len(p) for p in prompts) + steps
        sched = OracleScheduleStage(stage, prompts, batches, capacity)
        try:
            res = pipeline.run_schedule(rank, world, batches, [len(p) for p in prompts], steps, sched, link)
        except stagewire.StagewireError as e:
            with open(f"{out_path}.rank{rank}.err", "w") as f:
                f.write(f"{type(e).__name__}: {e}")
            res = None
        if rank == world - 1 and res is not None:
            with open(out_path, "w") as f:
                json.dump({str(k): v for k, v in pipeline.collect_tokens(res).items()}, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _chained_reference(package, prompts, world, steps):
    """One process: stage 0 -> F16 codec -> stage 1 -> ... per sequence."""
    from oracle import binding as ob

    meta = ob.OracleStage(package)
    layers = meta.model.layer_count
    meta.close()
    stages = [ob.OracleStage(package, a, b) for a, b in pipeline.stage_ranges(layers, world)]
    capacity = max(len(p) for p in prompts) + steps
    out = {}
    for s, prompt in enumerate(prompts):
        sessions = [st.session(capacity) for st in stages]
        tokens, feed = [], list(prompt)
        for step in range(steps):
            prefill = step == 0
            x = None
            for k, sess in enumerate(sessions):
                r = sess.forward(prefill, tokens=feed) if k == 0 else sess.forward(prefill, activations=x)
                if k + 1 < len(sessions):
                    x = r["activations"].astype(np.float16).astype(np.float32)
                else:
                    tokens.append(r["token"])
            feed = [tokens[-1]]
        out[s] = tokens
    return out


@pytest.mark.parametrize("world,micro", [(2, 2), (2, 3), (3, 2), (4, 4)])
def test_pipeline_matches_chained_stages(small_q4k_package, tmp_path, world, micro):
    import torch.multiprocessing as mp

    rng = np.random.default_rng(world * 10 + micro)
    prompts = [rng.integers(0, 1024, n).tolist() for n in (7, 3, 12, 5, 9)]
    steps = 6
    out_path = tmp_path / "tokens.json"
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    mp.spawn(_rank_main, args=(world, _free_port(), str(small_q4k_package), prompts, micro, steps, str(out_path)),
             nprocs=world, join=True)
    got = {int(k): v for k, v in json.loads(out_path.read_text()).items()}
    ref = _chained_reference(small_q4k_package, prompts, world, steps)
    assert got == ref
    assert all(len(v) == steps for v in got.values())


@pytest.mark.parametrize("world,micro", [(2, 3), (3, 2), (4, 4)])
def test_pipeline_over_stagewire_frames(small_q4k_package, tmp_path, world, micro):
    """Every activation and returned token as a Stagewire v2 frame (host
    checksums on gloo): same tokens as the chained reference, and every
    received frame passes the decoder's rules at the end of the schedule."""
    import torch.multiprocessing as mp

    rng = np.random.default_rng(world * 7 + micro)
    prompts = [rng.integers(0, 1024, n).tolist() for n in (6, 11, 4, 8)]
    steps = 5
    out_path = tmp_path / "tokens.json"
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    mp.spawn(_rank_main, args=(world, _free_port(), str(small_q4k_package), prompts, micro, steps, str(out_path),
                               True), nprocs=world, join=True)
    assert not list(tmp_path.glob("*.err"))
    got = {int(k): v for k, v in json.loads(out_path.read_text()).items()}
    assert got == _chained_reference(small_q4k_package, prompts, world, steps)


def test_stagewire_frame_corruption_is_detected(small_q4k_package, tmp_path):
    """A payload byte flipped on the wire: the receiving stage's checksum
    check fails the run when the schedule is verified."""
    import torch.multiprocessing as mp

    prompts = [[1, 2, 3, 4], [5, 6, 7]]
    out_path = tmp_path / "tokens.json"
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    mp.spawn(_rank_main, args=(2, _free_port(), str(small_q4k_package), prompts, 2, 3, str(out_path), True, 2),
             nprocs=2, join=True)
    errs = {p.name: p.read_text() for p in tmp_path.glob("*.err")}
    assert list(errs) == ["tokens.json.rank1.err"], errs
    assert errs["tokens.json.rank1.err"].startswith("ChecksumMismatch")


def test_eight_stage_framed_pipeline(tmp_path):
    """Eight gloo ranks, one layer each, eight micro-batches, every message a
    Stagewire frame: the schedule the 8-GPU benchmark runs, checked against the
    chained stages."""
    import torch.multiprocessing as mp

    from jetsonfabric_b200 import jfm

    package = tmp_path / "eight.jfm"
    jfm.write_synthetic_package(package, layer_count=8, embedding_length=256, head_count=2, kv_head_count=1,
                                feed_forward_length=512, vocabulary_size=512, context_length=128, seed=11,
                                draw_norms=True, draw_biases=True)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 512, n).tolist() for n in (5, 3, 6, 2, 4, 7, 3, 5)]
    steps = 4
    out_path = tmp_path / "tokens.json"
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    mp.spawn(_rank_main, args=(8, _free_port(), str(package), prompts, 8, steps, str(out_path), True),
             nprocs=8, join=True)
    assert not list(tmp_path.glob("*.err"))
    got = {int(k): v for k, v in json.loads(out_path.read_text()).items()}
    assert got == _chained_reference(package, prompts, 8, steps)
