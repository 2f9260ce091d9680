"""Pipeline-parallel greedy generation over contiguous layer ranges.

The reference splits a Qwen2 model into stages by contiguous layer ranges
(the first stage also owns token_embd, the last owns output_norm, output and
the argmax) and moves activations between stage workers over Stagewire with
the F16 activation codec (runtime/activation/builtin_activation_codecs.cpp:
51-206; the stage contract is native_inference.hpp:127-163 and
native_stage_executor.cpp:143-180). Here one process drives one stage on one
GPU:

  - the boundary carries the F16 codec of the f32 activations [rows, hidden]
    point to point to the next stage, which decodes it back to f32;
  - the last stage sends each micro-batch's greedy tokens back to the first
    stage, which feeds them into the next decode step;
  - the sequences are split into micro-batches so that, with at least as
    many micro-batches as stages, every stage is busy on a different
    micro-batch at the same time.

Every rank runs the same (step, micro-batch) sequence, so the messages of a
link always match in order. The activation links (rank r -> r+1) and the
token link (last -> first) are separate communicators: NCCL runs the point-
to-point operations of one communicator in order on its own stream, and with
a shared communicator the first stage's next activation send could wait
behind the token receive that it is itself needed for.

The compute of a stage and the transport are pluggable: `EngineStage` drives
a device-resident `NativeEngine` stage over NCCL (the benchmark path),
`HostEngineStage` the host-buffer C ABI, and the tests drive the CPU oracle
over gloo with the same schedule.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Protocol, Sequence

import numpy as np


def stage_ranges(layer_count: int, stages: int) -> list[tuple[int, int]]:
    """Even split of [0, layer_count) into `stages` contiguous ranges; the
    first `layer_count % stages` ranges get one layer more."""
    if stages < 1 or stages > layer_count:
        raise ValueError("stage count must be between 1 and the layer count")
    base, extra = divmod(layer_count, stages)
    out, start = [], 0
    for s in range(stages):
        end = start + base + (1 if s < extra else 0)
        out.append((start, end))
        start = end
    return out


def split_batches(sequences: int, micro_batches: int) -> list[list[int]]:
    """Sequences 0..n-1 in `micro_batches` contiguous groups of near-equal size."""
    if micro_batches < 1 or micro_batches > sequences:
        raise ValueError("micro-batch count must be between 1 and the sequence count")
    base, extra = divmod(sequences, micro_batches)
    out, start = [], 0
    for m in range(micro_batches):
        size = base + (1 if m < extra else 0)
        out.append(list(range(start, start + size)))
        start += size
    return out


class Stage(Protocol):
    """One pipeline stage: `forward` consumes the input of micro-batch `m`
    (token ids on the first stage, the decoded boundary activations
    elsewhere) and returns greedy tokens (last stage) or f32 activations."""

    first: bool
    last: bool
    hidden: int

    def forward(self, m: int, prefill: bool, inputs): ...

    def encode(self, activations, out=None): ...  # f32 -> F16 codec payload to send (into `out` if given)

    def decode(self, payload): ...  # F16 codec payload -> f32 stage input

    def empty_payload(self, rows: int): ...

    def empty_tokens(self, count: int): ...

    def prompt_tokens(self, m: int): ...


class Link(Protocol):
    def send_activation(self, stage, activations) -> None: ...  # encode and send to the next stage

    def recv_activation(self, stage, rows: int): ...  # the next F16 payload from the previous stage

    def send_next(self, payload) -> None: ...

    def recv_prev(self, payload) -> None: ...

    def send_tokens(self, tokens) -> None: ...

    def recv_tokens(self, tokens) -> None: ...

    def flush(self) -> None: ...


class TorchLink:
    """Point-to-point links over torch.distributed.

    `groups` holds one two-rank group per activation link (rank r, r + 1) and
    one for the token link (last, first); every rank must create all of them
    in the same order (see `make_groups`). Works for NCCL with CUDA tensors
    (operations ordered against the current CUDA stream) and for gloo with
    CPU tensors. Sends are asynchronous; each handle (and its buffer) is
    kept until the send has completed, and dropped at the next send after
    that, so a long schedule holds only the sends still in flight; `flush`
    waits for the rest."""

    def __init__(self, rank: int, world: int, groups: dict):
        import torch.distributed as dist

        self.dist = dist
        self.rank, self.world = rank, world
        self.next_group = groups.get(("act", rank))
        self.prev_group = groups.get(("act", rank - 1))
        self.tok_group = groups.get("tok")
        self.pending = []

    def _drop_completed(self) -> None:
        # never blocks: a send that has not completed stays pending
        self.pending = [(w, buf) for w, buf in self.pending if not w.is_completed()]

    def send_activation(self, stage, activations) -> None:
        self.send_next(stage.encode(activations))

    def recv_activation(self, stage, rows: int):
        payload = stage.empty_payload(rows)
        self.recv_prev(payload)
        return payload

    def send_next(self, payload) -> None:
        self._drop_completed()
        self.pending.append((self.dist.isend(payload, self.rank + 1, group=self.next_group), payload))

    def recv_prev(self, payload) -> None:
        self.dist.irecv(payload, self.rank - 1, group=self.prev_group).wait()

    def send_tokens(self, tokens) -> None:
        self._drop_completed()
        self.pending.append((self.dist.isend(tokens, 0, group=self.tok_group), tokens))

    def recv_tokens(self, tokens) -> None:
        self.dist.irecv(tokens, self.world - 1, group=self.tok_group).wait()

    def flush(self) -> None:
        for work, _ in self.pending:
            work.wait()
        self.pending.clear()


def make_groups(world: int, backend: str | None = None, timeout_s: float | None = None) -> dict:
    """The two-rank groups of `TorchLink`, created collectively by every rank.
    `timeout_s` bounds every operation on them (a peer that never posts the
    matching operation ends the wait with an error instead of a hang)."""
    import datetime

    import torch.distributed as dist

    groups = {}
    if world < 2:
        return groups
    kw = {} if timeout_s is None else {"timeout": datetime.timedelta(seconds=timeout_s)}
    for r in range(world - 1):
        groups[("act", r)] = dist.new_group([r, r + 1], backend=backend, **kw)
    groups["tok"] = dist.new_group([world - 1, 0], backend=backend, **kw)
    return groups


def warm_groups(rank: int, world: int, groups: dict, device=None) -> None:
    """Initialises every communicator of `make_groups` before the schedule
    starts: each rank joins a one-element all-reduce on each group it belongs
    to, in creation order (links 0-1, 1-2, ..., then last-first), an order in
    which no rank waits on a peer that waits on it."""
    import torch
    import torch.distributed as dist

    members = {("act", r): (r, r + 1) for r in range(world - 1)}
    members["tok"] = (world - 1, 0)
    for key in [("act", r) for r in range(world - 1)] + ["tok"]:
        if key in groups and rank in members[key]:
            t = torch.zeros(1, device=device) if device is not None else torch.zeros(1)
            dist.all_reduce(t, group=groups[key])


@dataclass
class ScheduleResult:
    tokens: dict  # sequence index -> generated token ids (last stage only)


def run_schedule(rank: int, world: int, batches: Sequence[Sequence[int]], prompt_lengths: Sequence[int],
                 steps: int, stage: Stage, link: Link | None,
                 on_output: Callable[[int, int, object], None] | None = None) -> ScheduleResult:
    """Prefill of every micro-batch, then `steps - 1` decode steps, in
    (step, micro-batch) order on every rank. The last stage calls
    `on_output(step, m, tokens)` after each micro-batch (the tokens may still
    be device-resident and in flight)."""
    first, last = rank == 0, rank == world - 1
    results = {s: [] for mb in batches for s in mb}
    carry = [None] * len(batches)  # single-stage: tokens of the previous step
    for step in range(steps):
        prefill = step == 0
        for m, mb in enumerate(batches):
            rows = sum(prompt_lengths[s] for s in mb) if prefill else len(mb)
            if first:
                if prefill:
                    inputs = stage.prompt_tokens(m)
                elif world == 1:
                    inputs = carry[m]
                else:
                    inputs = stage.empty_tokens(len(mb))
                    link.recv_tokens(inputs)
            else:
                inputs = stage.decode(link.recv_activation(stage, rows))
            out = stage.forward(m, prefill, inputs)
            if last:
                if on_output is not None:
                    on_output(step, m, out)
                results_tokens = out
                if world == 1:
                    carry[m] = out
                elif step + 1 < steps:
                    link.send_tokens(out)
                for i, s in enumerate(mb):
                    results[s].append((results_tokens, i))
            else:
                link.send_activation(stage, out)
    if link is not None:
        link.flush()
    return ScheduleResult(tokens=results)


def collect_tokens(result: ScheduleResult) -> dict:
    """Host token ids per sequence from a last-stage schedule result."""
    out = {}
    for s, entries in result.tokens.items():
        ids = []
        for buf, i in entries:
            host = buf.cpu().numpy() if hasattr(buf, "cpu") else np.asarray(buf)
            ids.append(int(host[i]))
        out[s] = ids
    return out


class EngineStage:
    """A device-resident NativeEngine stage for `run_schedule`.

    Sessions of all sequences live on this stage's engine; inputs, outputs
    and boundary payloads are CUDA tensors, and every operation runs on the
    engine's stream (the caller enters `torch.cuda.stream(stage.stream)` so
    that NCCL orders its transfers against it)."""

    def __init__(self, engine, prompts: Sequence[Sequence[int]], batches: Sequence[Sequence[int]],
                 capacity: int):
        import torch

        from . import kernels

        self.torch, self.kernels = torch, kernels
        self.engine = engine
        info = engine.model_info()
        self.first = info.resident_layer_start == 0
        self.last = info.resident_layer_end == info.layer_count
        self.hidden = info.embedding_length
        self.batches = [list(mb) for mb in batches]
        self.prompts = [list(p) for p in prompts]
        self.capacity = capacity
        self.sessions = [engine.create_session(capacity) for _ in prompts]
        self.handles = [engine._handles([self.sessions[s] for s in mb]) for mb in self.batches]
        self.stream = torch.cuda.ExternalStream(engine.stream())
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        with torch.cuda.stream(self.stream):
            self.prompt_dev = [torch.tensor([t for s in mb for t in self.prompts[s]], dtype=torch.int32, device=dev)
                               for mb in self.batches]
        self.counts = [[len(self.prompts[s]) for s in mb] for mb in self.batches]

    def reset(self) -> None:
        for s in self.sessions:
            s.reset()

    def close(self) -> None:
        for s in self.sessions:
            s.close()

    def prompt_tokens(self, m: int):
        return self.prompt_dev[m]

    def empty_tokens(self, count: int):
        return self.torch.empty(count, dtype=self.torch.int32, device=self.device)

    def empty_payload(self, rows: int):
        return self.torch.empty((rows, self.hidden), dtype=self.torch.float16, device=self.device)

    def encode(self, activations, out=None):
        payload = out if out is not None else self.torch.empty(activations.shape, dtype=self.torch.float16,
                                                                device=self.device)
        self.kernels.codec_f32_to_f16(activations, payload, stream=self.stream)
        return payload

    def decode(self, payload):
        act = self.torch.empty(payload.shape, dtype=self.torch.float32, device=self.device)
        self.kernels.codec_f16_to_f32(payload, act, stream=self.stream)
        return act

    def forward(self, m: int, prefill: bool, inputs):
        mb = self.batches[m]
        rows = sum(self.counts[m]) if prefill else len(mb)
        torch = self.torch
        tokens_out = acts_out = None
        if self.last:
            tokens_out = torch.empty(len(mb), dtype=torch.int32, device=self.device)
        else:
            acts_out = torch.empty((rows, self.hidden), dtype=torch.float32, device=self.device)
        self.engine.stage_batch_device(
            [self.sessions[s] for s in mb], prefill, self.counts[m] if prefill else None,
            tokens_ptr=inputs.data_ptr() if self.first else 0,
            activations_ptr=0 if self.first else inputs.data_ptr(),
            tokens_out_ptr=tokens_out.data_ptr() if self.last else 0,
            activations_out_ptr=0 if self.last else acts_out.data_ptr(),
            handles=self.handles[m])
        return tokens_out if self.last else acts_out


class HostEngineStage(EngineStage):
    """The same stage through the host-buffer C ABI (prefill_stage_batch /
    decode_stage_batch with host activations), the reference-facing calls a
    Stagewire worker makes; inputs and outputs are host arrays and the
    boundary payload is a CPU tensor of F16 codec bits."""

    def __init__(self, engine, prompts, batches, capacity):
        super().__init__(engine, prompts, batches, capacity)

    def prompt_tokens(self, m: int):
        return [self.prompts[s] for s in self.batches[m]]

    def empty_tokens(self, count: int):
        return self.torch.empty(count, dtype=self.torch.int32)

    def empty_payload(self, rows: int):
        return self.torch.empty((rows, self.hidden), dtype=self.torch.float16)

    def encode(self, activations, out=None):
        payload = self.torch.from_numpy(np.ascontiguousarray(activations, dtype=np.float32).astype(np.float16))
        if out is None:
            return payload
        out.copy_(payload)
        return out

    def decode(self, payload):
        return payload.numpy().astype(np.float32)

    def forward(self, m: int, prefill: bool, inputs):
        mb = self.batches[m]
        sessions = [self.sessions[s] for s in mb]
        if self.first:
            if prefill:
                res = self.engine.prefill_stage_batch(sessions, inputs)
            else:
                res = self.engine.decode_stage_batch(sessions, [int(t) for t in np.asarray(inputs).ravel()])
        else:
            x = np.asarray(inputs, dtype=np.float32)
            if prefill:
                parts, row = [], 0
                for n in self.counts[m]:
                    parts.append(x[row:row + n])
                    row += n
                res = self.engine.prefill_stage_batch_activations(sessions, parts)
            else:
                res = self.engine.decode_stage_batch_activations(sessions, x)
        if self.last:
            return self.torch.tensor([r.sampled_token for r in res], dtype=self.torch.int32)
        return np.concatenate([r.activation.reshape(-1, self.hidden) for r in res], axis=0)
