"""Device Stagewire v2 checksums (include/jfb/jfb_stagewire.h) and the framed
stage link on CUDA tensors.

- jfb_crc32 must equal zlib.crc32 (Go's crc32.ChecksumIEEE, the checksum of
  the reference's frame.go:221,272) bit for bit: empty, tiny, ragged, chunk
  boundary, unaligned and multi-level (hundreds of MB) inputs;
- the stamp writes the field the host codec decodes, and the check flags a
  wrong or malformed field without touching a correct one;
- a frame sent through StagewireLink on the device decodes with the host
  codec's full rules, and a payload byte flipped in flight is reported.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from jetsonfabric_b200 import kernels
    return kernels


def _device_crc(K, t, scratch=None) -> int:
    n = t.numel() * t.element_size()
    if scratch is None:
        scratch = torch.empty(K.crc32_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    K.crc32(t, out, scratch)
    return int(out.item()) & 0xFFFFFFFF


@pytest.mark.parametrize("n", [0, 1, 2, 15, 16, 17, 63, 64, 65, 1023, 1024, 1025, 4099, 65536, 458752,
                               (1 << 20) + 7, 58 * (1 << 20) + 333])
def test_crc32_matches_zlib(K, n):
    host = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8)
    dev = torch.from_numpy(host).cuda()
    assert _device_crc(K, dev) == zlib.crc32(host.tobytes())


def test_crc32_large_and_unaligned(K):
    n = 300 * (1 << 20) + 5
    dev = torch.randint(0, 256, (n + 16,), dtype=torch.uint8, device="cuda")
    host = dev.cpu().numpy()
    assert _device_crc(K, dev[:n]) == zlib.crc32(host[:n].tobytes())
    for off in (1, 3, 8):
        m = 1_000_003
        assert _device_crc(K, dev[off:off + m]) == zlib.crc32(host[off:off + m].tobytes())


def test_crc32_rejects_small_scratch(K):
    from jetsonfabric_b200.engine import InvalidArgument

    dev = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(InvalidArgument, match="scratch"):
        K.crc32(dev, out, torch.empty(16, dtype=torch.uint8, device="cuda"))


def test_stamp_and_check(K):
    for value in (0, 7, 1234567, 0xFFFFFFFF):
        crc = torch.tensor([value - (1 << 32) if value >= 1 << 31 else value], dtype=torch.int32, device="cuda")
        frame = torch.full((64,), ord("#"), dtype=torch.uint8, device="cuda")
        K.stagewire_stamp_crc(crc, frame, 20)
        got = bytes(frame.cpu().numpy())
        assert got[20:30] == f"{value:>10d}".encode() and got[:20] == b"#" * 20 and got[30:] == b"#" * 34
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        K.stagewire_check_crc(crc, frame, 20, flag)
        assert int(flag.item()) == 0
        other = crc + 1
        K.stagewire_check_crc(other, frame, 20, flag)
        assert int(flag.item()) == 1
    frame = torch.frombuffer(bytearray(b"   12x4567"), dtype=torch.uint8).cuda()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.stagewire_check_crc(torch.tensor([124567], dtype=torch.int32, device="cuda"), frame, 0, flag)
    assert int(flag.item()) == 1


class _Loopback:
    """A base link whose sends are the next receives (one process holds both
    ends), optionally flipping a byte of the `corrupt`-th message."""

    def __init__(self, corrupt=-1):
        self.q, self.corrupt, self.count = [], corrupt, 0

    def send_next(self, frame):
        frame = frame.clone()
        if self.count == self.corrupt:
            frame[-5] ^= 0x21
        self.count += 1
        self.q.append(frame)

    send_tokens = send_next

    def recv_prev(self, frame):
        frame.copy_(self.q.pop(0))

    recv_tokens = recv_prev

    def flush(self):
        pass


class _Codec:
    def __init__(self, K, hidden):
        self.K, self.hidden = K, hidden

    def encode(self, activations, out=None):
        self.K.codec_f32_to_f16(activations, out)
        return out


@pytest.mark.parametrize("corrupt", [-1, 3])
def test_framed_link_on_device(K, corrupt):
    from jetsonfabric_b200 import stagewire as sw

    hidden, batches, lengths, steps = 256, [[0, 1], [2]], [7, 5, 9], 3
    plan = sw.FramePlan(model_id="m", stage_layers=[(0, 2), (2, 4)], batches=batches, prompt_lengths=lengths,
                        steps=steps, hidden=hidden)
    base = _Loopback(corrupt)
    tx = sw.StagewireLink(base, 0, plan, device="cuda")
    rx = sw.StagewireLink(base, 1, plan, device="cuda")
    stage = _Codec(K, hidden)
    g = torch.Generator(device="cuda").manual_seed(5)
    for step in range(steps):
        for m in range(len(batches)):
            rows = plan.rows(step, m)
            act = torch.randn((rows, hidden), device="cuda", generator=g)
            tx.send_activation(stage, act)
            got = rx.recv_activation(stage, rows)
            if base.count - 1 != corrupt:
                assert torch.equal(got, act.half())
    # the frames on the wire decode with the host codec
    for k in range(len(rx.expect)):
        pre = bytes(rx.recv_log[k].cpu().numpy())
        meta_len, payload_len = sw.parse_prefix(pre)
        assert sw.HEADER_SIZE + meta_len == 1024 and payload_len == rx.expect[k][2]
    if corrupt < 0:
        tx.flush()
        rx.flush()
        assert rx.sent == rx.received == 0
    else:
        tx.flush()
        with pytest.raises(sw.ChecksumMismatch):
            rx.flush()


def test_framed_tokens_on_device(K):
    from jetsonfabric_b200 import stagewire as sw

    plan = sw.FramePlan(model_id="m", stage_layers=[(0, 1), (1, 2)], batches=[[0, 1, 2]], prompt_lengths=[3, 3, 3],
                        steps=3, hidden=8)
    base = _Loopback()
    last = sw.StagewireLink(base, 1, plan, device="cuda")
    first = sw.StagewireLink(base, 0, plan, device="cuda")
    for step in range(2):
        toks = torch.tensor([11 + step, 151935, 0], dtype=torch.int32, device="cuda")
        last.send_tokens(toks)
        out = torch.empty(3, dtype=torch.int32, device="cuda")
        first.recv_tokens(out)
        assert torch.equal(out, toks)
    assert first.verify() == 2
    tokens = np.array([12, 151935, 0], dtype=np.uint32).tobytes()
    frame = sw.unmarshal(bytes(first.recv_log[1].cpu().numpy()) + tokens)
    assert frame.metadata.payload_kind == "sampled_tokens" and frame.metadata.decode_step == 2
