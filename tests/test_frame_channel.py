"""The in-box frame channel (`jfb_frame_channel_*`, include/jfb/jfb_stagewire.h)
under the in-box StageTransport: request/reply hand-off, bounded waits,
capacity limits, a server that closes, a caller that gave up, and two
processes. CPU only: the channel is shared memory and futexes."""
from __future__ import annotations

import multiprocessing as mp
import os
import threading
import time

import pytest

from jetsonfabric_b200 import engine
from jetsonfabric_b200.stagewire import ChannelTimeout, FrameChannel


def _name(tag: str) -> str:
    return f"jfbtest-{tag}-{os.getpid()}-{time.monotonic_ns() % 1_000_000}"


def test_round_trips_in_order():
    name = _name("rt")
    with FrameChannel.create(name, capacity=1 << 16) as server:
        assert server.capacity == 1 << 16

        def serve():
            for _ in range(50):
                req = server.receive(timeout_ms=5000)
                server.reply(200, True, b"ack:" + req[:8], req[8:][::-1])

        t = threading.Thread(target=serve)
        t.start()
        with FrameChannel.open(name) as caller:
            for i in range(50):
                head, body = f"{i:08d}".encode(), os.urandom(i * 37)
                status, is_frame, reply = caller.call(head, body)
                assert status == 200 and is_frame
                assert reply == b"ack:" + head + body[::-1]
        t.join()


def test_json_error_replies_and_empty_frames():
    name = _name("err")
    with FrameChannel.create(name, capacity=4096) as server:
        def serve():
            server.receive()
            server.reply(401, False, b'{"error":"runtime_auth_failed","message":"no"}')
            assert server.receive() == b""
            server.reply(200, True, b"")

        t = threading.Thread(target=serve)
        t.start()
        with FrameChannel.open(name) as caller:
            assert caller.call(b"x") == (401, False, b'{"error":"runtime_auth_failed","message":"no"}')
            assert caller.call(b"") == (200, True, b"")
        t.join()


def test_limits_and_names():
    name = _name("lim")
    with FrameChannel.create(name, capacity=4096) as server:
        with pytest.raises(engine.InvalidArgument):  # the name is taken
            FrameChannel.create(name)
        with FrameChannel.open(name) as caller:
            with pytest.raises(engine.InvalidArgument):  # larger than the channel
                caller.call(b"h" * 100, b"b" * 4096)
        # a reply too large for the mailbox becomes a 502 error body
        def serve():
            server.receive()
            server.reply(200, True, b"r" * 5000)

        t = threading.Thread(target=serve)
        t.start()
        with FrameChannel.open(name) as caller:
            status, is_frame, reply = caller.call(b"q")
            assert status == 502 and not is_frame and b"runtime_stage_reply_too_large" in reply
        t.join()
    for bad in ("", "a/b", "x" * 201, "sp ace"):
        with pytest.raises(engine.InvalidArgument):
            FrameChannel.create(bad)
    with pytest.raises(engine.NativeExecutionError):  # nobody serves it
        FrameChannel.open(_name("absent"), timeout_ms=50)


def test_abandoned_request_and_late_reply():
    """A caller that times out leaves its request; the server's late reply is
    dropped by the next caller, which gets its own answer."""
    name = _name("late")
    with FrameChannel.create(name, capacity=4096) as server:
        with FrameChannel.open(name) as caller:
            with pytest.raises(ChannelTimeout):
                caller.call(b"first", timeout_ms=100)
            assert server.receive(timeout_ms=1000) == b"first"
            server.reply(200, True, b"late answer")

            def serve():
                req = server.receive(timeout_ms=5000)
                server.reply(200, True, b"answer to " + req)

            t = threading.Thread(target=serve)
            t.start()
            assert caller.call(b"second") == (200, True, b"answer to second")
            t.join()
        with pytest.raises(ChannelTimeout):  # no request pending
            server.receive(timeout_ms=50)


def test_server_close_wakes_a_waiting_caller():
    name = _name("close")
    server = FrameChannel.create(name, capacity=4096)
    caller = FrameChannel.open(name)
    errors = []

    def call():
        try:
            caller.call(b"never answered", timeout_ms=10000)
        except Exception as e:  # noqa: BLE001 - the error type is what the test checks
            errors.append(e)

    t = threading.Thread(target=call)
    t.start()
    assert server.receive(timeout_ms=5000) == b"never answered"
    t0 = time.monotonic()
    server.close()
    t.join(timeout=10)
    assert not t.is_alive() and time.monotonic() - t0 < 5
    assert len(errors) == 1 and isinstance(errors[0], engine.NativeExecutionError)
    assert "closed" in str(errors[0])
    caller.close()


def _serve_process(name: str, count: int, ready) -> None:
    with FrameChannel.create(name, capacity=1 << 20) as server:
        ready.set()
        for _ in range(count):
            req = server.receive(timeout_ms=20000)
            server.reply(200, True, req.upper())


def test_two_processes():
    name = _name("proc")
    ctx = mp.get_context("spawn")
    ready = ctx.Event()
    p = ctx.Process(target=_serve_process, args=(name, 20, ready))
    p.start()
    try:
        assert ready.wait(60)
        with FrameChannel.open(name, timeout_ms=10000) as caller:
            for i in range(20):
                body = bytes([97 + i % 26]) * (1000 * i)
                assert caller.call(b"frame-", body, timeout_ms=20000) == (200, True, b"FRAME-" + body.upper())
    finally:
        p.join(timeout=60)
    assert p.exitcode == 0


def _create_and_vanish(name: str) -> None:
    FrameChannel.create(name, capacity=4096)
    os._exit(0)  # exits without closing: the name stays behind


def _call_and_hang(name: str, started) -> None:
    with FrameChannel.open(name) as caller:
        started.set()
        caller.call(b"from a caller that will be killed", timeout_ms=60000)


def test_stale_server_name_and_dead_caller_are_taken_over():
    ctx = mp.get_context("spawn")
    name = _name("stale")
    p = ctx.Process(target=_create_and_vanish, args=(name,))
    p.start()
    p.join(60)
    assert p.exitcode == 0
    with FrameChannel.create(name, capacity=4096) as server:  # the dead server's name is reclaimed
        started = ctx.Event()
        hung = ctx.Process(target=_call_and_hang, args=(name, started))
        hung.start()
        assert started.wait(60)
        assert server.receive(timeout_ms=10000) == b"from a caller that will be killed"
        hung.kill()  # this test's own child, by its exact handle, while it holds the channel
        hung.join(30)

        def serve():
            server.reply(200, True, b"stale reply")  # the dead caller's answer
            req = server.receive(timeout_ms=10000)
            server.reply(200, True, b"fresh " + req)

        t = threading.Thread(target=serve)
        t.start()
        with FrameChannel.open(name) as caller:
            assert caller.call(b"call", timeout_ms=10000) == (200, True, b"fresh call")
        t.join()
