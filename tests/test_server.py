"""The daemon's Unix-socket protocol (gemma4_b200.server; reference gemma4_tpu/server.py
and the client side of session.py) with a stand-in engine on the CPU: ping / status /
shutdown, a token-id generation streamed as JSON lines (info, prompt, prefill, token...,
done), the context limit and over-long prompts, a text prompt without a tokenizer
reported as an error, and the one-generation-at-a-time lock ("daemon busy").  The GPU
test of the real Engine behind the daemon is in test_gpu_server.py."""
import os
import tempfile
import threading
import time

import pytest

from gemma4_b200.config import tiny_parity_config
from gemma4_b200.server import Daemon, daemon_alive, remote_events, send_command


class FakeEngine:
    """Enough of the Engine API for the daemon: generate() yields token events."""

    def __init__(self, delay=0.0):
        self.cfg = tiny_parity_config()
        self.max_len, self.n_devices, self.param_bytes = 64, 1, 1000
        self.active_params, self.cache_bytes, self.decode_step_seconds = 10, 100, 0.0
        self.delay = delay
        self.calls = []

    def compile_all(self):
        return {"prefill_compile_s": 0.0, "decode_compile_s": 0.0, "decode_step_s": 0.001}

    def generate(self, prompt_ids, max_new_tokens=512, temperature=1.0, top_p=0.95, seed=0, **kw):
        self.calls.append((list(prompt_ids), max_new_tokens, temperature, top_p, seed))
        for i in range(max_new_tokens):
            time.sleep(self.delay)
            ev = {"kind": "prefill" if i == 0 else "decode", "token": 100 + i, "t": time.perf_counter()}
            if i == 0:
                ev.update(ttft=0.01, prompt_tokens=len(prompt_ids))
            yield ev


@pytest.fixture
def daemon():
    d = tempfile.mkdtemp(prefix="g4d")
    path = os.path.join(d, "s.sock")
    eng = FakeEngine(delay=0.02)
    dm = Daemon(eng, "tiny", path)
    th = threading.Thread(target=dm.serve_forever, daemon=True)
    th.start()
    assert dm.ready.wait(10)
    yield dm, path
    send_command("shutdown", path)
    th.join(10)
    assert not th.is_alive() and not os.path.exists(path)


def test_commands(daemon):
    dm, path = daemon
    assert daemon_alive(path)
    st = send_command("status", path)
    assert st["kind"] == "status" and st["model"] == "tiny" and st["busy"] is False


def test_generation_stream(daemon):
    dm, path = daemon
    evs = list(remote_events({"prompt_ids": [1, 2, 3], "max_new_tokens": 5, "temperature": 0.0, "seed": 7}, path))
    kinds = [e["kind"] for e in evs]
    assert kinds == ["info", "prompt", "prefill", "token", "token", "token", "token", "done"]
    assert evs[0]["allowed_max_new_tokens"] == 5 and evs[1]["tokens"] == 3
    assert [e["token"] for e in evs[2:7]] == [100, 101, 102, 103, 104]
    assert dm.engine.calls[-1] == ([1, 2, 3], 5, 0.0, 0.95, 7)


def test_limits_and_errors(daemon):
    dm, path = daemon
    evs = list(remote_events({"prompt_ids": list(range(60)), "max_new_tokens": 10}, path))
    assert [e["kind"] for e in evs][:3] == ["info", "prompt", "limit"] and evs[2]["allowed"] == 4
    evs = list(remote_events({"prompt_ids": list(range(64)), "max_new_tokens": 10}, path))
    assert [e["kind"] for e in evs] == ["info", "prompt", "error", "done"]
    evs = list(remote_events({"prompt": "hello"}, path))  # no tokenizer loaded
    assert [e["kind"] for e in evs] == ["error", "done"]


def test_busy(daemon):
    dm, path = daemon
    first = []
    th = threading.Thread(target=lambda: first.extend(remote_events({"prompt_ids": [1], "max_new_tokens": 40},
                                                                    path)))
    th.start()
    time.sleep(0.3)
    second = list(remote_events({"prompt_ids": [1], "max_new_tokens": 2}, path))
    th.join(30)
    assert second == [{"kind": "error", "message": "daemon busy"}, {"kind": "done"}]
    assert first[-1]["kind"] == "done" and len(first) == 40 + 3
