"""The daemon on the real B200 Engine (tiny parity model on cuda:0): a token-id request over
the Unix socket streams the same greedy tokens as Engine.generate called directly, and a
sampled request with a seed is reproducible across requests."""
import os
import tempfile
import threading

import pytest
import torch

from gemma4_b200.config import tiny_parity_config
from gemma4_b200.engine import Engine
from gemma4_b200.model import Mesh
from gemma4_b200.server import Daemon, remote_events, send_command
from gemma4_b200.weights import random_params

pytestmark = pytest.mark.gpu


def test_daemon_streams_engine_tokens():
    cfg = tiny_parity_config()
    eng = Engine(None, max_len=128, cfg=cfg, params=random_params(cfg, 0), mesh=Mesh(0, 1, 0))
    path = os.path.join(tempfile.mkdtemp(prefix="g4d"), "s.sock")
    dm = Daemon(eng, "tiny", path)
    th = threading.Thread(target=dm.serve_forever, daemon=True)
    th.start()
    assert dm.ready.wait(30)
    try:
        prompt = list(range(11, 40))
        req = {"prompt_ids": prompt, "max_new_tokens": 12, "temperature": 0.0}
        evs = list(remote_events(req, path))
        got = [e["token"] for e in evs if e["kind"] in ("prefill", "token")]
        want = [e["token"] for e in eng.generate(prompt, 12, temperature=0.0, stop_ids=())]
        stop = set(cfg.eos_token_ids)
        cut = next((i + 1 for i, t in enumerate(want) if t in stop), len(want))
        assert got == want[:cut]
        s1 = [e["token"] for e in remote_events({**req, "temperature": 1.0, "seed": 9}, path) if "token" in e]
        s2 = [e["token"] for e in remote_events({**req, "temperature": 1.0, "seed": 9}, path) if "token" in e]
        assert s1 == s2
    finally:
        send_command("shutdown", path)
        th.join(30)
        torch.cuda.synchronize()
