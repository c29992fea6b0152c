#!/usr/bin/env python3
"""Persistent inference daemon over a Unix socket, on the B200 Engine.

The reference's daemon (gemma4_tpu/server.py:47-190, client side session.py:158-196)
loads the weights once, warms the step programs up once and then streams generations to
clients as JSON lines; this module keeps that protocol so existing clients work:

  request (one JSON line)            reply (JSON lines)
  {"cmd": "ping"}                    {"kind": "pong"}
  {"cmd": "status"}                  {"kind": "status", pid, model, uptime_s, requests,
                                      busy, max_len, decode_step_ms}
  {"cmd": "shutdown"}                {"kind": "bye"}, then the daemon stops
  {"prompt": "...", ...} or          {"kind": "info", ...}, {"kind": "prompt", ...},
  {"prompt_ids": [...], ...}         optional {"kind": "limit", ...} / {"kind": "error"},
    max_new_tokens, temperature,     {"kind": "prefill", token, ttft, prompt_tokens, ...},
    top_p, seed                      {"kind": "token", token, text, ...} ..., {"kind": "done"}

One generation runs at a time (a second concurrent request gets {"kind": "error",
"message": "daemon busy"} and "done"), as in the reference (server.py:117-138).  Text
prompts need a tokenizer (HF AutoTokenizer from the model directory, chat template
applied); ``prompt_ids`` requests need none.  The channel splitting, TPU monitor and
dashboard of the reference's session layer are outside the decode path and not carried.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import threading
import time
import traceback
from typing import Iterator

from .limits import MAX_OUTPUT_TOKENS, allowed_output_tokens

SOCKET_PATH = os.environ.get("GEMMA4_SOCKET", "/tmp/gemma4-b200.sock")


def log(msg: str):
    print(f"[{time.strftime('%H:%M:%S')}] {msg}", flush=True)


def model_info(engine, model_id: str, served_by: str | None = None) -> dict:
    """The "info" event (reference session.py:51-71)."""
    cfg = engine.cfg
    kv_bytes = sum(2 * 2 * cfg.kv_heads_for(lt) * cfg.head_dim_for(lt) for lt in cfg.layer_types)
    return {"kind": "info", "model": model_id, "param_bytes": engine.param_bytes,
            "active_params": engine.active_params, "cache_bytes": engine.cache_bytes,
            "max_len": engine.max_len, "n_devices": engine.n_devices,
            "num_layers": cfg.num_hidden_layers,
            "sliding_layers": sum(1 for x in cfg.layer_types if x == "sliding_attention"),
            "full_layers": sum(1 for x in cfg.layer_types if x == "full_attention"),
            "hidden_size": cfg.hidden_size, "vocab_size": cfg.vocab_size,
            "num_experts": cfg.num_experts, "top_k_experts": cfg.top_k_experts,
            "kv_bytes_per_token": kv_bytes, "decode_step_s": engine.decode_step_seconds,
            "max_output_tokens": MAX_OUTPUT_TOKENS, "served_by": served_by}


def prompt_ids_of(tok, request: dict) -> list[int]:
    """Token ids of a request: ``prompt_ids`` as given, or the chat-templated ``prompt``."""
    if "prompt_ids" in request:
        return [int(t) for t in request["prompt_ids"]]
    if tok is None:
        raise ValueError("a text prompt needs a tokenizer; send prompt_ids")
    messages = ([{"role": "system", "content": request["system"]}] if request.get("system") else [])
    messages.append({"role": "user", "content": request["prompt"]})
    enc = tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True,
                                  enable_thinking=request.get("think", True))
    ids = enc["input_ids"] if hasattr(enc, "keys") else enc
    while ids and isinstance(ids[0], list):
        ids = ids[0]
    return [int(t) for t in ids]


def generate_events(engine, tok, request: dict, info: dict) -> Iterator[dict]:
    """One generation's event stream (the protocol of reference session.py:85-155)."""
    ids = prompt_ids_of(tok, request)
    requested = max(1, int(request.get("max_new_tokens", 768)))
    allowed = allowed_output_tokens(requested, len(ids), engine.max_len)
    yield {**info, "requested_max_new_tokens": requested, "allowed_max_new_tokens": allowed}
    yield {"kind": "prompt", "text": request.get("prompt", ""), "tokens": len(ids)}
    if allowed < 1:
        yield {"kind": "error",
               "message": f"prompt uses {len(ids)} tokens and fills the {engine.max_len}-token context"}
        yield {"kind": "done"}
        return
    if allowed != requested:
        yield {"kind": "limit", "requested": requested, "allowed": allowed, "prompt_tokens": len(ids),
               "context_tokens": engine.max_len}
    stop = set(engine.cfg.eos_token_ids)
    for ev in engine.generate(ids, max_new_tokens=allowed, temperature=float(request.get("temperature", 1.0)),
                              top_p=float(request.get("top_p", 0.95)), seed=int(request.get("seed", 0))):
        tid = ev["token"]
        text = "" if tok is None or tid in stop else tok.decode([tid])
        out = {"kind": "prefill" if ev["kind"] == "prefill" else "token", "t": ev["t"], "token": tid,
               "text": text}
        if ev["kind"] == "prefill":
            out["ttft"] = ev["ttft"]
            out["prompt_tokens"] = ev["prompt_tokens"]
        yield out
    yield {"kind": "done"}


class Daemon:
    def __init__(self, engine, model_id: str, path: str = SOCKET_PATH, tokenizer=None, warm: bool = True):
        self.engine = engine
        self.model_id = model_id
        self.path = path
        self.tok = tokenizer
        self.lock = threading.Lock()
        self.requests = 0
        self.started = time.time()
        self._stop = threading.Event()
        self.ready = threading.Event()
        if warm:
            ct = engine.compile_all()
            log(f"step graphs captured; decode step {1000 * ct['decode_step_s']:.2f} ms")

    def info(self) -> dict:
        return model_info(self.engine, self.model_id, served_by=f"daemon pid {os.getpid()} ({self.path})")

    def status(self) -> dict:
        return {"kind": "status", "pid": os.getpid(), "model": self.model_id,
                "uptime_s": round(time.time() - self.started, 1), "requests": self.requests,
                "busy": self.lock.locked(), "max_len": self.engine.max_len,
                "max_output_tokens": MAX_OUTPUT_TOKENS,
                "decode_step_ms": round(1000 * self.engine.decode_step_seconds, 2)}

    def handle(self, conn: socket.socket):
        conn.settimeout(600.0)
        f = conn.makefile("rw")

        def send(obj):
            f.write(json.dumps(obj) + "\n")
            f.flush()

        try:
            line = f.readline()
            if not line.strip():
                return
            req = json.loads(line)
            cmd = req.get("cmd")
            if cmd == "ping":
                return send({"kind": "pong"})
            if cmd == "status":
                return send(self.status())
            if cmd == "shutdown":
                send({"kind": "bye"})
                self._stop.set()
                return
            if not self.lock.acquire(blocking=False):
                send({"kind": "error", "message": "daemon busy"})
                return send({"kind": "done"})
            try:
                self.requests += 1
                for ev in generate_events(self.engine, self.tok, req, self.info()):
                    send(ev)
            except (BrokenPipeError, ConnectionResetError):
                log("client disconnected mid-generation")
            except Exception:
                log(traceback.format_exc())
                try:
                    send({"kind": "error", "message": "generation failed"})
                    send({"kind": "done"})
                except OSError:
                    pass
            finally:
                self.lock.release()
        finally:
            try:
                f.close()
            except OSError:
                pass
            conn.close()

    def serve_forever(self):
        if os.path.exists(self.path):
            os.unlink(self.path)
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        srv.bind(self.path)
        os.chmod(self.path, 0o600)
        srv.listen(8)
        srv.settimeout(0.2)
        self.ready.set()
        log(f"READY listening on {self.path}")
        try:
            while not self._stop.is_set():
                try:
                    conn, _ = srv.accept()
                except socket.timeout:
                    continue
                threading.Thread(target=self.handle, args=(conn,), daemon=True).start()
        finally:
            srv.close()
            if os.path.exists(self.path):
                os.unlink(self.path)
            log("stopped")


# ------------------------------------------------------------------------ client
def daemon_alive(path: str = SOCKET_PATH, timeout: float = 2.0) -> bool:
    if not os.path.exists(path):
        return False
    try:
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
            s.settimeout(timeout)
            s.connect(path)
            s.sendall(json.dumps({"cmd": "ping"}).encode() + b"\n")
            return bool(s.makefile("r").readline())
    except OSError:
        return False


def remote_events(request: dict, path: str = SOCKET_PATH) -> Iterator[dict]:
    """Stream a generation request's events from the daemon."""
    with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
        s.settimeout(600.0)
        s.connect(path)
        s.sendall(json.dumps(request).encode() + b"\n")
        with s.makefile("r") as f:
            for line in f:
                if line.strip():
                    ev = json.loads(line)
                    yield ev
                    if ev["kind"] == "done":
                        return


def send_command(cmd: str, path: str = SOCKET_PATH, timeout: float = 5.0) -> dict | None:
    try:
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
            s.settimeout(timeout)
            s.connect(path)
            s.sendall(json.dumps({"cmd": cmd}).encode() + b"\n")
            line = s.makefile("r").readline()
            return json.loads(line) if line.strip() else None
    except OSError:
        return None


def main() -> int:
    from .engine import Engine

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--model", default="google/gemma-4-26B-A4B-it")
    ap.add_argument("--model-dir", required=True)
    ap.add_argument("--max-len", type=int, default=32768)
    ap.add_argument("--top-k", type=int, default=64)
    ap.add_argument("--socket", default=SOCKET_PATH)
    args = ap.parse_args()
    log(f"loading {args.model} from {args.model_dir}")
    t0 = time.time()
    engine = Engine(args.model_dir, max_len=args.max_len, top_k=args.top_k)
    log(f"weights on {engine.n_devices} GPU(s) in {time.time() - t0:.1f}s")
    tok = None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(args.model_dir)
    except Exception as exc:  # token-id requests still work
        log(f"no tokenizer ({exc!r}); serving prompt_ids requests only")
    Daemon(engine, args.model, args.socket, tok).serve_forever()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
