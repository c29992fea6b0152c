"""Decode engine: the reference ``Engine`` API on top of the B200 decode step.

Same constructor, attributes and generator protocol as gemma4_tpu/engine.py:25-221:
``Engine(model_dir, max_len, batch, top_k, progress)``, ``compile_all()``,
``generate(prompt_ids, max_new_tokens, temperature, top_p, seed, stop_ids, lookahead)``
yielding ``prefill`` then ``decode`` events, ``reset_cache()``, ``prefill_fn(t)``,
``decode_fn()`` and ``_put``.

What changes underneath: each rank owns one GPU (``torchrun`` for tensor parallelism,
rank/world from torch.distributed or the launcher env); the step is one captured CUDA
graph of the C-ABI kernels, replayed per token; a prompt is consumed by the same step
as forced tokens; tokens never leave the device between steps and the host reads
token i from a mapped pinned mirror once step i's event has completed, ``lookahead``
steps behind the dispatch, like the reference's lookahead-3 loop (engine.py:192-221).
"""

from __future__ import annotations

import time
from collections import deque
from typing import Iterator

import torch

from .config import TextConfig, load_text_config
from .limits import allowed_output_tokens
from .model import Mesh, cache_bytes, make_mesh
from .runtime import Comm, DecodeModel
from .weights import active_params_per_token, load_params, param_bytes, rank_shard, random_rank_shard

PREFILL_BUCKET = 256


def _seed_of(key) -> int:
    """The sampling seed of a step fn's ``key`` argument (an int, a 1-element tensor or
    array, or None = 0); the reference passes a JAX PRNG key built from the seed."""
    if key is None:
        return 0
    try:
        return int(key)
    except (TypeError, ValueError):
        import numpy as np

        return int(np.asarray(key).ravel()[-1])


def _round_up(x: int, m: int) -> int:
    return max(m, ((x + m - 1) // m) * m)


class Engine:
    def __init__(
        self,
        model_dir: str | None,
        max_len: int = 4096,
        batch: int = 1,
        top_k: int = 64,
        progress=None,
        *,
        cfg: TextConfig | None = None,
        params: dict | None = None,
        random_seed: int | None = None,
        random_std: float = 0.02,
        mesh: Mesh | None = None,
        engine: str = "step",
        prefill: bool = True,
        prefill_chunk: int = 0,
    ):
        if not 1 <= top_k <= 128:
            raise ValueError(f"top_k must be in [1, 128] on the B200 sampler, got {top_k}")
        if batch != 1:
            raise NotImplementedError("the B200 decode path runs batch 1 (engine.py:167 fills row 0)")
        self.model_dir = model_dir
        self.cfg: TextConfig = cfg if cfg is not None else load_text_config(model_dir)
        self.max_len = max_len
        self.batch = batch
        self.top_k = top_k
        self.use_prefill = prefill
        self.prefill_chunk = prefill_chunk
        self.mesh = mesh or make_mesh()
        self.n_devices = self.mesh.world
        self.device = torch.device("cuda", self.mesh.device)
        torch.cuda.set_device(self.device)

        t0 = time.time()
        if random_seed is not None:
            shard = random_rank_shard(self.cfg, random_seed, self.mesh, self.device, random_std)
        else:
            canon = params if params is not None else load_params(self.cfg, model_dir, progress)
            shard = rank_shard(self.cfg, canon.__getitem__, self.mesh, self.device)
            del canon
        torch.cuda.synchronize(self.device)
        self.load_seconds = time.time() - t0

        self.comm = Comm(self.mesh, self.cfg.hidden_size) if self.mesh.world > 1 else None
        self.model = DecodeModel(self.cfg, shard, self.mesh, max_len, self.comm, engine=engine)
        self.params = shard
        self.param_bytes = param_bytes(self.cfg)
        self.cache_bytes = cache_bytes(self.cfg, batch, max_len)
        self.active_params = active_params_per_token(self.cfg)
        self.decode_step_seconds = 0.0

    @property
    def cache(self) -> dict:
        return {"k": self.model.cache_k, "v": self.model.cache_v}

    # ---------------------------------------------------------------- step fns
    def _step_fn(self, n_steps: int | None):
        """Callable with the reference's jitted-step signature (engine.py:60, 74)."""

        def fn(params, tokens, cache, pos, key=None, temperature=0.0, top_p=1.0):
            del params, cache
            m = self.model
            m.set_sampling(float(temperature), float(top_p), self.top_k, _seed_of(key))
            if n_steps is not None:  # prefill: tokens [1, T], pos = prompt length
                plen = int(pos)
                m.reset(tokens[0, :plen].tolist())
                self._consume_prompt(plen)
                out_pos = plen
            else:                    # decode: token [1, 1] already in tokens_out at pos
                out_pos = int(pos) + 1
                m.step(1)
            tok = m.tokens_out[out_pos:out_pos + 1].reshape(1, 1)
            return tok, self.cache, out_pos

        return fn

    def prefill_fn(self, t: int):
        return self._step_fn(t)

    def decode_fn(self):
        return self._step_fn(None)

    # ---------------------------------------------------------------- helpers
    def _consume_prompt(self, n: int):
        """The prompt through the model: one tensor-core prefill (engine.py:57-69) when
        the library has it for this model (world 1), else ``n`` decode steps."""
        if not (self.use_prefill and self.model.prefill(n, self.prefill_chunk)):
            self.model.step(n)

    def reset_cache(self):
        for t in self.model.cache_k + self.model.cache_v:
            t.zero_()

    def _put(self, value, dtype=torch.int32):
        return torch.as_tensor(value, dtype=dtype, device=self.device)

    def compile_all(self, bucket: int = PREFILL_BUCKET) -> dict[str, float]:
        """Capture the step graph, warm it up and time blocking decode steps."""
        out = {}
        m = self.model
        t0 = time.perf_counter()
        m.set_sampling(0.0, 1.0, self.top_k, 0)
        m.reset([0, 0, 0, 0])
        m.step(1, use_graph=False)   # first launch configures the kernels
        m.capture()
        torch.cuda.synchronize(self.device)
        out["prefill_compile_s"] = time.perf_counter() - t0
        t0 = time.perf_counter()
        m.step(3)
        torch.cuda.synchronize(self.device)
        out["decode_compile_s"] = time.perf_counter() - t0
        n = 8
        t0 = time.perf_counter()
        m.step(n)
        torch.cuda.synchronize(self.device)
        self.decode_step_seconds = (time.perf_counter() - t0) / n
        out["decode_step_s"] = self.decode_step_seconds
        m.check_status()
        return out

    # ---------------------------------------------------------------- generation
    def generate(
        self,
        prompt_ids: list[int],
        max_new_tokens: int = 512,
        temperature: float = 1.0,
        top_p: float = 0.95,
        seed: int = 0,
        stop_ids: tuple[int, ...] | None = None,
        lookahead: int = 3,
    ) -> Iterator[dict]:
        """Yield one event per generated token (engine.py:143-221 protocol)."""
        stop = set(stop_ids if stop_ids is not None else self.cfg.eos_token_ids)
        p_len = len(prompt_ids)
        if self.max_len - p_len < 1:
            raise ValueError(f"prompt({p_len}) fills the resident context ({self.max_len})")
        max_new_tokens = allowed_output_tokens(max_new_tokens, p_len, self.max_len)
        bucket = min(_round_up(p_len, PREFILL_BUCKET), self.max_len)
        m = self.model
        host = m.tokens_host

        m.set_sampling(float(temperature), float(top_p), self.top_k, int(seed))
        t_start = time.perf_counter()
        m.reset(prompt_ids)
        self._consume_prompt(p_len)
        torch.cuda.current_stream(self.device).synchronize()
        m.check_status()
        first = int(host[p_len])
        ttft = time.perf_counter() - t_start
        yield {"kind": "prefill", "token": first, "ttft": ttft, "prompt_tokens": p_len,
               "prefill_bucket": bucket, "t": time.perf_counter()}
        if first in stop:
            return

        pending: deque = deque()
        emitted = 1
        pos = p_len  # position consumed by the next step
        stopped = False

        def drain(keep: int):
            nonlocal emitted, stopped
            while len(pending) > keep:
                ev, out_pos = pending.popleft()
                ev.synchronize()
                value = int(host[out_pos])
                emitted += 1
                yield {"kind": "decode", "token": value, "index": emitted - 1,
                       "t": time.perf_counter(), "total_tokens": emitted}
                if value in stop:
                    stopped = True
                    return

        for _ in range(max_new_tokens - 1):
            m.step(1)
            ev = torch.cuda.Event()
            ev.record()
            pos += 1
            pending.append((ev, pos))
            yield from drain(lookahead)
            if stopped:
                break
        if not stopped:
            yield from drain(0)
        torch.cuda.current_stream(self.device).synchronize()
        m.check_status()
