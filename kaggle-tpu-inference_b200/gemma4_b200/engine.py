"""Decode engine: the reference ``Engine`` API on top of the B200 decode step.

Same constructor, attributes and generator protocol as gemma4_tpu/engine.py:25-221:
``Engine(model_dir, max_len, batch, top_k, progress)``, ``compile_all()``,
``generate(prompt_ids, max_new_tokens, temperature, top_p, seed, stop_ids, lookahead)``
yielding ``prefill`` then ``decode`` events, ``reset_cache()``, ``prefill_fn(t)``,
``decode_fn()`` and ``_put``.

Devices: like the reference (``make_mesh`` over every device, model.py:159-161) an Engine
in a plain process owns every visible GPU as one tensor-parallel rank each, from one
host thread: the ranks' communicators address each other's exchange buffers directly
(``g4_comm_open_local``) and every step is launched on all devices in turn (the launches
are asynchronous, so the devices run the step together).  Under ``torchrun`` (an
initialised process group or RANK/WORLD_SIZE in the environment) each process owns its
own rank instead and the communicator handles travel over the process group.  An
explicit ``mesh`` (one rank) or ``devices`` list overrides both.

What changes underneath: the decode step is one captured CUDA graph of the C-ABI
kernels per device, replayed per token; a prompt goes through the tensor-core prefill
(``g4_prefill``, engine.py:57-69) on every rank, the ranks exchanging their partials
per layer under tensor parallelism; tokens never leave the device between steps and the host reads
token i from rank 0's mapped pinned mirror once step i's event has completed,
``lookahead`` steps behind the dispatch, like the reference's lookahead-3 loop
(engine.py:192-221).  ``temperature > 0`` samples on the device (model.py:414-424).
"""

from __future__ import annotations

import os
import threading
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


def _local_meshes(mesh: Mesh | None, devices) -> list[Mesh]:
    """The ranks this process owns: an explicit mesh; else the torchrun rank; else one
    rank per listed (or visible) device."""
    if mesh is not None:
        return [mesh]
    launched = False
    try:
        import torch.distributed as dist

        launched = dist.is_available() and dist.is_initialized()
    except ImportError:  # pragma: no cover
        pass
    if devices is None and (launched or int(os.environ.get("WORLD_SIZE", "1")) > 1):
        return [make_mesh()]
    if devices is None:
        devices = list(range(max(1, torch.cuda.device_count())))
    devices = list(devices)
    return [Mesh(r, len(devices), d) for r, d in enumerate(devices)]


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
        devices=None,
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
        self.meshes = _local_meshes(mesh, devices)
        self.mesh = self.meshes[0]
        self.n_devices = self.mesh.world
        self.device = torch.device("cuda", self.mesh.device)
        torch.cuda.set_device(self.device)

        t0 = time.time()
        shards = []
        for ms in self.meshes:
            dev = torch.device("cuda", ms.device)
            with torch.cuda.device(dev):
                if random_seed is not None:
                    shards.append(random_rank_shard(self.cfg, random_seed, ms, dev, random_std))
                elif params is not None:  # canonical tensors in host memory (tests, conversions)
                    shards.append(rank_shard(self.cfg, params.__getitem__, ms, dev))
                else:  # this rank's slices straight from the checkpoint's memory maps
                    shards.append(load_params(self.cfg, model_dir, ms, progress, dev))
                torch.cuda.synchronize(dev)
        self.load_seconds = time.time() - t0

        H = self.cfg.hidden_size
        if self.mesh.world == 1:
            self.comms = [None]
        elif len(self.meshes) == self.mesh.world:  # every rank in this process
            self.comms = Comm.local_group(self.meshes, H)
        else:  # one rank of a torchrun job
            self.comms = [Comm(self.mesh, H)]
        self.comm = self.comms[0]
        self.models = []
        for ms, shard, comm in zip(self.meshes, shards, self.comms):
            with torch.cuda.device(ms.device):
                self.models.append(DecodeModel(self.cfg, shard, ms, max_len, comm, engine=engine))
        self.model = self.models[0]
        self.params = shards[0]
        self.param_bytes = param_bytes(self.cfg)
        self.cache_bytes = cache_bytes(self.cfg, batch, max_len)
        self.active_params = active_params_per_token(self.cfg)
        self.decode_step_seconds = 0.0

    @property
    def cache(self) -> dict:
        return {"k": self.model.cache_k, "v": self.model.cache_v}

    def _all(self, fn):
        """fn(model) on every rank this process owns, each with its device current."""
        for m in self.models:
            with torch.cuda.device(m.device):
                fn(m)

    def _sync(self):
        for m in self.models:
            torch.cuda.current_stream(m.device).synchronize()

    def _check(self):
        for m in self.models:
            m.check_status()

    # ---------------------------------------------------------------- step fns
    def _step_fn(self, n_steps: int | None):
        """Callable with the reference's jitted-step signature (engine.py:60, 74)."""

        def fn(params, tokens, cache, pos, key=None, temperature=0.0, top_p=1.0):
            del params, cache
            seed = _seed_of(key)
            self._all(lambda m: m.set_sampling(float(temperature), float(top_p), self.top_k, seed))
            if n_steps is not None:  # prefill: tokens [1, T], pos = prompt length
                plen = int(pos)
                ids = tokens[0, :plen].tolist()
                self._all(lambda m: m.reset(ids))
                self._consume_prompt(plen)
                out_pos = plen
            else:                    # decode: token [1, 1] already in tokens_out at pos
                out_pos = int(pos) + 1
                self._all(lambda m: m.step(1))
            tok = self.model.tokens_out[out_pos:out_pos + 1].reshape(1, 1)
            return tok, self.cache, out_pos

        return fn

    def prefill_fn(self, t: int):
        return self._step_fn(t)

    def decode_fn(self):
        return self._step_fn(None)

    # ---------------------------------------------------------------- helpers
    def _all_threads(self, fn):
        """fn(model) on every rank this process owns, one host thread per rank when it owns
        several: a rank's launches that wait on its peers' exchange flags must not fill
        its device's launch queue (blocking the host) before the peers' launches exist."""
        if len(self.models) == 1:
            return self._all(fn)
        errors = []

        def run(m):
            try:
                with torch.cuda.device(m.device):
                    fn(m)
            except BaseException as e:  # re-raised on the calling thread
                errors.append(e)

        threads = [threading.Thread(target=run, args=(m,)) for m in self.models]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]

    def _consume_prompt(self, n: int):
        """The prompt through the model: one tensor-core prefill (engine.py:57-69) on every
        rank (under tensor parallelism the ranks exchange their partials per layer), or
        ``n`` forced decode steps when the engine was built with ``prefill=False``."""
        if self.use_prefill:
            self._all_threads(lambda m: m.prefill(n, self.prefill_chunk))
        else:
            self._all(lambda m: m.step(n))

    def reset_cache(self):
        for m in self.models:
            for t in m.cache_k + m.cache_v:
                t.zero_()

    def _put(self, value, dtype=torch.int32):
        return torch.as_tensor(value, dtype=dtype, device=self.device)

    def compile_all(self, bucket: int = PREFILL_BUCKET) -> dict[str, float]:
        """Capture the step graphs, warm them up and time blocking decode steps."""
        out = {}
        t0 = time.perf_counter()

        def first(m):
            m.set_sampling(0.0, 1.0, self.top_k, 0)
            m.reset([0, 0, 0, 0])
            m.step(1, use_graph=False)   # first launch configures the kernels

        self._all(first)
        self._all(lambda m: m.capture())
        if self.use_prefill:
            # one prefill of the largest chunk this engine uses: the tensor-core prefill
            # allocates its workspace and configures its kernels here, not in a request's TTFT
            n = min(self.max_len - 1, self.prefill_chunk or 4096)
            self._all(lambda m: m.reset([0] * n))
            self._all_threads(lambda m: m.prefill(n, self.prefill_chunk))
            self._sync()
            self._check()
            self._all(lambda m: m.reset([0, 0, 0, 0]))  # the warm-up decode steps start near the cache start
        self._sync()
        out["prefill_compile_s"] = time.perf_counter() - t0
        t0 = time.perf_counter()
        self._all(lambda m: m.step(3))
        self._sync()
        out["decode_compile_s"] = time.perf_counter() - t0
        n = 8
        t0 = time.perf_counter()
        for _ in range(n):
            self._all(lambda m: m.step(1))
        self._sync()
        self.decode_step_seconds = (time.perf_counter() - t0) / n
        out["decode_step_s"] = self.decode_step_seconds
        self._check()
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
        lead = self.model
        host = lead.tokens_host
        ids = list(prompt_ids)

        self._all(lambda m: m.set_sampling(float(temperature), float(top_p), self.top_k, int(seed)))
        t_start = time.perf_counter()
        self._all(lambda m: m.reset(ids))
        self._consume_prompt(p_len)
        self._sync()
        self._check()
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
            self._all(lambda m: m.step(1))
            with torch.cuda.device(lead.device):
                ev = torch.cuda.Event()
                ev.record()
            pos += 1
            pending.append((ev, pos))
            yield from drain(lookahead)
            if stopped:
                break
        if not stopped:
            yield from drain(0)
        self._sync()
        self._check()
