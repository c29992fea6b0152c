"""One rank's native decode model: device buffers, KV cache, communicator, CUDA graph.

``DecodeModel`` owns the per-rank state the C ABI needs (control block, token rings,
logits shard, KV cache per layer) and forwards the packed weight shards to
``g4_model_set_tensor``.  A decode step consumes the token at ``control[POS]`` and
writes the argmax of the next-token logits to ``tokens_out[pos + 1]``; prompts are
consumed by the same step ("forced" tokens taken from ``tokens_in``).

``Comm`` wraps ``g4_comm``: for world > 1 the 64-byte CUDA IPC handles of every rank's
exchange buffer are swapped through the torch.distributed process group (host
plumbing only); the all-reduces themselves are peer stores inside the kernels.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N
from .config import TextConfig
from .model import Mesh, local_cache_shapes


HANDLE_BYTES = 64  # one CUDA IPC memory handle


def exchange_handles(mine: bytes, world: int, group=None) -> bytes:
    """Every rank's exchange-buffer handle, concatenated in rank order (the layout
    ``g4_comm_open`` expects), swapped through the torch.distributed process group."""
    import torch.distributed as dist

    if len(mine) != HANDLE_BYTES:
        raise ValueError(f"an IPC handle is {HANDLE_BYTES} bytes, got {len(mine)}")
    allh: list = [None] * world
    dist.all_gather_object(allh, mine, group=group)
    if any(h is None or len(h) != HANDLE_BYTES for h in allh):
        raise RuntimeError("a rank sent no valid IPC handle")
    return b"".join(allh)


class Comm:
    def __init__(self, mesh: Mesh, hidden: int, group=None, _local: bool = False):
        L = N.lib()
        self.mesh = mesh
        self.handle = ctypes.c_void_p()
        N.check(L.g4_comm_create(mesh.device, mesh.rank, mesh.world, hidden, ctypes.byref(self.handle)),
                "g4_comm_create")
        if mesh.world > 1 and not _local:
            import torch.distributed as dist

            buf = ctypes.create_string_buffer(HANDLE_BYTES)
            N.check(L.g4_comm_get_handle(self.handle, buf), "g4_comm_get_handle")
            allh = exchange_handles(bytes(buf.raw), mesh.world, group)
            N.check(L.g4_comm_open(self.handle, allh), "g4_comm_open")
            dist.barrier(group=group)

    @classmethod
    def local_group(cls, meshes, hidden: int) -> list:
        """One communicator per device for ranks owned by this process (one device each):
        created on their devices and opened together with direct peer addressing
        (``g4_comm_open_local``), no IPC handles and no process group."""
        comms = [cls(m, hidden, _local=True) for m in meshes]
        arr = (ctypes.c_void_p * len(comms))(*[c.handle.value for c in comms])
        N.check(N.lib().g4_comm_open_local(arr, len(comms)), "g4_comm_open_local")
        return comms

    def close(self):
        if self.handle:
            N.lib().g4_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()


def _i32(v: int) -> int:
    """An unsigned 32-bit value as the int32 with the same bits."""
    return v - (1 << 32) if v >= (1 << 31) else v


class DecodeModel:
    """Per-rank native model.  ``shard``: native tensor name -> CUDA tensor."""

    def __init__(self, cfg: TextConfig, shard: dict, mesh: Mesh, max_len: int,
                 comm: Comm | None = None, timeout_us: int = 2_000_000, engine: str = "step"):
        L = N.lib()
        self.cfg, self.mesh, self.max_len = cfg, mesh, max_len
        self.device = torch.device("cuda", mesh.device)
        dev = self.device
        self.shard = shard  # keep the tensors alive: the library only holds pointers
        self.ctrl = torch.zeros(N.CTRL_WORDS, dtype=torch.int32, device=dev)
        self.ctrl[N.CTRL_TIMEOUT_US] = timeout_us
        self.tokens_in = torch.zeros(max_len, dtype=torch.int32, device=dev)
        self.tokens_out = torch.zeros(max_len + 1, dtype=torch.int32, device=dev)
        self.v_local = cfg.vocab_size // mesh.world
        self.logits = torch.zeros(self.v_local, dtype=torch.float32, device=dev)
        self.cache_k, self.cache_v = [], []
        for shape in local_cache_shapes(cfg, 1, max_len, mesh):
            self.cache_k.append(torch.zeros(shape, dtype=torch.bfloat16, device=dev))
            self.cache_v.append(torch.zeros(shape, dtype=torch.bfloat16, device=dev))

        ccfg = N.G4Config.from_text_config(cfg)
        full = bytes(1 if lt == "full_attention" else 0 for lt in cfg.layer_types)
        self.handle = ctypes.c_void_p()
        with torch.cuda.device(dev):
            N.check(L.g4_model_create(ctypes.byref(ccfg), full, mesh.rank, mesh.world, max_len,
                                      mesh.device, ctypes.byref(self.handle)), "g4_model_create")
            for name, t in shard.items():
                self._set(name, t)
            for i in range(cfg.num_hidden_layers):
                self._set(f"layers.{i}.cache_k", self.cache_k[i])
                self._set(f"layers.{i}.cache_v", self.cache_v[i])
            for name, t in (("control", self.ctrl), ("tokens_in", self.tokens_in),
                            ("tokens_out", self.tokens_out), ("logits", self.logits)):
                self._set(name, t)
            self.comm = comm
            if comm is not None:
                N.check(L.g4_model_set_comm(self.handle, comm.handle), "g4_model_set_comm")
            N.check(L.g4_model_finalize(self.handle), "g4_model_finalize")
            if engine not in N.ENGINES:
                raise ValueError(f"engine must be one of {sorted(N.ENGINES)}")
            self.engine = engine
            N.check(L.g4_model_set_engine(self.handle, N.ENGINES[engine]), "g4_model_set_engine")
            hp = ctypes.POINTER(ctypes.c_int)()
            N.check(L.g4_model_host_tokens(self.handle, ctypes.byref(hp)), "g4_model_host_tokens")
            self.tokens_host = np.ctypeslib.as_array(hp, shape=(max_len + 1,))
        self.graph_ready = False
        self.workspace_epoch = 0  # bumped by every prefill: it may re-allocate the prefill workspace
        self.batch_owner = None   # the BatchDecoder whose caches the library holds
        self.kernels_per_step = L.g4_model_kernel_count(self.handle)

    def _set(self, name: str, t: torch.Tensor):
        if not t.is_contiguous():
            raise ValueError(f"{name}: tensor must be contiguous")
        N.check(N.lib().g4_model_set_tensor(self.handle, name.encode(), N.ptr(t),
                                            t.numel() * t.element_size()), f"set_tensor({name})")

    # ------------------------------------------------------------------ control
    def reset(self, prompt_ids, write_logits: bool = False, clear_status: bool = True):
        """Start a new sequence: position 0, the prompt as forced tokens."""
        p = len(prompt_ids)
        if p < 1 or p > self.max_len:
            raise ValueError(f"prompt length {p} outside [1, {self.max_len}]")
        self.tokens_in[:p].copy_(torch.as_tensor(list(prompt_ids), dtype=torch.int32))
        self.ctrl[N.CTRL_POS] = 0
        self.ctrl[N.CTRL_FORCED_LEN] = p
        self.ctrl[N.CTRL_WRITE_LOGITS] = 1 if write_logits else 0
        if clear_status:
            self.ctrl[N.CTRL_STATUS] = 0

    def set_write_logits(self, on: bool):
        self.ctrl[N.CTRL_WRITE_LOGITS] = 1 if on else 0

    def set_sampling(self, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 64,
                     seed: int = 0):
        """Sampling parameters of the following steps (model.py:414-424).  temperature
        <= 0 is greedy; otherwise each step draws from top_k(logits / t) with the top-p
        mask, keyed by (seed, position) -- see include/g4b200.h G4_CTRL_TEMPERATURE."""
        if not 1 <= int(top_k) <= N.SAMPLE_MAX_TOP_K:
            raise ValueError(f"top_k must be in [1, {N.SAMPLE_MAX_TOP_K}], got {top_k}")
        f = torch.tensor([float(temperature), float(top_p)], dtype=torch.float32).view(torch.int32)
        s64 = int(seed) & (2 ** 64 - 1)
        words = torch.tensor([int(f[0]), int(f[1]), int(top_k),
                              _i32(s64 & 0xFFFFFFFF), _i32(s64 >> 32)], dtype=torch.int32)
        self.ctrl[N.CTRL_TEMPERATURE:N.CTRL_SEED_HI + 1].copy_(words)

    def step(self, n: int = 1, use_graph: bool = True):
        """Enqueue ``n`` decode steps on the current stream (asynchronous)."""
        L = N.lib()
        st = N.stream_handle()
        with torch.cuda.device(self.device):
            if use_graph:
                if not self.graph_ready:
                    self.capture()
                N.check(L.g4_graph_launch(self.handle, st, n), "g4_graph_launch")
            else:
                for _ in range(n):
                    N.check(L.g4_step(self.handle, st), "g4_step")

    def prefill(self, n_tokens: int, chunk: int = 0, dense_moe: bool = False):
        """Consume the first ``n_tokens`` forced tokens in one tensor-core pass per chunk
        (``g4_prefill``): cache rows [0, n), tokens_out[n] and POS = n, like ``n`` steps.
        ``dense_moe`` runs the reference's all-expert MoE as written instead of the routed
        pairs (same result up to fp32 summation order; world 1 only).  Under tensor
        parallelism every rank must make the same call: the layers' two all-reduces and
        the LM head's argmax run through the communicators' prefill exchange, in chunks of
        at most 4096 prompt rows.  Returns True (enqueued)."""
        flags = N.PREFILL_DENSE_MOE if dense_moe else 0
        self.workspace_epoch += 1
        with torch.cuda.device(self.device):
            N.check(N.lib().g4_prefill(self.handle, int(n_tokens), int(chunk), flags, N.stream_handle()),
                    "g4_prefill")
        return True

    def capture(self):
        with torch.cuda.device(self.device):
            N.check(N.lib().g4_graph_capture(self.handle, N.stream_handle()), "g4_graph_capture")
        self.graph_ready = True

    KERNEL_CLASSES = ("qkv", "attention", "o_proj", "router_mlp_up", "mlp_down_experts_up",
                      "experts_down", "lm_head_argmax")

    def profile(self, steps: int) -> dict:
        """Summed ms per kernel class over ``steps`` event-separated steps (always the
        per-op kernels, whatever the engine: a persistent step has no kernel classes)."""
        out = (ctypes.c_float * 7)()
        with torch.cuda.device(self.device):
            N.check(N.lib().g4_model_profile(self.handle, N.stream_handle(), steps, out, 7),
                    "g4_model_profile")
        return dict(zip(self.KERNEL_CLASSES, [float(v) for v in out]))

    def check_status(self):
        """Synchronise and raise if a status bit is set (a bounded device wait gave up,
        a bad token, a position overflow).  With the step kernel, steps after a set bit
        do nothing until ``reset`` clears it."""
        st = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            rc = N.lib().g4_model_status(self.handle, N.stream_handle(), ctypes.byref(st))
        if rc != N.G4_OK:
            raise N.G4Error(rc, "decode step", f"device status word 0x{st.value:x}")

    def close(self):
        if self.handle:
            torch.cuda.synchronize(self.device)
            N.lib().g4_model_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


class BatchDecoder:
    """``batch`` sequences decoded together on one rank's model (``g4_batch_*``): each has
    its own KV cache of ``ctx_len`` positions; prompts go through the tensor-core prefill,
    every step decodes one greedy token of every sequence (benchmark config 5's batch-8
    decode; the reference forward's batch axis, model.py:333-386)."""

    def __init__(self, model: DecodeModel, batch: int, ctx_len: int):
        self.model, self.batch, self.ctx_len = model, batch, ctx_len
        dev = model.device
        with torch.cuda.device(dev):
            N.check(N.lib().g4_batch_reserve(model.handle, batch, ctx_len), "g4_batch_reserve")
        model.batch_owner = self
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(batch, model.v_local, dtype=torch.float32, device=dev)
        self.positions = [0] * batch
        self._graph, self._graph_key, self._warm = None, None, None

    def _owned(self) -> DecodeModel:
        m = self.model
        if m.batch_owner is not self:
            raise RuntimeError("a newer BatchDecoder on this model has replaced this one's caches")
        return m

    def prefill(self, seq: int, prompt_ids) -> None:
        """Sequence ``seq``'s prompt into its cache; its first token becomes its next input."""
        m = self._owned()
        p = len(prompt_ids)
        if not 1 <= p < self.ctx_len:
            raise ValueError(f"prompt length {p} outside [1, {self.ctx_len})")
        m.workspace_epoch += 1
        with torch.cuda.device(m.device):
            m.tokens_in[:p].copy_(torch.as_tensor(list(prompt_ids), dtype=torch.int32))
            N.check(N.lib().g4_batch_prefill(m.handle, seq, p, N.ptr(self.tokens[seq:seq + 1]), N.stream_handle()),
                    "g4_batch_prefill")
        self.positions[seq] = p

    def _enqueue(self, write_logits: bool) -> None:
        m = self.model
        N.check(N.lib().g4_batch_step(m.handle, N.ptr(self.tokens),
                                      N.ptr(self.logits) if write_logits else None, N.stream_handle()),
                "g4_batch_step")

    def step(self, write_logits: bool = False, graph: bool = False) -> torch.Tensor:
        """One token of every sequence (asynchronous); returns the device tensor of the
        B tokens just produced (valid after the stream reaches this point).

        ``graph``: replay the step as a CUDA graph (one launch instead of ~27 per layer).
        Positions live in the device control blocks, so one captured step serves every
        later step.  The graph is captured once an eager step of the same kind has run
        since the last prefill (a prefill may re-allocate the workspace the graph reads)."""
        m = self._owned()
        if max(self.positions) + 1 >= self.ctx_len:
            raise ValueError("a sequence would pass the end of its cache")
        key = (m.workspace_epoch, bool(write_logits))
        with torch.cuda.device(m.device):
            if graph and self._warm == key:
                if self._graph_key != key:
                    self._graph = None
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, capture_error_mode="thread_local"):
                        self._enqueue(write_logits)
                    self._graph, self._graph_key = g, key
                self._graph.replay()
            else:
                self._enqueue(write_logits)
                self._warm = key
        self.positions = [p + 1 for p in self.positions]
        return self.tokens

    def check_status(self):
        st = ctypes.c_int(0)
        with torch.cuda.device(self.model.device):
            rc = N.lib().g4_batch_status(self.model.handle, N.stream_handle(), ctypes.byref(st))
        if rc != N.G4_OK:
            raise N.G4Error(rc, "batched decode", f"status word 0x{st.value:x}")
