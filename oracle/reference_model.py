"""CPU oracle for the Gemma-4 decode/prefill forward step -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the reference JAX forward pass of
YLiu95/kaggle-tpu-inference (``gemma4_tpu/model.py``).  It is the checker for the
CUDA path: only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  Nothing in the product
package imports or executes it.

Parity pinning: the reference itself cannot run here (``jax`` is not installed and
cannot be installed).  The reference pins its JAX forward against HuggingFace
``transformers`` on a tiny random model (``tests/test_parity.py:29-153``); this
oracle is pinned the same way (``tests/test_oracle.py``) against ``transformers``
5.5.0 on that exact tiny model and thresholds, with ``router_input="residual"``
because transformers 5.5.0 routes on the raw residual while ``model.py:315-316``
routes on the ``pre_feedforward_layernorm_2`` output.  Golden vectors produced by
``tests/golden/make_golden.py`` are committed under ``tests/golden/``.

Two numeric modes:

* ``"bf16"`` -- bf16-faithful: parameters, activations and the KV cache are bf16 and
  every rounding point of the reference is reproduced (einsum outputs rounded to
  bf16 after fp32 accumulation, fp32 norms/softmax, bf16 elementwise products,
  bf16 RoPE application, scores rounded to bf16 before the fp32 softmax,
  per-expert bf16 sums in the decode MoE).
* ``"fp32"`` -- the same graph entirely in float32 (the "truth" used to report how
  far both the reference semantics and the CUDA path are from exact arithmetic).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

FULL = "full_attention"
SLIDING = "sliding_attention"
NEG_INF = -1e30  # model.py:32


# ----------------------------------------------------------------------------- layout
def param_shapes(cfg) -> dict[str, tuple[int, ...]]:
    """Canonical parameter shapes keyed by flat name (model.py:84-117)."""
    h = cfg.hidden_size
    out: dict[str, tuple[int, ...]] = {"embed": (cfg.vocab_size, h), "norm": (h,)}
    for i, lt in enumerate(cfg.layer_types):
        d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
        g = cfg.num_attention_heads // kv
        p = f"layers.{i}."
        for n in ("input_layernorm", "post_attention_layernorm",
                  "pre_feedforward_layernorm", "post_feedforward_layernorm"):
            out[p + n] = (h,)
        out[p + "layer_scalar"] = (1,)
        out[p + "q_proj"] = (kv, g, d, h)
        out[p + "k_proj"] = (kv, d, h)
        if not cfg.k_eq_v_for(lt):
            out[p + "v_proj"] = (kv, d, h)
        out[p + "o_proj"] = (h, kv, g, d)
        out[p + "q_norm"] = (d,)
        out[p + "k_norm"] = (d,)
        out[p + "mlp.gate_proj"] = (cfg.intermediate_size, h)
        out[p + "mlp.up_proj"] = (cfg.intermediate_size, h)
        out[p + "mlp.down_proj"] = (h, cfg.intermediate_size)
        if cfg.enable_moe_block:
            for n in ("pre_feedforward_layernorm_2", "post_feedforward_layernorm_1",
                      "post_feedforward_layernorm_2", "router.scale"):
                out[p + n] = (h,)
            out[p + "router.proj"] = (cfg.num_experts, h)
            out[p + "router.per_expert_scale"] = (cfg.num_experts,)
            out[p + "experts.gate_up_proj"] = (cfg.num_experts, 2, cfg.moe_intermediate_size, h)
            out[p + "experts.down_proj"] = (cfg.num_experts, h, cfg.moe_intermediate_size)
    return out


# ----------------------------------------------------------------------------- primitives
def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    """fp32 RMSNorm, cast back to the input dtype (model.py:42-47)."""
    x32 = x.float()
    out = x32 * torch.rsqrt(x32.square().mean(-1, keepdim=True) + eps)
    if w is not None:
        out = out * w.float()
    return out.to(x.dtype)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """tanh-approximate GELU evaluated in fp32 and rounded once (model.py:50-51)."""
    y = x.float()
    cdf = 0.5 * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (y + 0.044715 * y.pow(3))))
    return (y * cdf).to(x.dtype)


def contract(eq: str, a: torch.Tensor, b: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    """einsum with fp32 accumulation and one rounding of the result to ``dt``."""
    return torch.einsum(eq, a.float(), b.float()).to(dt)


def rope_inv_freq(head_dim: int, theta: float, partial: float = 1.0) -> np.ndarray:
    """Rotate-half inverse frequencies with a zero-frequency NoPE tail (model.py:54-61)."""
    n_rot = int(partial * head_dim // 2)
    inv = 1.0 / (theta ** (np.arange(0, 2 * n_rot, 2, dtype=np.float64) / head_dim))
    tail = head_dim // 2 - n_rot
    if tail > 0:
        inv = np.concatenate([inv, np.zeros(tail, np.float64)])
    return inv.astype(np.float32)


def rope_tables(positions: torch.Tensor, inv_freq: np.ndarray):
    """fp32 cos/sin of position x inv_freq, duplicated over both halves (model.py:64-67)."""
    f = positions.float()[:, None] * torch.from_numpy(inv_freq)[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE with cos/sin cast to x's dtype before the products (model.py:70-78)."""
    d = x.shape[-1]
    rotated = torch.cat([-x[..., d // 2:], x[..., : d // 2]], dim=-1)
    shape = (1, cos.shape[0]) + (1,) * (x.ndim - 3) + (d,)
    c = cos.reshape(shape).to(x.dtype)
    s = sin.reshape(shape).to(x.dtype)
    return x * c + rotated * s


# ----------------------------------------------------------------------------- cache / masks
def init_cache(cfg, batch: int, max_len: int, dtype=torch.bfloat16) -> dict:
    """Per-layer zeroed K and V caches [B, max_len, kv, d] (model.py:174-185)."""
    ks, vs = [], []
    for lt in cfg.layer_types:
        shape = (batch, max_len, cfg.kv_heads_for(lt), cfg.head_dim_for(lt))
        ks.append(torch.zeros(shape, dtype=dtype))
        vs.append(torch.zeros(shape, dtype=dtype))
    return {"k": ks, "v": vs}


def prefill_masks(cfg, t: int, prompt_len: int) -> dict:
    """Causal & kv < prompt_len; sliding adds kv > q - window (model.py:392-399)."""
    q = torch.arange(t)[:, None]
    kv = torch.arange(t)[None, :]
    valid = (kv <= q) & (kv < prompt_len)
    return {FULL: valid, SLIDING: valid & (kv > q - cfg.sliding_window)}


def decode_masks(cfg, max_len: int, pos: int) -> dict:
    """kv <= pos; sliding adds kv > pos - window (model.py:402-408)."""
    kv = torch.arange(max_len)[None, :]
    valid = kv <= pos
    return {FULL: valid, SLIDING: valid & (kv > pos - cfg.sliding_window)}


# ----------------------------------------------------------------------------- model
@dataclass
class Oracle:
    cfg: object
    params: dict
    mode: str = "bf16"             # "bf16" (faithful) or "fp32" (truth)
    router_input: str = "normed"   # "normed" = model.py:315-316; "residual" = transformers 5.5.0
    moe_decode: str = "slice"      # model.py:252 GEMMA4_MOE_DECODE: "slice" (default) or "loop"

    def __post_init__(self):
        self.dt = torch.bfloat16 if self.mode == "bf16" else torch.float32
        self.p = {k: v.to(self.dt) for k, v in self.params.items()}
        self.inv = {
            SLIDING: rope_inv_freq(self.cfg.head_dim, self.cfg.rope_theta_sliding),
            FULL: rope_inv_freq(self.cfg.global_head_dim, self.cfg.rope_theta_full,
                                self.cfg.rope_partial_rotary_factor_full),
        }

    def lp(self, i: int) -> dict:
        pre = f"layers.{i}."
        return {k[len(pre):]: v for k, v in self.p.items() if k.startswith(pre)}

    # -- blocks ------------------------------------------------------------------
    def attention(self, lp, x, lt, cos, sin, ck, cv, write_at, mask, kv_len):
        """model.py:195-215 (scale 1.0; scores rounded to dtype before the fp32 softmax)."""
        cfg, dt, eps = self.cfg, self.dt, self.cfg.rms_norm_eps
        q = contract("bth,kgdh->btkgd", x, lp["q_proj"], dt)
        q = apply_rope(rms_norm(q, lp["q_norm"], eps), cos, sin)
        k_raw = contract("bth,kdh->btkd", x, lp["k_proj"], dt)
        v_raw = k_raw if cfg.k_eq_v_for(lt) else contract("bth,kdh->btkd", x, lp["v_proj"], dt)
        k = apply_rope(rms_norm(k_raw, lp["k_norm"], eps), cos, sin)
        v = rms_norm(v_raw, None, eps)
        t = x.shape[1]
        ck[:, write_at:write_at + t] = k.to(ck.dtype)
        cv[:, write_at:write_at + t] = v.to(cv.dtype)
        kk, vv = ck[:, :kv_len].to(dt), cv[:, :kv_len].to(dt)
        scores = contract("btkgd,bskd->bkgts", q, kk, dt).float()
        scores = torch.where(mask, scores, torch.tensor(NEG_INF, dtype=torch.float32))
        probs = torch.softmax(scores, dim=-1).to(dt)
        ctx = contract("bkgts,bskd->btkgd", probs, vv, dt)
        return contract("btkgd,hkgd->bth", ctx, lp["o_proj"], dt)

    def dense_mlp(self, lp, x):
        """model.py:218-221."""
        dt = self.dt
        gate = contract("bth,ih->bti", x, lp["mlp.gate_proj"], dt)
        up = contract("bth,ih->bti", x, lp["mlp.up_proj"], dt)
        return contract("bti,hi->bth", gelu(gate) * up, lp["mlp.down_proj"], dt)

    def router(self, lp, flat):
        """model.py:224-232 (top-k ties resolved to the lower expert index)."""
        cfg, dt = self.cfg, self.dt
        x = rms_norm(flat, None, cfg.rms_norm_eps)
        x = x * lp["router.scale"]
        x = x * torch.tensor(cfg.hidden_size ** -0.5, dtype=torch.float32).to(dt)
        scores = contract("nh,eh->ne", x, lp["router.proj"], dt).float()
        probs = torch.softmax(scores, dim=-1)
        order = torch.sort(-probs, dim=-1, stable=True).indices[:, : cfg.top_k_experts]
        top_w = torch.gather(probs, 1, order)
        top_w = top_w / top_w.sum(-1, keepdim=True)
        top_w = top_w * lp["router.per_expert_scale"].float()[order]
        return top_w, order

    def moe(self, lp, flat, dense: bool):
        """model.py:235-294: dense all-expert prefill, or per-expert slices for decode."""
        cfg, dt = self.cfg, self.dt
        top_w, top_i = self.router(lp, flat)
        gate_up, down = lp["experts.gate_up_proj"], lp["experts.down_proj"]
        if dense:
            w_full = torch.zeros(flat.shape[0], cfg.num_experts).scatter_add_(1, top_i, top_w)
            gu = contract("nh,ecfh->necf", flat, gate_up, dt)
            act = gelu(gu[:, :, 0]) * gu[:, :, 1]
            act = act * w_full[:, :, None].to(dt)
            return contract("nef,ehf->nh", act, down, dt)
        rows = []
        for n in range(flat.shape[0]):
            acc = None
            for k in range(cfg.top_k_experts):
                e = int(top_i[n, k])
                gu = contract("h,cfh->cf", flat[n], gate_up[e], dt)
                a = gelu(gu[0]) * gu[1] * top_w[n, k].to(dt)
                part = contract("f,hf->h", a, down[e], dt)
                if self.moe_decode == "loop":
                    acc = part.float() if acc is None else acc + part.float()
                else:
                    acc = part if acc is None else acc + part
            rows.append(acc.to(dt))
        return torch.stack(rows, 0)

    def layer(self, i, x, lt, cos, sin, ck, cv, write_at, mask, kv_len, dense_moe):
        """model.py:297-322."""
        cfg, eps, lp = self.cfg, self.cfg.rms_norm_eps, self.lp(i)
        residual = x
        h = rms_norm(x, lp["input_layernorm"], eps)
        h = self.attention(lp, h, lt, cos, sin, ck, cv, write_at, mask, kv_len)
        x = residual + rms_norm(h, lp["post_attention_layernorm"], eps)
        residual = x
        h = self.dense_mlp(lp, rms_norm(x, lp["pre_feedforward_layernorm"], eps))
        if cfg.enable_moe_block:
            h1 = rms_norm(h, lp["post_feedforward_layernorm_1"], eps)
            b, t, hid = residual.shape
            h2 = rms_norm(residual.reshape(-1, hid), lp["pre_feedforward_layernorm_2"], eps)
            if self.router_input == "residual":
                # transformers 5.5.0 routes on the raw residual (modeling_gemma4 decoder layer)
                top = self.router(lp, residual.reshape(-1, hid))
                h2 = self._moe_with_routing(lp, h2, top, dense_moe)
            else:
                h2 = self.moe(lp, h2, dense_moe)
            h2 = rms_norm(h2.reshape(b, t, hid), lp["post_feedforward_layernorm_2"], eps)
            h = h1 + h2
        h = rms_norm(h, lp["post_feedforward_layernorm"], eps)
        x = residual + h
        return x * lp["layer_scalar"].to(x.dtype)

    def _moe_with_routing(self, lp, flat, top, dense):
        saved = self.router
        self.router = lambda _lp, _flat: top
        try:
            return self.moe(lp, flat, dense)
        finally:
            self.router = saved

    def forward(self, tokens, positions, cache, write_at, masks, kv_len, dense_moe, last_index=None):
        """model.py:333-386 -> (fp32 softcapped logits [B, T', V], cache)."""
        cfg, dt = self.cfg, self.dt
        embed = self.p["embed"]
        x = embed[tokens.long()]
        x = x * torch.tensor(np.float32(cfg.embed_scale)).to(torch.bfloat16).to(dt)
        rope = {lt: rope_tables(positions, self.inv[lt]) for lt in (SLIDING, FULL)}
        for i, lt in enumerate(cfg.layer_types):
            cos, sin = rope[lt]
            x = self.layer(i, x, lt, cos, sin, cache["k"][i], cache["v"][i],
                           write_at, masks[lt], kv_len, dense_moe)
        x = rms_norm(x, self.p["norm"], cfg.rms_norm_eps)
        if last_index is not None:
            x = x[:, last_index:last_index + 1]
        logits = contract("bth,vh->btv", x, embed, dt).float()
        if cfg.final_logit_softcapping:
            cap = float(cfg.final_logit_softcapping)
            logits = torch.tanh(logits / cap) * cap
        return logits, cache

    # -- engine-style steps (engine.py:57-83) -------------------------------------
    def new_cache(self, batch: int, max_len: int) -> dict:
        return init_cache(self.cfg, batch, max_len, self.dt)

    def prefill(self, cache, tokens, prompt_len: int, bucket: int | None = None, dense_moe=True):
        """Prefill a padded bucket; returns logits at every bucket position [T, V]."""
        t = bucket or len(tokens)
        padded = torch.zeros(1, t, dtype=torch.int64)
        padded[0, :len(tokens)] = torch.as_tensor(tokens)
        masks = {k: v[None, None, None] for k, v in prefill_masks(self.cfg, t, prompt_len).items()}
        logits, cache = self.forward(padded, torch.arange(t), cache, 0, masks, t, dense_moe)
        return logits[0], cache

    def decode(self, cache, token: int, pos: int, max_len: int):
        """One decode step at ``pos`` (reads the whole cache under the mask like engine.py:77)."""
        masks = {k: v[None, None, None] for k, v in decode_masks(self.cfg, max_len, pos).items()}
        tok = torch.tensor([[token]], dtype=torch.int64)
        logits, cache = self.forward(tok, torch.tensor([pos]), cache, pos, masks, max_len, False)
        return logits[0, 0], cache

    def greedy_generate(self, prompt, n_new: int, max_len: int, teacher=None):
        """Token-by-token greedy decode over the prompt then ``n_new`` tokens.

        Every position, including the prompt, goes through :meth:`decode`, which is
        how the CUDA engine consumes a prompt.  With ``teacher`` given, the fed token
        after the prompt is ``teacher[j]`` instead of the oracle's own argmax
        (teacher-forced comparison).  Returns (logits [P+n_new-1... , V], argmax ids).
        """
        cache = self.new_cache(1, max_len)
        logits_all, ids = [], []
        seq = list(prompt)
        for pos in range(len(prompt) + n_new - 1):
            tok = seq[pos]
            lg, cache = self.decode(cache, tok, pos, max_len)
            logits_all.append(lg)
            nxt = int(torch.argmax(lg))
            if pos >= len(prompt) - 1:
                ids.append(nxt)
                j = pos - (len(prompt) - 1)
                seq.append(teacher[j] if teacher is not None else nxt)
        return torch.stack(logits_all), ids


def sample_greedy(logits: torch.Tensor) -> int:
    """Greedy branch of model.py:414-424 (first index of the maximum)."""
    return int(torch.argmax(logits))


# ----------------------------------------------------------------------------- sampling
def philox4x32_10(ctr, key):
    """Philox-4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, SC 2011) on Python ints:
    multipliers 0xD2511F53 / 0xCD9E8D57, key increments 0x9E3779B9 / 0xBB67AE85.  The
    counter-based generator the device sampler documents (keyed by the seed, counter =
    (position, 0, 0, 0))."""
    c0, c1, c2, c3 = (int(v) & 0xFFFFFFFF for v in ctr)
    k0, k1 = (int(v) & 0xFFFFFFFF for v in key)
    for _ in range(10):
        p0, p1 = 0xD2511F53 * c0, 0xCD9E8D57 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & 0xFFFFFFFF, p1 & 0xFFFFFFFF, \
            ((p0 >> 32) ^ c3 ^ k1) & 0xFFFFFFFF, p0 & 0xFFFFFFFF
        k0, k1 = (k0 + 0x9E3779B9) & 0xFFFFFFFF, (k1 + 0xBB67AE85) & 0xFFFFFFFF
    return c0, c1, c2, c3


def philox_uniform(seed: int, position: int) -> np.float32:
    """Uniform in [0, 1) of (seed, position): the top 24 bits of the first output word."""
    s = int(seed) & (2 ** 64 - 1)
    c = philox4x32_10((position, 0, 0, 0), (s & 0xFFFFFFFF, s >> 32))
    return np.float32(c[0] >> 8) * np.float32(1.0 / 16777216.0)


def sampling_distribution(logits: torch.Tensor, temperature: float, top_k: int, top_p: float):
    """model.py:414-424 up to the categorical draw, in fp32 with sequential sums:
    top_k(logits / t) (ties to the lower index, like lax.top_k), softmax, the top-p mask
    (cumsum - p) < top_p.  Returns (token ids, unnormalised kept probabilities, their sum)."""
    t = np.float32(max(float(temperature), 1e-6))
    v = (logits.float().numpy().astype(np.float32) / t).astype(np.float32)
    order = np.lexsort((np.arange(v.size), -v))[:top_k]  # value desc, index asc
    vals = v[order]
    mx = vals[0]
    e = np.exp((vals - mx).astype(np.float32)).astype(np.float32)
    total = np.float32(0.0)
    for x in e:
        total = np.float32(total + x)
    probs, csum, kept = [], np.float32(0.0), np.float32(0.0)
    for x in e:
        p = np.float32(x / total)
        csum = np.float32(csum + p)
        if np.float32(csum - p) < np.float32(top_p):
            probs.append(p)
            kept = np.float32(kept + p)
        else:
            break
    if not probs:
        probs, kept = [np.float32(e[0] / total)], np.float32(e[0] / total)
    return order[:len(probs)], np.array(probs, np.float32), kept


def sample_token(logits: torch.Tensor, temperature: float, top_k: int, top_p: float, u: float) -> int:
    """The token model.py:414-424 draws when its categorical sample is the inverse CDF of
    the renormalised kept probabilities at ``u`` (greedy for temperature <= 0)."""
    if temperature <= 0.0:
        return int(torch.argmax(logits))
    ids, probs, kept = sampling_distribution(logits, temperature, top_k, top_p)
    target = np.float32(np.float32(u) * kept)
    acc = np.float32(0.0)
    for i, p in zip(ids, probs):
        acc = np.float32(acc + p)
        if target < acc:
            return int(i)
    return int(ids[-1])
