"""Helpers shared by the GPU parity tests (comparison metrics, oracle block restatements)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import reference_model as R


def corr(a, b) -> float:
    a = np.asarray(torch.as_tensor(a).float().cpu(), np.float64).ravel()
    b = np.asarray(torch.as_tensor(b).float().cpu(), np.float64).ravel()
    return float(np.corrcoef(a, b)[0, 1])


def rel_err(got, ref) -> float:
    got, ref = torch.as_tensor(got).float().cpu(), torch.as_tensor(ref).float().cpu()
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def bf16_ulp_diff(a, b) -> torch.Tensor:
    """|a - b| in units of bf16 ulps (as integer distance of the bit patterns)."""
    ia = torch.as_tensor(a).cpu().to(torch.bfloat16).view(torch.int16).to(torch.int32)
    ib = torch.as_tensor(b).cpu().to(torch.bfloat16).view(torch.int16).to(torch.int32)
    # map sign-magnitude to a monotone integer line
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return (ia - ib).abs()


def attention_reference(qkv_raw, q_norm, k_norm, cache_k, cache_v, pos, n_q, n_kv, d, k_eq_v,
                        window, theta, partial, eps):
    """model.py:197-213 for one decode token, from the raw q|k|v projections (CPU, bf16).

    Returns (ctx [n_q*d] bf16, k_new [n_kv, d], v_new [n_kv, d]); the caches are updated.
    """
    g = n_q // n_kv
    q = qkv_raw[: n_q * d].reshape(1, 1, n_kv, g, d)
    k_raw = qkv_raw[n_q * d: n_q * d + n_kv * d].reshape(1, 1, n_kv, d)
    v_raw = k_raw if k_eq_v else qkv_raw[n_q * d + n_kv * d:].reshape(1, 1, n_kv, d)
    inv = R.rope_inv_freq(d, theta, partial)
    cos, sin = R.rope_tables(torch.tensor([pos]), inv)
    q = R.apply_rope(R.rms_norm(q, q_norm, eps), cos, sin)
    k = R.apply_rope(R.rms_norm(k_raw, k_norm, eps), cos, sin)
    v = R.rms_norm(v_raw, None, eps)
    cache_k[pos] = k[0, 0]
    cache_v[pos] = v[0, 0]
    max_len = cache_k.shape[0]
    kv = torch.arange(max_len)
    mask = kv <= pos
    if window:
        mask &= kv > pos - window
    lo = int(mask.nonzero().min())
    kk = cache_k[lo:pos + 1][None]
    vv = cache_v[lo:pos + 1][None]
    dt = torch.bfloat16
    scores = R.contract("btkgd,bskd->bkgts", q, kk, dt).float()
    probs = torch.softmax(scores, -1).to(dt)
    ctx = R.contract("bkgts,bskd->btkgd", probs, vv, dt)
    return ctx.reshape(-1), k[0, 0], v[0, 0]
