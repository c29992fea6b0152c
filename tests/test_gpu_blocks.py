"""Block-level parity of the CUDA kernels with the CPU oracle, through the C ABI.

* decode attention (benchmark config 3): sliding layer 16 q / 8 KV heads, d 256, window
  1024, cache 32768; full k==v layer 16 q / 2 KV heads, d 256 (and the real 512), cache
  32768 fully live; Q/K/V N(0,1), seed 2.
* MoE block (benchmark config 2): hidden 2816, 128 experts top-8, moe_intermediate 704,
  weights N(0, 0.02), x N(0, 1), seed 1, world 1.

Tolerances: the kernels reproduce every bf16 rounding point of the reference except
the accumulation order inside fp32 dot products and, in attention, the bf16 rounding
of the normalised probabilities (the kernel keeps them in fp32; see g4_attention.cuh).
So: routing (expert ids) must be identical, the new K/V cache rows must agree to
within 1 bf16 ulp on >= 99.9% of elements, and the outputs must have corr >= 0.9999
and max error <= 2% of the output's max magnitude.
"""

import ctypes

import pytest
import torch

from gemma4_b200 import _native as N
from gemma4_b200.config import make_config
from gemma4_b200.weights import random_param
from oracle.reference_model import Oracle
from gpu_util import attention_reference, bf16_ulp_diff, corr, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _attn_case(n_q, n_kv, d, k_eq_v, window, theta, partial, pos, max_len, seed=2):
    g = torch.Generator().manual_seed(seed * 7919 + pos)
    rows = n_q * d + n_kv * d + (0 if k_eq_v else n_kv * d)
    qkv = torch.randn(rows, generator=g).to(torch.bfloat16)
    q_norm = (0.3 + 0.2 * torch.rand(d, generator=g)).to(torch.bfloat16)
    k_norm = (0.3 + 0.2 * torch.rand(d, generator=g)).to(torch.bfloat16)
    ck = torch.randn(max_len, n_kv, d, generator=g).to(torch.bfloat16) * 0.5
    cv = torch.randn(max_len, n_kv, d, generator=g).to(torch.bfloat16)
    ck_g, cv_g = ck.to(DEV), cv.to(DEV)
    ctx_g = torch.empty(n_q * d, dtype=torch.bfloat16, device=DEV)
    qkv_g, qn_g, kn_g = qkv.to(DEV), q_norm.to(DEV), k_norm.to(DEV)
    rc = N.lib().g4_attention_decode(
        N.ptr(qkv_g), N.ptr(qn_g), N.ptr(kn_g), N.ptr(ck_g), N.ptr(cv_g), max_len, n_q, n_kv,
        d, int(k_eq_v), pos, window, theta, partial, 1e-6, N.ptr(ctx_g), N.stream_handle())
    N.check(rc, "g4_attention_decode")
    torch.cuda.synchronize()
    ref_ctx, k_new, v_new = attention_reference(qkv, q_norm, k_norm, ck, cv, pos, n_q, n_kv, d,
                                                k_eq_v, window, theta, partial, 1e-6)
    return ctx_g.cpu(), ref_ctx, ck_g[pos].cpu(), k_new, cv_g[pos].cpu(), v_new


def _check_attn(out):
    ctx, ref, kg, kr, vg, vr = out
    for a, b in ((kg, kr), (vg, vr)):
        ulp = bf16_ulp_diff(a, b)
        assert int(ulp.max()) <= 1 and float((ulp > 0).float().mean()) <= 1e-3
    assert corr(ctx, ref) >= 0.9999, corr(ctx, ref)
    assert rel_err(ctx, ref) <= 0.02, rel_err(ctx, ref)


@pytest.mark.parametrize("pos", [0, 1, 700, 1023, 1024, 5000, 32767])
def test_sliding_attention_config3(pos):
    _check_attn(_attn_case(16, 8, 256, False, 1024, 10000.0, 1.0, pos, 32768))


@pytest.mark.parametrize("pos", [0, 37, 4095, 32767])
def test_full_attention_k_eq_v_config3(pos):
    _check_attn(_attn_case(16, 2, 256, True, 0, 1e6, 0.25, pos, 32768))


@pytest.mark.parametrize("pos", [5, 9000])
def test_full_attention_real_head_dim_512(pos):
    _check_attn(_attn_case(16, 2, 512, True, 0, 1e6, 0.25, pos, 16384))


@pytest.mark.parametrize("d,n_q,n_kv", [(64, 4, 2), (128, 8, 1)])
def test_attention_small_head_dims(d, n_q, n_kv):
    _check_attn(_attn_case(n_q, n_kv, d, False, 64, 10000.0, 1.0, 300, 512))


def _moe_case(cfg, seed):
    names = {n: f"layers.0.{n}" for n in ("router.proj", "router.scale", "router.per_expert_scale",
                                            "experts.gate_up_proj", "experts.down_proj")}
    lp = {n: random_param(cfg, full, seed) for n, full in names.items()}
    x = torch.randn(1, cfg.hidden_size, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
    o = Oracle(cfg, {"layers.0." + k: v for k, v in lp.items()}, mode="bf16")
    top_w, top_i = o.router(lp, x)
    ref = o.moe(lp, x, dense=False)[0]
    dev = {k: v.to(DEV) for k, v in lp.items()}
    xg = x[0].to(DEV)
    out = torch.empty(cfg.hidden_size, dtype=torch.bfloat16, device=DEV)
    ti = torch.empty(16, dtype=torch.int32, device=DEV)
    tw = torch.empty(16, dtype=torch.float32, device=DEV)
    ctrl = torch.zeros(N.CTRL_WORDS, dtype=torch.int32, device=DEV)
    ccfg = N.G4Config.from_text_config(cfg)
    rc = N.lib().g4_moe_block(
        ctypes.byref(ccfg), 0, 1, None, N.ptr(xg), N.ptr(dev["router.proj"]),
        N.ptr(dev["router.scale"]), N.ptr(dev["router.per_expert_scale"]),
        N.ptr(dev["experts.gate_up_proj"]), N.ptr(dev["experts.down_proj"]), N.ptr(out),
        N.ptr(ti), N.ptr(tw), N.ptr(ctrl), N.stream_handle())
    N.check(rc, "g4_moe_block")
    torch.cuda.synchronize()
    assert int(ctrl[N.CTRL_STATUS]) == 0
    k = cfg.top_k_experts
    return out.cpu(), ref, ti[:k].cpu(), top_i[0], tw[:k].cpu(), top_w[0]


@pytest.mark.parametrize("seed", [1, 11])
def test_moe_block_config2(seed):
    cfg = make_config(num_hidden_layers=1, layer_types=("sliding_attention",))
    out, ref, ti, ri, tw, rw = _moe_case(cfg, seed)
    assert ti.tolist() == ri.tolist()
    torch.testing.assert_close(tw, rw.float(), rtol=1e-4, atol=1e-7)
    assert corr(out, ref) >= 0.9999 and rel_err(out, ref) <= 0.02
    assert float((bf16_ulp_diff(out, ref) <= 1).float().mean()) >= 0.99


def test_moe_block_tiny_shapes():
    cfg = make_config(hidden_size=256, num_hidden_layers=1, layer_types=("sliding_attention",),
                      num_experts=16, top_k_experts=4, moe_intermediate_size=128)
    out, ref, ti, ri, tw, rw = _moe_case(cfg, 5)
    assert ti.tolist() == ri.tolist()
    assert corr(out, ref) >= 0.9999 and rel_err(out, ref) <= 0.02
