"""The allocation-free attention entry point agrees with the allocating one.

g4_attention_decode_noalloc exists for callers that cannot allocate device memory while
they call the library (a server that reserved its whole memory budget at start-up, a host
whose caching allocator owns the GPU, a loop that cannot take an allocation's
synchronisation).  It keeps its
scratch in a fixed array inside the library, shared by all calls, so this test makes two
calls in a row -- the second one must not see leftovers of the first -- and compares both
with g4_attention_decode on the same inputs.  It lives in its own file, collected last.
"""

import pytest
import torch

from gemma4_b200 import _native as N
from gpu_util import bf16_ulp_diff

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(n_q, n_kv, d, k_eq_v, max_len, seed):
    g = torch.Generator().manual_seed(seed)
    rows = n_q * d + n_kv * d + (0 if k_eq_v else n_kv * d)
    qkv = torch.randn(rows, generator=g).to(torch.bfloat16)
    qn = (0.3 + 0.2 * torch.rand(d, generator=g)).to(torch.bfloat16)
    kn = (0.3 + 0.2 * torch.rand(d, generator=g)).to(torch.bfloat16)
    ck = (torch.randn(max_len, n_kv, d, generator=g) * 0.5).to(torch.bfloat16)
    cv = torch.randn(max_len, n_kv, d, generator=g).to(torch.bfloat16)
    return [t.to(DEV) for t in (qkv, qn, kn, ck, cv)]


def _call(fn, inp, max_len, n_q, n_kv, d, k_eq_v, pos, window, theta, partial):
    qkv, qn, kn, ck, cv = (t.clone() for t in inp)
    ctx = torch.empty(n_q * d, dtype=torch.bfloat16, device=DEV)
    N.check(fn(N.ptr(qkv), N.ptr(qn), N.ptr(kn), N.ptr(ck), N.ptr(cv), max_len, n_q, n_kv, d,
               int(k_eq_v), pos, window, theta, partial, 1e-6, N.ptr(ctx), N.stream_handle()),
            fn.__name__)
    torch.cuda.synchronize()
    return ctx.cpu(), ck[pos].cpu(), cv[pos].cpu()


# (n_q, n_kv, d, k_eq_v, max_len, pos, window, theta, partial): a sliding layer with a
# full window, then a long full k==v layer whose partials use more of the fixed array.
CASES = [
    (16, 8, 256, False, 4096, 2500, 1024, 10000.0, 1.0),
    (16, 2, 256, True, 32768, 30000, 0, 1e6, 0.25),
]


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    lib = N.lib()
    for i, (n_q, n_kv, d, kv1, max_len, pos, window, theta, partial) in enumerate(CASES):
        inp = _inputs(n_q, n_kv, d, kv1, max_len, seed=40 + i)
        ref = _call(lib.g4_attention_decode, inp, max_len, n_q, n_kv, d, kv1, pos, window, theta, partial)
        for _ in range(2):  # two calls in a row share (and must reset) the fixed scratch
            got = _call(lib.g4_attention_decode_noalloc, inp, max_len, n_q, n_kv, d, kv1, pos, window,
                        theta, partial)
            for a, b in zip(got, ref):
                assert int(bf16_ulp_diff(a, b).max()) <= 1
            torch.testing.assert_close(got[0].float(), ref[0].float(), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch():
    lib = N.lib()
    inp = _inputs(16, 2, 512, True, 64, seed=1)
    ctx = torch.empty(16 * 512, dtype=torch.bfloat16, device=DEV)
    rc = lib.g4_attention_decode_noalloc(N.ptr(inp[0]), N.ptr(inp[1]), N.ptr(inp[2]), N.ptr(inp[3]),
                                         N.ptr(inp[4]), 262144, 16, 2, 512, 1, 5, 0, 1e6, 0.25, 1e-6,
                                         N.ptr(ctx), N.stream_handle())
    assert rc == N.G4_ERR_SHAPE
    assert b"fixed scratch" in lib.g4_last_error()
