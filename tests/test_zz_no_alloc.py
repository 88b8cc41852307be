"""rwkv_moe_router_noalloc: the router entry point that allocates nothing.

It is for callers that cannot allocate device memory (an FFI binding holding only
buffers a framework gave it, or a serving loop that reserved all device memory at
start-up).  Called through the C ABI twice in a row, on different inputs, it must
give what rwkv_moe_router gives on the same inputs: identical expert indices and
counts, scores and loss statistics within 1e-6.  Collected last on purpose.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _route(lib, nat, x, gw, bias, k, noalloc):
    ntok, C = x.shape
    E = gw.shape[0]
    inds = torch.full((ntok, k), -1, device="cuda", dtype=torch.int32)
    scores = torch.zeros((ntok, k), device="cuda", dtype=x.dtype)
    stats = torch.zeros(2 + E, device="cuda", dtype=torch.float32)
    counts = torch.zeros(E, device="cuda", dtype=torch.int32)
    logits = torch.zeros((ntok, E), device="cuda", dtype=torch.float32)
    st = nat.stream_ptr()
    if noalloc:
        rc = lib.rwkv_moe_router_noalloc(nat.ptr(x), nat.ptr(gw), nat.ptr(bias), nat.ptr(logits), nat.ptr(inds),
                                         nat.ptr(scores), nat.ptr(stats), nat.ptr(counts), ntok, C, E, k,
                                         nat.dtype_code(x), st)
    else:
        ws_bytes = lib.rwkv_moe_router_workspace_size(ntok, E)
        ws = torch.empty(ws_bytes, device="cuda", dtype=torch.uint8)
        rc = lib.rwkv_moe_router(nat.ptr(x), nat.ptr(gw), nat.ptr(bias), nat.ptr(logits), nat.ptr(inds),
                                 nat.ptr(scores), nat.ptr(stats), nat.ptr(counts), nat.ptr(ws), ws_bytes, ntok,
                                 C, E, k, nat.dtype_code(x), st)
    assert rc == 0, nat.STATUS.get(rc, rc)
    torch.cuda.synchronize()
    return inds.cpu().numpy(), scores.float().cpu().numpy(), stats.cpu().numpy(), counts.cpu().numpy(), \
        logits.cpu().numpy()


def test_noalloc_router_matches_router_on_two_calls_in_a_row():
    from rwkv_mlx_b200 import _native as nat

    lib = nat.lib()
    assert lib.rwkv_moe_router_noalloc_scratch_bytes() > 0
    cases = [(65536, 768, 8, 2, True, 0), (3001, 512, 16, 3, False, 1)]
    for ntok, C, E, k, with_bias, seed in cases:  # two calls in a row, different shapes
        rng = np.random.default_rng(seed)
        x = torch.tensor(rng.standard_normal((ntok, C)), dtype=torch.float16, device="cuda")
        gw = torch.tensor(rng.standard_normal((E, C)) * 0.02, dtype=torch.float32, device="cuda")
        bias = torch.tensor(rng.normal(0, 1.5, E), dtype=torch.float32, device="cuda") if with_bias else None
        got = _route(lib, nat, x, gw, bias, k, noalloc=True)
        ref = _route(lib, nat, x, gw, bias, k, noalloc=False)
        np.testing.assert_array_equal(got[0], ref[0])
        np.testing.assert_allclose(got[1], ref[1], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(got[2], ref[2], rtol=1e-6, atol=1e-6)
        np.testing.assert_array_equal(got[3], ref[3])
        np.testing.assert_array_equal(got[4], ref[4])
        assert got[3].sum() == ntok * k


def test_noalloc_router_rejects_too_many_experts():
    from rwkv_mlx_b200 import _native as nat

    lib = nat.lib()
    x = torch.zeros((16, 64), dtype=torch.float16, device="cuda")
    gw = torch.zeros((33, 64), dtype=torch.float32, device="cuda")
    out = torch.zeros(64, device="cuda")
    rc = lib.rwkv_moe_router_noalloc(nat.ptr(x), nat.ptr(gw), None, None, nat.ptr(out), nat.ptr(out), nat.ptr(out),
                                     None, 16, 64, 33, 2, 1, nat.stream_ptr())
    assert rc == 1  # RWKV_ERR_SHAPE
