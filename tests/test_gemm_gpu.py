"""tcgen05 grouped GEMM (csrc/gemm_tc.cu) vs a float64 product of the same 16-bit
operands (needs a B200).

out[m] = a[m] @ w[g]^T over the rows of group g, rounded once to the activation dtype
(squared ReLU of the rounded product for epi 1, as rwkv_mlx/moe.py:234 computes it in
the activation dtype).  Tolerance: 2e-3 relative to RMS for fp16, 1e-2 for bf16 (one
rounding of the output; the fp32 accumulation order differs from float64's).
"""

import numpy as np
import pytest
import torch

from tests.inputs import rel_rms

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _ref(a, w, offs, relu_sq, dt):
    a64, w64 = a.double().cpu(), w.double().cpu()
    out = torch.zeros(a.shape[0], w.shape[1], dtype=torch.float64)
    for g in range(w.shape[0]):
        r0, r1 = int(offs[g]), int(offs[g + 1])
        if r1 > r0:
            y = (a64[r0:r1] @ w64[g].T).to(dt).double()
            out[r0:r1] = y.clamp(min=0) ** 2 if relu_sq else y
    return out


def _groups(sizes, device="cuda"):
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    return torch.tensor(offs, device=device), offs


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("sizes,N,K", [([300, 0, 128, 1, 517], 3072, 768), ([1000, 24], 768, 3072),
                                       ([5, 130, 77], 200, 72), ([129], 256, 64), ([3, 0, 0, 2], 40, 8)])
@pytest.mark.parametrize("relu_sq", [False, True])
def test_grouped_gemm_matches_float64(dt, sizes, N, K, relu_sq):
    """Empty groups, single rows, ragged row tiles, N and K not multiples of the tile."""
    from rwkv_mlx_b200.moe import grouped_gemm

    G, M = len(sizes), int(sum(sizes))
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(dt)
    w = (torch.randn(G, N, K, device="cuda", generator=g) / K ** 0.5).to(dt)
    offs_d, offs = _groups(sizes)
    out = grouped_gemm(a, w, offs_d, relu_sq=relu_sq)
    torch.cuda.synchronize()
    ref = _ref(a, w, offs, relu_sq, dt)
    assert rel_rms(out.double().cpu().numpy(), ref.numpy()) < TOL[dt]


def test_rows_outside_every_group_are_not_written():
    from rwkv_mlx_b200.moe import grouped_gemm

    M, N, K = 400, 512, 128
    a = torch.randn(M, K, device="cuda").half()
    w = torch.randn(2, N, K, device="cuda").half() / K ** 0.5
    offs_d, offs = _groups([100, 150])  # rows 250..399 belong to no group
    out = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    grouped_gemm(a, w, offs_d, out=out)
    torch.cuda.synchronize()
    assert (out[250:] == 7.0).all()
    ref = _ref(a, w, offs, False, torch.float16)
    assert rel_rms(out[:250].double().cpu().numpy(), ref[:250].numpy()) < TOL[torch.float16]


def test_plain_gemm_and_strided_output():
    """offsets None: one group over all rows; output rows with a larger stride."""
    from rwkv_mlx_b200.moe import grouped_gemm

    M, N, K = 1000, 768, 256
    a = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(1, N, K, device="cuda") / K ** 0.5).bfloat16()
    big = torch.zeros(M, N + 64, device="cuda", dtype=torch.bfloat16)
    grouped_gemm(a, w, None, out=big[:, :N])
    torch.cuda.synchronize()
    ref = (a.double() @ w[0].double().T).to(torch.bfloat16).double()
    assert rel_rms(big[:, :N].double().cpu().numpy(), ref.cpu().numpy()) < TOL[torch.bfloat16]
    assert (big[:, N:] == 0).all()


def test_grouped_gemm_captures_in_a_cuda_graph():
    """The group sizes are read on the device: one captured graph replays correctly after
    the offsets (and so the group sizes) change in place."""
    from rwkv_mlx_b200.moe import grouped_gemm

    M, N, K, G = 640, 512, 256, 4
    a = torch.randn(M, K, device="cuda").half()
    w = (torch.randn(G, N, K, device="cuda") / K ** 0.5).half()
    offs_d, _ = _groups([100, 200, 300, 40])
    out = torch.zeros(M, N, device="cuda", dtype=torch.float16)
    grouped_gemm(a, w, offs_d, out=out)  # warm-up (tensor maps, attributes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        grouped_gemm(a, w, offs_d, out=out)
    for sizes in ([10, 500, 0, 130], [640, 0, 0, 0]):
        offs_new, offs = _groups(sizes)
        offs_d.copy_(offs_new)
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        ref = _ref(a, w, offs, False, torch.float16)
        assert rel_rms(out.double().cpu().numpy(), ref.numpy()) < TOL[torch.float16]


def test_forced_wait_timeout_fills_outputs_with_nan():
    """Every bounded wait gives up at once (a flag set from the host): the kernel exits
    with NaN outputs and the error word set; the next call is correct again."""
    import rwkv_mlx_b200 as rb
    from rwkv_mlx_b200 import _native
    from rwkv_mlx_b200.moe import grouped_gemm

    M, N, K = 300, 512, 128
    a = torch.randn(M, K, device="cuda").half()
    w = (torch.randn(2, N, K, device="cuda") / K ** 0.5).half()
    offs_d, offs = _groups([120, 180])
    rb.check_device_error()
    L = _native.lib()
    _native.check(L.rwkv_debug_force_wait_timeout(1), "rwkv_debug_force_wait_timeout")
    try:
        out = grouped_gemm(a, w, offs_d)
        torch.cuda.synchronize()
    finally:
        _native.check(L.rwkv_debug_force_wait_timeout(0), "rwkv_debug_force_wait_timeout")
    assert torch.isnan(out).all()
    with pytest.raises(rb.RwkvDeviceError):
        rb.check_device_error()
    out = grouped_gemm(a, w, offs_d)
    torch.cuda.synchronize()
    rb.check_device_error()
    assert rel_rms(out.double().cpu().numpy(), _ref(a, w, offs, False, torch.float16).numpy()) < TOL[torch.float16]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,V,C", [(300, 1000, 64), (4096, 65568, 768), (129, 777, 96)])
def test_head_ce_stats_match_the_chunked_path(dt, M, V, C):
    """The per-token state {max, sum exp, target logit, argmax} of the fused head kernel
    equals the one the chunked kernel folds from the materialised logits (argmax exact,
    max and target logit exact: both read the same rounded logits)."""
    from rwkv_mlx_b200 import loss as ls

    g = torch.Generator(device="cuda").manual_seed(M + V)
    x = torch.randn(M, C, device="cuda", generator=g).to(dt)
    w = (torch.randn(V, C, device="cuda", generator=g) * (2.0 / C ** 0.5)).to(dt)
    tg = torch.randint(0, V, (M,), device="cuda", generator=g).to(torch.int32)
    st_fused = torch.empty(M, 4, device="cuda")
    ls._head_stats(x, w, tg, st_fused)
    lg = (x.double() @ w.double().T).to(dt)  # the same rounded logits, materialised
    st_ref = torch.empty(M, 4, device="cuda")
    ls._chunk_stats(lg, V, tg, st_ref, 0, V, True)
    torch.cuda.synchronize()
    a, b = st_fused.cpu(), st_ref.cpu()
    am_a, am_b = a[:, 3].view(torch.int32), b[:, 3].view(torch.int32)
    # logits whose fp32 accumulation lands on the other side of a rounding boundary may
    # differ by one ulp; allow a handful of such rows, never a gross difference
    same = (am_a == am_b) & (a[:, 0] == b[:, 0])
    assert same.float().mean() > 0.99
    assert torch.allclose(a[:, 0], b[:, 0], rtol=2e-3, atol=1e-2)
    assert torch.allclose(a[:, 2], b[:, 2], rtol=2e-3, atol=1e-2)
    assert torch.allclose(a[:, 1], b[:, 1], rtol=2e-3)
