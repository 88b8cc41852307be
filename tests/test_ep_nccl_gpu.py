"""Expert-parallel LoRA-MoE on 2+ GPUs over NCCL vs the single-GPU module on the
concatenated batch (skipped with fewer than 2 GPUs)."""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem(E=8, C=768, F=3072, R=16, ntok=4096, ws=2):
    g = torch.Generator().manual_seed(0)
    return dict(xk=torch.rand(1, 1, C, generator=g), key=torch.randn(F, C, generator=g) / C ** 0.5,
                value=torch.randn(C, F, generator=g) / F ** 0.5, gate=torch.randn(E, C, generator=g) / C ** 0.5,
                bias=torch.randn(E, generator=g) * 1.5, A=torch.randn(E, C, R, generator=g) * 0.02,
                B=torch.randn(E, R, C, generator=g) * 0.02, x=torch.randn(ws, 1, ntok, C, generator=g),
                E=E, C=C, F=F, R=R)


def _build(P, dev, ep):
    from rwkv_mlx_b200.ep import ExpertParallelLoRAMoE
    from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig
    from rwkv_mlx_b200.moe import LoRAMoE_CMix

    base = RWKV_CMix_x070(RWKVConfig(n_layer=2, n_embd=P["C"], dim_ffn=P["F"]), 1)
    with torch.no_grad():
        base.x_k.copy_(P["xk"])
        base.key.weight.copy_(P["key"])
        base.value.weight.copy_(P["value"])
    if ep:
        m = ExpertParallelLoRAMoE(base, P["E"], P["R"], 2)
        m.load_experts(P["A"], P["B"])
    else:
        m = LoRAMoE_CMix(base, P["E"], P["R"], 2)
        with torch.no_grad():
            m.lora_A.copy_(P["A"])
            m.lora_B.copy_(P["B"])
    with torch.no_grad():
        m.router.gate.weight.copy_(P["gate"])
    m = m.to(dev).half()
    m.router.bias = P["bias"].to(dev)
    return m


def _rank_main(rank, ws, port, P, results):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=60), device_id=dev)
        m = _build(P, dev, ep=True)
        with torch.no_grad():
            out, aux, z = m(P["x"][rank].to(dev).half())
            torch.cuda.synchronize()
        results[rank] = ("ok", out.float().cpu().numpy(), float(aux), float(z))
        dist.destroy_process_group()
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}", traceback.format_exc())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_nccl_matches_single_gpu():
    import torch.multiprocessing as mp

    ws = 2
    P = _problem(ws=ws)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    res = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, P, res)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = dict(res)
    for r in range(ws):
        assert r in res and res[r][0] == "ok", res.get(r)
    single = _build(P, torch.device("cuda", 0), ep=False)
    with torch.no_grad():
        out, aux, z = single(P["x"].reshape(1, -1, P["C"]).cuda().half())
    # the base ChannelMix token-shifts within each rank's own sequence
    with torch.no_grad():
        base_parts = torch.cat([single.base(P["x"][r].cuda().half()) for r in range(ws)], 1)
        base_full = single.base(P["x"].reshape(1, -1, P["C"]).cuda().half())
    ref = (out - base_full + base_parts).float().cpu().numpy().reshape(-1, P["C"])
    got = np.concatenate([res[r][1].reshape(-1, P["C"]) for r in range(ws)])
    err = np.sqrt(np.mean((got - ref) ** 2)) / np.sqrt(np.mean(ref ** 2))
    assert err < 2e-3, err
    for r in range(ws):
        assert abs(res[r][2] - float(aux)) < 1e-4 * max(1, float(aux))
        assert abs(res[r][3] - float(z)) < 1e-4 * max(1, float(z))
