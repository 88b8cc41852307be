"""Expert-parallel LoRA-MoE exchange logic on CPU ranks (gloo, world size 2 and 4).

The local compute steps are the numpy oracle (oracle/moe_oracle.py); what is tested
is the dispatch / return / combine bookkeeping of rwkv_mlx_b200/ep.py against the
single-process result on the concatenated batch, plus failure behaviour: a rank
that dies before the exchange makes the others fail with an error, not hang."""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as mo


class OracleOps:
    @staticmethod
    def router(x2, w, k, bias):
        lg = x2.double() @ w.double().T
        if bias is not None:
            lg = lg + bias.double()
        inds, scores, aux, z, _ = mo.router(None, None, k, logits=lg.numpy())
        return {"inds": torch.tensor(inds, dtype=torch.int32), "scores": torch.tensor(scores, dtype=x2.dtype),
                "aux": torch.tensor(aux), "z": torch.tensor(z), "logits": lg.float()}

    @staticmethod
    def permute(inds, E):
        flat = inds.reshape(-1).numpy()
        perm = np.argsort(flat, kind="stable")
        inv = np.empty_like(perm)
        inv[perm] = np.arange(len(perm))
        off = np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))])
        return (torch.tensor(perm, dtype=torch.int32), torch.tensor(inv, dtype=torch.int32),
                torch.tensor(off, dtype=torch.int32))

    @staticmethod
    def gather_rows(x2, perm, topk):
        return x2[perm.long() // topk].contiguous()

    @staticmethod
    def _experts(offsets, n):
        return np.searchsorted(offsets.numpy()[1:], np.arange(n), side="right")

    @staticmethod
    def lora_down(rows, A, perm, offsets):
        e = OracleOps._experts(offsets, perm.numel())
        return torch.einsum("pc,pcr->pr", rows[perm.long()].double(), A.double()[e]).float()

    @staticmethod
    def lora_up(h, Bw, offsets, out_index, dtype):
        e = OracleOps._experts(offsets, h.shape[0])
        y = torch.einsum("pr,prc->pc", h.double(), Bw.double()[e])
        out = torch.empty_like(y)
        out[out_index.long()] = y
        return out.to(dtype)

    @staticmethod
    def combine_rows(base2d, rows, scores, inv):
        ntok, k = scores.shape
        r = rows.double()[inv.long()].view(ntok, k, -1)
        return (base2d.double() + (scores.double().unsqueeze(-1) * r).sum(1)).to(base2d.dtype)

    @staticmethod
    def ortho_loss(A):
        return torch.tensor(mo.orthogonal_loss(A.double().numpy()))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup_problem(E=8, C=32, F=64, R=8, ntok_per_rank=24, ws=2):
    g = torch.Generator().manual_seed(0)
    xk = torch.rand(1, 1, C, generator=g)
    key = torch.randn(F, C, generator=g) / C ** 0.5
    value = torch.randn(C, F, generator=g) / F ** 0.5
    gate = torch.randn(E, C, generator=g) * 0.5
    bias = torch.randn(E, generator=g) * 1.5
    A = torch.randn(E, C, R, generator=g) * 0.2
    Bw = torch.randn(E, R, C, generator=g) * 0.2
    x = torch.randn(ws, 1, ntok_per_rank, C, generator=g)
    return dict(xk=xk, key=key, value=value, gate=gate, bias=bias, A=A, B=Bw, x=x, E=E, C=C, F=F, R=R)


def _rank_main(rank, ws, port, P, results, fail_rank):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=10))
        from rwkv_mlx_b200.ep import ExpertParallelLoRAMoE
        from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig

        base = RWKV_CMix_x070(RWKVConfig(n_layer=2, n_embd=P["C"], dim_ffn=P["F"]), 1)
        with torch.no_grad():
            base.x_k.copy_(P["xk"])
            base.key.weight.copy_(P["key"])
            base.value.weight.copy_(P["value"])
        m = ExpertParallelLoRAMoE(base, P["E"], P["R"], 2, ops=OracleOps)
        with torch.no_grad():
            m.router.gate.weight.copy_(P["gate"])
        m.router.bias = P["bias"]
        m.load_experts(P["A"], P["B"])
        if rank == fail_rank:
            raise RuntimeError("injected failure before the exchange")
        with torch.no_grad():
            out, aux, z = m(P["x"][rank])
            ortho = m.orthogonal_loss()
        results[rank] = ("ok", out.numpy(), float(aux), float(z), float(ortho))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        results[rank] = ("error", f"{type(e).__name__}: {e}", traceback.format_exc())


def _run(ws, fail_rank=-1, timeout=90):
    P = _setup_problem(ws=ws)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, P, results, fail_rank)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return P, dict(results)


@pytest.mark.parametrize("ws", [2, 4])
def test_expert_parallel_matches_single_process(ws):
    P, res = _run(ws)
    for r in range(ws):
        assert res[r][0] == "ok", res[r]
    E, C = P["E"], P["C"]
    x = P["x"].reshape(-1, C).double().numpy()
    base = mo.cmix(x.reshape(1, ws, -1, C).reshape(ws, -1, C), P["xk"], P["key"], P["value"])  # per-rank shift
    lg = mo.gate_logits(x, P["gate"], P["bias"])
    inds, scores, aux, z, _ = mo.router(None, None, 2, logits=lg)
    ref = base.reshape(-1, C) + mo.lora_moe_delta(x, P["A"].numpy(), P["B"].numpy(), inds, scores)
    got = np.concatenate([res[r][1].reshape(-1, C) for r in range(ws)])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    for r in range(ws):
        assert abs(res[r][2] - aux) < 1e-6 * max(1, aux) and abs(res[r][3] - z) < 1e-6 * max(1, z)
        assert abs(res[r][4] - mo.orthogonal_loss(P["A"].numpy())) < 1e-6 * max(1, res[r][4])


def test_rank_failure_surfaces_as_error_not_hang():
    P, res = _run(2, fail_rank=1, timeout=60)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error", res[0]  # the survivor's collective fails within the group timeout
