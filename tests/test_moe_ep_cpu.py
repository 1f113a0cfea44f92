"""Expert-parallel exchange logic on gloo CPU ranks (world size 2 and 4).

A float64 CPU backend stands in for the GPU stages (router top-k, layout,
gather, per-expert linear+SwiGLU experts, combine); the test checks that the
count exchange, the two uneven all_to_all_single calls and the segment order
reproduce a single-process forward over all tokens exactly.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ferrisres_b200.moe_ep import ep_forward


class CpuBackend:
    def __init__(self, R, Wg, Wu, Wd, K):
        self.R, self.Wg, self.Wu, self.Wd, self.K = R, Wg, Wu, Wd, K
        self.E, self.H = R.shape

    def route(self, x):
        p = torch.softmax(x @ self.R.T, dim=1)
        order = torch.argsort(-p, dim=1, stable=True)[:, :self.K]
        w = torch.gather(p, 1, order)
        w = w / w.sum(dim=1, keepdim=True)
        counts = torch.bincount(order.reshape(-1), minlength=self.E).to(torch.int32)
        return order.to(torch.int32), w, counts

    def layout(self, idx, counts):
        flat = idx.reshape(-1).long()
        order = torch.argsort(flat, stable=True)  # expert-major, then (token, k) order
        slot_of = torch.empty_like(order)
        slot_of[order] = torch.arange(order.numel())
        token_of = (order // self.K).to(torch.int32)
        return slot_of.to(torch.int32), token_of

    def gather(self, x, token_of):
        return x[token_of.long()]

    def experts(self, seg_e, seg_n, x_rows):
        out, r = [], 0
        for e, n in zip(seg_e, seg_n):
            xs = x_rows[r:r + n]
            g = xs @ self.Wg[e].T
            h = g / (1 + torch.exp(-g)) * (xs @ self.Wu[e].T)
            out.append(h @ self.Wd[e].T)
            r += n
        return torch.cat(out) if out else x_rows.new_zeros(0, self.H)

    def combine(self, o, slot_of, w):
        T = w.shape[0]
        o = o[slot_of.long()].view(T, self.K, self.H)
        return (o * w.unsqueeze(-1)).sum(dim=1)


def make(E=8, H=16, F=12, T=24, K=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    R = torch.randn(E, H, generator=g, dtype=torch.float64)
    Wg = torch.randn(E, F, H, generator=g, dtype=torch.float64)
    Wu = torch.randn(E, F, H, generator=g, dtype=torch.float64)
    Wd = torch.randn(E, H, F, generator=g, dtype=torch.float64)
    x = torch.randn(T, H, generator=g, dtype=torch.float64)
    return CpuBackend(R, Wg, Wu, Wd, K), x


def _worker(rank, world, port, out_q, micro):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be, x = make()
        shard = x.chunk(world)[rank]
        y = ep_forward(shard, be, be.E, rank, world, micro=micro)
        out_q.put((rank, y.numpy()))
    except Exception as e:  # surface the failure to the parent instead of a queue timeout
        out_q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,micro", [(2, 1), (4, 1), (2, 3)])
def test_ep_matches_single_process(world, micro):
    be, x = make()
    ref = ep_forward(x, be, be.E).numpy()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, micro)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert not isinstance(got[r], str), f"rank {r} failed: {got[r]}"
    y = np.concatenate([got[r] for r in range(world)])
    assert np.allclose(y, ref, rtol=1e-12, atol=1e-12)
