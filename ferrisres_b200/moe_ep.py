"""Expert-parallel MoE layer: experts sharded over the ranks of a process group.

Rank r holds experts [r*E/W, (r+1)*E/W) and routes its own tokens.  One layer
forward is:
  1. route (router GEMV + softmax + top-k, on the GPU) and build the
     expert-major layout of this rank's (token, k) entries;
  2. exchange the per-expert counts (all_gather of E int32 per rank) and
     read them on the host (a pinned copy and an event wait, while the GPU
     gathers the rows);
  3. dispatch: all_to_all_single of the gathered activation rows to the
     experts' owners (uneven splits from the counts);
  4. every owner runs ONE grouped expert launch over its (source rank,
     local expert) segments;
  5. combine: the reverse all_to_all_single brings the expert outputs back in
     the order they were sent, then the top-k weighted sum per token.
The reference has no expert parallelism (its distributed transports are
simulated, src/compute/distributed.rs:167-174); this is new.  Collectives run
on torch.distributed (NCCL over NVLink on B200, gloo in the CPU tests).  The
compute stages come from a backend: ``GpuMoEBackend`` calls
libferris_ternary.so; the tests plug in a CPU backend to check the exchange
bookkeeping on gloo ranks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from ._lib import ShapeError, call


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


class GpuMoEBackend:
    """Stages of ft_moe_* on the current CUDA stream.  Intermediate buffers are
    kept between calls (one set per name and shape): every stage of a step is
    ordered on the stream after the previous step's use of the same buffer, and
    the per-step allocations were a sizeable part of the host's time."""

    def __init__(self, layer):
        self.layer = layer
        self.E, self.K, self.H = layer.n_experts, layer.top_k, layer.hidden_dim
        self._bufs = {}
        self.tag = 0  # micro-batch in flight: buffers are kept per micro-batch

    def _s(self):
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def buf(self, name, shape, dtype, device):
        name = (name, self.tag)
        key = (name, tuple(shape), dtype, device)
        t = self._bufs.get(key)
        if t is None:
            for k in [k for k in self._bufs if k[0] == name]:  # one shape per name
                del self._bufs[k]
            t = self._bufs[key] = torch.empty(shape, dtype=dtype, device=device)
        return t

    def route(self, x):
        T = x.shape[0]
        dev = x.device
        idx = self.buf("idx", (T, self.K), torch.int32, dev)
        w = self.buf("w", (T, self.K), torch.float32, dev)
        counts = self.buf("counts", (self.E,), torch.int32, dev)
        call("ft_moe_route", self.layer.ctx.handle, self.layer.handle, T, _p(x),
             int(x.dtype == torch.bfloat16), _p(idx), _p(w), None, _p(counts), self._s())
        return idx, w, counts

    def layout(self, idx, counts):
        T = idx.shape[0]
        dev = idx.device
        offs = self.buf("offs", (self.E + 1,), torch.int32, dev)
        fill = self.buf("fill", (self.E,), torch.int32, dev)
        slot_of = self.buf("slot_of", (T * self.K,), torch.int32, dev)
        token_of = self.buf("token_of", (T * self.K,), torch.int32, dev)
        call("ft_moe_dispatch_layout", self.layer.ctx.handle, self.layer.handle, T, _p(idx),
             _p(counts), _p(offs), _p(fill), _p(slot_of), _p(token_of), self._s())
        return slot_of, token_of

    def gather(self, x, token_of):
        n = token_of.numel()
        out = self.buf("xg", (n, self.H), x.dtype, x.device)
        call("ft_moe_gather_rows", self.layer.ctx.handle, _p(x), x.element_size(), self.H,
             _p(token_of), n, _p(out), self._s())
        return out

    def experts(self, seg_experts, seg_rows, x_rows):
        total = int(sum(seg_rows))
        out = self.buf("o_recv", (total, self.H), torch.float32, x_rows.device)
        if len(seg_experts):
            e = np.ascontiguousarray(seg_experts, np.int32)
            r = np.ascontiguousarray(seg_rows, np.int64)
            call("ft_moe_expert_ffn", self.layer.ctx.handle, self.layer.handle, len(e),
                 e.ctypes.data_as(C.c_void_p), r.ctypes.data_as(C.c_void_p), _p(x_rows),
                 int(x_rows.dtype == torch.bfloat16), _p(out), self._s())
        return out

    def combine(self, o_rows, slot_of, w, out=None):
        T = w.shape[0]
        y = out if out is not None else torch.empty(T, self.H, dtype=torch.float32,
                                                     device=o_rows.device)
        call("ft_moe_combine", self.layer.ctx.handle, self.layer.handle, T, _p(o_rows),
             _p(slot_of), _p(w), _p(y), self._s())
        return y


_PINNED = {}


def _pinned_counts(world, E, dtype, tag=0):
    """A reused pinned host buffer for the gathered counts (one per micro-batch)."""
    key = (world, E, dtype, tag)
    if key not in _PINNED:
        _PINNED[key] = torch.empty(world, E, dtype=dtype).pin_memory()
    return _PINNED[key]


def ep_forward(x, backend, n_experts, rank=0, world=1, group=None, marks=None, stats=None,
               micro=1):
    """One expert-parallel MoE forward of this rank's tokens x [T, H].

    ``micro`` > 1 splits the tokens into that many micro-batches whose routes
    and count exchanges are all issued first: while the host waits for one
    micro-batch's counts (the step's host synchronisation) the GPU still has
    the others' work queued, and while it runs one micro-batch's experts the
    host issues the next one's exchange.  Results are identical (every token
    is computed from its own row).
    ``marks`` (optional list, micro = 1): a CUDA event is recorded on the
    current stream after each phase and appended as (phase name, event), for
    per-phase timing.  ``stats`` (optional dict) receives the rows this rank
    sent to and received from other ranks."""

    def mark(name):
        if marks is not None and micro <= 1:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    def set_tag(i):
        if hasattr(backend, "tag"):
            backend.tag = i

    E = n_experts
    if E % world:
        raise ShapeError(f"{E} experts do not split over {world} ranks")
    per = E // world
    T, H = x.shape[0], x.shape[1]
    parts = [x] if micro <= 1 or T < micro else list(x.chunk(micro))
    mark("start")
    # phase 1, every micro-batch: route, expert-major layout, counts of every
    # rank to the host (pinned copy + event), row gather
    st = []
    for i, xc in enumerate(parts):
        set_tag(i)
        idx, w, counts = backend.route(xc)
        slot_of, token_of = backend.layout(idx, counts)
        if world == 1:
            ac_dev = counts.view(1, E)
        else:
            ac_dev = torch.empty(world * E, dtype=counts.dtype, device=counts.device)
            dist.all_gather_into_tensor(ac_dev, counts, group=group)
            ac_dev = ac_dev.view(world, E)
        if ac_dev.is_cuda:
            ac_host = _pinned_counts(world, E, counts.dtype, i)
            ac_host.copy_(ac_dev, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record()
        else:
            ac_host, ready = ac_dev, None
        xg = backend.gather(xc, token_of)  # [rows, H], expert-major
        st.append((xc.shape[0], w, slot_of, xg, ac_host, ready))
    mark("route")
    out = None
    if len(parts) > 1 and x.is_cuda:
        out = torch.empty(T, backend.H if hasattr(backend, "H") else H, dtype=torch.float32,
                          device=x.device)
    ys, t0 = [], 0
    sent = recvd = 0
    for i, (tc, w, slot_of, xg, ac_host, ready) in enumerate(st):
        set_tag(i)
        if ready is not None:
            ready.synchronize()
        ac = ac_host.numpy().astype(np.int64)  # [src rank, expert]
        mark("counts")
        send_rows = ac[rank].reshape(world, per).sum(axis=1).tolist()
        recv_rows = ac[:, rank * per:(rank + 1) * per].sum(axis=1).tolist()
        sent += sum(n for d, n in enumerate(send_rows) if d != rank)
        recvd += sum(n for s, n in enumerate(recv_rows) if s != rank)
        if world == 1:
            recv = xg
        else:
            recv = torch.empty(sum(recv_rows), H, dtype=xg.dtype, device=xg.device)
            dist.all_to_all_single(recv.view(-1), xg.reshape(-1), [r * H for r in recv_rows],
                                   [r * H for r in send_rows], group=group)
        mark("dispatch")
        seg_e = np.tile(np.arange(rank * per, (rank + 1) * per, dtype=np.int32), world)
        seg_n = ac[:, rank * per:(rank + 1) * per].reshape(-1)
        o_recv = backend.experts(seg_e, seg_n, recv)
        mark("experts")
        if world == 1:
            o_send = o_recv
        else:
            o_send = torch.empty(xg.shape[0], H, dtype=o_recv.dtype, device=xg.device)
            dist.all_to_all_single(o_send.view(-1), o_recv.view(-1), [r * H for r in send_rows],
                                   [r * H for r in recv_rows], group=group)
        mark("combine")
        if out is not None:
            backend.combine(o_send, slot_of, w, out=out[t0:t0 + tc])
        else:
            ys.append(backend.combine(o_send, slot_of, w))
        t0 += tc
        mark("sum")
    set_tag(0)
    if stats is not None:
        stats["sent_rows_remote"] = sent
        stats["recv_rows_remote"] = recvd
    if out is not None:
        return out
    return ys[0] if len(ys) == 1 else torch.cat(ys)
