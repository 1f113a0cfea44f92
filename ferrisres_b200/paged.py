"""Paged 3-bit KV cache: PagedAttention's block metadata over a device page pool.

The reference's PagedAttention (src/inference/paged_attention.rs) is metadata
only: ``BlockAllocator`` (:44-150) hands out block ids with reference counts,
a ``BlockTable`` (:158-224) per request and layer maps logical block j to a
block id, ``PrefixSharingManager`` (:294-350) shares the blocks of a common
prompt, ``PagedAttentionManager`` (:354-527) creates, forks and frees requests.
It allocates no GPU memory.  This module keeps those classes with the same
methods and semantics (host metadata, as in the reference), and adds what the
reference lacks: ``PagedKv3Cache``, which stores the positions in a device
page pool (``ft_kvp``: page P = 32 positions of every kv head in the 3-bit
record format of the ring cache) and appends, reads and flash-decodes through
the block tables, with copy-on-write of a shared partially filled page.

The device block size is 32 positions (the reference's default is 16;
``BlockTable`` and ``BlockAllocator`` themselves accept any size).
"""
from __future__ import annotations

import ctypes as C
from collections import OrderedDict

import numpy as np
import torch

from ._lib import OOMError, ShapeError, call
from .gpu import _dptr, _stream_ptr, get_context

DEFAULT_BLOCK_SIZE = 16   # the reference's default (paged_attention.rs:21)
PAGE_POSITIONS = 32       # positions per device page
HEAD_DIM = 128
REC_BYTES = HEAD_DIM * 3 // 8


# ------------------------------------------------------------- metadata --
class BlockAllocator:
    """Pool of block ids with reference counts (paged_attention.rs:44-150)."""

    def __init__(self, num_blocks: int, block_size: int, hidden_dim: int):
        self._ref = [0] * int(num_blocks)
        self._allocated = [False] * int(num_blocks)
        # ids are handed out from the end of the free list, so a fresh pool
        # gives the highest id first, as the reference's Vec::pop does
        self._free = list(range(int(num_blocks)))
        self._block_size = int(block_size)
        self._hidden_dim = int(hidden_dim)

    def allocate(self):
        """A free block id with reference count 1, or None when the pool is empty."""
        if not self._free:
            return None
        b = self._free.pop()
        self._ref[b] = 1
        self._allocated[b] = True
        return b

    def free(self, block_id: int) -> None:
        """Drops one reference; the block returns to the pool at zero."""
        if self._ref[block_id] > 0:
            self._ref[block_id] -= 1
        if self._ref[block_id] == 0 and self._allocated[block_id]:
            self._allocated[block_id] = False
            self._free.append(block_id)

    def add_ref(self, block_id: int) -> None:
        self._ref[block_id] += 1

    def ref_count(self, block_id: int) -> int:
        return self._ref[block_id]

    def num_free(self) -> int:
        return len(self._free)

    def total_blocks(self) -> int:
        return len(self._ref)

    def block_size(self) -> int:
        return self._block_size

    def hidden_dim(self) -> int:
        return self._hidden_dim

    def utilization(self) -> float:
        n = len(self._ref)
        return 0.0 if n == 0 else 1.0 - len(self._free) / n

    def memory_used_bytes(self) -> int:
        """The reference's fp32 K+V figure for the used blocks (:142-146)."""
        return (len(self._ref) - len(self._free)) * self._block_size * self._hidden_dim * 4 * 2


class BlockTable:
    """Logical block -> block id of one request and layer (:158-224)."""

    def __init__(self, block_size: int):
        self._table: list[int] = []
        self._tokens = 0
        self._bs = int(block_size)

    def num_blocks_needed(self) -> int:
        return -(-self._tokens // self._bs)

    def num_blocks_allocated(self) -> int:
        return len(self._table)

    def block_for_position(self, pos: int):
        j = pos // self._bs
        return self._table[j] if j < len(self._table) else None

    def append_block(self, block_id: int) -> None:
        self._table.append(int(block_id))

    def add_tokens(self, n: int) -> None:
        self._tokens += int(n)

    def num_tokens(self) -> int:
        return self._tokens

    def table(self) -> list[int]:
        return self._table

    def clear(self) -> None:
        self._table = []
        self._tokens = 0

    def slot_in_block(self, pos: int) -> int:
        return pos % self._bs


class RequestState:
    """Per-request block tables, one per layer (:229-283)."""

    def __init__(self, request_id: int, num_layers: int, block_size: int):
        self._tables = [BlockTable(block_size) for _ in range(int(num_layers))]
        self._id = int(request_id)
        self._bs = int(block_size)
        self._tokens = 0

    def layer_table(self, layer_idx: int) -> BlockTable:
        return self._tables[layer_idx]

    layer_table_mut = layer_table

    def num_tokens(self) -> int:
        return self._tokens

    def add_tokens(self, n: int) -> None:
        self._tokens += int(n)

    def request_id(self) -> int:
        return self._id

    def num_layers(self) -> int:
        return len(self._tables)


class PrefixSharingManager:
    """Token prefix -> per-layer block ids, shared by reference count (:294-350)."""

    def __init__(self, allocator: BlockAllocator, block_size: int):
        self._prefixes: dict[tuple, list[list[int]]] = {}
        self._alloc = allocator
        self._bs = int(block_size)

    def register_prefix(self, prefix_tokens, layer_blocks) -> None:
        self._prefixes[tuple(prefix_tokens)] = [list(b) for b in layer_blocks]

    def lookup_prefix(self, prefix_tokens):
        """The blocks of a registered prefix, one more reference on each; None if absent."""
        blocks = self._prefixes.get(tuple(prefix_tokens))
        if blocks is None:
            return None
        for layer_blocks in blocks:
            for b in layer_blocks:
                self._alloc.add_ref(b)
        return [list(b) for b in blocks]

    def num_prefixes(self) -> int:
        return len(self._prefixes)

    def has_prefix(self, tokens) -> bool:
        return tuple(tokens) in self._prefixes

    def remove_prefix(self, tokens) -> None:
        self._prefixes.pop(tuple(tokens), None)


class PagedAttentionManager:
    """Requests over a shared block pool (:354-527)."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, hidden_dim: int):
        self.allocator = BlockAllocator(num_blocks, block_size, hidden_dim)
        self._prefix = PrefixSharingManager(self.allocator, block_size)
        self._requests: OrderedDict[int, RequestState] = OrderedDict()
        self._bs = int(block_size)
        self._hidden = int(hidden_dim)
        self._layers = int(num_layers)
        self._next = 0

    def create_request(self, prefill_len: int) -> int:
        return self.create_request_with_layers(prefill_len, self._layers)

    def create_request_with_layers(self, prefill_len: int, num_layers: int) -> int:
        """A new request with blocks for ``prefill_len`` tokens in each layer
        (an exhausted pool leaves the table short, as in the reference)."""
        rid = self._next
        self._next += 1
        st = RequestState(rid, num_layers, self._bs)
        need = -(-int(prefill_len) // self._bs)
        for layer in range(num_layers):
            t = st.layer_table(layer)
            for _ in range(need):
                b = self.allocator.allocate()
                if b is not None:
                    t.append_block(b)
            t.add_tokens(prefill_len)
        st.add_tokens(prefill_len)
        self._requests[rid] = st
        return rid

    def fork_request(self, parent_id: int):
        """A child sharing every block of the parent (one more reference each)."""
        parent = self._requests.get(parent_id)
        if parent is None:
            return None
        cid = self._next
        self._next += 1
        child = RequestState(cid, parent.num_layers(), self._bs)
        child._tokens = parent.num_tokens()
        for layer in range(parent.num_layers()):
            pt, ct = parent.layer_table(layer), child.layer_table(layer)
            for b in pt.table():
                self.allocator.add_ref(b)
                ct.append_block(b)
            ct.add_tokens(pt.num_tokens())
        self._requests[cid] = child
        return cid

    def free_request(self, request_id: int) -> None:
        st = self._requests.pop(request_id, None)
        if st is None:
            return
        for layer in range(st.num_layers()):
            for b in st.layer_table(layer).table():
                self.allocator.free(b)

    def get_request(self, request_id: int):
        return self._requests.get(request_id)

    get_request_mut = get_request

    def num_requests(self) -> int:
        return len(self._requests)

    def utilization(self) -> float:
        return self.allocator.utilization()

    def num_free_blocks(self) -> int:
        return self.allocator.num_free()

    def block_size(self) -> int:
        return self._bs

    def prefix_manager(self) -> PrefixSharingManager:
        return self._prefix

    prefix_manager_mut = prefix_manager


# ----------------------------------------------------------- device pool --
class PagedKv3Cache:
    """3-bit KV cache of many requests over ``num_layers`` layers, paged.

    Metadata: a ``PagedAttentionManager`` with 32-position blocks; block id P
    is page P of one device pool shared by all layers (``ft_kvp``).  A
    request's positions are appended layer by layer; pages are allocated as
    they fill, and a page that a fork shares is copied before a request
    writes into it (copy-on-write).  Flash decode, get_range and export run
    on the device through the requests' block tables.
    """

    def __init__(self, num_layers: int, num_pages: int, kv_heads: int,
                 head_dim: int = HEAD_DIM, device=None, mode: str = "R", seed: int = 0):
        if mode not in ("R", "T"):
            raise ShapeError("mode must be 'R' or 'T'")
        self.ctx = get_context(device)
        self.device = torch.device("cuda", self.ctx.device)
        self.kv_heads, self.mode = int(kv_heads), mode
        self.manager = PagedAttentionManager(num_layers, num_pages, PAGE_POSITIONS,
                                             self.kv_heads * int(head_dim))
        h = C.c_void_p()
        call("ft_kvp_create", self.ctx.handle, int(num_pages), self.kv_heads, int(head_dim),
             PAGE_POSITIONS, 0 if mode == "R" else 1, int(seed) & (2**64 - 1), C.byref(h))
        self.handle = h

    # ---- requests
    def create_request(self) -> int:
        return self.manager.create_request(0)

    def fork_request(self, parent_id: int) -> int:
        cid = self.manager.fork_request(parent_id)
        if cid is None:
            raise ShapeError(f"no request {parent_id}")
        return cid

    def free_request(self, request_id: int) -> None:
        self.manager.free_request(request_id)

    def seq_len(self, request_id: int, layer: int = 0) -> int:
        return self._state(request_id).layer_table(layer).num_tokens()

    def block_table(self, request_id: int, layer: int = 0) -> list[int]:
        return list(self._state(request_id).layer_table(layer).table())

    def signs(self) -> np.ndarray:
        out = np.empty(HEAD_DIM, np.float32)
        call("ft_kvp_signs", self.handle, out.ctypes.data_as(C.c_void_p))
        return out

    def _state(self, rid: int) -> RequestState:
        st = self.manager.get_request(rid)
        if st is None:
            raise ShapeError(f"no request {rid}")
        return st

    # ---- page bookkeeping
    def _prepare(self, layer: int, rid: int, n_pos: int, copies: list):
        """Pages for positions [len, len + n_pos) of (rid, layer): the shared
        partial page is replaced by a private copy, new pages are appended."""
        t = self._state(rid).layer_table(layer)
        alloc = self.manager.allocator
        length = t.num_tokens()
        tab = t.table()
        j = length // PAGE_POSITIONS
        cow = bool(length % PAGE_POSITIONS and n_pos and alloc.ref_count(tab[j]) > 1)
        need = -(-(length + n_pos) // PAGE_POSITIONS)
        if int(cow) + max(0, need - len(tab)) > alloc.num_free():
            raise OOMError(f"page pool exhausted: request {rid} needs "
                           f"{int(cow) + max(0, need - len(tab))} pages, {alloc.num_free()} free")
        if cow:
            old, new = tab[j], alloc.allocate()
            copies.append((old, new))
            tab[j] = new
            alloc.free(old)
        while len(tab) < need:
            tab.append(alloc.allocate())
        return length

    def _tables(self, layer: int, rids):
        tabs = [self._state(r).layer_table(layer).table() for r in rids]
        stride = max(1, max(len(t) for t in tabs))
        a = np.zeros((len(rids), stride), np.int32)
        for i, t in enumerate(tabs):
            a[i, :len(t)] = t
        return torch.from_numpy(a).to(self.device), stride

    def _kv_view(self, t: torch.Tensor, n_req: int) -> torch.Tensor:
        if t.device != self.device or t.dtype not in (torch.float32, torch.bfloat16):
            raise ShapeError("k, v must be fp32 or bf16 tensors on the cache's device")
        if t.dim() != 4 or t.shape[0] != n_req or t.shape[2] != self.kv_heads or \
                t.shape[3] != HEAD_DIM:
            raise ShapeError(f"k, v must be [requests={n_req}, n_pos, {self.kv_heads}, {HEAD_DIM}]")
        return t.contiguous()

    # ---- data
    def append(self, layer: int, request_ids, k: torch.Tensor, v: torch.Tensor, stream=None):
        """Appends n_pos positions to each request of ``request_ids`` in
        ``layer``: k, v [len(request_ids), n_pos, kv_heads, 128]."""
        rids = list(request_ids)
        if len(set(rids)) != len(rids):
            raise ShapeError("a request may appear once per append")
        k, v = self._kv_view(k, len(rids)), self._kv_view(v, len(rids))
        if k.shape != v.shape or k.dtype != v.dtype:
            raise ShapeError("k and v differ in shape or dtype")
        n_pos = int(k.shape[1])
        if n_pos == 0 or not rids:
            return
        copies = []
        starts = np.array([self._prepare(layer, r, n_pos, copies) for r in rids], np.int32)
        if copies:
            src = np.array([c[0] for c in copies], np.int32)
            dst = np.array([c[1] for c in copies], np.int32)
            call("ft_kvp_copy_pages", self.ctx.handle, self.handle, len(copies),
                 src.ctypes.data_as(C.c_void_p), dst.ctypes.data_as(C.c_void_p),
                 _stream_ptr(stream))
        tables, stride = self._tables(layer, rids)
        start_dev = torch.from_numpy(starts).to(self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        # the uploads above ran on the current stream; order the append after them
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream(self.device))
        call("ft_kvp_append", self.ctx.handle, self.handle, len(rids), n_pos, _dptr(tables),
             stride, _dptr(start_dev), _dptr(k), _dptr(v), 1 if k.dtype == torch.bfloat16 else 0,
             _stream_ptr(s))
        tables.record_stream(s)
        start_dev.record_stream(s)
        for r in rids:
            self._state(r).layer_table(layer).add_tokens(n_pos)
            if layer == 0:
                self._state(r).add_tokens(n_pos)

    def flash_decode(self, layer: int, request_ids, q: torch.Tensor, scale: float = 0.0,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """q [len(request_ids), q_heads, 128] fp32 -> softmax attention over
        each request's positions in ``layer`` (ragged lengths)."""
        rids = list(request_ids)
        if q.dim() != 3 or q.shape[0] != len(rids) or q.shape[2] != HEAD_DIM or \
                q.dtype != torch.float32 or q.device != self.device:
            raise ShapeError(f"q must be fp32 [{len(rids)}, q_heads, {HEAD_DIM}] on the device")
        q = q.contiguous()
        lens = np.array([self.seq_len(r, layer) for r in rids], np.int32)
        if lens.max(initial=0) == 0:
            raise ShapeError("flash decode over empty requests")
        tables, stride = self._tables(layer, rids)
        lens_dev = torch.from_numpy(lens).to(self.device)
        if out is None:
            out = torch.empty_like(q)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream(self.device))
        call("ft_kvp_flash_decode", self.ctx.handle, self.handle, len(rids), _dptr(tables),
             stride, _dptr(lens_dev), int(lens.max()), _dptr(q), int(q.shape[1]), float(scale),
             _dptr(out), _stream_ptr(s))
        tables.record_stream(s)
        lens_dev.record_stream(s)
        return out

    def _range_check(self, layer, rids, start, end):
        for r in rids:
            if not (0 <= start <= end <= self.seq_len(r, layer)):
                raise ShapeError(f"range [{start}, {end}) outside request {r} "
                                 f"({self.seq_len(r, layer)} positions)")

    def get_range(self, layer: int, request_ids, start: int, end: int, stream=None):
        """Dequantised K, V [len(request_ids), end-start, kv_heads, 128] fp32."""
        rids = list(request_ids)
        self._range_check(layer, rids, start, end)
        shape = (len(rids), end - start, self.kv_heads, HEAD_DIM)
        k = torch.empty(shape, dtype=torch.float32, device=self.device)
        v = torch.empty_like(k)
        tables, stride = self._tables(layer, rids)
        call("ft_kvp_get_range", self.ctx.handle, self.handle, len(rids), _dptr(tables), stride,
             int(start), int(end), _dptr(k), _dptr(v), _stream_ptr(stream))
        return k, v

    def export_range(self, layer: int, request_ids, start: int, end: int, stream=None):
        """The reference's stored form of positions [start, end): codes
        [n, end-start, kv_heads*48] uint8 and (min, max) [n, end-start, kv_heads, 2]."""
        rids = list(request_ids)
        self._range_check(layer, rids, start, end)
        n = end - start
        kc = torch.empty((len(rids), n, self.kv_heads * REC_BYTES), dtype=torch.uint8,
                         device=self.device)
        vc = torch.empty_like(kc)
        km = torch.empty((len(rids), n, self.kv_heads, 2), dtype=torch.float32, device=self.device)
        vm = torch.empty_like(km)
        tables, stride = self._tables(layer, rids)
        call("ft_kvp_export_range", self.ctx.handle, self.handle, len(rids), _dptr(tables), stride,
             int(start), int(end), _dptr(kc), _dptr(km), _dptr(vc), _dptr(vm),
             _stream_ptr(stream))
        return kc, km, vc, vm

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            call("ft_kvp_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
