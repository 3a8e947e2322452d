"""A paged, routed K/V cache that feeds ``ultrametric_decode``.

sparse-ai's routed paged decode (``src/ultrametric/kernel_decode.py:188-247``) takes a paged
cache -- K/V pools indexed by physical page, per-request block tables, context lengths and a
routing vector per physical page -- but nothing in the reference fills one: its surgery layer
decodes from a dense cache with an eager token mask (``src/llama_surgery/surgery.py:883-891``).
``PagedKVCache`` is that missing caller side:

* a host-side page allocator (``PageAllocator``: free list, per-request page lists, no device
  synchronisation) that assigns a new physical page whenever a request's next token starts one;
* ``prefill``: writes a prompt's K/V rows into freshly allocated pages with their routes;
* ``append``: one new token per request, written on the device by ``sa_paged_kv_append``
  (K/V rows scattered into the tail page, the tail page's routing vector refreshed -- the
  reference recomputes its tail block's route at every decode step, surgery.py:350-374 --
  and the context length advanced);
* ``decode``: ``ultrametric_decode`` over the cache.

Routes follow the decode's convention: ``router`` is (num_pages, H, TD), indexed by the
PHYSICAL page id (kernel_decode.py:79).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from . import _native as nat
from .kernel_decode import ultrametric_decode


class PageAllocator:
    """Physical pages on the host: a free list and each request's pages in logical order.
    Pure bookkeeping, no device work."""

    def __init__(self, num_pages: int, page_size: int):
        self.page_size = int(page_size)
        self.free: List[int] = list(range(num_pages - 1, -1, -1))  # pop() hands out 0, 1, ...
        self.pages: Dict[int, List[int]] = {}
        self.length: Dict[int, int] = {}

    def add(self, rid: int) -> None:
        if rid in self.pages:
            raise ValueError(f"request {rid} already exists")
        self.pages[rid] = []
        self.length[rid] = 0

    def reserve(self, rid: int, n_tokens: int) -> List[int]:
        """Make room for ``n_tokens`` more tokens of ``rid``; returns the pages it added."""
        need = -(-(self.length[rid] + n_tokens) // self.page_size) - len(self.pages[rid])
        if need > len(self.free):
            raise RuntimeError(f"out of pages: request {rid} needs {need}, {len(self.free)} free")
        added = [self.free.pop() for _ in range(max(0, need))]
        self.pages[rid].extend(added)
        self.length[rid] += n_tokens
        return added

    def release(self, rid: int) -> None:
        self.free.extend(reversed(self.pages.pop(rid)))
        del self.length[rid]


class PagedKVCache:
    """K/V pools (num_pages, Hkv, page_size, D), block tables (max_requests, max_pages) int32,
    context lengths (max_requests,) int32 and page routes (num_pages, H, TD) int32 on one
    device.  Request slots are rows of the block table; ``decode`` runs the given slots."""

    def __init__(self, num_pages: int, num_kv_heads: int, page_size: int, head_dim: int,
                 num_heads: int, tree_depth: int, max_requests: int, max_pages_per_request: int,
                 dtype=torch.bfloat16, device="cuda"):
        self.page_size, self.H, self.TD = int(page_size), int(num_heads), int(tree_depth)
        shape = (num_pages, num_kv_heads, page_size, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.v_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.router = torch.zeros((num_pages, num_heads, tree_depth), dtype=torch.int32, device=device)
        self.block_tables = torch.zeros((max_requests, max_pages_per_request), dtype=torch.int32,
                                        device=device)
        self.context_lens = torch.zeros((max_requests,), dtype=torch.int32, device=device)
        self.alloc = PageAllocator(num_pages, page_size)
        self.max_pages = int(max_pages_per_request)

    # -- host bookkeeping -------------------------------------------------------------------
    def add_request(self, rid: int) -> None:
        if not 0 <= rid < self.block_tables.shape[0]:
            raise ValueError(f"request slot {rid} out of range")
        self.alloc.add(rid)

    def free_request(self, rid: int) -> None:
        self.alloc.release(rid)
        self.context_lens[rid] = 0

    def _grow(self, rid: int, n_tokens: int) -> None:
        start = len(self.alloc.pages[rid])
        added = self.alloc.reserve(rid, n_tokens)
        if len(self.alloc.pages[rid]) > self.max_pages:
            raise RuntimeError(f"request {rid} exceeds {self.max_pages} pages")
        if added:
            self.block_tables[rid, start:start + len(added)] = torch.tensor(
                added, dtype=torch.int32).to(self.block_tables.device, non_blocking=True)

    # -- device writes ------------------------------------------------------------------------
    def prefill(self, rid: int, k: torch.Tensor, v: torch.Tensor, page_routes: torch.Tensor) -> None:
        """Write a prompt: k, v (S, Hkv, D); page_routes (ceil(S / page_size), H, TD)."""
        S = k.shape[0]
        if self.alloc.length[rid] != 0:
            raise ValueError("prefill expects an empty request")
        self._grow(rid, S)
        pages = torch.tensor(self.alloc.pages[rid], dtype=torch.long, device=k.device)
        n = pages.numel()
        pad = n * self.page_size - S
        kk = torch.nn.functional.pad(k, (0, 0, 0, 0, 0, pad)).view(n, self.page_size, *k.shape[1:])
        vv = torch.nn.functional.pad(v, (0, 0, 0, 0, 0, pad)).view(n, self.page_size, *v.shape[1:])
        self.k_cache[pages] = kk.transpose(1, 2).to(self.k_cache.dtype)
        self.v_cache[pages] = vv.transpose(1, 2).to(self.v_cache.dtype)
        self.router[pages] = page_routes.to(self.router.dtype)
        self.context_lens[rid] = S

    def append(self, rids: Sequence[int], k: torch.Tensor, v: torch.Tensor,
               tail_routes: Optional[torch.Tensor] = None) -> None:
        """One new token for each request in ``rids`` (given in slot order, ``rids`` a
        contiguous range of slots): k, v (len(rids), Hkv, D); ``tail_routes`` (len(rids), H, TD)
        becomes the routing vector of the page that receives the token."""
        rids = list(rids)
        if rids != list(range(rids[0], rids[0] + len(rids))):
            raise ValueError("append expects a contiguous range of request slots")
        for r in rids:
            self._grow(r, 1)
        sl = slice(rids[0], rids[0] + len(rids))
        bt, ctx = self.block_tables[sl], self.context_lens[sl]
        kk = k if k.stride(-1) == 1 else k.contiguous()
        vv = v if v.stride(-1) == 1 else v.contiguous()
        tr = tail_routes
        nat.check(nat.lib().sa_paged_kv_append(
            nat.float_code(self.k_cache.dtype), len(rids), self.k_cache.shape[1], self.k_cache.shape[3],
            self.page_size, self.k_cache.shape[0], kk.data_ptr(), nat.strides(kk), vv.data_ptr(),
            nat.strides(vv), bt.data_ptr(), nat.strides(bt), bt.shape[1], ctx.data_ptr(),
            self.k_cache.data_ptr(), nat.strides(self.k_cache), self.v_cache.data_ptr(),
            nat.strides(self.v_cache), nat.ptr(tr), nat.int_code(tr.dtype) if tr is not None else 0,
            nat.strides(tr) if tr is not None else None, self.H, self.TD, self.router.data_ptr(),
            nat.int_code(self.router.dtype), nat.strides(self.router), nat.stream_of(self.k_cache)),
            "paged append")

    def decode(self, q: torch.Tensor, q_routes: torch.Tensor, req_depth: int, rids: Sequence[int],
               local_blocks: int = 1, sink_block: bool = True) -> torch.Tensor:
        """``ultrametric_decode`` of one query token per request over a contiguous range of slots."""
        rids = list(rids)
        sl = slice(rids[0], rids[0] + len(rids))
        return ultrametric_decode(q, self.k_cache, self.v_cache, self.block_tables[sl],
                                  self.context_lens[sl], self.router, q_routes, req_depth,
                                  local_blocks=local_blocks, sink_block=sink_block)
