"""Multi-GPU drivers for sparse_attn_sharedkv (one process per GPU).

The op has no exchange step between requests, so it shards two ways:

* request-parallel: every rank owns a subset of the requests with their
  paged caches, block tables, indices and query rows, and runs the op on its
  own batch; nothing is communicated. ``partition_requests`` balances the
  requests (longest first, capped at ceil(B / world) per rank) and
  ``select_requests`` cuts a rank's batch out of a full one.
* head-sharded: every rank computes ``H / world`` query heads of every
  request and every rank ends with all heads. ``head_sharded_forward_p2p``
  (GPUs, NCCL group) has the attention kernel itself store each result into
  every rank's output buffer through peer pointers into symmetric memory
  (NVLink), so the gather happens while the kernel computes;
  ``head_sharded_forward`` runs the kernel and then an NCCL all-gather (also
  the form the gloo CPU tests use). The KV rows are shared by all heads, so
  each rank still reads every KV row: this mode trades bandwidth for latency
  by construction.
"""

from __future__ import annotations

import math
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist


def partition_requests(ctx: Sequence[int], world: int) -> List[List[int]]:
    """Request ids per rank: longest-processing-time order on context length,
    at most ceil(B / world) requests per rank (per-token work is O(window + K)
    and nearly context-independent, so request counts balance the compute and
    context lengths balance the cache footprint)."""
    order = sorted(range(len(ctx)), key=lambda i: (-int(ctx[i]), i))
    cap = math.ceil(len(ctx) / world) if len(ctx) else 0
    loads = [0] * world
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        cand = [p for p in range(world) if len(parts[p]) < cap]
        p = min(cand, key=lambda j: (loads[j], j))
        parts[p].append(i)
        loads[p] += int(ctx[i])
    return [sorted(p) for p in parts]


def select_requests(batch: Dict[str, torch.Tensor], req_ids: Sequence[int]) -> Dict[str, torch.Tensor]:
    """The sub-batch of ``req_ids`` from a TND batch given as the keyword set of
    ``sparse_attn_sharedkv`` plus ``q``. Paged pools are shared by reference;
    per-request rows (block tables, lengths) and per-token rows (q, indices)
    are gathered."""
    cu = batch["cu_seqlens_q"].to("cpu", torch.int64)
    ids = torch.as_tensor(list(req_ids), dtype=torch.int64)
    lens = (cu[1:] - cu[:-1])[ids]
    tok = torch.cat([torch.arange(int(cu[i]), int(cu[i + 1])) for i in ids.tolist()]) if len(ids) else \
        torch.zeros(0, dtype=torch.int64)
    dev = batch["q"].device
    tok_d = tok.to(dev)
    ids_d = ids.to(dev)
    out = dict(batch)
    out["q"] = batch["q"].index_select(0, tok_d)
    new_cu = torch.zeros(len(ids) + 1, dtype=torch.int32)
    new_cu[1:] = torch.cumsum(lens, 0).to(torch.int32)
    out["cu_seqlens_q"] = new_cu.to(batch["cu_seqlens_q"].device)
    out["seqused_kv"] = batch["seqused_kv"].index_select(0, ids_d.to(batch["seqused_kv"].device))
    out["ori_block_table"] = batch["ori_block_table"].index_select(0, ids_d.to(batch["ori_block_table"].device))
    if batch.get("cmp_block_table") is not None:
        out["cmp_block_table"] = batch["cmp_block_table"].index_select(0, ids_d.to(batch["cmp_block_table"].device))
    if batch.get("cmp_sparse_indices") is not None:
        out["cmp_sparse_indices"] = batch["cmp_sparse_indices"].index_select(
            0, tok_d.to(batch["cmp_sparse_indices"].device))
    out.pop("metadata", None)
    return out


def _all_gather(dst: torch.Tensor, src: torch.Tensor, group) -> None:
    """dst[r] = src of rank r (one NCCL all-gather on GPUs; list form on gloo)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(dst, src, group=group)
    else:
        dist.all_gather(list(dst.unbind(0)), src, group=group)


def head_range(num_heads: int, world: int, rank: int):
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    h = num_heads // world
    return rank * h, (rank + 1) * h


def head_sharded_forward(q: torch.Tensor, *, group: Optional[dist.ProcessGroup] = None,
                         local_fn: Optional[Callable] = None, **kw):
    """Run ``H / world`` heads of every request on this rank and all-gather the
    outputs. Returns ``(out [T, H, 512], lse [T, H])`` on every rank.

    ``local_fn(q_local, sinks=..., **kw) -> (out_local, lse_local)`` defaults to
    ``sparse_attn_sharedkv(..., return_softmax_lse=True)``; tests pass a CPU
    stand-in to exercise the sharding logic on gloo ranks."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, H, D = q.shape
    h0, h1 = head_range(H, world, rank)
    sinks = kw.pop("sinks")
    if local_fn is None:
        from .api import sparse_attn_sharedkv

        def local_fn(ql, **k):
            return sparse_attn_sharedkv(ql, return_softmax_lse=True, **k)

    o_loc, l_loc = local_fn(q[:, h0:h1].contiguous(), sinks=sinks[h0:h1].contiguous(), **kw)
    hs = h1 - h0
    o_all = torch.empty((world, T, hs, D), dtype=o_loc.dtype, device=o_loc.device)
    l_all = torch.empty((world, T, hs), dtype=l_loc.dtype, device=l_loc.device)
    _all_gather(o_all, o_loc.contiguous(), group)
    _all_gather(l_all, l_loc.contiguous(), group)
    out = o_all.permute(1, 0, 2, 3).reshape(T, H, D)
    lse = l_all.permute(1, 0, 2).reshape(T, H)
    return out, lse


_SYMM: Dict[tuple, tuple] = {}


def _symmetric_outputs(T: int, H: int, dtype, device, group):
    """Cached symmetric-memory output and LSE buffers of this rank, with the
    device pointers of every rank's copies."""
    import os

    # plain peer pointers are all the kernel uses: no NVLink multicast object
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import torch.distributed._symmetric_memory as symm_mem

    key = (T, H, dtype, device.index, id(group))
    if key not in _SYMM:
        out = symm_mem.empty((T, H, 512), dtype=dtype, device=device)
        lse = symm_mem.empty((T, H), dtype=torch.float32, device=device)
        gname = group.group_name if group is not None else dist.group.WORLD.group_name
        ho = symm_mem.rendezvous(out, gname)
        hl = symm_mem.rendezvous(lse, gname)
        _SYMM[key] = (out, lse, ho, hl, list(ho.buffer_ptrs), list(hl.buffer_ptrs))
    return _SYMM[key]


def head_sharded_forward_p2p(q: torch.Tensor, *, group: Optional[dist.ProcessGroup] = None, **kw):
    """Head-sharded forward whose gather is done by the attention kernel's own
    peer stores (``sas_sparse_attn_sharedkv_fwd_gather``): this rank computes
    heads ``[rank * H / world, (rank + 1) * H / world)`` and writes them into
    the symmetric output buffers of all ranks. Returns this rank's buffers
    ``(out [T, H, 512], lse [T, H])``, complete once every rank has written;
    they are reused by the next call with the same shape."""
    from .api import sparse_attn_sharedkv

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, H, D = q.shape
    h0, h1 = head_range(H, world, rank)
    out, lse, ho, hl, optrs, lptrs = _symmetric_outputs(T, H, q.dtype, q.device, group)
    sinks = kw.pop("sinks")
    kw.pop("out", None)
    kw.pop("lse_out", None)
    ho.barrier(channel=0)  # every rank is done reading the buffers' previous contents
    sparse_attn_sharedkv(q[:, h0:h1].contiguous(), sinks=sinks[h0:h1].contiguous(),
                         _gather=(optrs, lptrs, H, h0), **kw)
    ho.barrier(channel=1)  # every rank's stores into this rank's buffers are done
    return out, lse
