"""Seeded synthetic inputs for the sparse_attn_sharedkv path.

The reference ships dense-tensor generators (``golden.py:315-473``:
``gen_ori_kv_paged``, ``gen_cmp_kv_paged``, ``gen_cmp_sparse_indices_tnd``)
that build a dense ``[B, N2, max_s, D]`` copy first and therefore cannot reach
the 64k-256k contexts of the long-context configurations. These generators
build the paged pools directly:

* raw (``ori``) cache: ``ceil(ctx/bs)`` blocks per request, physical block ids
  drawn from a random permutation of the pool (a shuffled block table, as in
  ``golden.py:342-348``), unused table slots ``-1``;
* compressed (``cmp``) cache: ``ctx // ratio`` rows per request, paged the
  same way;
* top-k indices: per query token, ``min(K, threshold)`` distinct ids drawn
  uniformly from the causally valid range ``[0, (s_g+1)//ratio)`` in random
  order, ``-1`` padded at the tail (``golden.py:442-473``).

``make_case`` returns numpy arrays (used by the parity tests and the CPU
oracle); ``make_case_torch`` builds the same structure directly on a CUDA
device for benchmark-sized configurations.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np


def _round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return _round_bf16(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    return x.astype(np.float32)


@dataclass
class Case:
    """One seeded input set in the reference's TND / PA_ND layout."""

    B: int
    H: int
    D: int
    dtype: str
    scenario: int  # 1 SWA, 2 CFA, 3 SCFA
    K: int
    cmp_ratio: int
    win_left: int
    cu_seqlens_q: np.ndarray  # [B+1] int32
    seqused_kv: np.ndarray  # [B] int32
    q: np.ndarray  # [T, H, D] float32 (dtype-rounded)
    ori_kv: np.ndarray  # [nblk, bs, 1, D]
    ori_bt: np.ndarray  # [B, L] int32
    cmp_kv: Optional[np.ndarray]
    cmp_bt: Optional[np.ndarray]
    idx: Optional[np.ndarray]  # [T, 1, K] int32
    sinks: np.ndarray  # [H] float32
    softmax_scale: float
    meta: dict = field(default_factory=dict)

    @property
    def T(self) -> int:
        return int(self.cu_seqlens_q[-1])


def _paged_table(rng, lens: Sequence[int], bs: int, spare: int):
    nb = [(int(l) + bs - 1) // bs for l in lens]
    total = sum(nb) + spare
    total = max(total, 1)
    perm = rng.permutation(total).astype(np.int32)
    width = max(max(nb) if nb else 0, 1)
    table = np.full((len(lens), width), -1, np.int32)
    cur = 0
    for b, n in enumerate(nb):
        table[b, :n] = perm[cur:cur + n]
        cur += n
    return table, total


def topk_indices(rng, thr: int, K: int) -> np.ndarray:
    row = np.full(K, -1, np.int32)
    take = min(max(thr, 0), K)
    if take > 0:
        row[:take] = rng.choice(thr, size=take, replace=False).astype(np.int32)
    return row


def make_case(
    *,
    ctx: Sequence[int],
    q_lens: Sequence[int],
    H: int,
    D: int = 512,
    K: int = 512,
    scenario: int = 3,
    cmp_ratio: int = 4,
    win_left: int = 127,
    bs_ori: int = 128,
    bs_cmp: int = 128,
    dtype: str = "bf16",
    seed: int = 0,
    dist: str = "normal",
    spare_blocks: int = 3,
    softmax_scale: Optional[float] = None,
) -> Case:
    """Numpy case. ``dist='normal'`` draws Q/KV/sinks from N(0,1) (the
    BASELINE configs); ``'uniform'`` mirrors the reference tests' ranges
    (Q, raw KV ~ U(-10,10); compressed KV ~ U(-5,10); sinks ~ U(-1,1))."""
    rng = np.random.default_rng(seed)
    B = len(ctx)
    assert len(q_lens) == B
    cu = np.zeros(B + 1, np.int32)
    cu[1:] = np.cumsum(np.asarray(q_lens, np.int64))
    T = int(cu[-1])
    seqused = np.asarray(ctx, np.int32)

    def draw(shape, lo, hi):
        if dist == "normal":
            return rng.standard_normal(shape, dtype=np.float32)
        return rng.uniform(lo, hi, size=shape).astype(np.float32)

    q = _round(draw((T, H, D), -10, 10), dtype)
    ori_bt, n_ori = _paged_table(rng, ctx, bs_ori, spare_blocks)
    ori_kv = _round(draw((n_ori, bs_ori, 1, D), -10, 10), dtype)
    cmp_kv = cmp_bt = idx = None
    if scenario >= 2:
        cmp_lens = [int(c) // cmp_ratio for c in ctx]
        cmp_bt, n_cmp = _paged_table(rng, cmp_lens, bs_cmp, spare_blocks)
        cmp_kv = _round(draw((n_cmp, bs_cmp, 1, D), -5, 10), dtype)
    if scenario == 3:
        idx = np.full((T, 1, K), -1, np.int32)
        for b in range(B):
            aq = int(q_lens[b])
            for s in range(aq):
                s_g = int(ctx[b]) - aq + s
                idx[cu[b] + s, 0] = topk_indices(rng, (s_g + 1) // cmp_ratio, K)
    if dist == "normal":
        sinks = rng.standard_normal(H, dtype=np.float32)
    else:
        sinks = rng.uniform(-1, 1, size=H).astype(np.float32)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    return Case(B=B, H=H, D=D, dtype=dtype, scenario=scenario, K=K if scenario == 3 else 0,
                cmp_ratio=cmp_ratio, win_left=win_left, cu_seqlens_q=cu, seqused_kv=seqused,
                q=q, ori_kv=ori_kv, ori_bt=ori_bt, cmp_kv=cmp_kv, cmp_bt=cmp_bt, idx=idx,
                sinks=sinks, softmax_scale=float(scale))


# ---------------------------------------------------------------------------
# Benchmark-scale generation on the device (torch, seeded).
# ---------------------------------------------------------------------------

def config_contexts(name: str, seed: int = 0) -> dict:
    """Context lengths / shapes of the named BASELINE configurations.

    C1 CPU-golden decode, C2 bf16 decode, C3 MTP decode, C4 prefill,
    C5 request-parallel long-context decode (the full 512-request batch; a
    GPU takes its share of it)."""
    rng = np.random.default_rng(seed)
    if name == "C1":
        return dict(ctx=[1024, 2048, 3000, 4096], q_lens=[1] * 4, H=16, K=256, bs=64)
    if name == "C2":
        return dict(ctx=rng.integers(8192, 65536 + 1, size=64).tolist(), q_lens=[1] * 64, H=64, K=512, bs=128)
    if name == "C3":
        ctx = np.exp(rng.uniform(math.log(128), math.log(131072), size=128)).astype(np.int64)
        ctx = np.maximum(ctx, 2)
        return dict(ctx=ctx.tolist(), q_lens=[2] * 128, H=128, K=512, bs=128)
    if name == "C4":
        return dict(ctx=[8192, 8192], q_lens=[8192, 8192], H=64, K=512, bs=128)
    if name == "C5":
        return dict(ctx=rng.integers(65536, 262144 + 1, size=512).tolist(), q_lens=[1] * 512, H=128, K=1024, bs=128)
    raise ValueError(name)


def balance_requests(ctx: Sequence[int], n_parts: int) -> List[List[int]]:
    """Longest-processing-time assignment of requests to ``n_parts`` GPUs.

    Per-token work is O(window + K), nearly independent of the context, so
    the balance key is the request's query-token count plus its context
    length as a tie-breaker for the paged-cache footprint."""
    order = sorted(range(len(ctx)), key=lambda i: -int(ctx[i]))
    loads = [0] * n_parts
    counts = [0] * n_parts
    parts: List[List[int]] = [[] for _ in range(n_parts)]
    per = math.ceil(len(ctx) / n_parts)
    for i in order:
        cand = [p for p in range(n_parts) if counts[p] < per]
        p = min(cand, key=lambda j: (loads[j], j))
        parts[p].append(i)
        loads[p] += int(ctx[i])
        counts[p] += 1
    return [sorted(p) for p in parts]


def make_case_torch(*, ctx, q_lens, H, K, bs=128, D=512, scenario=3, cmp_ratio=4, win_left=127,
                    dtype="bf16", seed=0, device="cuda"):
    """Device-resident case as a dict of torch tensors (values ~ N(0,1))."""
    import torch

    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    B = len(ctx)
    ctx_t = torch.tensor([int(c) for c in ctx], dtype=torch.int64)
    ql = torch.tensor([int(x) for x in q_lens], dtype=torch.int64)
    cu = torch.zeros(B + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(ql, 0)
    T = int(cu[-1])

    def pool_and_table(lens, bsz):
        nb = [(int(l) + bsz - 1) // bsz for l in lens]
        total = max(sum(nb) + 1, 1)
        perm = torch.randperm(total, generator=g, device=device).to(torch.int32)
        width = max(max(nb) if nb else 0, 1)
        table = torch.full((B, width), -1, dtype=torch.int32, device=device)
        cur = 0
        for b, n in enumerate(nb):
            if n:
                table[b, :n] = perm[cur:cur + n]
            cur += n
        per_block = bsz * D
        if total * per_block <= (1 << 31):
            pool = torch.randn((total, bsz, 1, D), generator=g, device=device, dtype=torch.float32).to(tdt)
        else:
            # large caches (long-context decode): fill in pieces of ~2 GB of fp32
            pool = torch.empty((total, bsz, 1, D), device=device, dtype=tdt)
            step = max(1, (1 << 29) // per_block)
            for b0 in range(0, total, step):
                n = min(step, total - b0)
                pool[b0:b0 + n] = torch.randn((n, bsz, 1, D), generator=g, device=device,
                                              dtype=torch.float32).to(tdt)
        return pool, table

    q = torch.randn((T, H, D), generator=g, device=device, dtype=torch.float32).to(tdt)
    ori_kv, ori_bt = pool_and_table(ctx, bs)
    out = dict(q=q, ori_kv=ori_kv, ori_block_table=ori_bt,
               cu_seqlens_q=cu.to(torch.int32).to(device), seqused_kv=ctx_t.to(torch.int32).to(device),
               sinks=torch.randn(H, generator=g, device=device, dtype=torch.float32),
               softmax_scale=1.0 / math.sqrt(D), cmp_ratio=cmp_ratio, ori_win_left=win_left)
    if scenario >= 2:
        cmp_kv, cmp_bt = pool_and_table([int(c) // cmp_ratio for c in ctx], bs)
        out.update(cmp_kv=cmp_kv, cmp_block_table=cmp_bt)
    if scenario == 3:
        # per token: threshold = (s_g + 1) // ratio; top-K distinct ids of random keys
        s_g = []
        for b in range(B):
            aq = int(ql[b])
            s_g += [int(ctx[b]) - aq + s for s in range(aq)]
        thr = torch.tensor([(x + 1) // cmp_ratio for x in s_g], dtype=torch.int64, device=device)
        idx = torch.full((T, 1, K), -1, dtype=torch.int32, device=device)
        chunk = max(1, (1 << 26) // max(int(thr.max().item()), 1))
        tmax = int(thr.max().item()) if T else 0
        for t0 in range(0, T, chunk):
            t1 = min(T, t0 + chunk)
            th = thr[t0:t1]
            if tmax == 0:
                break
            keys = torch.rand((t1 - t0, tmax), generator=g, device=device)
            ar = torch.arange(tmax, device=device)
            keys = torch.where(ar[None, :] < th[:, None], keys, torch.full_like(keys, -1.0))
            kk = min(K, tmax)
            vals, ids = torch.topk(keys, kk, dim=1)
            ids = torch.where(vals >= 0, ids, torch.full_like(ids, -1)).to(torch.int32)
            idx[t0:t1, 0, :kk] = ids
        out.update(cmp_sparse_indices=idx, topk_cmp=K)
    return out
