"""TEST INFRASTRUCTURE ONLY: CPU restatement of the sparse_attn_sharedkv forward.

This module is the checker the CUDA path is compared against. The product
path (``dsv4_b200``) never imports it; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
do.

It restates ``sparse_attn_sharedkv_tilelang/golden.py`` in numpy:

* ``forward``: ``sparse_attn_sharedkv_golden_bnsd`` (golden.py:69-204) --
  per query token, the causal sliding window ``[max(s_g - win_left, 0), s_g]``
  over the raw cache, then the compressed rows selected by
  ``_gather_cmp_kv_tokens`` (golden.py:28-66: scan the first
  ``min(K, threshold)`` index slots, stop at the first ``-1``, skip slots with
  ``idx >= threshold``), or all ``[0, threshold)`` rows for the dense (CFA)
  scenario; online softmax over tiles of 512 rows (window tiles first), state
  seeded with ``(max, sum) = (sink_h, 1)``; ``P`` rounded to the I/O dtype
  before ``P @ V`` while the running sum uses the unrounded ``P``
  (golden.py:156-200); ``out = acc / sum`` rounded to the dtype and
  ``lse = max + ln(sum)``.
* ``single_shot``: ``sinks_softmax_reference`` (golden.py:207-244).

Differences from golden.py, all outside its defined domain:

* paged caches are read through the block tables directly instead of being
  unpacked to dense BNSD first (same rows);
* a token with ``s_g < 0`` (more query tokens than kv tokens) attends to no
  rows; golden.py slices ``[0:s_g+1]`` there, which Python wraps around;
* index values below ``-1`` are skipped; golden.py would index from the end.

Parity of this restatement with golden.py itself is pinned by
``tests/golden/attn_cases.npz`` (made by ``tests/golden/make_golden.py``,
which runs the reference golden on the same seeded inputs).
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

GOLDEN_S2_TILE = 512


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def round_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "fp16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    if dtype == "fp32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dtype)


def paged_row_ids(table: np.ndarray, b: int, pos: np.ndarray, bs: int) -> np.ndarray:
    """Flat pool row (block * bs + offset) of positions ``pos`` of request ``b``."""
    pos = np.asarray(pos, np.int64)
    return table[b, pos // bs].astype(np.int64) * bs + pos % bs


def _paged_rows(pool: np.ndarray, table: np.ndarray, b: int, pos: np.ndarray) -> np.ndarray:
    """Rows ``pos`` of request ``b`` from a paged pool [nblk, bs, 1, D]."""
    bs = pool.shape[1]
    phys = table[b, pos // bs]
    return pool[phys, pos % bs, 0, :].astype(np.float32)


def token_positions(*, s_g: int, idx_row: Optional[np.ndarray], has_cmp: bool, cmp_ratio: int, win_left: int):
    """(window positions, compressed positions) one query token attends
    (golden.py:28-66 and the window of golden.py:120-150)."""
    win = np.arange(max(s_g - win_left, 0), s_g + 1) if s_g >= 0 else np.zeros(0, np.int64)
    if not has_cmp:
        return win, np.zeros(0, np.int64)
    threshold = (s_g + 1) // cmp_ratio
    if idx_row is not None:
        return win, cmp_selected_positions(idx_row, threshold)
    return win, np.arange(max(threshold, 0))


def token_forward(q_t: np.ndarray, win: np.ndarray, cmp: np.ndarray, sinks: np.ndarray, softmax_scale: float,
                  dtype: str = "bf16", s2_tile: int = GOLDEN_S2_TILE):
    """One query token: ``q_t`` [H, D], attended rows ``win`` / ``cmp`` [n, D]
    (float32 holding dtype values). Returns the dtype-rounded output [H, D]
    and the LSE [H] (golden.py:156-204)."""
    tiles = [win[i:i + s2_tile] for i in range(0, max(win.shape[0], 1), s2_tile)]
    tiles += [cmp[i:i + s2_tile] for i in range(0, cmp.shape[0], s2_tile)]
    o, l = _online_softmax(np.asarray(q_t, np.float32), tiles, np.asarray(sinks, np.float32), softmax_scale, dtype)
    return round_dtype(o, dtype), l


def cmp_selected_positions(idx_row: np.ndarray, threshold: int) -> np.ndarray:
    """Compressed row ids attended by one token (golden.py:28-66, block size 1)."""
    K = idx_row.shape[0]
    valid_count = min(K, threshold)
    sel = []
    for i in range(max(valid_count, 0)):
        v = int(idx_row[i])
        if v == -1:
            break
        if v < 0 or v >= threshold:
            continue
        sel.append(v)
    return np.asarray(sel, dtype=np.int64)


def token_rows(
    *,
    b: int,
    s_g: int,
    ori_kv: np.ndarray,
    ori_bt: np.ndarray,
    cmp_kv: Optional[np.ndarray],
    cmp_bt: Optional[np.ndarray],
    idx_row: Optional[np.ndarray],
    cmp_ratio: int,
    win_left: int,
):
    """(window rows, compressed rows) as float32 arrays for one query token."""
    D = ori_kv.shape[-1]
    lo = max(s_g - win_left, 0)
    if s_g >= 0:
        win = _paged_rows(ori_kv, ori_bt, b, np.arange(lo, s_g + 1))
    else:
        win = np.zeros((0, D), np.float32)
    if cmp_kv is None:
        cmp = np.zeros((0, D), np.float32)
    else:
        threshold = (s_g + 1) // cmp_ratio
        if idx_row is not None:
            sel = cmp_selected_positions(idx_row, threshold)
        else:
            sel = np.arange(max(threshold, 0))
        cmp = _paged_rows(cmp_kv, cmp_bt, b, sel) if sel.size else np.zeros((0, D), np.float32)
    return win, cmp


def _online_softmax(q, tiles, sinks, scale, dtype):
    G = q.shape[0]
    row_max = sinks.astype(np.float32).copy()
    row_sum = np.ones(G, np.float32)
    acc = np.zeros((G, q.shape[1]), np.float32)
    for k in tiles:
        if k.shape[0] == 0:
            continue
        score = (q @ k.T) * np.float32(scale)
        old = row_max
        row_max = np.maximum(row_max, score.max(axis=1))
        alpha = np.exp(old - row_max)
        p = np.exp(score - row_max[:, None])
        row_sum = alpha * row_sum + p.sum(axis=1)
        pv = round_dtype(p, dtype) @ k
        acc = acc * alpha[:, None] + pv
    out = acc / row_sum[:, None]
    lse = row_max + np.log(row_sum)
    return out, lse


def forward(
    q: np.ndarray,  # [T, H, D] float32 holding dtype values
    *,
    ori_kv: np.ndarray,  # [nblk, bs, 1, D]
    ori_bt: np.ndarray,  # [B, L]
    cmp_kv: Optional[np.ndarray],
    cmp_bt: Optional[np.ndarray],
    idx: Optional[np.ndarray],  # [T, 1, K] (SCFA) or None (CFA / SWA)
    cu_seqlens_q: Sequence[int],
    seqused_kv: Sequence[int],
    sinks: np.ndarray,  # [H]
    softmax_scale: float,
    cmp_ratio: int = 4,
    win_left: int = 127,
    dtype: str = "bf16",
    tokens: Optional[Sequence[int]] = None,
    s2_tile: int = GOLDEN_S2_TILE,
):
    """Reference output ``[T, H, D]`` (dtype-rounded float32) and LSE ``[T, H]``.

    ``tokens`` restricts the work to a subset of flat token ids (other rows
    stay zero), which is how large configurations are checked on a sample.
    """
    T, H, D = q.shape
    out = np.zeros((T, H, D), np.float32)
    lse = np.zeros((T, H), np.float32)
    cu = [int(x) for x in cu_seqlens_q]
    B = len(cu) - 1
    want = None if tokens is None else set(int(t) for t in tokens)
    for b in range(B):
        act_q = cu[b + 1] - cu[b]
        act_kv = int(seqused_kv[b])
        for s in range(act_q):
            t = cu[b] + s
            if want is not None and t not in want:
                continue
            s_g = act_kv - act_q + s
            win, cmp = token_rows(
                b=b, s_g=s_g, ori_kv=ori_kv, ori_bt=ori_bt, cmp_kv=cmp_kv, cmp_bt=cmp_bt,
                idx_row=None if idx is None else idx[t, 0], cmp_ratio=cmp_ratio, win_left=win_left,
            )
            out[t], lse[t] = token_forward(q[t], win, cmp, sinks, softmax_scale, dtype, s2_tile)
    return out, lse


def single_shot(q: np.ndarray, k: np.ndarray, sinks: np.ndarray, softmax_scale: float, dtype: str = "fp32"):
    """One-shot ``softmax([q k^T * scale, sink]) @ [k; 0]`` (golden.py:207-244)."""
    q = q.astype(np.float32)
    k = k.astype(np.float32)
    score = (q @ k.T) * np.float32(softmax_scale)
    s = sinks.astype(np.float32)[:, None]
    x_max = np.maximum(score.max(axis=1, keepdims=True) if score.shape[1] else s, s)
    y = np.exp(score - x_max)
    denom = y.sum(axis=1, keepdims=True) + np.exp(s - x_max)
    p = y / denom
    out = round_dtype(round_dtype(p, dtype) @ k, dtype)
    lse = (x_max + np.log(denom))[:, 0]
    return out, lse


def token_work(cu_seqlens_q, seqused_kv, idx, *, cmp_ratio=4, win_left=127, scenario=3):
    """Per-token (n_window_rows, n_cmp_rows) actually attended (for FLOP/byte accounting)."""
    cu = [int(x) for x in cu_seqlens_q]
    res = []
    for b in range(len(cu) - 1):
        act_q = cu[b + 1] - cu[b]
        act_kv = int(seqused_kv[b])
        for s in range(act_q):
            s_g = act_kv - act_q + s
            n_win = 0 if s_g < 0 else s_g - max(s_g - win_left, 0) + 1
            thr = (s_g + 1) // cmp_ratio
            if scenario == 1:
                n_cmp = 0
            elif scenario == 2:
                n_cmp = max(thr, 0)
            else:
                n_cmp = int(cmp_selected_positions(idx[cu[b] + s, 0], thr).size)
            res.append((n_win, n_cmp))
    return res


__all__ = [
    "forward", "single_shot", "round_bf16", "round_dtype", "cmp_selected_positions", "paged_row_ids",
    "token_positions", "token_forward",
    "token_rows", "token_work", "GOLDEN_S2_TILE",
]
