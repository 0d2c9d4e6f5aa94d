"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

This script is the only place that executes the reference implementation
(``sparse_attn_sharedkv_tilelang/golden.py`` and ``metadata.py``, both plain
CPU PyTorch). It needs the reference checkout, so it runs in the development
container only; the fixtures it writes are committed and travel with the
repository. Inputs are regenerated from seeds by ``dsv4_b200.synth``, so a
fixture stores only the case parameters and the reference outputs.

Usage::

    python tests/golden/make_golden.py --ref <path to sparse_attn_sharedkv_tilelang>

Writes:

* ``metadata_cases.npz`` -- ``configs`` (JSON list of keyword sets) and
  ``outputs`` (``int32[N, 1024]``) from ``metadata.sparse_attn_sharedkv_metadata``.
* ``metadata_fd_cases.npz`` -- the same for the flash-decode schedule: the
  reference scheduler class (``metadata._MetadataScheduler``) with its
  ``supportFd`` attribute set to True before ``run()``; the configs add
  ``aiv_core_num``. Configurations on which the reference's row walk does not
  end within a time limit (its inner loop has no bound) are left out.
* ``attn_cases.npz`` -- ``configs`` (JSON list of ``synth.make_case`` keyword
  sets plus index edits) and, per case ``i``, ``out_i`` (raw 16-bit pattern of
  the bf16/fp16 output, ``[T, H, D]``) and ``lse_i`` (``float32[T, H]``) from
  ``golden.sparse_attn_sharedkv_golden_bnsd``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from dsv4_b200 import synth  # noqa: E402


def metadata_configs(rng: np.random.Generator, n_random: int):
    cfgs = []
    # the reference test scenarios (test_sparse_attn_sharedkv.py:81-220)
    for sc, S1, ratio in [(3, 1, 4), (3, 8192, 4), (1, 1, 4), (1, 8192, 4), (2, 1, 128), (2, 8192, 128)]:
        kv = 8193 if S1 == 1 else 8192
        cfgs.append(dict(num_heads_q=64, num_heads_kv=1, head_dim=512, cu_seqlens_q=[0, S1], seqused_kv=[kv],
                         batch_size=1, max_seqlen_q=S1, max_seqlen_kv=kv, layout_q="TND",
                         has_cmp_kv=sc >= 2, cmp_ratio=ratio if sc >= 2 else -1, cmp_topk=512 if sc == 3 else 0))
    # BASELINE-shaped configurations
    for name in ["C1", "C2", "C3", "C4", "C5"]:
        c = synth.config_contexts(name)
        ql = c["q_lens"]
        cu = [0] + list(np.cumsum(ql).astype(int))
        cfgs.append(dict(num_heads_q=c["H"], num_heads_kv=1, head_dim=512, cu_seqlens_q=[int(x) for x in cu],
                         seqused_kv=[int(x) for x in c["ctx"]], batch_size=len(ql), max_seqlen_q=max(ql),
                         max_seqlen_kv=int(max(c["ctx"])), layout_q="TND", has_cmp_kv=True, cmp_ratio=4,
                         cmp_topk=c["K"]))
    for i in range(n_random):
        kind = rng.integers(0, 4)
        B = int(rng.integers(1, [8, 64, 300, 4][kind] + 1))
        if kind == 3:
            ql = rng.integers(0, 3000, size=B)
        elif kind == 2:
            ql = rng.integers(0, 3, size=B)
        else:
            ql = rng.integers(0, 40, size=B)
        if rng.random() < 0.7:
            ql = np.maximum(ql, 1)
        kv = rng.integers(0, [5000, 70000, 300000, 9000][kind], size=B)
        if rng.random() < 0.5:
            kv = np.maximum(kv, ql)  # the usual case: at least as many kv as q tokens
        nkv = int(rng.choice([1, 1, 1, 2, 4]))
        nq = nkv * int(rng.choice([1, 8, 16, 64, 128]))
        layout = str(rng.choice(["TND", "BSND"]))
        sc = int(rng.choice([1, 2, 3, 3]))
        mask = int(rng.choice([4, 4, 4, 3, 0, 1]))
        win = int(rng.choice([127, 127, 0, 63, 300, -1]))
        aic = int(rng.choice([24, 24, 1, 8, 36, 48]))
        cu = [0] + list(np.cumsum(ql).astype(int))
        cfg = dict(num_heads_q=nq, num_heads_kv=nkv, head_dim=512, seqused_kv=[int(x) for x in kv],
                   batch_size=B, max_seqlen_q=int(max(ql)) if B else 0, max_seqlen_kv=int(max(kv)) if B else 0,
                   layout_q=layout, has_cmp_kv=sc >= 2, ori_mask_mode=mask, ori_win_left=win, aic_core_num=aic)
        if layout == "TND":
            cfg["cu_seqlens_q"] = [int(x) for x in cu]
        if sc >= 2:
            cfg["cmp_ratio"] = int(rng.choice([4, 128]))
        if sc == 3:
            cfg["cmp_topk"] = int(rng.choice([64, 256, 512, 1024]))
        cfgs.append(cfg)
    return cfgs


def _to_torch_kwargs(cfg):
    kw = dict(cfg)
    for k in ("cu_seqlens_q", "seqused_kv"):
        if k in kw:
            kw[k] = torch.tensor(kw[k], dtype=torch.int32)
    return kw


ATTN_CASES = [
    # BASELINE config 1 exactly (CPU golden decode)
    dict(name="c1_decode", ctx=[1024, 2048, 3000, 4096], q_lens=[1, 1, 1, 1], H=16, K=256, bs_ori=64, bs_cmp=64,
         scenario=3, seed=0),
    # MTP: 2 tokens, a request shorter than the window, fewer than K valid
    dict(name="mtp_short", ctx=[100, 1500, 5000], q_lens=[2, 2, 2], H=128, K=512, scenario=3, seed=1),
    # small prefill from position 0, ragged requests
    dict(name="prefill_small", ctx=[300, 9], q_lens=[12, 9], H=64, K=64, scenario=3, seed=2),
    # sliding window only
    dict(name="swa", ctx=[50, 700], q_lens=[1, 5], H=64, K=0, scenario=1, seed=3),
    # dense compressed, ratio 128
    dict(name="cfa", ctx=[8193, 3000], q_lens=[1, 3], H=64, K=0, scenario=2, cmp_ratio=128, seed=4),
    # fp16 I/O
    dict(name="fp16", ctx=[2000, 777], q_lens=[1, 2], H=64, K=256, scenario=3, dtype="fp16", seed=5),
    # the reference test's distribution and decode case (scfa_decode)
    dict(name="uniform_decode", ctx=[8193], q_lens=[1], H=64, K=512, scenario=3, dist="uniform", seed=6,
         softmax_scale=0.04419417),
    # index edits: a -1 in the middle (golden stops there) and out-of-range ids (skipped)
    dict(name="idx_edits", ctx=[3000, 4000], q_lens=[1, 2], H=64, K=512, scenario=3, seed=7,
         edits=[[0, 100, -1], [1, 5, 999999], [1, 6, 750], [2, 0, -1]]),
    # narrower window
    dict(name="win63", ctx=[1000, 90], q_lens=[3, 2], H=64, K=256, scenario=3, win_left=63, seed=8),
]


def build_attn_case(cfg):
    kw = {k: v for k, v in cfg.items() if k not in ("name", "edits")}
    case = synth.make_case(**kw)
    for t, pos, val in cfg.get("edits", []):
        case.idx[t, 0, pos] = val
    return case


def run_reference_golden(G, case):
    tdt = torch.bfloat16 if case.dtype == "bf16" else torch.float16
    cu = torch.tensor(case.cu_seqlens_q, dtype=torch.int32)
    q = torch.from_numpy(case.q).to(tdt)
    q_bnsd = G.tnd_to_bnsd_q(q, cu)
    S1 = q_bnsd.shape[2]
    ori = torch.from_numpy(case.ori_kv).to(tdt)
    ori_bnsd = G.unpack_paged_kv(ori, torch.from_numpy(case.ori_bt), int(case.seqused_kv.max()))
    kw = {}
    if case.scenario >= 2:
        max_cmp = max(int(c) // case.cmp_ratio for c in case.seqused_kv)
        cmp = torch.from_numpy(case.cmp_kv).to(tdt)
        kw["cmp_k_bnsd"] = G.unpack_paged_kv(cmp, torch.from_numpy(case.cmp_bt), max(max_cmp, 1))
        kw["cmp_ratio"] = case.cmp_ratio
    if case.scenario == 3:
        idx = torch.full((case.B, S1, 1, case.K), -1, dtype=torch.int32)
        for b in range(case.B):
            s0, s1 = int(case.cu_seqlens_q[b]), int(case.cu_seqlens_q[b + 1])
            idx[b, : s1 - s0] = torch.from_numpy(case.idx[s0:s1])
        kw["cmp_sparse_indices"] = idx
    act_q = [int(case.cu_seqlens_q[b + 1] - case.cu_seqlens_q[b]) for b in range(case.B)]
    out, lse = G.sparse_attn_sharedkv_golden_bnsd(
        q_bnsd, ori_bnsd, torch.from_numpy(case.sinks), act_q_lens=act_q, act_kv_lens=case.seqused_kv.tolist(),
        softmax_scale=case.softmax_scale, ori_win_left=case.win_left, return_lse=True, **kw)
    out_t = G.bnsd_to_tnd_out(out, cu)
    lse_t = G.bnsd_to_tnd_lse(lse, cu)
    return out_t.view(torch.int16).numpy().view(np.uint16), lse_t.numpy().astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of sparse_attn_sharedkv_tilelang")
    ap.add_argument("--n-random", type=int, default=1500)
    ap.add_argument("--only", choices=["meta", "fd", "attn", "all"], default="all")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import golden as G  # reference
    import metadata as M  # reference

    if args.only in ("meta", "all"):
        rng = np.random.default_rng(20261201)
        cfgs = metadata_configs(rng, args.n_random)
        outs = np.zeros((len(cfgs), 1024), np.int32)
        for i, cfg in enumerate(cfgs):
            outs[i] = M.sparse_attn_sharedkv_metadata(**_to_torch_kwargs(cfg)).numpy()
        np.savez_compressed(os.path.join(HERE, "metadata_cases.npz"), configs=np.array(json.dumps(cfgs)),
                            outputs=outs)
        print(f"metadata: {len(cfgs)} cases")

    if args.only in ("fd", "all"):
        import signal

        rng = np.random.default_rng(20261202)
        cand = metadata_configs(rng, 700)
        for i, cfg in enumerate(cand):
            cfg["aiv_core_num"] = int(rng.choice([48, 48, 72, 8, 1, 0]))
        # decode-shaped batches with few cores, where rows are cut between cores
        for B, kv, aic in [(1, 70000, 24), (2, 200000, 24), (4, 9000, 24), (3, 130000, 36), (1, 8193, 8)]:
            cand.append(dict(num_heads_q=64, num_heads_kv=1, head_dim=512, cu_seqlens_q=list(range(B + 1)),
                             seqused_kv=[kv + 977 * j for j in range(B)], batch_size=B, max_seqlen_q=1,
                             max_seqlen_kv=kv + 977 * B, layout_q="TND", has_cmp_kv=True, cmp_ratio=4,
                             cmp_topk=1024, aic_core_num=aic, aiv_core_num=48))

        def on_alarm(*_):
            raise TimeoutError

        signal.signal(signal.SIGALRM, on_alarm)
        keep, outs = [], []
        for cfg in cand:
            kw = _to_torch_kwargs(cfg)
            sched = M._MetadataScheduler(**kw)
            sched.supportFd = True
            signal.alarm(5)
            try:
                o = sched.run().numpy()
            except (TimeoutError, IndexError):
                continue
            finally:
                signal.alarm(0)
            keep.append(cfg)
            outs.append(o)
        np.savez_compressed(os.path.join(HERE, "metadata_fd_cases.npz"), configs=np.array(json.dumps(keep)),
                            outputs=np.stack(outs).astype(np.int32))
        n_fd = int(sum((o[36 * 8:36 * 8 + 72 * 8].reshape(72, 8)[:, 0] != 0).any() for o in outs))
        print(f"metadata fd: {len(keep)} of {len(cand)} cases ({n_fd} with flash-decode rows)")

    if args.only in ("attn", "all"):
        arrays = {}
        for i, cfg in enumerate(ATTN_CASES):
            case = build_attn_case(cfg)
            o, l = run_reference_golden(G, case)
            arrays[f"out_{i}"] = o
            arrays[f"lse_{i}"] = l
            print(f"attn case {cfg['name']}: T={case.T} H={case.H}")
        np.savez_compressed(os.path.join(HERE, "attn_cases.npz"), configs=np.array(json.dumps(ATTN_CASES)), **arrays)


if __name__ == "__main__":
    main()
