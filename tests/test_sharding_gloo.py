"""CPU: multi-GPU host logic on gloo ranks (world size 2).

The CUDA op is replaced by the CPU oracle inside each rank, so these tests
check the sharding itself: request partitioning and per-rank sub-batches
(request-parallel), head slicing and the all-gather layout (head-sharded),
and that a rank failing before a collective surfaces as an error on the
other rank instead of a hang (failure detection made on the host)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv4_b200 import sharding, synth
from oracle import golden_oracle as O

CASE = dict(ctx=[900, 1300, 200, 2500, 640], q_lens=[1, 2, 1, 3, 1], H=16, K=128, seed=5)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_tensors(case, heads=None, sinks=None, tokens=None):
    q = case.q if heads is None else case.q[:, heads[0]:heads[1]]
    sk = case.sinks if sinks is None else sinks
    o, l = O.forward(np.ascontiguousarray(q), ori_kv=case.ori_kv, ori_bt=case.ori_bt, cmp_kv=case.cmp_kv,
                     cmp_bt=case.cmp_bt, idx=case.idx, cu_seqlens_q=case.cu_seqlens_q, seqused_kv=case.seqused_kv,
                     sinks=sk, softmax_scale=case.softmax_scale, cmp_ratio=case.cmp_ratio, win_left=case.win_left,
                     dtype=case.dtype, tokens=tokens)
    return torch.from_numpy(o), torch.from_numpy(l)


def test_partition_requests_covers_each_request_once():
    rng = np.random.default_rng(0)
    for world in (1, 2, 4, 8):
        ctx = rng.integers(64 * 1024, 256 * 1024, size=512).tolist()
        parts = sharding.partition_requests(ctx, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(512))
        assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 1
        loads = [sum(ctx[i] for i in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.02


def test_select_requests_cuts_consistent_sub_batch():
    case = synth.make_case(**CASE)
    full = dict(q=torch.from_numpy(case.q), cu_seqlens_q=torch.from_numpy(case.cu_seqlens_q),
                seqused_kv=torch.from_numpy(case.seqused_kv), ori_block_table=torch.from_numpy(case.ori_bt),
                cmp_block_table=torch.from_numpy(case.cmp_bt), cmp_sparse_indices=torch.from_numpy(case.idx))
    sub = sharding.select_requests(full, [1, 3])
    assert sub["cu_seqlens_q"].tolist() == [0, 2, 5]
    assert sub["seqused_kv"].tolist() == [1300, 2500]
    assert torch.equal(sub["q"][:2], full["q"][1:3]) and torch.equal(sub["q"][2:], full["q"][4:7])
    assert torch.equal(sub["cmp_sparse_indices"][2:], full["cmp_sparse_indices"][4:7])


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        case = synth.make_case(**CASE)
        if mode == "heads":
            def local_fn(ql, sinks, **kw):
                h0, h1 = sharding.head_range(case.H, world, rank)
                return _oracle_tensors(case, heads=(h0, h1), sinks=sinks.numpy())
            out, lse = sharding.head_sharded_forward(torch.from_numpy(case.q), sinks=torch.from_numpy(case.sinks),
                                                     local_fn=local_fn)
            ref_o, ref_l = _oracle_tensors(case)
            # per-head math is independent; BLAS blocking may move the last fp32 bit
            ok = (torch.allclose(out, ref_o, rtol=2 ** -7, atol=1e-4) and torch.allclose(lse, ref_l, atol=1e-5)
                  and out.shape == ref_o.shape)
            q.put((rank, bool(ok)))
        elif mode == "requests":
            parts = sharding.partition_requests(case.seqused_kv.tolist(), world)
            cu = case.cu_seqlens_q
            toks = [t for b in parts[rank] for t in range(cu[b], cu[b + 1])]
            o, l = _oracle_tensors(case, tokens=toks)
            mine = torch.zeros(case.T, dtype=torch.bool)
            mine[toks] = True
            o = o * mine[:, None, None]
            dist.all_reduce(o)  # assemble on every rank: ranks own disjoint tokens
            ref_o, _ = _oracle_tensors(case)
            q.put((rank, bool(torch.equal(o, ref_o))))
        elif mode == "fail":
            if rank == 1:
                raise SystemExit(3)  # leaves between steps, before the collective
            try:
                dist.all_reduce(torch.ones(4))
                q.put((rank, False))
            except Exception:
                q.put((rank, True))
    finally:
        if mode != "fail":
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "requests"])
def test_two_rank_sharding_matches_single_rank(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, "fail", q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    assert q.get(timeout=5) == (0, True)
