"""Head-sharded forward on 2 GPUs (skipped with fewer): the attention kernel
of each rank stores its heads into both ranks' symmetric output buffers
(sas_sparse_attn_sharedkv_fwd_gather), and every rank must end with exactly
the single-GPU result for all heads, bit for bit (heads are independent and
every token stays on one CTA, so the split does not change any rounding).
The NCCL all-gather form is checked the same way."""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CFG = dict(ctx=[5000, 129, 9000, 20000], q_lens=[1, 2, 1, 1], H=128, K=512, seed=91)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q_out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import sas_testutil as U
        from dsv4_b200 import sharding, sparse_attn_sharedkv

        case = U.build_case(CFG)
        d = U.to_device(case, device=f"cuda:{rank}")
        q = d.pop("q")
        ref_o, ref_l = sparse_attn_sharedkv(q, return_softmax_lse=True, **d)
        res = {}
        for name, fn in (("p2p", sharding.head_sharded_forward_p2p), ("nccl", sharding.head_sharded_forward)):
            for _ in range(2):  # the second call reuses the symmetric buffers
                o, l = fn(q, **dict(d))
            torch.cuda.synchronize()
            res[name] = (bool(torch.equal(o, ref_o)), bool(torch.equal(l, ref_l)))
        q_out.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_head_sharded_two_gpus_match_single_gpu(sas_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    here = os.path.dirname(os.path.abspath(__file__))
    os.environ["PYTHONPATH"] = os.pathsep.join([os.path.dirname(here), here, os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    codes = [p.exitcode for p in procs]
    assert codes == [0, 0], codes
    res = dict(q_out.get(timeout=10) for _ in range(2))
    for rank in (0, 1):
        assert res[rank]["p2p"] == (True, True), res
        assert res[rank]["nccl"] == (True, True), res
