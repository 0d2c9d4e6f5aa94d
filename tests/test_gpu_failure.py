"""Failure paths on the GPU, exercised without faulting it.

* A bounded wait that runs out: the wait limit is lowered to 1 us for one
  normal call, so real waits of the attention kernel give up. The call must
  return, the status word must read SAS_ERR_TIMEOUT_BASE + the wait's id, and
  the next call with the default limit must be correct (the aborted CTAs
  drained their copies and MMAs and freed their TMEM).
* The scheduler's row-scan cap: lowered so that a prefill schedule hits it,
  which records SAS_ERR_SCHED_OVERRUN; with the default cap the schedule is
  bit-exact again.
* Block-table entries outside the table or the pool (the reference's kernel
  clamps -1 entries, kernel.py:735-742, and reads up to act_kv,
  kernel.py:285-300): such rows are dropped exactly like -1 entries and the
  non-fatal status SAS_ERR_BAD_BLOCK_ENTRY is set. The pool is declared
  smaller than its allocation, so even a kernel without the check would only
  read allocated memory.
"""

import numpy as np
import pytest

import sas_testutil as U

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True)
def _gpu(sas_lib):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dsv4_b200 import reset_device_status

    reset_device_status()
    yield
    reset_device_status()


def _status():
    from dsv4_b200 import device_status

    torch.cuda.synchronize()
    return device_status()


def _set(opt, value):
    from dsv4_b200 import _lib as L

    L.check(L.lib().sas_fwd_set_option(opt, float(value), None), "sas_fwd_set_option")


def _run(d, **over):
    from dsv4_b200 import sparse_attn_sharedkv

    kw = dict(d)
    kw.update(over)
    q = kw.pop("q")
    o, l = sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
    return o.float().cpu().numpy(), l.cpu().numpy()


CASES = [
    dict(ctx=[9000, 20000, 130, 40000] * 4, q_lens=[1] * 16, H=64, K=512, seed=51),  # fused plan
    dict(ctx=[3000, 900], q_lens=[400, 300], H=64, K=256, seed=52),                  # plan kernel
]


@pytest.mark.parametrize("cfg", CASES, ids=["decode", "prefill"])
def test_wait_timeout_returns_status_and_recovers(cfg):
    from dsv4_b200 import _lib as L, reset_device_status

    case = U.build_case(cfg)
    d = U.to_device(case)
    try:
        _set(L.OPT_WAIT_LIMIT_NS, 1000)
        _run(d)
        st = _status()
    finally:
        _set(L.OPT_WAIT_LIMIT_NS, 0)
    assert st >= L.STATUS_TIMEOUT_BASE, f"no wait ran out (status {st})"
    reset_device_status()
    out, lse = _run(d)
    assert _status() == 0
    ro, rl = U.oracle_forward(case)
    U.check_close(out, ro, lse, rl, what="after a timed-out launch")
    U.check_result_ref(out, ro, case.dtype)


def test_scheduler_scan_cap_reports_overrun():
    from dsv4_b200 import _lib as L, reset_device_status
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata
    from oracle import meta_oracle as M

    # 4 x 8192 prefill rows do not fit the scheduler's shared-memory row
    # cache, so the greedy walk scans rows 32 at a time and a core takes
    # ~1400 of them: far past a cap of 64
    cfg = dict(num_heads_q=64, num_heads_kv=1, head_dim=512, cu_seqlens_q=[0, 8192, 16384, 24576, 32768],
               seqused_kv=[8192] * 4, batch_size=4, max_seqlen_q=8192, max_seqlen_kv=8192, layout_q="TND",
               has_cmp_kv=True, cmp_ratio=4, cmp_topk=512, aic_core_num=24)
    kw = {k: (torch.tensor(v, dtype=torch.int32) if isinstance(v, list) else v) for k, v in cfg.items()}
    try:
        _set(L.OPT_SCHED_SCAN_CAP, 64)
        sparse_attn_sharedkv_metadata(device="cuda", **kw)
        st = _status()
    finally:
        _set(L.OPT_SCHED_SCAN_CAP, 0)
    assert st == 5, f"status {st}"
    reset_device_status()
    md = sparse_attn_sharedkv_metadata(device="cuda", **kw).cpu().numpy()
    assert _status() == 0
    assert np.array_equal(md, M.metadata(**cfg))


def _bad_entry_case(seed):
    case = U.build_case(dict(ctx=[5000, 12000, 700, 30000], q_lens=[1, 2, 1, 1], H=64, K=512, seed=seed,
                             spare_blocks=0))
    return case, U.to_device(case)


def test_block_entries_past_the_pool_are_dropped():
    case, d = _bad_entry_case(61)
    for pool, table in (("ori_kv", "ori_block_table"), ("cmp_kv", "cmp_block_table")):
        n = d[pool].shape[0]
        decl = n - max(2, n // 8)  # declared pool size; the last blocks stay allocated
        bt = d[table]
        masked = torch.where(bt >= decl, torch.full_like(bt, -1), bt)
        assert int((bt >= decl).sum()) > 0
        out_a, lse_a = _run(d, **{pool: d[pool][:decl]})
        st_a = _status()
        from dsv4_b200 import reset_device_status

        reset_device_status()
        out_b, lse_b = _run(d, **{pool: d[pool][:decl], table: masked})
        st_b = _status()
        assert st_a == 7, f"{pool}: status {st_a}"
        assert st_b == 0, f"{pool}: status {st_b} with -1 entries"
        assert np.array_equal(out_a, out_b) and np.array_equal(lse_a, lse_b), pool
        reset_device_status()


def test_seqused_kv_longer_than_table_is_dropped():
    from dsv4_b200 import reset_device_status

    case, d = _bad_entry_case(62)
    bt = d["ori_block_table"]
    short = bt[:, :-1].contiguous()   # the last column is missing
    masked = bt.clone()
    masked[:, -1] = -1                # the same table with that column unused
    out_a, lse_a = _run(d, ori_block_table=short)
    st_a = _status()
    reset_device_status()
    out_b, lse_b = _run(d, ori_block_table=masked)
    assert st_a == 7 and _status() == 0
    assert np.array_equal(out_a, out_b) and np.array_equal(lse_a, lse_b)
