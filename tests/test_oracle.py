"""CPU: pin the oracle (the parity checker) against the reference's outputs.

* The C scheduler restatement must reproduce every fixture produced by the
  reference metadata.py (tests/golden/metadata_cases.npz) bit for bit.
* The numpy golden restatement must reproduce the reference golden.py
  outputs (tests/golden/attn_cases.npz) to within fp32 summation-order noise.
* The reference's own CPU tests are restated here against the oracle:
  test_golden_math_matches_single_shot_softmax (test_sparse_attn_sharedkv.py:930-1002)
  and the metadata invariants (:721-924).
"""

import math

import numpy as np
import pytest

from oracle import golden_oracle as O
from oracle import meta_oracle as M
import sas_testutil as U


def test_metadata_oracle_matches_reference_fixtures():
    cfgs, outs = U.load_meta_fixtures()
    assert len(cfgs) > 1000
    bad = [i for i, c in enumerate(cfgs) if not np.array_equal(M.metadata(**c), outs[i])]
    assert not bad, f"{len(bad)} mismatching cases, first {bad[:5]}"


@pytest.mark.parametrize("i", range(9))
def test_golden_oracle_matches_reference_fixtures(i):
    fx = U.load_attn_fixtures()
    cfg, ref_out, ref_lse = fx[i]
    case = U.build_case(cfg)
    out, lse = U.oracle_forward(case)
    # identical inputs and math; only fp32 summation order differs
    d = np.abs(out - ref_out)
    # one output ulp, plus a small absolute floor for near-zero outputs where
    # the weighted sum cancels and summation order moves the last bits
    ulp = np.maximum(np.abs(ref_out), np.abs(out)) * (2.0 ** -7 if case.dtype == "bf16" else 2.0 ** -10)
    assert (d <= ulp + 1e-4).all(), cfg["name"]
    assert d.mean() < 1e-6, cfg["name"]
    assert (out == ref_out).mean() > 0.99, cfg["name"]
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=2e-6)


def test_golden_math_matches_single_shot_softmax():
    rng = np.random.default_rng(0)
    S1, N1, D, ratio, K = 4, 64, 512, 4, 8
    kv_len = 128
    scale = 1.0 / math.sqrt(D)
    q = rng.uniform(-1, 1, (S1, N1, D)).astype(np.float32)
    ori = rng.uniform(-1, 1, (kv_len, D)).astype(np.float32)
    cmpk = rng.uniform(-1, 1, (kv_len // ratio, D)).astype(np.float32)
    sinks = (rng.random(N1) * 0.1).astype(np.float32)
    idx = np.full((S1, 1, K), -1, np.int32)
    for s in range(S1):
        thr = (kv_len - S1 + s + 1) // ratio
        take = min(K, max(thr, 0))
        idx[s, 0, :take] = np.arange(take)
    # paged with one block per cache, identity table
    out, lse = O.forward(q, ori_kv=ori[None, :, None, :], ori_bt=np.zeros((1, 1), np.int32),
                         cmp_kv=cmpk[None, :, None, :], cmp_bt=np.zeros((1, 1), np.int32), idx=idx,
                         cu_seqlens_q=[0, S1], seqused_kv=[kv_len], sinks=sinks, softmax_scale=scale,
                         cmp_ratio=ratio, dtype="fp32")
    for s in range(S1):
        s_g = kv_len - S1 + s
        k = np.concatenate([ori[max(s_g - 127, 0): s_g + 1],
                            cmpk[idx[s, 0][(idx[s, 0] >= 0) & (idx[s, 0] < (s_g + 1) // ratio)]]])
        ro, rl = O.single_shot(q[s], k, sinks, scale, dtype="fp32")
        np.testing.assert_allclose(out[s], ro, rtol=2e-4, atol=2e-4)
        np.testing.assert_allclose(lse[s], rl, rtol=1e-4, atol=1e-4)


SCENARIOS = {
    "scfa_decode": dict(S1=1, kv=8193, sc=3, ratio=4),
    "scfa_prefill": dict(S1=8192, kv=8192, sc=3, ratio=4),
    "swa_decode": dict(S1=1, kv=8193, sc=1, ratio=4),
    "swa_prefill": dict(S1=8192, kv=8192, sc=1, ratio=4),
    "cfa_decode": dict(S1=1, kv=8193, sc=2, ratio=128),
    "cfa_prefill": dict(S1=8192, kv=8192, sc=2, ratio=128),
}


def _meta_kwargs(c, aic=24):
    kw = dict(num_heads_q=64, num_heads_kv=1, head_dim=512, cu_seqlens_q=[0, c["S1"]], seqused_kv=[c["kv"]],
              batch_size=1, max_seqlen_q=c["S1"], max_seqlen_kv=c["kv"], layout_q="TND",
              has_cmp_kv=c["sc"] >= 2, aic_core_num=aic)
    if c["sc"] >= 2:
        kw["cmp_ratio"] = c["ratio"]
    if c["sc"] == 3:
        kw["cmp_topk"] = 512
    return kw


@pytest.mark.parametrize("name", list(SCENARIOS))
def test_metadata_shape_and_continuity(name):
    md = M.metadata(**_meta_kwargs(SCENARIOS[name]))
    assert md.dtype == np.int32 and md.shape == (1024,)
    fa = md[:288].reshape(36, 8)
    used = fa[fa[:, 0] == 1]
    assert len(used) >= 1
    prev = (0, 0, 0)
    for row in used.tolist():
        assert tuple(row[1:4]) == prev
        prev = tuple(row[4:7])
    assert prev[0] in (1, 0)


@pytest.mark.parametrize("name", list(SCENARIOS))
def test_metadata_drives_complete_coverage(name):
    c = SCENARIOS[name]
    md = M.metadata(**_meta_kwargs(c))
    fa = md[:288].reshape(36, 8)
    seen = []
    for cid in range(24):
        en, bs, ms, _, be, me, _, _ = fa[cid].tolist()
        if en:
            seen += [p for p in range(bs * c["S1"] + ms, be * c["S1"] + me) if p // c["S1"] < 1]
    assert sorted(seen) == list(range(c["S1"]))


def test_metadata_prefill_uses_many_cores():
    md = M.metadata(**_meta_kwargs(SCENARIOS["scfa_prefill"]))
    assert md[:288].reshape(36, 8)[:, 0].sum() == 24


def test_sampled_oracle_matches_full_oracle():
    """The sampled oracle used at full config shapes (rows gathered from
    torch tensors) gives exactly what the full oracle gives on the same data."""
    import torch
    import sas_testutil as U
    from dsv4_b200 import synth
    from oracle import golden_oracle as O

    d = synth.make_case_torch(ctx=[300, 2000, 130], q_lens=[2, 1, 3], H=16, K=256, bs=64, seed=5, device="cpu")
    toks = [0, 1, 2, 4, 5]
    so, sl = U.oracle_sampled(d, toks)
    f32 = lambda t: t.float().numpy()
    fo, fl = O.forward(f32(d["q"]), ori_kv=f32(d["ori_kv"]), ori_bt=d["ori_block_table"].numpy(),
                       cmp_kv=f32(d["cmp_kv"]), cmp_bt=d["cmp_block_table"].numpy(),
                       idx=d["cmp_sparse_indices"].numpy(), cu_seqlens_q=d["cu_seqlens_q"].numpy(),
                       seqused_kv=d["seqused_kv"].numpy(), sinks=d["sinks"].numpy(),
                       softmax_scale=d["softmax_scale"], cmp_ratio=4, tokens=toks)
    assert np.array_equal(so, fo[toks]) and np.array_equal(sl, fl[toks])


def test_meta_oracle_flash_decode_matches_reference_fixtures():
    """The flash-decode branches (metadata.py:777-870, 925-954), pinned by the
    reference scheduler run with supportFd on (tests/golden/make_golden.py)."""
    import sas_testutil as U
    from oracle import meta_oracle as M

    cfgs, outs = U.load_meta_fd_fixtures()
    n_fd = sum(int((o[288:288 + 576].reshape(72, 8)[:, 0] != 0).any()) for o in outs)
    assert len(cfgs) > 500 and n_fd > 100
    bad = [i for i, c in enumerate(cfgs) if not np.array_equal(M.metadata(support_fd=True, **c), outs[i])]
    assert not bad, bad[:5]
