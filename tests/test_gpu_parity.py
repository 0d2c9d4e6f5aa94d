"""GPU parity: the CUDA path (through the public API / C ABI) against the
reference fixtures and the pinned oracle.

Bounds: max-abs <= 2e-2, mean-abs <= 2e-3, LSE abs <= 1e-3, and the
reference's _check_result / _check_lse; the scheduler is bit-exact.
"""

import json

import numpy as np
import pytest

import sas_testutil as U

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _gpu(sas_lib):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dsv4_b200 import reset_device_status

    reset_device_status()
    yield
    from dsv4_b200 import check_device_status

    check_device_status()


def _meta_gpu(cfg):
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata

    kw = dict(cfg)
    for k in ("cu_seqlens_q", "seqused_kv"):
        if k in kw:
            kw[k] = torch.tensor(kw[k], dtype=torch.int32)
    return sparse_attn_sharedkv_metadata(device="cuda", **kw).cpu().numpy()


def test_metadata_gpu_bit_exact_vs_reference_fixtures():
    cfgs, outs = U.load_meta_fixtures()
    bad = [i for i, c in enumerate(cfgs) if not np.array_equal(_meta_gpu(c), outs[i])]
    assert not bad, f"{len(bad)} mismatches, first {bad[:5]}: {[cfgs[i] for i in bad[:2]]}"


def test_metadata_gpu_fuzz_vs_oracle():
    from oracle import meta_oracle as M

    rng = np.random.default_rng(7)
    bad = []
    for it in range(300):
        B = int(rng.integers(1, 200))
        ql = rng.integers(1, rng.choice([2, 3, 50, 600]), size=B)
        kv = np.maximum(rng.integers(1, rng.choice([300, 5000, 100000]), size=B), ql)
        cfg = dict(num_heads_q=int(rng.choice([16, 64, 128])), num_heads_kv=1, head_dim=512,
                   cu_seqlens_q=[0] + np.cumsum(ql).tolist(), seqused_kv=kv.tolist(), batch_size=B,
                   max_seqlen_q=int(ql.max()), max_seqlen_kv=int(kv.max()), layout_q="TND",
                   has_cmp_kv=bool(rng.random() < 0.8), cmp_ratio=int(rng.choice([4, 128])),
                   cmp_topk=int(rng.choice([0, 256, 512, 1024])), aic_core_num=int(rng.choice([24, 36, 8])))
        if not np.array_equal(_meta_gpu(cfg), M.metadata(**cfg)):
            bad.append(cfg)
    assert not bad, f"{len(bad)} mismatches; first {json.dumps(bad[0])[:400]}"


@pytest.mark.parametrize("i", range(9))
def test_attention_vs_reference_fixtures(i):
    cfg, ref_out, ref_lse = U.load_attn_fixtures()[i]
    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    U.check_close(out, ref_out, lse, ref_lse, what=cfg["name"])
    U.check_result_ref(out, ref_out, case.dtype)
    U.check_lse_ref(lse, ref_lse, case.dtype)


RANDOM_CASES = [
    dict(ctx=[5000, 129, 127, 1, 20000], q_lens=[1, 1, 1, 1, 1], H=64, K=512, seed=11),
    dict(ctx=[700, 3000, 64], q_lens=[2, 2, 2], H=128, K=512, seed=12),
    dict(ctx=[9000, 4000], q_lens=[1, 1], H=128, K=1024, seed=13),
    dict(ctx=[1500, 260], q_lens=[70, 5], H=64, K=512, seed=14),
    dict(ctx=[3000], q_lens=[1], H=16, K=256, bs_ori=64, bs_cmp=64, seed=15),
    dict(ctx=[2000, 1000], q_lens=[3, 4], H=32, K=128, seed=16),
    dict(ctx=[6000, 300], q_lens=[1, 2], H=96, K=384, seed=17),
    # the CPU-golden decode configuration at its full shape: B4, H16, K256, blocks of 64
    dict(ctx=[1024, 2048, 3000, 4096], q_lens=[1, 1, 1, 1], H=16, K=256, bs_ori=64, bs_cmp=64, seed=0),
]


@pytest.mark.parametrize("cfg", RANDOM_CASES, ids=[f"r{i}" for i in range(len(RANDOM_CASES))])
def test_attention_vs_oracle(cfg):
    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    ro, rl = U.oracle_forward(case)
    U.check_close(out, ro, lse, rl, what=str(cfg))
    U.check_result_ref(out, ro, case.dtype)


def test_attention_c2_scale_sampled():
    """BASELINE config 2 shapes (B=64, H=64, K=512, ctx U[8k,64k], block 128),
    checked against the oracle on a sample of 8 requests."""
    from dsv4_b200 import synth

    c = synth.config_contexts("C2")
    case = U.build_case(dict(ctx=c["ctx"], q_lens=c["q_lens"], H=64, K=512, seed=21))
    out, lse = U.run_api(case)
    toks = list(range(0, 64, 8))
    ro, rl = U.oracle_forward(case, tokens=toks)
    U.check_close(out, ro, lse, rl, rows=toks, what="C2 sample")
    U.check_result_ref(out[toks], ro[toks], case.dtype)


# Cases that cut tokens across CTAs (a token longer than a range plus the cut
# cost is split at range boundaries), covering both split-KV merge paths:
#  - 40 dense-CFA tokens of ~22 chunks over 148 ranges of ~7: each token cut
#    into 3-5 pieces (merged from TMEM up to 4 pieces, through L2 beyond);
#  - one long token among short ones: a 9-chunk SCFA token cut into a few
#    ranges (merged from TMEM), and a 41-chunk CFA token cut into many ranges
#    (merged through L2).
SPLIT_CASES = [
    (dict(ctx=[10000 + 37 * i for i in range(40)], q_lens=[1] * 40, H=64, K=0, scenario=2, seed=31),
     [0, 13, 27, 39]),
    (dict(ctx=[200] * 149 + [20000], q_lens=[1] * 150, H=64, K=1024, seed=32), [0, 77, 148, 149]),
    (dict(ctx=[100] * 149 + [20000], q_lens=[1] * 150, H=64, K=0, scenario=2, seed=33), [0, 148, 149]),
]


@pytest.fixture
def split_tokens():
    """Enable splitting long tokens across CTAs (SAS_OPT_SPLIT_TOKENS, cut cost
    one tile) for one test; the default keeps every token on one CTA."""
    from dsv4_b200 import _lib as L

    L.check(L.lib().sas_fwd_set_option(L.OPT_SPLIT_TOKENS, 1.0, None), "set_option")
    yield
    L.check(L.lib().sas_fwd_set_option(L.OPT_SPLIT_TOKENS, -1.0, None), "set_option")


@pytest.mark.parametrize("cfg,toks", SPLIT_CASES, ids=["long_tokens", "one_long_tmem", "one_long_l2"])
def test_attention_split_tokens(cfg, toks, split_tokens):
    """Split-KV path: within the accuracy bounds (a piece after the first
    rounds P against its own running max, so not the reference's rounding
    points), and bit-identical replays whichever piece lands last."""
    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    ro, rl = U.oracle_forward(case, tokens=toks)
    U.check_close(out, ro, lse, rl, rows=toks, what=str(cfg)[:80])
    out2, lse2 = U.run_api(case)
    assert np.array_equal(out, out2) and np.array_equal(lse, lse2), "split-token merge is not deterministic"


@pytest.mark.parametrize("cfg,toks", SPLIT_CASES[1:], ids=["one_long_a", "one_long_b"])
def test_long_tokens_whole_by_default(cfg, toks):
    """By default no token is split, so even a token far longer than a
    range meets the reference's own acceptance criterion."""
    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    ro, rl = U.oracle_forward(case, tokens=toks)
    U.check_close(out, ro, lse, rl, rows=toks, what=str(cfg)[:80])
    U.check_result_ref(out[toks], ro[toks], case.dtype)


def _covered_tokens(md, cu):
    """Tokens inside some enabled core window of the metadata (kernel.py:254-278)."""
    fa = md[:36 * 8].reshape(36, 8)
    ql = np.diff(cu)
    smax = int(ql.max())
    wins = [(int(r[1]) * smax + int(r[2]), int(r[4]) * smax + int(r[5])) for r in fa if r[0]]
    cov = []
    for b in range(len(ql)):
        for s in range(int(ql[b])):
            pid = b * smax + s
            cov.append(any(lo <= pid < hi for lo, hi in wins))
    return np.array(cov)


@pytest.mark.parametrize("cfg", [
    dict(ctx=[3000, 5000, 800, 12000], q_lens=[1, 2, 1, 3], H=64, K=512, seed=41),  # plan in the attention kernel
    dict(ctx=[3000, 900], q_lens=[400, 300], H=64, K=256, seed=42),                 # plan kernel
], ids=["fused_plan", "plan_kernel"])
def test_uncovered_tokens_are_zero(cfg):
    """Metadata with a core disabled: the tokens of its window get zero output
    and LSE, every other token is unchanged."""
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata

    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    cu = np.asarray(case.cu_seqlens_q)
    md = sparse_attn_sharedkv_metadata(
        num_heads_q=case.H, num_heads_kv=1, head_dim=512, cu_seqlens_q=torch.tensor(cu, dtype=torch.int32),
        seqused_kv=torch.tensor(case.seqused_kv, dtype=torch.int32), batch_size=len(cu) - 1, layout_q="TND",
        cmp_topk=case.K, cmp_ratio=case.cmp_ratio, device="cpu").numpy().copy()
    used = [i for i in range(36) if md[i * 8] == 1]
    md[used[len(used) // 2] * 8] = 0  # disable a core in the middle
    cov = _covered_tokens(md, cu)
    assert (~cov).any() and cov.any()
    out2, lse2 = U.run_api(case, metadata=torch.tensor(md, dtype=torch.int32, device="cuda"))
    assert np.all(out2[~cov] == 0) and np.all(lse2[~cov] == 0)
    assert np.array_equal(out2[cov], out[cov]) and np.array_equal(lse2[cov], lse[cov])


def test_bsnd_layout_and_return_types():
    from dsv4_b200 import sparse_attn_sharedkv

    case = U.build_case(dict(ctx=[900, 1200], q_lens=[3, 3], H=64, K=256, seed=31))
    d = U.to_device(case)
    q = d.pop("q")
    B, S = 2, 3
    idx = d.pop("cmp_sparse_indices")
    o_tnd, l_tnd = sparse_attn_sharedkv(q, cmp_sparse_indices=idx, return_softmax_lse=True, **d)
    o_only = sparse_attn_sharedkv(q, cmp_sparse_indices=idx, **d)
    assert isinstance(o_only, torch.Tensor) and torch.equal(o_only, o_tnd)
    assert o_tnd.shape == q.shape and l_tnd.shape == (B * S, 64) and l_tnd.dtype == torch.float32
    d.pop("cu_seqlens_q")
    o_b, l_b = sparse_attn_sharedkv(q.reshape(B, S, 64, 512), cmp_sparse_indices=idx.reshape(B, S, 1, 256),
                                    layout_q="BSND", return_softmax_lse=True, **d)
    assert o_b.shape == (B, S, 64, 512) and l_b.shape == (B, S, 64)
    assert torch.equal(o_b.reshape(B * S, 64, 512), o_tnd)
    assert torch.equal(l_b.reshape(B * S, 64), l_tnd)


def test_bsnd_padding_rows_are_zero():
    from dsv4_b200 import sparse_attn_sharedkv

    case = U.build_case(dict(ctx=[900, 1200], q_lens=[4, 4], H=64, K=256, seed=32))
    d = U.to_device(case)
    q = d.pop("q").reshape(2, 4, 64, 512)
    idx = d.pop("cmp_sparse_indices").reshape(2, 4, 1, 256)
    d["cu_seqlens_q"] = torch.tensor([0, 2, 5], dtype=torch.int32, device="cuda")  # act_q = 2, 3
    o, l = sparse_attn_sharedkv(q, cmp_sparse_indices=idx, layout_q="BSND", return_softmax_lse=True, **d)
    assert torch.count_nonzero(o[0, 2:]) == 0 and torch.count_nonzero(l[0, 2:]) == 0
    assert torch.count_nonzero(o[1, 3:]) == 0
    assert torch.count_nonzero(o[0, :2]) > 0


def test_deterministic_replay():
    case = U.build_case(dict(ctx=[20000, 30000, 5000], q_lens=[1, 2, 1], H=128, K=512, seed=41))
    a, la = U.run_api(case)
    b, lb = U.run_api(case)
    assert np.array_equal(a, b) and np.array_equal(la, lb)


def test_metadata_default_returns_cpu_tensor():
    """As the reference (metadata.py:1083-1086): a CPU tensor unless a device is named."""
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata

    kw = dict(num_heads_q=64, num_heads_kv=1, head_dim=512, cu_seqlens_q=torch.tensor([0, 1, 3], dtype=torch.int32),
              seqused_kv=torch.tensor([5000, 900], dtype=torch.int32), batch_size=2, layout_q="TND", cmp_topk=512,
              cmp_ratio=4)
    a = sparse_attn_sharedkv_metadata(**kw)
    b = sparse_attn_sharedkv_metadata(device="cuda", **kw)
    assert a.device.type == "cpu" and b.is_cuda and torch.equal(a, b.cpu())


def _meta_gpu_fd(cfg):
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata

    kw = dict(cfg)
    for k in ("cu_seqlens_q", "seqused_kv"):
        if k in kw:
            kw[k] = torch.tensor(kw[k], dtype=torch.int32)
    return sparse_attn_sharedkv_metadata(device="cuda", support_fd=True, **kw).cpu().numpy()


def test_metadata_fd_gpu_bit_exact_vs_reference_fixtures():
    cfgs, outs = U.load_meta_fd_fixtures()
    bad = [i for i, c in enumerate(cfgs) if not np.array_equal(_meta_gpu_fd(c), outs[i])]
    assert not bad, f"{len(bad)} mismatches, first {bad[:5]}: {[cfgs[i] for i in bad[:2]]}"


def test_metadata_fd_gpu_fuzz_vs_oracle():
    from oracle import meta_oracle as M

    rng = np.random.default_rng(8)
    bad = []
    for it in range(150):
        B = int(rng.integers(1, 40))
        ql = rng.integers(1, rng.choice([2, 3, 50, 600]), size=B)
        kv = np.maximum(rng.integers(1, rng.choice([300, 5000, 200000]), size=B), ql)
        cfg = dict(num_heads_q=int(rng.choice([16, 64, 128])), num_heads_kv=1, head_dim=512,
                   cu_seqlens_q=[0] + np.cumsum(ql).tolist(), seqused_kv=kv.tolist(), batch_size=B,
                   max_seqlen_q=int(ql.max()), max_seqlen_kv=int(kv.max()), layout_q="TND",
                   has_cmp_kv=bool(rng.random() < 0.8), cmp_ratio=int(rng.choice([4, 128])),
                   cmp_topk=int(rng.choice([0, 256, 512, 1024])), aic_core_num=int(rng.choice([24, 36, 8])),
                   aiv_core_num=int(rng.choice([48, 72, 8])))
        if not np.array_equal(_meta_gpu_fd(cfg), M.metadata(support_fd=True, **cfg)):
            bad.append(cfg)
    assert not bad, f"{len(bad)} mismatches; first {json.dumps(bad[0])[:400]}"


@pytest.mark.parametrize("cfg", [
    dict(ctx=[70000, 9000, 200000, 130], q_lens=[1, 1, 1, 1], H=64, K=1024, seed=43),   # rows cut between cores
    dict(ctx=[3000, 900], q_lens=[400, 300], H=64, K=256, seed=44),                     # plan kernel
], ids=["decode", "prefill"])
def test_attention_accepts_flash_decode_schedule(cfg):
    """A flash-decode schedule covers the same tokens (a row cut between two
    cores belongs to the core that starts with it, kernel.py:254-278), so the
    forward gives the same bits with either schedule."""
    from dsv4_b200.metadata import sparse_attn_sharedkv_metadata

    case = U.build_case(cfg)
    out, lse = U.run_api(case)
    cu = torch.tensor(np.asarray(case.cu_seqlens_q), dtype=torch.int32)
    md = sparse_attn_sharedkv_metadata(
        num_heads_q=case.H, num_heads_kv=1, head_dim=512, cu_seqlens_q=cu,
        seqused_kv=torch.tensor(case.seqused_kv, dtype=torch.int32), batch_size=len(cu) - 1, layout_q="TND",
        cmp_topk=case.K, cmp_ratio=case.cmp_ratio, device="cuda", support_fd=True)
    out2, lse2 = U.run_api(case, metadata=md)
    assert np.array_equal(out2, out) and np.array_equal(lse2, lse)
