"""Backward (the gradient the reference's LSE output is documented for,
api.py:32-35, 176-184) against a plain PyTorch autograd reference (float64).

The reference builds, per query token, the attended rows exactly as the
oracle does (window, then the top-k scan of golden.py:28-66), gathers them
from fp32 leaf copies of the caches (so the pool gradients come out of the
gather), and differentiates softmax([q K^T * scale, sink]) @ [K; 0] against
a random output gradient. Bounds: each gradient's max-abs error is at most
2e-2 of its largest magnitude (the kernel reads bf16/fp16 inputs and writes
dq in that type; everything else is fp32).
"""

import numpy as np
import pytest

import sas_testutil as U

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

REL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _gpu(sas_lib):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dsv4_b200 import check_device_status, reset_device_status

    reset_device_status()
    yield
    check_device_status()


def torch_reference(case, dout):
    """fp32 autograd gradients (dq, d_ori, d_cmp, d_sinks) of sum(out * dout)."""
    from oracle import golden_oracle as O

    q = torch.from_numpy(case.q).double().requires_grad_()
    ori = torch.from_numpy(case.ori_kv).double().requires_grad_()
    cmp = torch.from_numpy(case.cmp_kv).double().requires_grad_() if case.scenario >= 2 else None
    sinks = torch.from_numpy(case.sinks).double().requires_grad_()
    cu = np.asarray(case.cu_seqlens_q)
    outs = []
    for b in range(case.B):
        aq = int(cu[b + 1] - cu[b])
        for s in range(aq):
            t = int(cu[b]) + s
            s_g = int(case.seqused_kv[b]) - aq + s
            wpos, cpos = O.token_positions(s_g=s_g, idx_row=None if case.idx is None else case.idx[t, 0],
                                           has_cmp=case.scenario >= 2, cmp_ratio=case.cmp_ratio,
                                           win_left=case.win_left)
            rows = []
            if len(wpos):
                ids = torch.from_numpy(O.paged_row_ids(case.ori_bt, b, wpos, case.ori_kv.shape[1]))
                rows.append(ori.reshape(-1, 512)[ids])
            if cmp is not None and len(cpos):
                ids = torch.from_numpy(O.paged_row_ids(case.cmp_bt, b, cpos, case.cmp_kv.shape[1]))
                rows.append(cmp.reshape(-1, 512)[ids])
            k = torch.cat(rows) if rows else torch.zeros(0, 512, dtype=torch.float64)
            sc = q[t] @ k.T * case.softmax_scale
            logits = torch.cat([sc, sinks[:, None]], dim=1)
            p = torch.softmax(logits, dim=1)
            outs.append(p[:, : k.shape[0]] @ k)
    out = torch.stack(outs)
    (out * torch.from_numpy(dout).double()).sum().backward()
    return (q.grad.numpy(), ori.grad.numpy(), None if cmp is None else cmp.grad.numpy(), sinks.grad.numpy())


def _check(name, got, ref):
    got = np.asarray(got, np.float64)
    err = np.abs(got - ref).max()
    scale = max(np.abs(ref).max(), 1e-6)
    print(f"{name}: max-abs err {err:.3e}, max |ref| {scale:.3e}")
    assert err <= REL * scale, f"{name}: {err:.3e} > {REL} * {scale:.3e}"


CASES = [
    dict(ctx=[3000, 5000, 129], q_lens=[1, 2, 1], H=64, K=512, seed=81),
    dict(ctx=[700, 260], q_lens=[40, 5], H=32, K=256, seed=82, edits=[[3, 10, -1]]),
    dict(ctx=[2000, 900], q_lens=[1, 3], H=64, K=0, scenario=2, cmp_ratio=128, seed=83),
    dict(ctx=[300, 90], q_lens=[4, 2], H=16, K=0, scenario=1, seed=84),
    dict(ctx=[1500], q_lens=[2], H=64, K=256, dtype="fp16", seed=85),
]


@pytest.mark.parametrize("cfg", CASES, ids=["scfa_decode", "scfa_prefill", "cfa", "swa", "fp16"])
def test_backward_vs_torch_autograd(cfg):
    from dsv4_b200 import sparse_attn_sharedkv, sparse_attn_sharedkv_backward

    case = U.build_case(cfg)
    d = U.to_device(case)
    q = d.pop("q")
    out, lse = sparse_attn_sharedkv(q, return_softmax_lse=True, **d)
    rng = np.random.default_rng(cfg["seed"])
    dout = rng.standard_normal(case.q.shape).astype(np.float32)
    dout_t = torch.from_numpy(dout).to(q.dtype).cuda()
    dq, d_ori, d_cmp, dsinks = sparse_attn_sharedkv_backward(dout_t, q, out, lse, **d)
    dout_r = dout_t.float().cpu().numpy()
    rq, rori, rcmp, rsinks = torch_reference(case, dout_r)
    _check("dq", dq.float().cpu().numpy(), rq)
    _check("d_ori_kv", d_ori.float().cpu().numpy(), rori)
    if rcmp is not None:
        _check("d_cmp_kv", d_cmp.float().cpu().numpy(), rcmp)
    _check("d_sinks", dsinks.cpu().numpy(), rsinks)


def test_autograd_function_matches_direct_backward():
    from dsv4_b200 import sparse_attn_sharedkv_backward, sparse_attn_sharedkv_train, sparse_attn_sharedkv

    case = U.build_case(CASES[0])
    d = U.to_device(case)
    q = d.pop("q").requires_grad_()
    ori = d.pop("ori_kv").requires_grad_()
    cmp = d.pop("cmp_kv").requires_grad_()
    sinks = d.pop("sinks").requires_grad_()
    o = sparse_attn_sharedkv_train(q, ori_kv=ori, cmp_kv=cmp, sinks=sinks, **d)
    g = torch.randn_like(o)
    o.backward(g)
    with torch.no_grad():
        o2, lse2 = sparse_attn_sharedkv(q, ori_kv=ori, cmp_kv=cmp, sinks=sinks, return_softmax_lse=True, **d)
        dq, d_ori, d_cmp, dsinks = sparse_attn_sharedkv_backward(g, q, o2, lse2, ori_kv=ori, cmp_kv=cmp,
                                                                 sinks=sinks, **d)
    assert torch.equal(o, o2)
    assert torch.equal(q.grad, dq)
    # pool gradients accumulate with atomics, so their summation order varies
    torch.testing.assert_close(ori.grad, d_ori, rtol=1e-2, atol=1e-3)
    torch.testing.assert_close(cmp.grad, d_cmp, rtol=1e-2, atol=1e-3)
    torch.testing.assert_close(sinks.grad, dsinks, rtol=1e-4, atol=1e-4)
