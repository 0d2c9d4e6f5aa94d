"""GPU parity at the BASELINE configurations' full shapes.

The public API runs on the whole seeded batch of each configuration, with the
inputs generated on the device (``synth.make_case_torch``); the oracle checks
a sample of tokens chosen where the edge cases are (``oracle_sampled``):

* C4 prefill, 2 x 8192 tokens, H64, K512 (above 512 tokens: the plan kernel
  and the non-fused attention variant): the first and last token of each
  request, tokens whose window is clipped at the start (s_g < 127), tokens
  with fewer than K valid compressed entries (s_g < 2047), and random ones;
* C3 MTP, 128 requests x 2 tokens, H128, K512, contexts log-U[128, 128k]:
  both tokens of the shortest requests (contexts of 130-160 rows, so windows
  that start at row 0 or 1 and fewer than K valid compressed entries), the
  longest ones, and random ones;
* C5 long-context decode, H128, K1024, contexts U[64k, 256k]: the 64 requests
  one GPU owns when the 512-request batch is length-balanced over 8 GPUs
  (every token checked);
* a prefill batch of 900 tokens checked on every token (plan-kernel path).

Every check asserts the BASELINE bounds and the reference's own
``_check_result`` criterion on the sampled rows.
"""

import numpy as np
import pytest

import sas_testutil as U

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _gpu(sas_lib):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dsv4_b200 import check_device_status, reset_device_status

    reset_device_status()
    yield
    check_device_status()


def _run_sampled(d, tokens, what):
    from dsv4_b200 import sparse_attn_sharedkv

    kw = dict(d)
    q = kw.pop("q")
    out, lse = sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
    sel = torch.tensor(tokens, dtype=torch.long, device=out.device)
    o = out.index_select(0, sel).float().cpu().numpy()
    l = lse.index_select(0, sel).cpu().numpy()
    ro, rl = U.oracle_sampled(d, tokens)
    U.check_close(o, ro, l, rl, what=what)
    U.check_result_ref(o, ro, "bf16")
    U.check_lse_ref(l, rl, "bf16")


def _device_case(name, seed, ctx=None, q_lens=None):
    from dsv4_b200 import synth

    c = synth.config_contexts(name, seed=0)
    return synth.make_case_torch(ctx=ctx if ctx is not None else c["ctx"],
                                 q_lens=q_lens if q_lens is not None else c["q_lens"],
                                 H=c["H"], K=c["K"], bs=c["bs"], seed=seed)


def test_c4_prefill_full_shape_sampled():
    d = _device_case("C4", seed=71)
    rng = np.random.default_rng(71)
    edges = [0, 1, 5, 100, 126, 127, 128, 129, 1000, 2046, 2047, 2048, 4000, 8190, 8191]
    toks = sorted(set(edges + [8192 + e for e in edges] + rng.integers(0, 16384, size=14).tolist()))
    _run_sampled(d, toks, "C4 prefill sample")
    del d
    torch.cuda.empty_cache()


def test_c3_mtp_full_shape_sampled():
    from dsv4_b200 import synth

    c = synth.config_contexts("C3", seed=0)
    ctx = np.asarray(c["ctx"])
    d = _device_case("C3", seed=72)
    order = np.argsort(ctx)
    reqs = list(order[:6]) + list(order[-3:])
    reqs += [int(r) for r in np.random.default_rng(72).choice(order[6:-3], size=7, replace=False)]
    assert (ctx[order[:6]] // 4 < 512).all()  # fewer than K valid compressed entries
    toks = sorted({2 * int(r) + s for r in reqs for s in (0, 1)})
    _run_sampled(d, toks, "C3 MTP sample")
    del d
    torch.cuda.empty_cache()


def test_c5_long_context_one_gpu_share():
    from dsv4_b200 import synth

    c = synth.config_contexts("C5", seed=0)
    part = synth.balance_requests(c["ctx"], 8)[0]
    ctx = [c["ctx"][i] for i in part]
    d = _device_case("C5", seed=73, ctx=ctx, q_lens=[1] * len(ctx))
    _run_sampled(d, list(range(len(ctx))), f"C5 ({len(ctx)} requests of 512)")
    del d
    torch.cuda.empty_cache()


def test_prefill_900_tokens_every_row():
    case = U.build_case(dict(ctx=[700, 2600], q_lens=[600, 300], H=64, K=512, seed=74))
    out, lse = U.run_api(case)
    ro, rl = U.oracle_forward(case)
    U.check_close(out, ro, lse, rl, what="900-token prefill, every row")
    U.check_result_ref(out, ro, case.dtype)
    U.check_lse_ref(lse, rl, case.dtype)
