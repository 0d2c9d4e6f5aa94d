"""Shared helpers for the parity tests: fixture loading, running a case
through the public API, and the acceptance checks.

Acceptance bounds (bf16 / fp16 output against the golden reference):
max-abs <= 2e-2, mean-abs <= 2e-3, LSE abs <= 1e-3, plus the reference's own
``_check_result`` / ``_check_lse`` criteria
(test_sparse_attn_sharedkv.py:394-481), restated in ``check_result_ref``.
"""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
LSE_ABS = 1e-3


def load_attn_fixtures():
    z = np.load(os.path.join(GOLDEN, "attn_cases.npz"))
    cfgs = json.loads(str(z["configs"]))
    res = []
    for i, c in enumerate(cfgs):
        raw = z[f"out_{i}"]
        if c.get("dtype", "bf16") == "bf16":
            out = (raw.astype(np.uint32) << 16).view(np.float32)
        else:
            out = raw.view(np.float16).astype(np.float32)
        res.append((c, out, z[f"lse_{i}"]))
    return res


def load_meta_fixtures():
    z = np.load(os.path.join(GOLDEN, "metadata_cases.npz"))
    return json.loads(str(z["configs"])), z["outputs"]


def build_case(cfg):
    from dsv4_b200 import synth

    kw = {k: v for k, v in cfg.items() if k not in ("name", "edits")}
    case = synth.make_case(**kw)
    for t, pos, val in cfg.get("edits", []):
        case.idx[t, 0, pos] = val
    return case


def oracle_forward(case, tokens=None):
    from oracle import golden_oracle as O

    return O.forward(case.q, ori_kv=case.ori_kv, ori_bt=case.ori_bt, cmp_kv=case.cmp_kv, cmp_bt=case.cmp_bt,
                     idx=case.idx, cu_seqlens_q=case.cu_seqlens_q, seqused_kv=case.seqused_kv, sinks=case.sinks,
                     softmax_scale=case.softmax_scale, cmp_ratio=case.cmp_ratio, win_left=case.win_left,
                     dtype=case.dtype, tokens=tokens)


def to_device(case, device="cuda"):
    import torch

    tdt = torch.bfloat16 if case.dtype == "bf16" else torch.float16
    d = dict(
        q=torch.from_numpy(case.q).to(tdt).to(device),
        ori_kv=torch.from_numpy(case.ori_kv).to(tdt).to(device),
        ori_block_table=torch.from_numpy(case.ori_bt).to(device),
        cu_seqlens_q=torch.from_numpy(case.cu_seqlens_q).to(device),
        seqused_kv=torch.from_numpy(case.seqused_kv).to(device),
        sinks=torch.from_numpy(case.sinks).to(device),
        softmax_scale=case.softmax_scale,
        ori_win_left=case.win_left,
    )
    if case.scenario >= 2:
        d["cmp_kv"] = torch.from_numpy(case.cmp_kv).to(tdt).to(device)
        d["cmp_block_table"] = torch.from_numpy(case.cmp_bt).to(device)
        d["cmp_ratio"] = case.cmp_ratio
    if case.scenario == 3:
        d["cmp_sparse_indices"] = torch.from_numpy(case.idx).to(device)
    return d


def run_api(case, device="cuda", **extra):
    from dsv4_b200 import sparse_attn_sharedkv

    kw = to_device(case, device)
    kw.update(extra)
    q = kw.pop("q")
    out, lse = sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
    return out.float().cpu().numpy(), lse.float().cpu().numpy()


def check_close(out, ref_out, lse, ref_lse, rows=None, what=""):
    """BASELINE bounds. They are absolute bounds for N(0,1) data, whose
    outputs are O(1); for inputs drawn at a larger scale (the reference
    tests' U(-10, 10)) the output bounds scale with the RMS of the reference
    output, so that they keep meaning "a few output ulps"."""
    if rows is not None:
        out, ref_out, lse, ref_lse = out[rows], ref_out[rows], lse[rows], ref_lse[rows]
    d = np.abs(out.astype(np.float64) - ref_out.astype(np.float64))
    dl = np.abs(lse.astype(np.float64) - ref_lse.astype(np.float64))
    scale = max(1.0, float(np.sqrt(np.mean(ref_out.astype(np.float64) ** 2))))
    ref_ok = float(np.isclose(out, ref_out, rtol=2.0 ** -7, atol=1e-4).mean())
    msg = (f"{what}: max-abs {d.max():.3e} mean-abs {d.mean():.3e} lse max-abs {dl.max():.3e} "
           f"(output scale {scale:.2f}; reference isclose criterion {100 * ref_ok:.2f}%)")
    print(msg)
    assert np.isfinite(out).all(), msg + " (non-finite output)"
    assert d.max() <= MAX_ABS * scale, msg
    assert d.mean() <= MEAN_ABS * scale, msg
    assert dl.max() <= LSE_ABS * max(1.0, float(np.abs(ref_lse).max()) / 10.0), msg
    return msg


def check_result_ref(real, expt, dtype="bf16"):
    """The reference's own criterion (test_sparse_attn_sharedkv.py:394-437)."""
    if dtype == "bf16":
        rtol, atol = 0.0078125, 0.0001
    else:
        rtol, atol = 0.005, 0.000025
    real = np.asarray(real, np.float32).ravel()
    expt = np.asarray(expt, np.float32).ravel()
    ok = np.isclose(real, expt, rtol=rtol, atol=atol, equal_nan=True)
    n_err = int((~ok).sum())
    pct = (real.size - n_err) / max(real.size, 1) * 100.0
    floor = (1.0 / (1 << 14)) / 0.005
    b = np.maximum(np.maximum(np.abs(real), np.abs(expt)), floor) + 1e-9
    rel = np.abs(real - expt) / b
    max_rel = float(rel[~ok].max()) if n_err else 0.0
    assert pct >= 99.5, f"only {pct:.4f}% within tolerance"
    assert max_rel < 10.0, f"max normalised relative error {max_rel:.3f}"


def check_lse_ref(real, expt, dtype="bf16"):
    """Reference ``_check_lse`` (test_sparse_attn_sharedkv.py:440-481)."""
    rtol, atol = (0.015, 0.005) if dtype == "bf16" else (0.01, 0.001)
    real = np.asarray(real, np.float32).ravel()
    expt = np.asarray(expt, np.float32).ravel()
    ok = np.isclose(real, expt, rtol=rtol, atol=atol, equal_nan=True)
    pct = ok.mean() * 100.0 if ok.size else 100.0
    assert pct >= 99.5, f"lse: only {pct:.4f}% within tolerance"


def oracle_sampled(d, tokens, dtype="bf16", win_left=127):
    """Oracle output and LSE for a sample of tokens of a device-resident case
    ``d`` (the keyword dict of ``sparse_attn_sharedkv``, as built by
    ``synth.make_case_torch``), at sizes whose full inputs the CPU could not
    hold: only the sampled tokens' q rows and their attended KV rows are
    gathered on the device and copied to the host; positions and the top-k
    scan follow the oracle (``token_positions``), the math is ``token_forward``.
    Returns ``(out [n, H, D], lse [n, H])`` in the order of ``tokens``."""
    import torch
    from oracle import golden_oracle as O

    cu = d["cu_seqlens_q"].cpu().numpy().astype(np.int64)
    skv = d["seqused_kv"].cpu().numpy().astype(np.int64)
    ori_bt = d["ori_block_table"].cpu().numpy()
    ori_bs = d["ori_kv"].shape[1]
    ori_flat = d["ori_kv"].view(-1, d["ori_kv"].shape[-1])
    has_cmp = "cmp_kv" in d
    if has_cmp:
        cmp_bt = d["cmp_block_table"].cpu().numpy()
        cmp_bs = d["cmp_kv"].shape[1]
        cmp_flat = d["cmp_kv"].view(-1, d["cmp_kv"].shape[-1])
    idx = d.get("cmp_sparse_indices")
    sinks = d["sinks"].float().cpu().numpy()
    ratio = int(d.get("cmp_ratio", 4))
    outs, lses = [], []
    for t in tokens:
        b = int(np.searchsorted(cu, t, side="right") - 1)
        act_q = int(cu[b + 1] - cu[b])
        s_g = int(skv[b]) - act_q + (t - int(cu[b]))
        idx_row = idx[t, 0].cpu().numpy() if idx is not None else None
        wpos, cpos = O.token_positions(s_g=s_g, idx_row=idx_row, has_cmp=has_cmp, cmp_ratio=ratio,
                                       win_left=win_left)

        def rows(flat, table, bs, pos):
            if len(pos) == 0:
                return np.zeros((0, flat.shape[1]), np.float32)
            ids = torch.from_numpy(O.paged_row_ids(table, b, pos, bs)).to(flat.device)
            return flat.index_select(0, ids).float().cpu().numpy()

        win = rows(ori_flat, ori_bt, ori_bs, wpos)
        cmp = rows(cmp_flat, cmp_bt, cmp_bs, cpos) if has_cmp else np.zeros((0, win.shape[1]), np.float32)
        o, l = O.token_forward(d["q"][t].float().cpu().numpy(), win, cmp, sinks, float(d["softmax_scale"]), dtype)
        outs.append(o)
        lses.append(l)
    return np.stack(outs), np.stack(lses)


def load_meta_fd_fixtures():
    """Flash-decode schedules from the reference scheduler with supportFd on."""
    z = np.load(os.path.join(GOLDEN, "metadata_fd_cases.npz"))
    return json.loads(str(z["configs"])), z["outputs"]
