"""CPU model of the cluster decode kernel's arithmetic (csrc/sas_dec.cu).

Four CTAs share a query token: the window tile is split 32 rows per CTA, and
compressed tile i puts its chunk 4i + rank on CTA `rank`. For each tile every
CTA publishes max(its rows' max, running max), all four take the max of the
four values, and round P against it; at the end the four partial outputs and
row sums are added. The model restates that order of operations in numpy and
checks it against the oracle (golden.py's tiles of 512 rows): same running
maxima, so the reference's own `_check_result` criterion holds as tightly as
for the single-CTA order.
"""

import numpy as np
import pytest

import sas_testutil as U

CL, CH, WP = 4, 128, 32


def cluster_token(q, win, cmp, sinks, scale, dtype="bf16"):
    from oracle import golden_oracle as O

    H, D = q.shape
    qs = q.astype(np.float32)
    m = sinks.astype(np.float32).copy()  # running max, natural units
    l = np.zeros((CL, H), np.float32)
    acc = np.zeros((CL, H, D), np.float32)
    # steps: the window tile split over the CTAs, then compressed tiles of 4 chunks
    steps = [[win[r * WP:(r + 1) * WP] for r in range(CL)]]
    nch = (cmp.shape[0] + CH - 1) // CH
    for t in range((nch + CL - 1) // CL):
        steps.append([cmp[(t * CL + r) * CH:(t * CL + r + 1) * CH] for r in range(CL)])
    for rows in steps:
        scores = [qs @ k.T * np.float32(scale) if k.shape[0] else np.zeros((H, 0), np.float32) for k in rows]
        local = [s.max(axis=1) if s.shape[1] else np.full(H, -np.inf, np.float32) for s in scores]
        m_new = np.maximum(m, np.max(np.stack(local), axis=0))
        alpha = np.exp(m - m_new)
        for r in range(CL):
            l[r] *= alpha
            acc[r] *= alpha[:, None]
            if rows[r].shape[0]:
                p = np.exp(scores[r] - m_new[:, None])
                l[r] += p.sum(axis=1)
                acc[r] += O.round_dtype(p, dtype) @ rows[r]
        m = m_new
    L = l.sum(axis=0) + np.exp(sinks.astype(np.float32) - m)
    out = acc.sum(axis=0) / L[:, None]
    return O.round_dtype(out, dtype), m + np.log(L)


CASES = [
    dict(ctx=[5000, 129, 127, 1, 20000], q_lens=[1, 1, 1, 1, 1], H=64, K=512, seed=11),
    dict(ctx=[9000, 4000], q_lens=[1, 1], H=128, K=1024, seed=13),
    dict(ctx=[3000], q_lens=[1], H=16, K=256, bs_ori=64, bs_cmp=64, seed=15),
    dict(ctx=[700, 3000, 64], q_lens=[2, 2, 2], H=128, K=512, seed=12),
]


@pytest.mark.parametrize("cfg", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_cluster_order_matches_oracle(cfg):
    from oracle import golden_oracle as O

    case = U.build_case(cfg)
    ro, rl = U.oracle_forward(case)
    cu = case.cu_seqlens_q
    outs, lses = [], []
    for b in range(case.B):
        aq = int(cu[b + 1] - cu[b])
        for s in range(aq):
            t = int(cu[b]) + s
            s_g = int(case.seqused_kv[b]) - aq + s
            win, cmp = O.token_rows(b=b, s_g=s_g, ori_kv=case.ori_kv, ori_bt=case.ori_bt, cmp_kv=case.cmp_kv,
                                    cmp_bt=case.cmp_bt, idx_row=case.idx[t, 0], cmp_ratio=case.cmp_ratio,
                                    win_left=case.win_left)
            o, lse = cluster_token(case.q[t], win, cmp, case.sinks, case.softmax_scale)
            outs.append(o)
            lses.append(lse)
    out, lse = np.stack(outs), np.stack(lses)
    U.check_close(out, ro, lse, rl, what=str(cfg))
    U.check_result_ref(out, ro, case.dtype)
