"""Backward of ``sparse_attn_sharedkv``, consuming the forward's LSE.

The reference documents the LSE output as the input of a FlashAttention-2
style backward (``sparse_attn_sharedkv_tilelang/api.py:32-35, 176-184``) and
ships none. ``sparse_attn_sharedkv_backward`` takes the forward's inputs, its
output and LSE and the output gradient, and returns the gradients of ``q``,
of the two paged caches (K = V: a row's key and value gradients are summed)
and of the sink logits. ``SparseAttnSharedkv.apply`` / ``sparse_attn_sharedkv_train``
wire forward and backward into ``torch.autograd``.

The gradient is that of the exact softmax with the sink in the denominator
(P is not rounded to the I/O type as the forward's P.V is, golden.py:191-195).
Every query token is taken as covered by the schedule (the forward leaves
tokens outside every core window at zero; a backward of such a call would
differ for those tokens).

One C-ABI call (``sas_sparse_attn_sharedkv_bwd``) computes dq and accumulates
the cache gradients in fp32 buffers shaped like the caches; ``sas_bwd_cast``
converts them to the caches' type.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _i32(t, dev):
    return t.to(device=dev, dtype=torch.int32).contiguous()


def sparse_attn_sharedkv_backward(
    dout: torch.Tensor,
    q: torch.Tensor,
    out: torch.Tensor,
    lse: torch.Tensor,
    *,
    ori_kv: torch.Tensor,
    cmp_kv: Optional[torch.Tensor] = None,
    cmp_sparse_indices: Optional[torch.Tensor] = None,
    ori_block_table: torch.Tensor,
    cmp_block_table: Optional[torch.Tensor] = None,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    seqused_q: Optional[torch.Tensor] = None,
    seqused_kv: torch.Tensor,
    sinks: torch.Tensor,
    softmax_scale: float,
    cmp_ratio: Optional[int] = None,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "TND",
    layout_kv: str = "PA_ND",
    topk_cmp: Optional[int] = None,
    **unused,
):
    """Returns ``(dq, d_ori_kv, d_cmp_kv, d_sinks)``; ``d_cmp_kv`` is None
    without a compressed cache. Arguments are those of the forward plus
    ``dout`` (the gradient of its output), ``out`` and ``lse`` (its results,
    ``lse`` as returned with ``return_softmax_lse=True``)."""
    del seqused_q, unused
    assert ori_mask_mode == 4, "only ori_mask_mode=4 supported"
    assert cmp_mask_mode == 3 or cmp_kv is None, "only cmp_mask_mode=3 supported"
    assert ori_win_right == 0, "only ori_win_right=0 supported"
    assert layout_kv == "PA_ND", "only layout_kv=PA_ND supported"
    assert layout_q in ("TND", "BSND"), f"unsupported layout_q={layout_q!r}"
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported dtype {q.dtype}")
    dcode = 0 if q.dtype == torch.bfloat16 else 1
    if not q.is_cuda:
        raise RuntimeError("sparse_attn_sharedkv_backward needs CUDA tensors (no CPU path)")
    dev = q.device
    scenario = 1 if cmp_kv is None else (2 if cmp_sparse_indices is None else 3)
    if layout_q == "TND":
        assert cu_seqlens_q is not None, "cu_seqlens_q is required for TND"
        T, H, D = q.shape
        cu = _i32(cu_seqlens_q, dev)
        B, S = cu.numel() - 1, 0
        idx = cmp_sparse_indices
    else:
        B, S, H, D = q.shape
        T = B * S
        cu = _i32(cu_seqlens_q, dev) if cu_seqlens_q is not None else None
        idx = None
        if cmp_sparse_indices is not None:
            idx = cmp_sparse_indices.reshape(T, cmp_sparse_indices.shape[2], cmp_sparse_indices.shape[3])
    if D != 512 or H <= 0:
        raise ValueError(f"only D=512 supported (got H={H}, D={D})")
    K = 0
    if scenario == 3:
        K = topk_cmp if topk_cmp is not None else idx.shape[-1]
        idx = _i32(idx, dev)
    ratio = cmp_ratio if cmp_ratio is not None else 4
    qf = q.contiguous().reshape(T, H, D)
    of = out.contiguous().reshape(T, H, D)
    dof = dout.to(q.dtype).contiguous().reshape(T, H, D)
    lf = lse.to(torch.float32).contiguous().reshape(T, H)
    ori = ori_kv.contiguous()
    obt = _i32(ori_block_table, dev)
    skv = _i32(seqused_kv, dev)
    snk = sinks.to(device=dev, dtype=torch.float32).contiguous()
    d_ori32 = torch.zeros(ori.shape, dtype=torch.float32, device=dev)
    cmp = cbt = d_cmp32 = None
    if scenario >= 2:
        cmp = cmp_kv.contiguous()
        cbt = _i32(cmp_block_table, dev)
        d_cmp32 = torch.zeros(cmp.shape, dtype=torch.float32, device=dev)
    dq = torch.empty_like(qf)
    dsinks = torch.zeros(H, dtype=torch.float32, device=dev)
    lib = _lib.lib()
    st = _lib.state(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.sas_sparse_attn_sharedkv_bwd(
        dof.data_ptr(), qf.data_ptr(), of.data_ptr(), lf.data_ptr(), T, H, D, dcode,
        1 if layout_q == "TND" else 0, int(B), int(S), _lib.ptr(cu), skv.data_ptr(),
        ori.data_ptr(), ori.shape[0], ori.shape[1], obt.data_ptr(), obt.shape[1],
        _lib.ptr(cmp), cmp.shape[0] if cmp is not None else 0, cmp.shape[1] if cmp is not None else 0,
        _lib.ptr(cbt), cbt.shape[1] if cbt is not None else 0, _lib.ptr(idx), int(K), snk.data_ptr(),
        float(softmax_scale), int(ratio), int(ori_win_left), scenario, dq.data_ptr(), d_ori32.data_ptr(),
        _lib.ptr(d_cmp32), dsinks.data_ptr(), st.status.data_ptr(), stream)
    if rc in (1, 2):
        raise ValueError(f"sparse_attn_sharedkv_backward: {_lib.ERRORS[rc]}")
    _lib.check(rc, "sas_sparse_attn_sharedkv_bwd")

    def cast(src, like):
        dst = torch.empty(like.shape, dtype=like.dtype, device=dev)
        _lib.check(lib.sas_bwd_cast(src.data_ptr(), dst.data_ptr(), src.numel(), dcode, stream), "sas_bwd_cast")
        return dst

    d_ori = cast(d_ori32, ori)
    d_cmp = cast(d_cmp32, cmp) if cmp is not None else None
    return dq.reshape(q.shape), d_ori, d_cmp, dsinks.to(sinks.dtype)


class SparseAttnSharedkv(torch.autograd.Function):
    """``sparse_attn_sharedkv`` as an autograd function of (q, ori_kv, cmp_kv, sinks)."""

    @staticmethod
    def forward(ctx, q, ori_kv, cmp_kv, sinks, kwargs):
        from .api import sparse_attn_sharedkv

        o, lse = sparse_attn_sharedkv(q, ori_kv=ori_kv, cmp_kv=cmp_kv, sinks=sinks, return_softmax_lse=True,
                                      **kwargs)
        ctx.kwargs = kwargs
        ctx.save_for_backward(q, ori_kv, cmp_kv if cmp_kv is not None else torch.empty(0), sinks, o, lse)
        ctx.has_cmp = cmp_kv is not None
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        del dlse
        q, ori_kv, cmp_kv, sinks, o, lse = ctx.saved_tensors
        kw = {k: v for k, v in ctx.kwargs.items() if k not in ("metadata", "core_num", "out", "lse_out")}
        dq, d_ori, d_cmp, dsinks = sparse_attn_sharedkv_backward(
            dout, q, o, lse, ori_kv=ori_kv, cmp_kv=cmp_kv if ctx.has_cmp else None, sinks=sinks, **kw)
        return dq, d_ori, d_cmp, dsinks, None


def sparse_attn_sharedkv_train(q, *, ori_kv, cmp_kv=None, sinks, return_softmax_lse=False, **kwargs):
    """Forward with autograd: gradients flow to ``q``, ``ori_kv``, ``cmp_kv`` and ``sinks``."""
    o, lse = SparseAttnSharedkv.apply(q, ori_kv, cmp_kv, sinks, kwargs)
    return (o, lse) if return_softmax_lse else o
