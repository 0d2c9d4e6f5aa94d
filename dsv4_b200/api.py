"""Host entry point ``sparse_attn_sharedkv`` (drop-in for the reference api.py).

Same keyword set, defaults, scenario routing and return convention as
``sparse_attn_sharedkv_tilelang/api.py:129-397``:

* ``cmp_kv=None, cmp_sparse_indices=None`` -> SWA (scenario 1),
  ``cmp_kv`` only -> CFA (2), both -> SCFA (3) (api.py:196-202);
* ``layout_q`` ``"TND"`` (``cu_seqlens_q`` required) or ``"BSND"``
  (api.py:208-240); ``layout_kv`` must be ``"PA_ND"``;
* ``metadata`` is the ``int32[1024]`` SparseAttnSharedkvMetadata contract;
  when omitted it is produced on the GPU with the same arguments the
  reference passes (api.py:335-366);
* returns ``out`` or ``(out, lse)`` with ``lse`` fp32 ``[T1, N1]`` (TND) or
  ``[B, S1, N1]`` (BSND) (api.py:388-397).

Underneath, one C-ABI call (``libsas_b200.so``) enqueues the plan, fused
attention and combine kernels on the current stream. There is no host
synchronisation on this path and no CPU fallback: a tensor that is not on a
CUDA device, or a missing library, raises.

Constraints (``ValueError``, widened from the reference's N1=64 only,
api.py:279-282): N2 = 1, D = 512, N1 a multiple of 8, bf16 or fp16.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple, Union

import torch

from . import _lib
from .metadata import SAS_META_SIZE, sparse_attn_sharedkv_metadata

DEFAULT_CORE_NUM = 24
DEFAULT_BLOCK_I = 128


def _dtype_code(t: torch.dtype) -> int:
    if t == torch.bfloat16:
        return 0
    if t == torch.float16:
        return 1
    raise ValueError(f"unsupported torch dtype {t}")


def _i32(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    return t.to(device=dev, dtype=torch.int32).contiguous()


def sparse_attn_sharedkv(
    q: torch.Tensor,
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
    metadata: Optional[torch.Tensor] = None,
    softmax_scale: float,
    cmp_ratio: Optional[int] = None,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "TND",
    layout_kv: str = "PA_ND",
    return_softmax_lse: bool = False,
    core_num: int = DEFAULT_CORE_NUM,
    topk_cmp: Optional[int] = None,
    out: Optional[torch.Tensor] = None,
    lse_out: Optional[torch.Tensor] = None,
    _stages: int = _lib.STAGE_ALL,
    _gather=None,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Forward pass; returns ``attention_out`` with the layout of ``q``.

    ``out`` / ``lse_out`` optionally supply preallocated result buffers
    (same shapes as the returned tensors), which CUDA-graph capture wants.
    ``seqused_q`` is accepted for API parity and unused (api.py:186).
    ``_gather`` (internal, ``dsv4_b200.sharding``) is ``(out_ptrs, lse_ptrs,
    heads_total, head_offset)``: the call computes heads ``[head_offset,
    head_offset + N1)`` and writes them into every buffer of ``out_ptrs`` /
    ``lse_ptrs`` (one per rank, outputs of ``heads_total`` heads); nothing is
    returned.
    """
    del seqused_q
    assert ori_mask_mode == 4, "only ori_mask_mode=4 supported"
    assert cmp_mask_mode == 3 or cmp_kv is None, "only cmp_mask_mode=3 supported"
    assert ori_win_right == 0, "only ori_win_right=0 supported"
    assert layout_kv == "PA_ND", "only layout_kv=PA_ND supported"
    assert layout_q in ("TND", "BSND"), f"unsupported layout_q={layout_q!r}"
    dcode = _dtype_code(q.dtype)
    dev = q.device

    if cmp_kv is None:
        scenario = 1
    elif cmp_sparse_indices is None:
        scenario = 2
    else:
        scenario = 3

    if layout_q == "TND":
        assert cu_seqlens_q is not None, "cu_seqlens_q is required for TND"
        T1, N1, D = q.shape
        cu = _i32(cu_seqlens_q, dev)
        B = cu.numel() - 1
        S = 0
        q_flat = q.contiguous()
        idx = cmp_sparse_indices
    else:
        B, S, N1, D = q.shape
        T1 = B * S
        cu = _i32(cu_seqlens_q, dev) if cu_seqlens_q is not None else None
        q_flat = q.contiguous().reshape(T1, N1, D)
        idx = None
        if cmp_sparse_indices is not None:
            ci = cmp_sparse_indices
            idx = ci.reshape(T1, ci.shape[2], ci.shape[3])

    if scenario == 3:
        N2 = idx.shape[1]
        K = topk_cmp if topk_cmp is not None else idx.shape[2]
        assert K == idx.shape[2], "topk_cmp does not match cmp_sparse_indices last dim"
        idx_dev = _i32(idx, dev)
    elif scenario == 2:
        N2 = cmp_kv.shape[2]
        K = 0
        idx_dev = None
    else:
        N2 = ori_kv.shape[2]
        K = 0
        idx_dev = None
    if N2 != 1 or D != 512 or N1 % 8 != 0 or N1 <= 0:
        raise ValueError(f"only N2=1, D=512 and N1 a multiple of 8 supported (got N1={N1}, N2={N2}, D={D})")
    if metadata is not None:
        assert metadata.numel() == SAS_META_SIZE, \
            f"metadata must have {SAS_META_SIZE} int32 entries (got {metadata.numel()})"
    # every host-side check above runs before the device is needed
    if not q.is_cuda:
        raise RuntimeError("sparse_attn_sharedkv needs q on a CUDA device (no CPU path)")
    cmp_ratio_eff = cmp_ratio if cmp_ratio is not None else 4

    ori_kv_dev = ori_kv.to(dev).contiguous()
    if ori_kv_dev.dtype != q.dtype:
        raise ValueError("ori_kv must have the dtype of q")
    ori_bt = _i32(ori_block_table, dev)
    skv = _i32(seqused_kv, dev)
    sinks_dev = sinks.to(device=dev, dtype=torch.float32).contiguous()
    if scenario >= 2:
        cmp_kv_dev = cmp_kv.to(dev).contiguous()
        if cmp_kv_dev.dtype != q.dtype:
            raise ValueError("cmp_kv must have the dtype of q")
        cmp_bt = _i32(cmp_block_table, dev)
    else:
        cmp_kv_dev = None
        cmp_bt = None

    lib = _lib.lib()
    st = _lib.state(dev)
    # the workspace first: a first-use allocation zero-fills it with a kernel,
    # which must not sit between the scheduler and the attention launch
    ws = st.workspace(lib.sas_fwd_workspace_bytes(T1, N1, st.num_sms))
    flags = 0
    if metadata is None:
        meta_kwargs = dict(
            num_heads_q=N1, num_heads_kv=N2, head_dim=D,
            cu_seqlens_q=cu if layout_q == "TND" else None,
            seqused_kv=skv, batch_size=int(B),
            # only read when cu_seqlens_q / seqused_kv are absent (BSND q length)
            max_seqlen_q=int(S), max_seqlen_kv=0,
            ori_mask_mode=ori_mask_mode, ori_win_left=ori_win_left, ori_win_right=ori_win_right,
            layout_q=layout_q, layout_kv=layout_kv, has_ori_kv=True, has_cmp_kv=cmp_kv is not None,
            aic_core_num=core_num, device=dev,
        )
        if scenario >= 2:
            meta_kwargs["cmp_ratio"] = cmp_ratio_eff
            meta_kwargs["cmp_mask_mode"] = cmp_mask_mode
        if scenario == 3:
            meta_kwargs["cmp_topk"] = K
        metadata = sparse_attn_sharedkv_metadata(**meta_kwargs)
        # nothing is enqueued between it and the attention launch, which may
        # then overlap it
        flags = _lib.FLAG_AFTER_METADATA if _gather is None else 0
    md = metadata.to(device=dev, dtype=torch.int32)
    assert md.numel() == SAS_META_SIZE, f"metadata must have {SAS_META_SIZE} int32 entries (got {md.numel()})"
    md = md.reshape(SAS_META_SIZE).contiguous()

    stream = torch.cuda.current_stream(dev).cuda_stream
    if _gather is not None:
        out_ptrs, lse_ptrs, heads_total, head_offset = _gather
        n = len(out_ptrs)
        optrs = (ctypes.c_void_p * n)(*out_ptrs)
        lptrs = (ctypes.c_void_p * n)(*lse_ptrs)
        rc = lib.sas_sparse_attn_sharedkv_fwd_gather(
            q_flat.data_ptr(), T1, N1, D, dcode, 1 if layout_q == "TND" else 0, int(B), int(S), _lib.ptr(cu),
            skv.data_ptr(),
            ori_kv_dev.data_ptr(), ori_kv_dev.shape[0], ori_kv_dev.shape[1], ori_bt.data_ptr(), ori_bt.shape[1],
            _lib.ptr(cmp_kv_dev), cmp_kv_dev.shape[0] if cmp_kv_dev is not None else 0,
            cmp_kv_dev.shape[1] if cmp_kv_dev is not None else 0, _lib.ptr(cmp_bt),
            cmp_bt.shape[1] if cmp_bt is not None else 0,
            _lib.ptr(idx_dev), int(K), sinks_dev.data_ptr(), md.data_ptr(), float(softmax_scale),
            int(cmp_ratio_eff), int(ori_win_left), scenario, optrs, lptrs, n, int(heads_total), int(head_offset),
            st.num_sms, int(_stages), st.status.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        if rc in (1, 2):
            raise ValueError(f"sparse_attn_sharedkv: {_lib.ERRORS[rc]}")
        _lib.check(rc, "sas_sparse_attn_sharedkv_fwd_gather")
        return None
    out_flat = out.view(T1, N1, D) if out is not None else torch.empty((T1, N1, D), dtype=q.dtype, device=dev)
    lse_flat = lse_out.view(T1, N1) if lse_out is not None else torch.empty((T1, N1), dtype=torch.float32,
                                                                              device=dev)
    rc = lib.sas_sparse_attn_sharedkv_fwd(
        q_flat.data_ptr(), T1, N1, D, dcode, 1 if layout_q == "TND" else 0, int(B), int(S), _lib.ptr(cu),
        skv.data_ptr(),
        ori_kv_dev.data_ptr(), ori_kv_dev.shape[0], ori_kv_dev.shape[1], ori_bt.data_ptr(), ori_bt.shape[1],
        _lib.ptr(cmp_kv_dev), cmp_kv_dev.shape[0] if cmp_kv_dev is not None else 0,
        cmp_kv_dev.shape[1] if cmp_kv_dev is not None else 0, _lib.ptr(cmp_bt),
        cmp_bt.shape[1] if cmp_bt is not None else 0,
        _lib.ptr(idx_dev), int(K), sinks_dev.data_ptr(), md.data_ptr(), float(softmax_scale), int(cmp_ratio_eff),
        int(ori_win_left), scenario, out_flat.data_ptr(), lse_flat.data_ptr(), st.num_sms, int(_stages) | flags,
        st.status.data_ptr(),
        ws.data_ptr(), ws.numel(), stream)
    if rc in (1, 2):
        raise ValueError(f"sparse_attn_sharedkv: {_lib.ERRORS[rc]}")
    _lib.check(rc, "sas_sparse_attn_sharedkv_fwd")

    if layout_q == "TND":
        o, l = out_flat, lse_flat
    else:
        o = out_flat.reshape(B, S, N1, D)
        l = lse_flat.reshape(B, S, N1)
    if return_softmax_lse:
        return o, l
    return o
