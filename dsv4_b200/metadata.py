"""SparseAttnSharedkvMetadata on the GPU (drop-in for the reference metadata.py).

``sparse_attn_sharedkv_metadata(**kw)`` takes the keyword set of the
reference (``sparse_attn_sharedkv_tilelang/metadata.py:1018-1045``) and
returns the same ``int32[SAS_META_SIZE]`` tensor, computed by the
single-CTA scheduler kernel in ``csrc/sas_meta.cu``. Differences from the
reference, by design:

* the result lives on a CUDA device (``device`` argument, default the
  current device) and is produced without a host round trip; pass
  ``device="cpu"`` to get a host copy, as the reference returns by default;
* ``max_seqlen_q`` / ``max_seqlen_kv`` are only read where the reference
  reads them (no ``cu_seqlens_q`` / ``seqused_kv`` given), so callers need
  not compute them on the host.

The module keeps the reference's layout constants, which callers index the
result with (metadata.py:38-81).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

AIC_CORE_NUM = 36
AIV_CORE_NUM = 72
SAS_META_SIZE = 1024

FA_METADATA_SIZE = 8
FD_METADATA_SIZE = 8

FA_CORE_ENABLE_INDEX = 0
FA_BN2_START_INDEX = 1
FA_M_START_INDEX = 2
FA_S2_START_INDEX = 3
FA_BN2_END_INDEX = 4
FA_M_END_INDEX = 5
FA_S2_END_INDEX = 6
FA_FIRST_FD_DATA_WORKSPACE_IDX_INDEX = 7

FD_CORE_ENABLE_INDEX = 0
FD_BN2_IDX_INDEX = 1
FD_M_IDX_INDEX = 2
FD_WORKSPACE_IDX_INDEX = 3
FD_WORKSPACE_NUM_INDEX = 4
FD_M_START_INDEX = 5
FD_M_NUM_INDEX = 6

WIN_NORMAL_BLOCK = 0
WIN_TAIL_BLOCK = 1
CMP_NORMAL_BLOCK = 2
CMP_TAIL_BLOCK = 3
BLOCK_MAX_TYPE = 4

FA_TOLERANCE_RATIO = 2


class SparseMode:
    DEFAULT_MASK = 0
    ALL_MASK = 1
    LEFT_UP_CAUSAL = 2
    RIGHT_DOWN_CAUSAL = 3
    BAND = 4
    SPARSE_BUTT = 5


_LAYOUT_Q = {"BSND": 0, "TND": 1, "BSH": 2}
_LAYOUT_KV = {"PA_ND": 0, "TND": 1}


def _dev_i32(t, device):
    """Device int32 view of an optional length tensor (None or empty -> None)."""
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    if t.numel() == 0:
        return None
    return t.to(device=device, dtype=torch.int32).contiguous().reshape(-1)


def sparse_attn_sharedkv_metadata(
    *,
    num_heads_q: int,
    num_heads_kv: int,
    head_dim: int,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    cu_seqlens_ori_kv: Optional[torch.Tensor] = None,
    cu_seqlens_cmp_kv: Optional[torch.Tensor] = None,
    seqused_q: Optional[torch.Tensor] = None,
    seqused_kv: Optional[torch.Tensor] = None,
    batch_size: int = 0,
    max_seqlen_q: int = 0,
    max_seqlen_kv: int = 0,
    ori_topk: int = 0,
    cmp_topk: int = 0,
    cmp_ratio: int = -1,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "BSND",
    layout_kv: str = "PA_ND",
    has_ori_kv: bool = True,
    has_cmp_kv: bool = True,
    aic_core_num: int = 24,
    aiv_core_num: int = 48,
    device: Optional[str] = None,
    out: Optional[torch.Tensor] = None,
    support_fd: bool = False,
) -> torch.Tensor:
    """Scheduler output ``int32[1024]`` (faMetadata[36][8] then fdMetadata[72][8]).

    The schedule is always computed on a CUDA device. As in the reference
    (metadata.py:1083-1086) the result is a CPU tensor unless ``device`` names
    a CUDA device, in which case it stays there (no host synchronisation).
    ``out`` may supply a preallocated device ``int32[1024]`` buffer (e.g. for
    CUDA-graph capture); it is filled and returned on its device.
    ``support_fd=True`` computes the flash-decode schedule: the reference
    scheduler with its ``supportFd`` switch on (metadata.py:323-325, left
    False by the reference), whose cores may end inside a row and whose
    ``fdMetadata`` rows spread the cut rows over ``aiv_core_num`` vector cores.
    """
    del cu_seqlens_cmp_kv, ori_topk, cmp_mask_mode, ori_win_right, has_ori_kv
    want_cpu = out is None and (device is None or torch.device(device).type == "cpu")
    if out is not None:
        dev = out.device
    elif device is not None and not want_cpu:
        dev = torch.device(device)
    else:
        dev = None
        for t in (seqused_kv, cu_seqlens_q, seqused_q, cu_seqlens_ori_kv):
            if isinstance(t, torch.Tensor) and t.is_cuda:
                dev = t.device
                break
        if dev is None:
            dev = torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise RuntimeError("sparse_attn_sharedkv_metadata runs on a CUDA device")
    cu_q = _dev_i32(cu_seqlens_q, dev)
    cu_kv = _dev_i32(cu_seqlens_ori_kv, dev)
    sq = _dev_i32(seqused_q, dev)
    skv = _dev_i32(seqused_kv, dev)
    lq = _LAYOUT_Q.get(layout_q, 3)
    lkv = _LAYOUT_KV.get(layout_kv, 0)
    B = batch_size
    if sq is not None:
        B = sq.numel()
    elif layout_q == "TND" and cu_q is not None:
        B = cu_q.numel() - 1
    if num_heads_kv == 0 or num_heads_q // num_heads_kv == 0:
        raise ZeroDivisionError("num_heads_q // num_heads_kv must be positive")
    lib = _lib.lib()
    st = _lib.state(dev)
    nbytes = lib.sas_metadata_workspace_bytes(max(int(B), 1), int(aic_core_num))
    ws = st.meta_workspace(nbytes)
    if out is None:
        out = torch.empty(SAS_META_SIZE, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def n(t):
        return 0 if t is None else t.numel()

    args = (_lib.ptr(cu_q), n(cu_q), _lib.ptr(cu_kv), n(cu_kv), _lib.ptr(sq), n(sq), _lib.ptr(skv), n(skv),
            int(batch_size), int(max_seqlen_q), int(max_seqlen_kv), int(num_heads_q), int(num_heads_kv),
            int(head_dim), int(cmp_topk), int(cmp_ratio), int(ori_mask_mode), int(ori_win_left), lq, lkv,
            int(bool(has_cmp_kv)), int(aic_core_num))
    tail = (out.data_ptr(), st.status.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    if support_fd:
        rc = lib.sas_metadata_fd(*args, int(aiv_core_num), *tail)
    else:
        rc = lib.sas_metadata(*args, *tail)
    if rc == 1:
        raise ValueError("sparse_attn_sharedkv_metadata: invalid arguments (array lengths / heads / ratio)")
    _lib.check(rc, "sas_metadata")
    if want_cpu:
        return out.cpu()
    return out
