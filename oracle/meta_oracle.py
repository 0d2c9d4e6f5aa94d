"""TEST INFRASTRUCTURE ONLY: Python binding of the C scheduler restatement.

``sas_meta_oracle.c`` restates the reference ``metadata.py`` scheduler
(``sparse_attn_sharedkv_metadata``, metadata.py:1018-1086) in plain C. This
module compiles it with ``gcc`` into ``oracle/_build/libsas_meta_oracle.so``
(``build()``) and exposes ``metadata(...)`` with the reference's keyword
arguments, returning ``numpy.int32[1024]``. Only tests, the smoke check and
the bench's CPU arm use it, as the bit-exact checker of the GPU kernel.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "sas_meta_oracle.c")
_BUILD = os.path.join(_HERE, "_build")
_SO = os.path.join(_BUILD, "libsas_meta_oracle.so")
_lib = None

LAYOUT_Q = {"BSND": 0, "TND": 1, "BSH": 2}
LAYOUT_KV = {"PA_ND": 0, "TND": 1}


def build(force: bool = False) -> str:
    os.makedirs(_BUILD, exist_ok=True)
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(_SRC):
        subprocess.check_call(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-o", _SO, _SRC])
    return _SO


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.POINTER(ctypes.c_int64)
        I = ctypes.c_int64
        _lib.sas_meta_oracle.argtypes = [I, I, I, P, I, P, I, P, I, P, I, I, I, I, I, I, I, I, I, I, I, I, I, I,
                                         ctypes.POINTER(ctypes.c_int32)]
        _lib.sas_meta_oracle.restype = ctypes.c_int
    return _lib


def _arr(x):
    if x is None:
        return None, 0
    a = np.ascontiguousarray(np.asarray(x, dtype=np.int64).reshape(-1))
    if a.size == 0:
        return None, 0
    return a, a.size


def metadata(*, num_heads_q, num_heads_kv, head_dim, cu_seqlens_q=None, cu_seqlens_ori_kv=None,
             cu_seqlens_cmp_kv=None, seqused_q=None, seqused_kv=None, batch_size=0, max_seqlen_q=0,
             max_seqlen_kv=0, ori_topk=0, cmp_topk=0, cmp_ratio=-1, ori_mask_mode=4, cmp_mask_mode=3,
             ori_win_left=127, ori_win_right=0, layout_q="BSND", layout_kv="PA_ND", has_ori_kv=True,
             has_cmp_kv=True, aic_core_num=24, aiv_core_num=48, support_fd=False) -> np.ndarray:
    """The scheduler's int32[1024] output; ``support_fd`` runs the reference
    scheduler's flash-decode branches (its ``supportFd`` switch)."""
    lib = _load()
    keep = []

    def ptr(x):
        a, n = _arr(x)
        keep.append(a)
        if a is None:
            return None, 0
        return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), n

    cq, ncq = ptr(cu_seqlens_q)
    ck, nck = ptr(cu_seqlens_ori_kv)
    sq, nsq = ptr(seqused_q)
    sk, nsk = ptr(seqused_kv)
    out = np.zeros(1024, np.int32)
    rc = lib.sas_meta_oracle(
        int(num_heads_q), int(num_heads_kv), int(head_dim), cq, ncq, ck, nck, sq, nsq, sk, nsk,
        int(batch_size), int(max_seqlen_q), int(max_seqlen_kv), int(cmp_topk), int(cmp_ratio),
        int(ori_mask_mode), int(ori_win_left), LAYOUT_Q.get(layout_q, 3), LAYOUT_KV.get(layout_kv, 0),
        int(bool(has_cmp_kv)), int(aic_core_num), int(aiv_core_num), int(bool(support_fd)),
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    if rc != 0:
        raise RuntimeError(f"metadata oracle failed with status {rc}")
    return out
