"""B200-native sparse_attn_sharedkv (DeepSeek-V4 style shared-KV sparse attention).

Drop-in replacements for the reference entry points:

* ``sparse_attn_sharedkv`` (``api.py``) -- the fused forward;
* ``sparse_attn_sharedkv_metadata`` (``metadata.py``) -- the scheduler;

and the backward the reference documents but does not ship
(``sparse_attn_sharedkv_backward``, ``sparse_attn_sharedkv_train``).

Both run hand-written sm_100a kernels from ``libsas_b200.so`` (C ABI in
``include/sas_b200.h``). ``sharding`` holds the request-parallel and
head-sharded multi-GPU drivers; ``synth`` the seeded input generators.
"""

from .api import sparse_attn_sharedkv  # noqa: F401
from .backward import SparseAttnSharedkv, sparse_attn_sharedkv_backward, sparse_attn_sharedkv_train  # noqa: F401
from .metadata import SAS_META_SIZE, sparse_attn_sharedkv_metadata  # noqa: F401
from ._lib import check_device_status, device_status, reset_device_status  # noqa: F401

__all__ = [
    "sparse_attn_sharedkv",
    "sparse_attn_sharedkv_backward",
    "sparse_attn_sharedkv_train",
    "SparseAttnSharedkv",
    "sparse_attn_sharedkv_metadata",
    "SAS_META_SIZE",
    "check_device_status",
    "device_status",
    "reset_device_status",
]
