"""ctypes binding of ``libsas_b200.so`` (declared in ``include/sas_b200.h``).

The product path has no fallback: if the shared library is missing or does
not load, every call raises. Workspace and status buffers are cached per
device as torch tensors; the library itself never allocates.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsas_b200.so")

SAS_OK = 0
STAGE_PLAN, STAGE_ATTENTION, STAGE_COMBINE, STAGE_ALL = 1, 2, 4, 7
FLAG_AFTER_METADATA = 8  # the preceding kernel on the stream is sas_metadata for the same call
OPT_RESCALE_THRESHOLD, OPT_TRACE_BUFFER, OPT_SPLIT_TOKENS, OPT_WAIT_LIMIT_NS, OPT_SCHED_SCAN_CAP = 1, 2, 3, 4, 5
ERRORS = {
    1: "invalid argument",
    2: "unsupported configuration",
    3: "CUDA error",
    4: "workspace too small",
    5: "scheduler row scan overran its cap",
    6: "request exceeds the fixed scratch of the allocation-free scheduler",
    7: "block-table entry outside the table or the pool (rows dropped)",
}
STATUS_BAD_BLOCK_ENTRY = 7
STATUS_TIMEOUT_BASE = 16

_lib = None
_lock = threading.Lock()

i32 = ctypes.c_int32
i64 = ctypes.c_int64
vp = ctypes.c_void_p
f32 = ctypes.c_float
sz = ctypes.c_size_t

EXPORTS = {
    "sas_version": ([], ctypes.c_int),
    "sas_metadata_workspace_bytes": ([i32, i32], sz),
    "sas_metadata": ([vp, i32, vp, i32, vp, i32, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32,
                      i32, i32, i32, vp, vp, vp, sz, vp], ctypes.c_int),
    "sas_metadata_fd": ([vp, i32, vp, i32, vp, i32, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32,
                         i32, i32, i32, i32, vp, vp, vp, sz, vp], ctypes.c_int),
    "sas_sparse_attn_sharedkv_fwd_gather": ([vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, i64, i32, vp, i32, vp,
                                             i64, i32, vp, i32, vp, i32, vp, vp, f32, i32, i32, i32, vp, vp, i32,
                                             i32, i32, i32, i32, vp, vp, sz, vp], ctypes.c_int),
    "sas_sparse_attn_sharedkv_bwd": ([vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, i64, i32, vp,
                                      i32, vp, i64, i32, vp, i32, vp, i32, vp, f32, i32, i32, i32, vp, vp, vp, vp,
                                      vp, vp], ctypes.c_int),
    "sas_bwd_cast": ([vp, vp, i64, i32, vp], ctypes.c_int),
    "sas_fwd_workspace_bytes": ([i32, i32, i32], sz),
    "sas_fwd_set_option": ([i32, ctypes.c_double, vp], ctypes.c_int),
    "sas_sparse_attn_sharedkv_fwd": ([vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, i64, i32, vp, i32, vp, i64,
                                      i32, vp, i32, vp, i32, vp, vp, f32, i32, i32, i32, vp, vp, i32, i32, vp, vp, sz, vp],
                                     ctypes.c_int),
}


def lib():
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m dsv4_b200.build` "
                        "(there is no CPU or fallback path)")
                h = ctypes.CDLL(LIB_PATH)
                for name, (args, res) in EXPORTS.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    if rc != SAS_OK:
        raise RuntimeError(f"{what} failed: {ERRORS.get(rc, rc)} (status {rc})")


class _DeviceState:
    def __init__(self, device: torch.device):
        self.device = device
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.ws = torch.empty(0, dtype=torch.uint8, device=device)
        self.meta_ws = torch.empty(0, dtype=torch.uint8, device=device)
        props = torch.cuda.get_device_properties(device)
        self.num_sms = props.multi_processor_count

    def workspace(self, nbytes: int) -> torch.Tensor:
        if self.ws.numel() < nbytes:
            # zeroed: the split-token counters in it start at zero and every
            # launch leaves them zero
            self.ws = torch.zeros(max(nbytes, 2 * self.ws.numel()), dtype=torch.uint8, device=self.device)
        return self.ws

    def meta_workspace(self, nbytes: int) -> torch.Tensor:
        """The scheduler's own scratch: it may run concurrently with an
        attention launch (SAS_FLAG_AFTER_METADATA), so it never shares the
        attention workspace."""
        if self.meta_ws.numel() < nbytes:
            self.meta_ws = torch.empty(max(nbytes, 2 * self.meta_ws.numel()), dtype=torch.uint8, device=self.device)
        return self.meta_ws


_states: Dict[int, _DeviceState] = {}


def state(device: torch.device) -> _DeviceState:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _states.get(idx)
    if st is None:
        st = _DeviceState(torch.device("cuda", idx))
        _states[idx] = st
    return st


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def device_status(device=None) -> int:
    """Read (synchronously) the sticky device status word; 0 = no device-side error."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(state(dev).status.item())


def check_device_status(device=None) -> None:
    code = device_status(device)
    if code != 0:
        if code >= 16:
            raise RuntimeError(f"device-side bounded wait {code - 16} ran out (status {code})")
        raise RuntimeError(f"device-side error: {ERRORS.get(code, code)} (status {code})")


def reset_device_status(device=None) -> None:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    state(dev).status.zero_()
