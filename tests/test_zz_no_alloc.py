"""GPU: the allocation-free scheduler entry point, through the C ABI.

``sas_metadata_noalloc`` serves callers that cannot allocate device memory
when they need a schedule (code inside an allocator or teardown path, plugins
whose host owns all device memory, loops that must not synchronise). It keeps
its scratch in a fixed array inside the library instead of a caller
workspace. This file checks, over two calls in a row, that it produces
exactly what ``sas_metadata`` (with a caller workspace) produces: a decode
batch, and a 3000-request batch large enough that the per-request arrays
live in the fixed scratch rather than in shared memory. It also checks that
a batch beyond its limit is refused. It is named so pytest collects it last.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SAS_ERR_NOALLOC_LIMIT = 6
i32 = ctypes.c_int32
vp = ctypes.c_void_p
ARGS = [vp, i32, vp, i32, vp, i32, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32,
        vp, vp]


@pytest.fixture(scope="module")
def lib():
    from dsv4_b200 import build, _lib

    build.build()
    h = _lib.lib()
    h.sas_metadata_noalloc.argtypes = ARGS + [vp]
    h.sas_metadata_noalloc.restype = ctypes.c_int
    return h


def _case(B, q_max, kv_max, seed):
    rng = np.random.default_rng(seed)
    ql = rng.integers(1, q_max + 1, size=B)
    kv = np.maximum(rng.integers(1, kv_max, size=B), ql)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(ql)]), dtype=torch.int32, device="cuda")
    skv = torch.tensor(kv, dtype=torch.int32, device="cuda")
    return cu, skv


def _common(cu, skv, B):
    # cu_seqlens_q, -, -, seqused_kv, batch, max_q, max_kv, H, Hkv, D, topk, ratio, mask, win, TND, PA_ND, cmp, cores
    return [cu.data_ptr(), cu.numel(), None, 0, None, 0, skv.data_ptr(), skv.numel(), B, 0, 0, 64, 1, 512, 512, 4, 4,
            127, 1, 0, 1, 24]


@pytest.mark.parametrize("B,q_max,kv_max", [(64, 1, 65536), (3000, 2, 131072)])
def test_noalloc_matches_workspace_entry_point(lib, B, q_max, kv_max):
    cu, skv = _case(B, q_max, kv_max, seed=B)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_bytes = lib.sas_metadata_workspace_bytes(B, 24)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ref = torch.full((1024,), -7, dtype=torch.int32, device="cuda")
    rc = lib.sas_metadata(*_common(cu, skv, B), ref.data_ptr(), status.data_ptr(), ws.data_ptr(), ws_bytes, stream)
    assert rc == 0
    for call in range(2):
        out = torch.full((1024,), -7, dtype=torch.int32, device="cuda")
        rc = lib.sas_metadata_noalloc(*_common(cu, skv, B), out.data_ptr(), status.data_ptr(), stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(out, ref), f"call {call} differs from sas_metadata"
    assert int(ref[:288].view(36, 8)[:, 0].sum().item()) >= 1


def test_noalloc_rejects_batches_beyond_its_scratch(lib):
    B = 5000
    cu, skv = _case(B, 1, 1000, seed=1)
    out = torch.zeros(1024, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sas_metadata_noalloc(*_common(cu, skv, B), out.data_ptr(), status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == SAS_ERR_NOALLOC_LIMIT
