"""CPU: the C-ABI library builds for sm_100a, loads, and exports every entry
point declared in include/sas_b200.h; host-only entry points answer."""

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "sas_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sas_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "sas_metadata" in names and "sas_sparse_attn_sharedkv_fwd" in names


def test_library_exports_every_declared_symbol(sas_lib):
    missing = [n for n in _declared() if not hasattr(sas_lib, n)]
    assert not missing, missing


def test_host_only_entry_points(sas_lib):
    assert sas_lib.sas_version() >= 1
    a = sas_lib.sas_metadata_workspace_bytes(64, 24)
    b = sas_lib.sas_metadata_workspace_bytes(4096, 24)
    assert 0 < a < b
    w = sas_lib.sas_fwd_workspace_bytes(64, 64, 148)
    w2 = sas_lib.sas_fwd_workspace_bytes(64, 128, 148)
    assert w > 148 * 2 * 64 * 512 * 4 and w2 >= w - 4096


def test_library_is_sm100a_only():
    from dsv4_b200 import build

    assert "arch=compute_100a,code=sm_100a" in build.ARCH


def test_bench_fused_plan_threshold_matches_kernel():
    """bench.py counts launches per step from the fused-plan threshold; it must
    be the attention kernel's own (kFusedMaxT in csrc/sas_fwd.cu)."""
    import bench

    src = open(os.path.join(ROOT, "dsv4_b200", "csrc", "sas_fwd.cu")).read()
    m = re.search(r"constexpr int kFusedMaxT = (\d+);", src)
    assert m and int(m.group(1)) == bench.FUSED_PLAN_MAX_TOKENS
