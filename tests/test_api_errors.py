"""Host-side argument checks of ``sparse_attn_sharedkv`` (CPU, no GPU).

The reference raises ``AssertionError`` for unsupported modes
(api.py:187-191), ``ValueError`` for shapes and dtypes (api.py:51-56,
279-282) and requires ``metadata.numel() == 1024`` (api.py:362-364). All of
these are checked before the device is touched, so they run here; a
well-formed call with CPU tensors then fails loudly (there is no CPU path).
"""

import pytest

torch = pytest.importorskip("torch")


def _args(N1=64, D=512, N2=1, T=2, K=128, dtype=torch.bfloat16):
    q = torch.zeros(T, N1, D, dtype=dtype)
    kv = torch.zeros(4, 128, N2, D, dtype=dtype)
    return dict(
        q=q, ori_kv=kv, cmp_kv=kv.clone(), cmp_sparse_indices=torch.zeros(T, N2, K, dtype=torch.int32),
        ori_block_table=torch.zeros(2, 2, dtype=torch.int32), cmp_block_table=torch.zeros(2, 2, dtype=torch.int32),
        cu_seqlens_q=torch.tensor([0, 1, 2], dtype=torch.int32), seqused_kv=torch.tensor([200, 300], dtype=torch.int32),
        sinks=torch.zeros(N1), softmax_scale=D ** -0.5, cmp_ratio=4)


def _call(**over):
    from dsv4_b200 import sparse_attn_sharedkv

    kw = _args(**{k: over.pop(k) for k in ("N1", "D", "N2", "K", "dtype") if k in over})
    kw.update(over)
    q = kw.pop("q")
    return sparse_attn_sharedkv(q, **kw)


@pytest.mark.parametrize("over", [dict(N1=12), dict(N1=0), dict(D=256), dict(N2=2), dict(dtype=torch.float32)],
                         ids=["N1%8", "N1=0", "D256", "N2=2", "fp32"])
def test_shape_and_dtype_value_errors(over):
    with pytest.raises(ValueError):
        _call(**over)


@pytest.mark.parametrize("over", [
    dict(ori_mask_mode=3), dict(cmp_mask_mode=1), dict(ori_win_right=1), dict(layout_kv="TND"),
    dict(layout_q="BSH"), dict(metadata=torch.zeros(512, dtype=torch.int32)), dict(topk_cmp=64),
], ids=["ori_mask_mode", "cmp_mask_mode", "win_right", "layout_kv", "layout_q", "metadata_numel", "topk_mismatch"])
def test_unsupported_modes_assert(over):
    with pytest.raises(AssertionError):
        _call(**over)


def test_tnd_needs_cu_seqlens():
    with pytest.raises(AssertionError):
        _call(cu_seqlens_q=None)


def test_cpu_tensors_have_no_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        _call()
