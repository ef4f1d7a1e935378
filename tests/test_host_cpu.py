"""Host-side behaviour of the Python mirror that needs no GPU: the reference's
NotImplementedError guards, argument validation, and no silent CPU fallback."""
import pytest
import torch

import tilelang_fa_v100 as fa
from tilelang_fa_v100 import _ext


def _qkv(dtype=torch.float16):
    g = torch.Generator().manual_seed(0)
    return [torch.randn(1, 8, 2, 64, generator=g).to(dtype) for _ in range(3)]


def test_exports_match_reference_api():
    assert set(fa.__all__) == {"tilelang_flash_attn_func", "tilelang_flash_attn_gpu",
                               "tilelang_paged_forward", "tilelang_decode_forward"}
    assert fa.tilelang_flash_attn_gpu is fa.tilelang_flash_attn_func
    assert fa.__version__ == "1.0.0"


@pytest.mark.parametrize("kw,msg", [(dict(dropout_p=0.1), "dropout"),
                                    (dict(alibi_slopes=torch.ones(2)), "alibi")])
def test_unsupported_features_raise_like_reference(kw, msg):
    q, k, v = _qkv()
    with pytest.raises(NotImplementedError, match=msg):
        fa.tilelang_flash_attn_func(q, k, v, **kw)


def test_softcap_is_accepted_and_still_needs_cuda():
    # softcap is honoured (the reference raises NotImplementedError for it): the call gets
    # past the guards and is refused only for its CPU tensors.
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="CUDA"):
        fa.tilelang_flash_attn_func(q, k, v, softcap=30.0)


def test_cpu_tensors_are_rejected_not_computed():
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="CUDA"):
        fa.tilelang_flash_attn_func(q, k, v, causal=True)


def test_paged_adapter_validates_cache_shape():
    q = torch.zeros(4, 4, 64, dtype=torch.float16)
    kc = torch.zeros(2, 16, 1, 64, dtype=torch.float16)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    sl = torch.tensor([4], dtype=torch.int32)
    qsl = torch.tensor([0, 4], dtype=torch.int32)
    pkl = torch.zeros(1, dtype=torch.int32)
    with pytest.raises(ValueError, match="block_size"):
        fa.tilelang_paged_forward(q, kc, kc, bt, sl, qsl, pkl, block_size=32)
    with pytest.raises(ValueError, match="query_start_loc"):
        fa.tilelang_paged_forward(q, kc, kc, bt, sl, qsl[:1], pkl)


def test_decode_adapter_validates_dtype():
    q = torch.zeros(1, 4, 64, dtype=torch.float16)
    kc = torch.zeros(2, 16, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="dtype"):
        fa.tilelang_decode_forward(q, kc, kc, torch.zeros(1, 2, dtype=torch.int32),
                                   torch.tensor([3], dtype=torch.int32))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_ext, "_lib", None)
    monkeypatch.setattr(_ext, "_LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not built"):
        _ext.load()


def test_backward_arity_matches_reference():
    # interface.py:56 of the reference returns 12 values (3 grads + 9 None)
    import inspect
    src = inspect.getsource(fa.interface.FlashAttnTileLangVFunc.backward)
    assert src.count("None") == 9
