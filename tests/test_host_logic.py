"""Host-side logic of the Python entry points that needs no GPU."""
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import ops


def test_slot_view_of_the_reference_pool_is_a_view():
    pool = torch.zeros(5, 64, 512, dtype=torch.bfloat16)
    v = ops._slot_view(pool, 512, "ckv_cache")
    assert v.shape == (320, 512) and v.data_ptr() == pool.data_ptr()


def test_slot_view_of_a_concatenated_cache_keeps_its_slot_stride():
    cat = torch.zeros(3, 64, 576, dtype=torch.bfloat16)
    ckv = ops._slot_view(cat[..., :512], 512, "ckv_cache")
    kpe = ops._slot_view(cat[..., 512:], 64, "kpe_cache")
    assert ckv.shape == (192, 512) and ckv.stride() == (576, 1)
    assert kpe.shape == (192, 64) and kpe.stride() == (576, 1)
    assert kpe.data_ptr() == cat.data_ptr() + 512 * 2


def test_slot_view_refuses_to_copy_a_pool():
    pool = torch.zeros(4, 64, 512, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="unit inner stride"):
        ops._slot_view(pool.transpose(1, 2), 64, "ckv_cache")
    with pytest.raises(ValueError, match="uniform slot table"):
        ops._slot_view(pool[::2, :32], 512, "ckv_cache")  # pages not evenly spaced as slots
