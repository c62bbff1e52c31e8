"""The C-ABI library loads, exports every symbol include/b200attn.h declares,
and its host-only logic behaves (no GPU needed for any of this)."""
import ctypes

import numpy as np
import pytest

import b200attn


def test_library_exports_every_declared_symbol():
    names = b200attn.declared_symbols()
    assert len(names) >= 15
    lib = b200attn.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []


def test_abi_version_and_status_strings():
    lib = b200attn.lib()
    assert lib.b2a_abi_version() == 1
    assert lib.b2a_status_string(b200attn.B2A_EINVAL) == b"B2A_EINVAL"
    assert lib.b2a_status_string(b200attn.B2A_EDEVICE) == b"B2A_EDEVICE"
    assert lib.b2a_status_string(99) == b"B2A_UNKNOWN"


def test_calls_with_null_context_are_rejected():
    lib = b200attn.lib()
    assert lib.b2a_decode(None, 0, 1, 0, None, None, None, None, None, 0, None, 1, 1, 1, 64, 16, 0.125, 0, 0.0, 0,
                          None, None, 0.0, None, None) == b200attn.B2A_EINVAL
    assert lib.b2a_mha(None, 0, 0, None, None, None, None, None, None, 1, 1, 1, 8, 0.3, 0, None) == \
        b200attn.B2A_EINVAL
    assert lib.b2a_set_decode_early_start(None, 1) == b200attn.B2A_EINVAL
    assert lib.b2a_set_workspace_limit(None, 0) == b200attn.B2A_EINVAL


def test_create_reports_missing_device_without_crashing():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        b200attn.Context(0)
    assert "B2A_ECUDA" in str(ei.value)


def test_partition_units_equal_counts_and_balance():
    rng = np.random.default_rng(3)
    cost = rng.integers(512, 8193, size=128).astype(np.int64) * 256
    for n_ranks in (1, 2, 4, 8):
        r = b200attn.partition_units(cost, n_ranks)
        counts = np.bincount(r, minlength=n_ranks)
        assert np.all(counts == 128 // n_ranks)
        loads = np.array([cost[r == k].sum() for k in range(n_ranks)])
        assert loads.max() / loads.mean() < 1.05


def test_partition_units_rejects_uneven_split():
    with pytest.raises(ValueError):
        b200attn.partition_units(np.ones(10, np.int64), 4)


def test_group_without_an_nccl_library_is_b2a_enccl(monkeypatch):
    """The multi-GPU group loads NCCL at run time; a missing library is an NCCL failure (B2A_ENCCL)
    reported before any device is touched."""
    monkeypatch.setenv("B2A_NCCL_LIBRARY", "/nonexistent/libnccl.so.2")
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        b200attn.Group([0])
    assert ei.value.status == b200attn.B2A_ENCCL
    assert "NCCL could not be loaded" in str(ei.value)


def test_group_with_a_bad_rank_count_is_b2a_enccl():
    """A clique of zero ranks is rejected by NCCL's own argument check (no device is touched)."""
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        b200attn.Group([])
    assert ei.value.status == b200attn.B2A_ENCCL
    assert "ncclCommInitAll(0 ranks)" in str(ei.value)


def test_catalog_backend_has_cuda_with_its_token():
    from b200attn.catalog import CatalogBackend
    assert [b.token() for b in CatalogBackend] == ["cpu", "directml", "warp", "auto", "cuda"]
    assert CatalogBackend.parse("cuda") is CatalogBackend.CUDA
    assert CatalogBackend.parse(" CUDA ") is CatalogBackend.CUDA
    with pytest.raises(ValueError):
        CatalogBackend.parse("metal")
