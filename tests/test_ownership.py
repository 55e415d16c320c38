"""Storage-lifetime contract (mirrors the reference's tests/test_tensor_ownership.py
over torch tensors; CPU only)."""

import gc

import numpy as np
import pytest
import torch

from glm53_flash_mlx_b200.ownership import (
    TensorLayout,
    TensorOwnership,
    TensorOwnershipError,
    borrowed_ephemeral_tensor,
    borrowed_stable_tensor,
    materialize_owned,
    owned_tensor,
    require_resident,
    resident_concatenate,
    storage_descriptor,
)


def test_row_contiguous_does_not_promote_ephemeral_storage_to_resident():
    staging = np.arange(64, dtype=np.float32).reshape(8, 8)
    lease = borrowed_ephemeral_tensor(torch.from_numpy(staging), owner=staging,
                                      layout=TensorLayout.ROW_MAJOR_CONTIGUOUS)
    with pytest.raises(TensorOwnershipError, match="materialize_owned"):
        require_resident(lease)
    resident = materialize_owned(lease)
    assert storage_descriptor(resident) == {"ownership": "owned", "layout": "row-major-contiguous"}
    expected = staging.copy()
    staging.fill(-91.0)
    assert np.array_equal(resident.value.numpy(), expected)


def test_layout_and_ownership_contracts_are_independent():
    wide = torch.arange(8 * 16, dtype=torch.float32).reshape(8, 16)
    strided = wide[:, 1::2]
    resident = require_resident(owned_tensor(strided))
    assert resident.ownership is TensorOwnership.OWNED
    assert resident.layout is TensorLayout.ROW_MAJOR_CONTIGUOUS
    assert resident.value.is_contiguous()
    assert torch.equal(resident.value, strided.contiguous())
    with pytest.raises(TypeError, match="explicit TensorLease"):
        require_resident(strided.contiguous())


def test_reusable_staging_views_cannot_corrupt_resident_fused_projection():
    staging = np.empty((3, 32), dtype=np.float32)
    q_expected = np.arange(staging.size, dtype=np.float32).reshape(staging.shape)
    staging[...] = q_expected
    unsafe_q = torch.from_numpy(staging)
    q = materialize_owned(borrowed_ephemeral_tensor(unsafe_q, owner=staging,
                                                    layout=TensorLayout.ROW_MAJOR_CONTIGUOUS))
    kv_expected = (q_expected * -0.25) + 17.0
    staging[...] = kv_expected
    kv = materialize_owned(borrowed_ephemeral_tensor(torch.from_numpy(staging), owner=staging,
                                                     layout=TensorLayout.ROW_MAJOR_CONTIGUOUS))
    # the external failure mode: an unowned view observes the reuse
    assert np.array_equal(unsafe_q.numpy(), kv_expected)
    fused = resident_concatenate([owned_tensor(q.value, layout=q.layout), owned_tensor(kv.value, layout=kv.layout)],
                                 axis=0)
    expected = np.concatenate([q_expected, kv_expected], axis=0)
    staging.fill(12345.0)
    del unsafe_q, staging
    gc.collect()
    assert np.array_equal(q.value.numpy(), q_expected)
    assert np.array_equal(kv.value.numpy(), kv_expected)
    assert np.array_equal(fused.value.numpy(), expected)


def test_borrowed_stable_requires_owner_and_bank_keeps_it():
    from glm53_flash_mlx_b200.packed import PackedFP8ExpertBank

    with pytest.raises(TensorOwnershipError):
        borrowed_stable_tensor(torch.zeros(2), owner=None)
    owner = object()
    gu = torch.zeros((2, 256, 128), dtype=torch.uint8)
    gus = torch.ones((2, 2, 1), dtype=torch.float32)
    dw = torch.zeros((2, 128, 128), dtype=torch.uint8)
    ds = torch.ones((2, 1, 1), dtype=torch.float32)
    layout = TensorLayout.ROW_MAJOR_CONTIGUOUS
    bank = PackedFP8ExpertBank(borrowed_stable_tensor(gu, owner=owner, layout=layout), owned_tensor(gus),
                               owned_tensor(dw), owned_tensor(ds), intermediate_size=128)
    assert bank.storage_contracts["gate_up_weight"] == {"ownership": "borrowed-stable",
                                                        "layout": "row-major-contiguous"}
    assert owner in bank._storage_owners
    with pytest.raises(TensorOwnershipError):
        PackedFP8ExpertBank(borrowed_ephemeral_tensor(gu), owned_tensor(gus), owned_tensor(dw), owned_tensor(ds),
                            intermediate_size=128)
    with pytest.raises(TypeError):
        PackedFP8ExpertBank(gu, owned_tensor(gus), owned_tensor(dw), owned_tensor(ds), intermediate_size=128)


def test_packed_bank_owns_reusable_staging_weights():
    from glm53_flash_mlx_b200.fp8 import DirectFP8Expert
    from glm53_flash_mlx_b200.packed import PackedFP8ExpertBank

    experts = [DirectFP8Expert(128, 128, 3.0) for _ in range(4)]
    staging = torch.zeros((128, 128), dtype=torch.uint8)
    for i, e in enumerate(experts):
        staging.fill_(i + 1)
        e.gate_proj.weight = staging.clone()
        e.up_proj.weight = staging.clone() + 10
        e.down_proj.weight = staging.clone() + 20
    bank = PackedFP8ExpertBank.pack(experts)
    staging.fill_(99)
    for i, e in enumerate(experts):
        e.gate_proj.weight.fill_(0)
        assert int(bank.gate_up_weight[i, 0, 0]) == i + 1
        assert int(bank.gate_up_weight[i, 128, 0]) == i + 11
        assert int(bank.down_weight[i, 0, 0]) == i + 21
    assert all(v == {"ownership": "owned", "layout": "row-major-contiguous"} for v in bank.storage_contracts.values())
