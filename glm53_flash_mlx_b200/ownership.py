"""Storage lifetime contract for tensors kept by long-lived structures.

The drop-in surface of glm53_flash_mlx/ownership.py:13-198 over
``torch.Tensor``: the enum values, the lease / resident dataclasses and their
fields, the exception types, the constructor names and the message fragments
the reference's tests match ("materialize_owned", "explicit TensorLease",
"requires an owner") are interface and kept.  The rule: a structure that
outlives a load step (the packed expert bank) keeps only storage it owns or
storage borrowed from an owner it keeps alive; staging and scratch storage
(borrowed-ephemeral) has to be copied into owned storage first.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Iterable

import torch


class TensorOwnership(str, Enum):
    OWNED = "owned"
    BORROWED_STABLE = "borrowed-stable"
    BORROWED_EPHEMERAL = "borrowed-ephemeral"


class TensorLayout(str, Enum):
    UNKNOWN = "unknown"
    ROW_MAJOR_CONTIGUOUS = "row-major-contiguous"


class TensorOwnershipError(ValueError):
    """A tensor's lifetime does not allow it to be kept where it was offered."""


@dataclass(frozen=True)
class TensorLease:
    """A tensor offered together with who owns its storage."""

    value: torch.Tensor
    ownership: TensorOwnership
    layout: TensorLayout = TensorLayout.UNKNOWN
    owner: object | None = None

    def __post_init__(self) -> None:
        if self.ownership is TensorOwnership.BORROWED_STABLE and self.owner is None:
            raise TensorOwnershipError("a borrowed-stable lease requires an owner to keep alive with it")


@dataclass(frozen=True)
class ResidentTensor:
    """A tensor accepted into a long-lived structure: owned or borrowed with
    its owner, row-major contiguous."""

    value: torch.Tensor
    ownership: TensorOwnership
    layout: TensorLayout
    owner: object | None = None

    def __post_init__(self) -> None:
        if self.ownership is TensorOwnership.BORROWED_EPHEMERAL:
            raise TensorOwnershipError("ephemeral (borrowed-ephemeral) storage cannot be kept resident")
        if self.layout is not TensorLayout.ROW_MAJOR_CONTIGUOUS:
            raise TensorOwnershipError("a resident tensor must be declared row-major contiguous")
        if self.ownership is TensorOwnership.BORROWED_STABLE and self.owner is None:
            raise TensorOwnershipError("a borrowed-stable resident tensor requires an owner to keep alive")


def owned_tensor(value: torch.Tensor, *, layout: TensorLayout = TensorLayout.UNKNOWN) -> TensorLease:
    """Lease of storage this runtime allocated and frees."""
    return TensorLease(value, TensorOwnership.OWNED, layout)


def borrowed_stable_tensor(
    value: torch.Tensor, *, owner: object, layout: TensorLayout = TensorLayout.UNKNOWN
) -> TensorLease:
    """Lease of storage owned by `owner`, which the keeper holds as long as it
    keeps the tensor."""
    return TensorLease(value, TensorOwnership.BORROWED_STABLE, layout, owner)


def borrowed_ephemeral_tensor(
    value: torch.Tensor, *, owner: object | None = None, layout: TensorLayout = TensorLayout.UNKNOWN
) -> TensorLease:
    """Lease of storage that its owner may overwrite once the current step is
    done (a staging or scratch buffer)."""
    return TensorLease(value, TensorOwnership.BORROWED_EPHEMERAL, layout, owner)


def _contiguous(value: torch.Tensor) -> torch.Tensor:
    return value.contiguous()


def _private_copy(value: torch.Tensor) -> torch.Tensor:
    # a fresh allocation: nothing written to the source afterwards reaches it
    return value.contiguous().clone(memory_format=torch.contiguous_format)


def require_resident(lease: TensorLease | ResidentTensor) -> ResidentTensor:
    """Accept a lease for keeping, or refuse it; never copies behind the
    caller's back (an ephemeral lease is refused, not copied)."""
    if isinstance(lease, ResidentTensor):
        return lease
    if not isinstance(lease, TensorLease):
        raise TypeError("keeping a tensor needs an explicit TensorLease: a bare tensor states no owner or lifetime")
    if lease.ownership is TensorOwnership.BORROWED_EPHEMERAL:
        raise TensorOwnershipError("ephemeral storage is refused here; copy it with materialize_owned() first")
    return ResidentTensor(_contiguous(lease.value), lease.ownership, TensorLayout.ROW_MAJOR_CONTIGUOUS, lease.owner)


def materialize_owned(lease: TensorLease | ResidentTensor) -> ResidentTensor:
    """An owned resident tensor: owned storage as it is (made contiguous),
    borrowed storage copied into a private allocation."""
    if isinstance(lease, ResidentTensor) and lease.ownership is TensorOwnership.OWNED:
        return lease
    if not isinstance(lease, (TensorLease, ResidentTensor)):
        raise TypeError("materialize_owned() takes a TensorLease or ResidentTensor, not a bare tensor")
    if lease.ownership is TensorOwnership.OWNED:
        value = _contiguous(lease.value)
    else:
        value = _private_copy(lease.value)
    return ResidentTensor(value, TensorOwnership.OWNED, TensorLayout.ROW_MAJOR_CONTIGUOUS)


def resident_concatenate(leases: Iterable[TensorLease | ResidentTensor], *, axis: int) -> ResidentTensor:
    """Concatenate keepable leases along `axis` into one owned tensor."""
    residents = [require_resident(lease) for lease in leases]
    if not residents:
        raise ValueError("resident_concatenate() needs at least one tensor")
    value = torch.cat([item.value for item in residents], dim=axis).contiguous()
    return ResidentTensor(value, TensorOwnership.OWNED, TensorLayout.ROW_MAJOR_CONTIGUOUS)


def storage_descriptor(value: TensorLease | ResidentTensor) -> dict[str, str]:
    """The lease's contract as strings (the bank's ``storage_contracts``)."""
    return {"ownership": value.ownership.value, "layout": value.layout.value}
