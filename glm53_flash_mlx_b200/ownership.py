"""Tensor storage lifetime contracts for persistent runtime structures.

Counterpart of glm53_flash_mlx/ownership.py:13-198 over ``torch.Tensor``:
the same enums, lease types, errors and constructors.  A resident structure
(the packed expert bank) may only retain owned or borrowed-stable storage;
borrowed-ephemeral storage (staging buffers, scratch) must be copied with
``materialize_owned`` before it crosses a resident boundary.
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
    """Raised when a storage lifetime cannot satisfy a resident boundary."""


@dataclass(frozen=True)
class TensorLease:
    value: torch.Tensor
    ownership: TensorOwnership
    layout: TensorLayout = TensorLayout.UNKNOWN
    owner: object | None = None

    def __post_init__(self) -> None:
        if self.ownership is TensorOwnership.BORROWED_STABLE and self.owner is None:
            raise TensorOwnershipError(
                "borrowed-stable storage requires an owner retained for its lifetime"
            )


@dataclass(frozen=True)
class ResidentTensor:
    value: torch.Tensor
    ownership: TensorOwnership
    layout: TensorLayout
    owner: object | None = None

    def __post_init__(self) -> None:
        if self.ownership is TensorOwnership.BORROWED_EPHEMERAL:
            raise TensorOwnershipError(
                "resident structures cannot retain borrowed-ephemeral storage"
            )
        if self.layout is not TensorLayout.ROW_MAJOR_CONTIGUOUS:
            raise TensorOwnershipError(
                "resident tensors require the row-major contiguous layout contract"
            )
        if self.ownership is TensorOwnership.BORROWED_STABLE and self.owner is None:
            raise TensorOwnershipError(
                "borrowed-stable resident storage must retain its owner"
            )


def owned_tensor(value: torch.Tensor, *, layout: TensorLayout = TensorLayout.UNKNOWN) -> TensorLease:
    """Declare storage created and lifetime-controlled by this runtime."""
    return TensorLease(value, TensorOwnership.OWNED, layout)


def borrowed_stable_tensor(
    value: torch.Tensor, *, owner: object, layout: TensorLayout = TensorLayout.UNKNOWN
) -> TensorLease:
    """Borrow storage whose owner is retained for the resident lifetime."""
    return TensorLease(value, TensorOwnership.BORROWED_STABLE, layout, owner)


def borrowed_ephemeral_tensor(
    value: torch.Tensor, *, owner: object | None = None, layout: TensorLayout = TensorLayout.UNKNOWN
) -> TensorLease:
    """Borrow staging/scratch storage that may be reused after the load step."""
    return TensorLease(value, TensorOwnership.BORROWED_EPHEMERAL, layout, owner)


def _row_major(value: torch.Tensor) -> torch.Tensor:
    return value.contiguous()


def _owned_copy(value: torch.Tensor) -> torch.Tensor:
    # clone() allocates storage of its own: later writes to the borrowed
    # source (or its owner) cannot reach the copy.
    return value.contiguous().clone(memory_format=torch.contiguous_format)


def require_resident(lease: TensorLease | ResidentTensor) -> ResidentTensor:
    """Validate a resident boundary without silently copying ephemeral data."""
    if isinstance(lease, ResidentTensor):
        return lease
    if not isinstance(lease, TensorLease):
        raise TypeError(
            "resident tensors require an explicit TensorLease; bare arrays "
            "have no storage lifetime contract"
        )
    if lease.ownership is TensorOwnership.BORROWED_EPHEMERAL:
        raise TensorOwnershipError(
            "borrowed-ephemeral storage must call materialize_owned() before "
            "crossing a resident boundary"
        )
    return ResidentTensor(
        _row_major(lease.value), lease.ownership, TensorLayout.ROW_MAJOR_CONTIGUOUS, lease.owner
    )


def materialize_owned(lease: TensorLease | ResidentTensor) -> ResidentTensor:
    """Create storage independent of every borrowed source and source owner."""
    if isinstance(lease, ResidentTensor) and lease.ownership is TensorOwnership.OWNED:
        return lease
    if not isinstance(lease, (TensorLease, ResidentTensor)):
        raise TypeError("materialize_owned() requires an explicit storage contract")
    if lease.ownership is TensorOwnership.OWNED:
        value = _row_major(lease.value)
    else:
        value = _owned_copy(lease.value)
    return ResidentTensor(value, TensorOwnership.OWNED, TensorLayout.ROW_MAJOR_CONTIGUOUS)


def resident_concatenate(leases: Iterable[TensorLease | ResidentTensor], *, axis: int) -> ResidentTensor:
    """Build an owned fusion from non-ephemeral source tensors."""
    residents = [require_resident(lease) for lease in leases]
    if not residents:
        raise ValueError("cannot concatenate an empty resident tensor list")
    value = torch.cat([item.value for item in residents], dim=axis).contiguous()
    return ResidentTensor(value, TensorOwnership.OWNED, TensorLayout.ROW_MAJOR_CONTIGUOUS)


def storage_descriptor(value: TensorLease | ResidentTensor) -> dict[str, str]:
    return {"ownership": value.ownership.value, "layout": value.layout.value}
