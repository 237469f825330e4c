"""Group-wise Hadamard rotation (ConvRot), same API as the reference's
convrot.py (convrot.py:18-118).

``build_hadamard`` returns the normalised matrix exactly as the reference
builds it (callers serialise or inspect it).  The rotations themselves run in
the fused CUDA kernel: ``rotate_activation`` and ``rotate_weight`` identify
the matrix family from ``H`` and never perform a dense matmul.  Two families:

* "regular": the reference's H4 Kronecker powers (sizes 16, 64, 256);
* "sylvester": ``scipy.linalg.hadamard`` normalised the same way (sizes that
  are not powers of 4, e.g. 128, where no regular Hadamard exists).
"""
from __future__ import annotations

import torch

from . import library as kops  # the kernels as registered torch.library operators

_HADAMARD_CACHE: dict = {}
_H4 = [[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]]


def _int_matrix(size: int, kind: str) -> torch.Tensor:
    if kind == "regular":
        if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
            raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
        h4 = torch.tensor(_H4, dtype=torch.float32)
        h = h4
        while h.shape[0] < size:
            h = torch.kron(h, h4)
        return h
    if kind == "sylvester":
        if size < 2 or size & (size - 1):
            raise ValueError(f"Sylvester Hadamard size must be a power of 2, got {size}")
        h = torch.ones((1, 1), dtype=torch.float32)
        while h.shape[0] < size:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        return h
    raise ValueError(f"unknown Hadamard kind {kind!r}")


def build_hadamard(size: int, device="cpu", dtype: torch.dtype = torch.float32, kind: str = "regular") -> torch.Tensor:
    """Normalised Hadamard ``H_int / size**0.5`` (convrot.py:18-55).

    kind="regular" (default) is the reference's construction and rejects sizes
    that are not powers of 4, like the reference.  The returned tensor carries
    its family so ``rotate_*`` can dispatch to the kernel."""
    key = (size, str(device), dtype, kind)
    if key in _HADAMARD_CACHE:
        return _HADAMARD_CACHE[key]
    h = (_int_matrix(size, kind) / (size ** 0.5)).to(device=device, dtype=dtype)
    h._qlin_kind = kind
    _HADAMARD_CACHE[key] = h
    return h


def hadamard_kind(H: torch.Tensor) -> str:
    """Family of a normalised Hadamard matrix (by tag, else by inspection)."""
    kind = getattr(H, "_qlin_kind", None)
    if kind is not None:
        return kind
    g = H.shape[-1]
    sign = torch.sign(H.detach().float().cpu())
    for k in ("regular", "sylvester"):
        try:
            if torch.equal(sign, _int_matrix(g, k)):
                return k
        except ValueError:
            continue
    raise ValueError("H is neither a regular (H4 Kronecker) nor a Sylvester Hadamard matrix")


def rotate_activation(x: torch.Tensor, H: torch.Tensor, group_size: int) -> torch.Tensor:
    """x_rot = x @ blockdiag(H) (convrot.py:89-118); result in x.dtype."""
    if x.shape[-1] % group_size != 0:
        raise ValueError(f"features {x.shape[-1]} not divisible by group_size {group_size}")
    return kops.rotate(x, hadamard_kind(H), group_size)


def rotate_weight(weight: torch.Tensor, H: torch.Tensor, group_size: int) -> torch.Tensor:
    """W_rot = W @ blockdiag(H)^T (convrot.py:58-86); H is symmetric."""
    if weight.dim() != 2:
        raise ValueError("rotate_weight expects a 2-D weight")
    if weight.shape[1] % group_size != 0:
        raise ValueError(f"in_features {weight.shape[1]} not divisible by group_size {group_size}")
    return kops.rotate(weight, hadamard_kind(H), group_size)
