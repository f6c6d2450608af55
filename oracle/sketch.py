"""
Seeded random sketches of large gradient tensors, for golden fixtures.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). A fixture that must pin a
model's full parameter gradient to 1e-10 in float64 would store every element
(megabytes of incompressible doubles). Instead, tensors above ``FULL_LIMIT``
elements are stored as ``ROWS`` projections onto seeded Rademacher (+-1)
vectors: for any error e of a gradient g, the projections satisfy
E ||S e||^2 = ROWS ||e||^2 (Johnson-Lindenstrauss), so the relative error of
the sketch estimates the relative error of the tensor itself. The seed of each
tensor's sign matrix is the CRC32 of its name: generator and checker draw the
same matrix.
"""

from __future__ import annotations

import zlib

import torch

FULL_LIMIT = 4096
ROWS = 256


def _signs(name: str, numel: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    return torch.randint(0, 2, (ROWS, numel), generator=gen).to(torch.float64).mul_(2.0).sub_(1.0)


def sketch(name: str, t: torch.Tensor) -> torch.Tensor:
    """The full tensor (float64, flattened) when small, else its ROWS signed sums."""
    flat = t.detach().to(torch.float64).flatten().cpu()
    if flat.numel() <= FULL_LIMIT:
        return flat
    return _signs(name, flat.numel()) @ flat
