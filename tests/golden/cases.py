"""Seeded inputs shared by make_golden.py and the tests.

Fixtures whose inputs are large store only a SHA-256 digest of them; the
tests rebuild the inputs with these functions (torch's CPU generator) and
check the digest before comparing outputs.
"""

from __future__ import annotations

import torch


def sphere_cloud(n: int, seed: int) -> torch.Tensor:
    """BASELINE config 3's input: a unit sphere with N(0, 0.01) radial jitter."""
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(1, n, 3, generator=g)
    p = p / p.norm(dim=-1, keepdim=True)
    return p * (1 + 0.01 * torch.randn(1, n, 1, generator=g))


def nd_cloud_pair(B: int, P: int, Q: int, D: int, seed: int, lattice: bool = False):
    """Inputs of the feature-space Chamfer fixtures (chamfer_nd.npz)."""
    g = torch.Generator().manual_seed(seed)
    if lattice:
        return (torch.randint(0, 3, (B, P, D), generator=g).float(),
                torch.randint(0, 3, (B, Q, D), generator=g).float())
    return torch.randn(B, P, D, generator=g), torch.randn(B, Q, D, generator=g)


ND_CASES = {  # name: (B, P, Q, D, seed, (x_lengths, y_lengths) or None)
    "d1": (2, 700, 1100, 1, 901, None),
    "d2_ragged": (3, 900, 650, 2, 902, ([900, 513, 1], [650, 2, 600])),
    "d5": (2, 1030, 777, 5, 903, None),
    "d64": (1, 300, 260, 64, 904, None),
    "d100": (1, 280, 200, 100, 905, None),
    "d8_lattice": (2, 256, 300, 8, 906, None),
}
