"""Code tables of the NF4 format (host constants, built once).

* ``nf4_code()``: the 16 NormalFloat-4 values of QLoRA (Dettmers et al., 2023):
  N(0,1) quantiles over 8 positive and 7 negative equal-probability ranges with
  one shared zero, normalised to [-1, 1].
* ``dynamic_map()``: the signed 8-bit dynamic-tree map ("8-bit Optimizers via
  Block-wise Quantization", Dettmers et al., 2022) used for the double
  quantisation of the NF4 absmax vector: for exponent level i in 0..6 the
  interval [0.1, 1] split into 2^i equal parts, midpoints scaled by 10^(i-6),
  both signs, plus 0 and 1.

These are the ``{key}_nf4_code`` / ``{key}_nf4_ncode`` buffers the reference
stores next to NF4 weights (experts.py:1028-1031).  Kernels always read the
tables from the buffers, so artifacts carrying other tables decode correctly.
"""

from __future__ import annotations

import functools
from statistics import NormalDist

import torch


@functools.lru_cache(maxsize=None)
def _nf4_values() -> tuple[float, ...]:
    inv = NormalDist().inv_cdf
    offset = 0.9677083

    def lin(a, b, n):
        return [a + (b - a) * i / (n - 1) for i in range(n)]

    pos = [inv(p) for p in lin(offset, 0.5, 9)[:-1]]
    neg = [-inv(p) for p in lin(offset, 0.5, 8)[:-1]]
    vals = sorted(pos + [0.0] + neg)
    top = max(vals)
    return tuple(v / top for v in vals)


@functools.lru_cache(maxsize=None)
def _dynamic_values() -> tuple[float, ...]:
    vals: list[float] = []
    for i in range(7):
        n = 2 ** i
        edges = [0.1 + 0.9 * j / n for j in range(n + 1)]
        mids = [(edges[j] + edges[j + 1]) / 2.0 for j in range(n)]
        scale = 10.0 ** (i - 6)
        vals += [scale * m for m in mids] + [-scale * m for m in mids]
    vals += [0.0, 1.0]
    return tuple(sorted(vals))


def nf4_code(device=None) -> torch.Tensor:
    return torch.tensor(_nf4_values(), dtype=torch.float32, device=device)


def dynamic_map(device=None) -> torch.Tensor:
    return torch.tensor(_dynamic_values(), dtype=torch.float32, device=device)
