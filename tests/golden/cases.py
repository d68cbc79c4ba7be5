"""Seeded input cases shared by the golden-fixture generator and the parity tests.

Every case regenerates bit-identically from its seed with torch's CPU generator, so the
fixtures only store the reference's outputs plus an input checksum that detects generator drift.
Inputs are drawn N(0, 1) in fp32 in the order q, k, v and cast to the case dtype.
"""
from __future__ import annotations

import os
import sys

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from usagi_b200 import patterns as P  # noqa: E402

BLOCK = 128


def qkv(B, H, T, seed=0, dtype=torch.float16, D=128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T, D, generator=g)
    k = torch.randn(B, H, T, D, generator=g)
    v = torch.randn(B, H, T, D, generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def _irregular_rows():
    """Rows that exercise what the reference accepts without checking (v4 :78-107):
    empty rows, unsorted and duplicated off-diagonals, a last entry that is not the diagonal
    (ignored: the diagonal is always qb), and a future block listed as off-diagonal (unmasked)."""
    return [
        [],             # row 0: empty -> diagonal only
        [3, 1],         # row 1: future block 3 (unmasked), then diag entry
        [0, 0, 2],      # row 2: duplicate off-diagonal 0
        [2, 0, 1],      # row 3: unsorted; last entry 1 is skipped, diagonal 3 used
        [3, 1, 4],      # row 4: off-diag 3, 1
    ]


def case(name):
    """Return dict(q, k, v, row_ptr, col_idx, seq_lens) on the CPU for a named case."""
    if name == "cfg0_window4":
        # The CPU configuration: B=1, H=2, T=1024, window of 4 blocks, seed 0.
        q, k, v = qkv(1, 2, 1024, seed=0)
        pat = P.window_pattern(1, 2, 1024, 4, shared=False)
        sl = None
    elif name == "prefix_window":
        q, k, v = qkv(1, 1, 1024, seed=2)
        pat = P.prefix_window_pattern(1, 1, 1024, 4, 4)
        sl = None
    elif name == "retrieval":
        q, k, v = qkv(1, 2, 1024, seed=3)
        pat = P.retrieval_pattern(1, 2, 1024, 8, seed=1)
        sl = None
    elif name == "seqlens":
        q, k, v = qkv(2, 1, 512, seed=4)
        pat = P.window_pattern(2, 1, 512, 3, shared=False)
        sl = torch.tensor([512, 300], dtype=torch.int32)
    elif name == "irregular":
        q, k, v = qkv(1, 1, 640, seed=5)
        pat = P.pattern_from_rows([_irregular_rows()], 1, 1, 5, "irregular")
        sl = None
    elif name == "bf16_window":
        q, k, v = qkv(1, 1, 512, seed=6, dtype=torch.bfloat16)
        pat = P.window_pattern(1, 1, 512, 4, shared=False)
        sl = None
    else:
        raise KeyError(name)
    return dict(q=q, k=k, v=v, row_ptr=pat.row_ptr.contiguous(), col_idx=pat.col_idx.contiguous(),
                seq_lens=sl)


# bf16_window is generated on demand only: the Triton interpreter's bf16 tl.dot returns
# meaningless scores (lse ~ 1e10), so it cannot serve as a golden reference.
CASES = ["cfg0_window4", "prefix_window", "retrieval", "seqlens", "irregular"]


def checksum(t: torch.Tensor) -> float:
    return float(t.double().sum()) + float((t.double() * torch.arange(t.numel(), dtype=torch.float64)
                                             .reshape(t.shape).remainder(7)).sum())
