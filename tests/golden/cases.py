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


# ---------------------------------------------------------------------------------------------
# Full-size cases: the benchmark configurations on their exact seeded inputs.  The fixtures
# (full_<name>.npz, made by make_golden_full.py) hold the reference's outputs for the listed
# (b, h) heads; ``qblocks`` None means every query block of the head is stored.
# ---------------------------------------------------------------------------------------------
FULL_CONFIGS = {
    # B, H, T of the three family configurations and of the head-sharded scaling mix
    "family": (2, 16, 8192),
    "mix": (4, 32, 32768),
}

_MIX_QBLOCKS = [0, 1, 2, 7, 8, 15, 16, 17, 64, 127, 128, 200, 253, 254, 255]

FULL_CASES = {
    "window8": {"config": "family", "heads": [(0, 0)], "qblocks": None},
    "prefix4_window4": {"config": "family", "heads": [(1, 7)], "qblocks": None},
    "retrieval8": {"config": "family", "heads": [(0, 0), (1, 9)], "qblocks": None},
    # bh = b * 32 + h; bh % 3 picks window16 (0), prefix8+window8 (1), retrieval 2+16 (2)
    "mix": {"config": "mix", "heads": [(0, 0), (0, 1), (0, 2), (2, 1), (3, 31)],
            "qblocks": _MIX_QBLOCKS},
}


def full_inputs(config: str):
    """(q, k, v) fp16 of a full-size configuration: N(0,1) fp32 from CPU seed 0 in the order
    q, k, v, cast to fp16 one tensor at a time (the scaling mix is 2.1 GB per fp32 draw)."""
    B, H, T = FULL_CONFIGS[config]
    g = torch.Generator().manual_seed(0)
    return tuple(torch.randn(B, H, T, 128, generator=g).half() for _ in range(3))


def full_pattern(name: str, inputs=None) -> "P.CsrPattern":
    """The CSR pattern of a full-size case at its configuration's shape."""
    cfg = FULL_CASES[name]["config"]
    B, H, T = FULL_CONFIGS[cfg]
    if name == "window8":
        return P.window_pattern(B, H, T, 8, shared=True)
    if name == "prefix4_window4":
        return P.prefix_window_pattern(B, H, T, 4, 4)
    if name == "retrieval8":
        return P.retrieval_pattern(B, H, T, 8, seed=1)
    if name == "mix":
        return P.mixed_pattern(B, H, T, seed=1)
    raise KeyError(name)


def head_slice(q, k, v, pat, b: int, h: int) -> dict:
    """Single-head (B=1, H=1) slice of a problem: inputs and that head's CSR rows."""
    one = lambda t: t[b:b + 1, h:h + 1].contiguous()  # noqa: E731
    return dict(q=one(q), k=one(k), v=one(v), row_ptr=one(pat.row_ptr), col_idx=one(pat.col_idx))


def head_checksums(sl: dict) -> list:
    """Checksums of a head slice: q, k, v, and the head's listed CSR entries."""
    rp = sl["row_ptr"].reshape(-1).to(torch.int64)
    ci = sl["col_idx"].reshape(-1)[: int(rp[-1])].to(torch.int64)
    w = torch.arange(ci.numel(), dtype=torch.int64) % 13 + 1
    return [checksum(sl["q"]), checksum(sl["k"]), checksum(sl["v"]), float(rp.sum()),
            float((ci * w).sum())]
