"""CSR block-sparsity patterns over 128x128 blocks (the caller-side step of the path).

The reference entry point ``block_sparse_attn_fwd(q, k, v, row_ptr, col_idx, seq_lens)``
(kernels/v4_leaderboard_0740ms.py:242-243) receives, per (batch, head), a CSR list of live key
blocks for every query block:

* ``row_ptr``  int32 [B, H, nqb + 1]  -- offsets into that head's column list
* ``col_idx``  int32 [B, H, max_nnz]  -- key-block indices, padded to ``max_nnz``

The kernel walks ``col_idx[row_start : row_end - 1]`` as unmasked off-diagonal blocks and then
always processes block ``qb`` itself as the causal diagonal (v4 :78-124).  So every row produced
here is sorted ascending and ends with its own diagonal.

The three families and the mixed scaling pattern follow the benchmark configurations of this
path (sliding window, global prefix + window, random retrieval).  Generation is seeded and uses
``torch.Generator`` on the CPU so fixtures regenerate bit-identically on any host with the same
torch build.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Sequence

import torch

BLOCK = 128
HEAD_DIM = 128

__all__ = [
    "BLOCK",
    "HEAD_DIM",
    "CsrPattern",
    "window_rows",
    "prefix_window_rows",
    "retrieval_rows",
    "pattern_from_rows",
    "shared_pattern",
    "window_pattern",
    "prefix_window_pattern",
    "retrieval_pattern",
    "mixed_pattern",
    "family_pattern",
    "live_blocks",
    "FAMILIES",
    "device_window_pattern",
    "device_prefix_window_pattern",
    "device_retrieval_pattern",
]


@dataclass
class CsrPattern:
    """A CSR block pattern for every (b, h) pair.

    ``row_ptr`` and ``col_idx`` may be stride-0 expanded views when one pattern is shared by
    all heads (the window families); ``live_blocks`` counts every listed block once per head.
    """

    row_ptr: torch.Tensor  # int32 [B, H, nqb + 1]
    col_idx: torch.Tensor  # int32 [B, H, max_nnz]
    name: str = ""

    @property
    def B(self) -> int:
        return int(self.row_ptr.shape[0])

    @property
    def H(self) -> int:
        return int(self.row_ptr.shape[1])

    @property
    def nqb(self) -> int:
        return int(self.row_ptr.shape[2]) - 1

    def live_blocks(self) -> int:
        """Total number of (query block, key block) tiles the kernel computes.

        Each row costs ``max(n - 1, 0) + 1`` tiles: the listed off-diagonals plus the diagonal,
        which the reference computes even for an empty row (v4 :85 ``range(num_kv - 1)``, :107).
        """
        rp = self.row_ptr.reshape(-1, self.nqb + 1).to(torch.int64)
        n = rp[:, 1:] - rp[:, :-1]
        return int(((n - 1).clamp(min=0) + 1).sum())

    def contiguous(self) -> "CsrPattern":
        return CsrPattern(self.row_ptr.contiguous(), self.col_idx.contiguous(), self.name)

    def to(self, device) -> "CsrPattern":
        return CsrPattern(self.row_ptr.to(device), self.col_idx.to(device), self.name)


def window_rows(nqb: int, window: int) -> List[List[int]]:
    """Row i attends blocks max(0, i - window + 1) .. i (diagonal included)."""
    return [list(range(max(0, i - window + 1), i + 1)) for i in range(nqb)]


def prefix_window_rows(nqb: int, prefix: int, window: int) -> List[List[int]]:
    """Row i attends {0 .. min(prefix-1, i)} U {max(0, i-window+1) .. i}, sorted, deduplicated."""
    rows = []
    for i in range(nqb):
        s = set(range(0, min(prefix - 1, i) + 1)) | set(range(max(0, i - window + 1), i + 1))
        rows.append(sorted(s))
    return rows


def retrieval_rows(nqb: int, n_random: int, gen: torch.Generator) -> List[List[int]]:
    """Row i attends blocks i and i-1 plus min(n_random, i-1) distinct blocks drawn uniformly
    without replacement from 0 .. i-2 (``randperm(i - 1)[:r]``), sorted."""
    rows = []
    for i in range(nqb):
        s = {i}
        if i >= 1:
            s.add(i - 1)
        if i >= 2:
            r = min(n_random, i - 1)
            picks = torch.randperm(i - 1, generator=gen)[:r]
            s.update(int(x) for x in picks)
        rows.append(sorted(s))
    return rows


def _pack(rows_per_head: Sequence[List[List[int]]], nqb: int):
    max_nnz = max(sum(len(r) for r in rows) for rows in rows_per_head)
    n_heads = len(rows_per_head)
    rp = torch.zeros(n_heads, nqb + 1, dtype=torch.int32)
    ci = torch.zeros(n_heads, max(max_nnz, 1), dtype=torch.int32)
    for h, rows in enumerate(rows_per_head):
        flat = [c for r in rows for c in r]
        lens = torch.tensor([len(r) for r in rows], dtype=torch.int64)
        rp[h, 1:] = torch.cumsum(lens, 0).to(torch.int32)
        if flat:
            ci[h, : len(flat)] = torch.tensor(flat, dtype=torch.int32)
    return rp, ci


def pattern_from_rows(rows_per_head: Sequence[List[List[int]]], B: int, H: int, nqb: int,
                      name: str = "") -> CsrPattern:
    """Pack per-(b,h) row lists (ordered b-major, then h) into a dense [B, H, ...] CSR."""
    assert len(rows_per_head) == B * H
    rp, ci = _pack(rows_per_head, nqb)
    return CsrPattern(rp.reshape(B, H, nqb + 1), ci.reshape(B, H, -1), name)


def shared_pattern(rows: List[List[int]], B: int, H: int, nqb: int, name: str = "") -> CsrPattern:
    """One pattern broadcast to every (b, h) as a stride-0 expanded view."""
    rp, ci = _pack([rows], nqb)
    return CsrPattern(rp.reshape(1, 1, nqb + 1).expand(B, H, nqb + 1),
                      ci.reshape(1, 1, -1).expand(B, H, ci.shape[1]), name)


def window_pattern(B: int, H: int, T: int, window: int = 8, shared: bool = True) -> CsrPattern:
    nqb = T // BLOCK
    rows = window_rows(nqb, window)
    if shared:
        return shared_pattern(rows, B, H, nqb, f"window{window}")
    return pattern_from_rows([rows] * (B * H), B, H, nqb, f"window{window}")


def prefix_window_pattern(B: int, H: int, T: int, prefix: int = 4, window: int = 4,
                          shared: bool = False) -> CsrPattern:
    nqb = T // BLOCK
    rows = prefix_window_rows(nqb, prefix, window)
    name = f"prefix{prefix}+window{window}"
    if shared:
        return shared_pattern(rows, B, H, nqb, name)
    return pattern_from_rows([rows] * (B * H), B, H, nqb, name)


def retrieval_pattern(B: int, H: int, T: int, n_random: int = 8, seed: int = 1) -> CsrPattern:
    """Per-(b,h) retrieval rows; one generator seeded once, drawn in b, h, row order."""
    nqb = T // BLOCK
    gen = torch.Generator().manual_seed(seed)
    rows = [retrieval_rows(nqb, n_random, gen) for _ in range(B * H)]
    return pattern_from_rows(rows, B, H, nqb, f"retrieval{n_random}")


def mixed_pattern(B: int, H: int, T: int, seed: int = 1) -> CsrPattern:
    """Head-sharded scaling mix: head index bh % 3 selects window16 / prefix8+window8 /
    retrieval (diagonal + previous + 16 random); retrieval rows drawn in b, h, row order."""
    nqb = T // BLOCK
    gen = torch.Generator().manual_seed(seed)
    w = window_rows(nqb, 16)
    pw = prefix_window_rows(nqb, 8, 8)
    rows = []
    for bh in range(B * H):
        kind = bh % 3
        if kind == 0:
            rows.append(w)
        elif kind == 1:
            rows.append(pw)
        else:
            rows.append(retrieval_rows(nqb, 16, gen))
    return pattern_from_rows(rows, B, H, nqb, "mixed")


FAMILIES: dict = {
    "window8": lambda B, H, T: window_pattern(B, H, T, 8, shared=True),
    "prefix4+window4": lambda B, H, T: prefix_window_pattern(B, H, T, 4, 4),
    "retrieval8": lambda B, H, T: retrieval_pattern(B, H, T, 8, seed=1),
}


def family_pattern(name: str, B: int, H: int, T: int) -> CsrPattern:
    if name == "mixed":
        return mixed_pattern(B, H, T)
    return FAMILIES[name](B, H, T)


def live_blocks(pattern: CsrPattern) -> int:
    return pattern.live_blocks()


# ---------------------------------------------------------------------------------------------
# The same families built on the GPU by the library (bsattn_build_csr), for callers that keep the
# whole step on the device.  Window families are bit-identical to the host builders above and are
# built once and shared by every head (stride 0); retrieval rows use the library's counter-based
# generator keyed by (seed, head, row): the same distribution as retrieval_rows, other draws.
# ---------------------------------------------------------------------------------------------
def _device_csr(kind: int, n_heads: int, nqb: int, prefix: int, window: int, n_random: int,
                seed: int, device) -> tuple:
    import ctypes
    from . import _lib
    lib = _lib.load()
    nnz = ctypes.c_int64(0)
    rc = lib.bsattn_csr_nnz(kind, nqb, prefix, window, n_random, ctypes.byref(nnz))
    if rc != 0:
        raise ValueError(f"bsattn_csr_nnz: {_lib.strerror(rc)}")
    dev = torch.device(device)
    rp = torch.empty((n_heads, nqb + 1), dtype=torch.int32, device=dev)
    ci = torch.empty((n_heads, max(int(nnz.value), 1)), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = lib.bsattn_build_csr(kind, nqb, prefix, window, n_random,
                                  seed & 0xFFFFFFFFFFFFFFFF, n_heads, rp.data_ptr(),
                                  ci.data_ptr(), ci.shape[1],
                                  torch.cuda.current_stream(dev).cuda_stream)
    if rc != 0:
        raise RuntimeError(f"bsattn_build_csr: {_lib.strerror(rc)}")
    return rp, ci


def device_window_pattern(B: int, H: int, T: int, window: int = 8,
                          device="cuda") -> CsrPattern:
    nqb = T // BLOCK
    rp, ci = _device_csr(0, 1, nqb, 0, window, 0, 0, device)
    return CsrPattern(rp.reshape(1, 1, -1).expand(B, H, nqb + 1),
                      ci.reshape(1, 1, -1).expand(B, H, ci.shape[1]), f"window{window}")


def device_prefix_window_pattern(B: int, H: int, T: int, prefix: int = 4, window: int = 4,
                                 device="cuda") -> CsrPattern:
    nqb = T // BLOCK
    rp, ci = _device_csr(1, 1, nqb, prefix, window, 0, 0, device)
    return CsrPattern(rp.reshape(1, 1, -1).expand(B, H, nqb + 1),
                      ci.reshape(1, 1, -1).expand(B, H, ci.shape[1]),
                      f"prefix{prefix}+window{window}")


def device_retrieval_pattern(B: int, H: int, T: int, n_random: int = 8, seed: int = 1,
                             device="cuda") -> CsrPattern:
    nqb = T // BLOCK
    rp, ci = _device_csr(2, B * H, nqb, 0, 0, n_random, seed, device)
    return CsrPattern(rp.reshape(B, H, nqb + 1), ci.reshape(B, H, -1), f"retrieval{n_random}")
