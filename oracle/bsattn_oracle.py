"""CPU oracle for block-sparse causal attention forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this module.  It is the checker, never the product: the product path
(``usagi_b200``) runs only the CUDA kernel and fails loudly when that is missing.

It restates, in fp32 PyTorch/numpy on the CPU, what the reference computes in
``_fwd_csr`` (sissississi-013/usagi, kernels/v4_leaderboard_0740ms.py:31-136; identical math in
kernels/v7_blockptr_warpspec.py:30-148).  Per (b, h) and 128-row query block ``qb``:

* off-diagonal key blocks are ``col_idx[row_start : row_end - 1]`` (v4 :78-86), taken as listed
  (duplicates count twice, no sortedness needed), unmasked except that query rows at or past
  ``seq_len`` are masked out (v4 :93);
* the diagonal block is always ``qb`` itself, whatever the last CSR entry says (v4 :107), with
  mask ``key <= query  and  key < seq_len  and  query < seq_len`` (v4 :111-114);
* a query block starting at or past ``seq_len`` writes o = 0 and lse = -inf (v4 :63-68);
* o = sum_j p_j v_j / sum_j p_j with p = exp(q.k * scale); rows whose sum is 0 give o = 0 and
  lse = -inf; otherwise lse = natural-log logsumexp of the scaled scores (v4 :126-136).

Three restatements are provided:

``attn_blockwise``   exact fp32 softmax over the listed blocks, batched per query block
                     (fast enough for the full benchmark sizes on a few heads).
``attn_dense_masked`` the dense-masked form: a [T, T] per-element multiplicity mask per head
                     (listed-block count + causal diagonal), masked softmax over all T keys.  This
                     is the "dense-masked PyTorch CPU path" the benchmark names as CPU baseline.
``attn_online_literal`` a literal numpy transcription of the reference's online-softmax loop
                     (exp2, running max initialised to -1e30, fp16-rounded P, fp32 accumulation)
                     for small cases; it pins the restatements against the reference's own
                     outputs (tests/golden).

Parity pinning: tests/golden/*.npz hold outputs of the reference Triton kernels (v1, v4, v7)
executed under ``TRITON_INTERPRET=1`` in the build container (generator script committed next
to them).  The interpreter rounds fp32 -> bf16 toward zero, so its ``o`` carries up to one bf16
ulp of error; the golden tests allow exactly that.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch

BLOCK = 128

__all__ = [
    "row_blocks",
    "attn_blockwise",
    "attn_dense_masked",
    "attn_online_literal",
    "live_flops",
]


def _flat_meta(q, row_ptr, col_idx, seq_lens):
    B, H, T, D = q.shape
    BH = B * H
    nqb = T // BLOCK
    rp = torch.as_tensor(row_ptr).reshape(BH, nqb + 1).to(torch.int64).cpu()
    ci = torch.as_tensor(col_idx).reshape(BH, -1).to(torch.int64).cpu()
    if seq_lens is None:
        sl = torch.full((BH,), T, dtype=torch.int64)
    else:
        # v4 :163  seq_lens.repeat_interleave(H)
        sl = torch.as_tensor(seq_lens).to(torch.int64).cpu().repeat_interleave(H)
    return B, H, T, D, BH, nqb, rp, ci, sl


def row_blocks(rp_bh: torch.Tensor, ci_bh: torch.Tensor, qb: int):
    """Off-diagonal key blocks of query block ``qb`` in walk order, then the diagonal.

    Follows v4 :78-86 and :107: ``num_kv = row_end - row_start``; the loop runs
    ``range(num_kv - 1)`` (empty when num_kv <= 1) and the diagonal is ``qb``.
    """
    rs = int(rp_bh[qb])
    re = int(rp_bh[qb + 1])
    n_off = max(re - rs - 1, 0)
    off = [int(x) for x in ci_bh[rs: rs + n_off]]
    return off, qb


def attn_blockwise(q, k, v, row_ptr, col_idx, seq_lens=None, scale: Optional[float] = None,
                   heads: Optional[list] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact fp32 block-sparse attention.  Returns (o fp32 [B,H,T,D], lse fp32 [B,H,T]).

    ``heads`` optionally restricts the computation to some flattened (b*H + h) indices; the
    other heads are left as NaN so a caller cannot mistake them for checked values.
    """
    B, H, T, D, BH, nqb, rp, ci, sl = _flat_meta(q, row_ptr, col_idx, seq_lens)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qf = q.reshape(BH, T, D).float().cpu()
    kf = k.reshape(BH, T, D).float().cpu()
    vf = v.reshape(BH, T, D).float().cpu()
    o = torch.full((BH, T, D), float("nan"), dtype=torch.float32)
    lse = torch.full((BH, T), float("nan"), dtype=torch.float32)
    ar = torch.arange(BLOCK)
    causal = ar[None, :] <= ar[:, None]  # [m, n]: key n <= query m
    for bh in (range(BH) if heads is None else heads):
        seq_len = int(sl[bh])
        for qb in range(nqb):
            q0 = qb * BLOCK
            if q0 >= seq_len:  # v4 :63-68
                o[bh, q0:q0 + BLOCK] = 0.0
                lse[bh, q0:q0 + BLOCK] = float("-inf")
                continue
            off, diag = row_blocks(rp[bh], ci[bh], qb)
            blocks = off + [diag]
            idx = torch.cat([torch.arange(b * BLOCK, (b + 1) * BLOCK) for b in blocks])
            kk = kf[bh, idx]
            vv = vf[bh, idx]
            s = (qf[bh, q0:q0 + BLOCK] @ kk.T) * scale
            q_valid = (q0 + ar) < seq_len
            mask = torch.ones(BLOCK, len(blocks) * BLOCK, dtype=torch.bool)
            mask[~q_valid, :] = False
            dmask = causal & ((diag * BLOCK + ar)[None, :] < seq_len) & q_valid[:, None]
            mask[:, -BLOCK:] = dmask
            s = s.masked_fill(~mask, float("-inf"))
            m = s.max(dim=1, keepdim=True).values
            m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
            p = torch.exp(s - m_safe)
            l = p.sum(dim=1, keepdim=True)
            l_safe = torch.where(l > 0, l, torch.ones_like(l))
            ob = (p @ vv) / l_safe
            ob[~q_valid] = 0.0
            o[bh, q0:q0 + BLOCK] = ob
            lrow = torch.where(l[:, 0] > 0, m_safe[:, 0] + torch.log(l_safe[:, 0]),
                               torch.full_like(l[:, 0], float("-inf")))
            lrow[~q_valid] = float("-inf")
            lse[bh, q0:q0 + BLOCK] = lrow
    return o.reshape(B, H, T, D), lse.reshape(B, H, T)


def dense_weights(rp_bh, ci_bh, nqb: int, T: int, seq_len: int) -> torch.Tensor:
    """[T, T] float multiplicity mask of one head (row = query, column = key).

    Each listed off-diagonal block adds 1 to its whole 128x128 tile (rows < seq_len only); the
    diagonal adds 1 where key <= query and key < seq_len and query < seq_len.
    """
    W = torch.zeros(T, T, dtype=torch.float32)
    ar = torch.arange(BLOCK)
    causal = (ar[None, :] <= ar[:, None]).float()
    for qb in range(nqb):
        q0 = qb * BLOCK
        if q0 >= seq_len:
            continue
        off, diag = row_blocks(rp_bh, ci_bh, qb)
        for kb in off:
            W[q0:q0 + BLOCK, kb * BLOCK:(kb + 1) * BLOCK] += 1.0
        d0 = diag * BLOCK
        dm = causal * ((d0 + ar)[None, :] < seq_len).float()
        W[q0:q0 + BLOCK, d0:d0 + BLOCK] += dm
    rows_invalid = torch.arange(T) >= seq_len
    W[rows_invalid] = 0.0
    return W


def attn_dense_masked(q, k, v, row_ptr, col_idx, seq_lens=None, scale: Optional[float] = None,
                      heads: Optional[list] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Dense-masked fp32 attention over all T keys with the CSR multiplicity mask."""
    B, H, T, D, BH, nqb, rp, ci, sl = _flat_meta(q, row_ptr, col_idx, seq_lens)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qf = q.reshape(BH, T, D).float().cpu()
    kf = k.reshape(BH, T, D).float().cpu()
    vf = v.reshape(BH, T, D).float().cpu()
    o = torch.full((BH, T, D), float("nan"), dtype=torch.float32)
    lse = torch.full((BH, T), float("nan"), dtype=torch.float32)
    for bh in (range(BH) if heads is None else heads):
        W = dense_weights(rp[bh], ci[bh], nqb, T, int(sl[bh]))
        s = (qf[bh] @ kf[bh].T) * scale
        s = s.masked_fill(W == 0, float("-inf"))
        m = s.max(dim=1, keepdim=True).values
        m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        p = torch.exp(s - m_safe) * W
        l = p.sum(dim=1, keepdim=True)
        l_safe = torch.where(l > 0, l, torch.ones_like(l))
        o[bh] = (p @ vf[bh]) / l_safe
        lse[bh] = torch.where(l[:, 0] > 0, m_safe[:, 0] + torch.log(l_safe[:, 0]),
                              torch.full_like(l[:, 0], float("-inf")))
    return o.reshape(B, H, T, D), lse.reshape(B, H, T)


def _exp2(x):
    with np.errstate(over="ignore", invalid="ignore"):
        return np.exp2(x)


def attn_online_literal(q, k, v, row_ptr, col_idx, seq_lens=None):
    """Literal transcription of the reference program loop (v4 :57-136), numpy fp32.

    QK_SCALE = log2(e)/sqrt(128) post-multiplies the fp32 dot (v4 :19-22, :91); m starts at
    -1e30 (:74); alpha = exp2(m - m_new), p = exp2(s - m_new) (:97-98); l sums fp32 p (:99);
    acc += fp16(p) @ fp16(v) in fp32 (:103); o = acc / l_safe, lse = m*ln2 + ln(l_safe) (:126-136).
    Returns fp32 (o, lse) before the final bf16 store.
    """
    B, H, T, D, BH, nqb, rp, ci, sl = _flat_meta(q, row_ptr, col_idx, seq_lens)
    qk_scale = np.float32((1.0 / math.sqrt(D)) * math.log2(math.e))
    ln2 = np.float32(math.log(2.0))
    # fp16 and bf16 values are exact in fp32.  V goes through fp16 below whatever its input type:
    # the reference multiplies fp16(P) by v.to(tl.float16) (v4 :103, :123).
    qn = q.reshape(BH, T, D).float().cpu().numpy()
    kn = k.reshape(BH, T, D).float().cpu().numpy()
    vn = v.reshape(BH, T, D).float().cpu().numpy()
    o = np.zeros((BH, T, D), np.float32)
    lse = np.full((BH, T), -np.inf, np.float32)
    offs = np.arange(BLOCK)
    for bh in range(BH):
        seq_len = int(sl[bh])
        for qb in range(nqb):
            q0 = qb * BLOCK
            if q0 >= seq_len:
                continue
            q_valid = (q0 + offs) < seq_len
            qt = qn[bh, q0:q0 + BLOCK].astype(np.float32)
            m_i = np.full(BLOCK, -1e30, np.float32)
            l_i = np.zeros(BLOCK, np.float32)
            acc = np.zeros((BLOCK, D), np.float32)
            off, diag = row_blocks(rp[bh], ci[bh], qb)

            def update(kb, mask):
                nonlocal m_i, l_i, acc
                kt = kn[bh, kb * BLOCK:(kb + 1) * BLOCK].astype(np.float32)
                vt = vn[bh, kb * BLOCK:(kb + 1) * BLOCK].astype(np.float16).astype(np.float32)
                s = (qt @ kt.T).astype(np.float32) * qk_scale
                s = np.where(mask, s, np.float32(-np.inf)).astype(np.float32)
                m_new = np.maximum(m_i, s.max(axis=1))
                alpha = _exp2(m_i - m_new).astype(np.float32)
                p = _exp2(s - m_new[:, None]).astype(np.float32)
                l_i = (alpha * l_i + p.sum(axis=1)).astype(np.float32)
                p16 = p.astype(np.float16).astype(np.float32)
                acc = (acc * alpha[:, None] + p16 @ vt).astype(np.float32)
                m_i = m_new

            for kb in off:
                update(kb, np.broadcast_to(q_valid[:, None], (BLOCK, BLOCK)))
            dmask = (offs[None, :] <= offs[:, None]) & ((diag * BLOCK + offs)[None, :] < seq_len) \
                & q_valid[:, None]
            update(diag, dmask)
            l_safe = np.where(l_i > 0, l_i, np.float32(1.0))
            ob = acc / l_safe[:, None]
            ob[~q_valid] = 0.0
            o[bh, q0:q0 + BLOCK] = ob
            with np.errstate(divide="ignore"):
                lr = np.where(l_i > 0, m_i * ln2 + np.log(l_safe), -np.inf).astype(np.float32)
            lr[~q_valid] = -np.inf
            lse[bh, q0:q0 + BLOCK] = lr
    return (torch.from_numpy(o).reshape(B, H, T, D), torch.from_numpy(lse).reshape(B, H, T))


def live_flops(row_ptr, B: int, H: int, T: int, D: int = 128) -> int:
    """Algorithmic FLOPs: every computed 128x128 tile counted in full, QK^T + PV, 2 flop/MAC."""
    nqb = T // BLOCK
    rp = torch.as_tensor(row_ptr).reshape(B * H, nqb + 1).to(torch.int64)
    n = rp[:, 1:] - rp[:, :-1]
    tiles = int(((n - 1).clamp(min=0) + 1).sum())
    return tiles * 4 * BLOCK * BLOCK * D
