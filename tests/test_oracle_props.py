"""The oracle's two exact restatements (blockwise and dense multiplicity mask) agree on random
CSR rows with the irregularities the reference's loop accepts: duplicated, unsorted and future
blocks, empty rows (the diagonal alone), and seq_lens shorter than T (v4 :63-68, :78-113).
They are independent codings of the same rules, so agreement to fp32 rounding checks both."""
import pytest
import torch

from oracle.bsattn_oracle import attn_blockwise, attn_dense_masked


def test_exact_restatements_agree_on_random_csr():
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=40, deadline=None, derandomize=True)
    @hyp.given(st.data())
    def check(data):
        B = data.draw(st.integers(1, 2))
        H = data.draw(st.integers(1, 2))
        nqb = data.draw(st.integers(1, 4))
        T, BH = 128 * nqb, B * H
        rows = [[data.draw(st.lists(st.integers(0, nqb - 1), min_size=0, max_size=5))
                 for _ in range(nqb)] for _ in range(BH)]
        width = max(1, max(sum(len(r) for r in head) for head in rows))
        rp = torch.zeros(BH, nqb + 1, dtype=torch.int32)
        ci = torch.zeros(BH, width, dtype=torch.int32)
        for bh, head in enumerate(rows):
            pos = 0
            for i, r in enumerate(head):
                ci[bh, pos:pos + len(r)] = torch.tensor(r, dtype=torch.int32)
                pos += len(r)
                rp[bh, i + 1] = pos
        seq_lens = None
        if data.draw(st.booleans()):
            seq_lens = torch.tensor(data.draw(st.lists(st.integers(0, T), min_size=B, max_size=B)))
        g = torch.Generator().manual_seed(data.draw(st.integers(0, 2 ** 31 - 1)))
        q, k, v = [torch.randn(B, H, T, 128, generator=g) for _ in range(3)]
        rp, ci = rp.reshape(B, H, -1), ci.reshape(B, H, -1)
        o1, l1 = attn_blockwise(q, k, v, rp, ci, seq_lens)
        o2, l2 = attn_dense_masked(q, k, v, rp, ci, seq_lens)
        assert torch.isfinite(o1).all() and torch.isfinite(o2).all()
        assert (o1 - o2).abs().max().item() <= 1e-4
        fin = torch.isfinite(l1)
        assert torch.equal(fin, torch.isfinite(l2))
        assert (l1[fin] - l2[fin]).abs().max().item() <= 1e-4 if fin.any() else True

    check()
