"""bf16 inputs on the GPU: the reference's original dtype contract.

The reference computes Q K^T on bf16 operands (fp32 accumulation) and P V as fp16(P) . fp16(V)
(kernels/v4_leaderboard_0740ms.py:91, :103, :123), and stores o in bf16 (:132).  The kernel runs
Q K^T on bf16 tensor-core operands and P V on fp16 ones after the library converts V to fp16.

Tolerances: against the fp32 oracle on the same bf16 inputs, fp16 o obeys the regression bound of
the fp16 tests (max 4e-3, mean 2e-4: the error budget after Q K^T is identical); bf16 o may differ
by one bf16 ulp of the oracle value plus 2e-3 (its own rounding plus fp16 P), mean <= 1e-3.
"""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import _lib
from usagi_b200 import patterns as P
from oracle.bsattn_oracle import attn_blockwise, attn_online_literal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
REG_MAX, REG_MEAN = 4e-3, 2e-4
LSE_TOL = 2e-4


@pytest.fixture(scope="module", autouse=True)
def _setup():
    ub.setup(device="cuda:0")
    yield
    ub.check_errors(DEV)


def _bf16_ulp(x):
    return torch.exp2(torch.floor(torch.log2(x.abs().clamp(min=2.0 ** -126))) - 7)


def _check(o, lse, ro, rl, tag):
    of = o.float().cpu()
    assert torch.isfinite(of).all(), tag
    d = (of - ro).abs()
    if o.dtype == torch.bfloat16:
        assert (d <= _bf16_ulp(ro) + 2e-3).all(), (tag, d.max().item())
        assert d.mean().item() <= 1e-3, (tag, d.mean().item())
    else:
        assert d.max().item() <= REG_MAX and d.mean().item() <= REG_MEAN, (tag, d.max().item())
    if lse is not None:
        lc = lse.cpu()
        fin = torch.isfinite(rl)
        assert torch.equal(fin, torch.isfinite(lc)), tag
        if fin.any():
            assert (lc[fin] - rl[fin]).abs().max().item() <= LSE_TOL, tag


def test_converter_matches_torch_bitwise():
    g = torch.Generator(device=DEV).manual_seed(5)
    x = (torch.randn(1 << 20, generator=g, device=DEV) * 4).bfloat16()
    edge = torch.tensor([0.0, -0.0, 1e-8, -3e-6, 6.1e-5, 65504.0, 70000.0, -1e6, float("inf"),
                         -float("inf"), 2.0 ** -24, 2.0 ** -25, 1.0, -1.5, 3.140625, 100.5],
                        device=DEV).bfloat16()
    x[:edge.numel()] = edge
    y = torch.empty(x.shape, device=DEV, dtype=torch.float16)
    rc = _lib.load().bsattn_bf16_to_f16(x.data_ptr(), y.data_ptr(), x.numel(),
                                        torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), x.to(torch.float16).view(torch.int16))


@pytest.mark.parametrize("fam", ["window8", "prefix4+window4", "retrieval8"])
@pytest.mark.parametrize("out_dtype", [None, torch.float16])
def test_small_families(fam, out_dtype):
    B, H, T = 1, 2, 2048
    g = torch.Generator().manual_seed(21)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).bfloat16() for _ in range(3)]
    pat = P.family_pattern(fam, B, H, T)
    o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr.to(DEV),
                                      pat.col_idx.to(DEV), out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert o.dtype == (torch.bfloat16 if out_dtype is None else out_dtype)
    ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx)
    _check(o, lse, ro, rl, fam)
    lo, ll = attn_online_literal(q, k, v, pat.row_ptr, pat.col_idx)
    _check(o, lse, lo, ll, fam + " literal")


@pytest.mark.parametrize("seq", [(0, 256), (1, 129), (256, 255), (5000, 384)])
def test_seq_lens_edges(seq):
    B, H, T = 2, 3, 384
    g = torch.Generator().manual_seed(22)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).bfloat16() for _ in range(3)]
    pat = P.retrieval_pattern(B, H, T, 8, seed=1)
    sl = torch.tensor(seq, dtype=torch.int32)
    o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr.to(DEV),
                                      pat.col_idx.to(DEV), sl.to(DEV))
    torch.cuda.synchronize()
    ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx, sl)
    _check(o, lse, ro, rl, str(seq))
    if seq[0] == 0:
        assert (o[0] == 0).all() and (lse[0] == float("-inf")).all()


def test_fp16_v_equals_converted_bf16_v():
    """Passing V already in fp16 is the same computation as passing it in bf16."""
    B, H, T = 2, 4, 4096
    g = torch.Generator(device=DEV).manual_seed(23)
    q, k, v = [torch.randn(B, H, T, 128, generator=g, device=DEV).bfloat16() for _ in range(3)]
    pat = P.family_pattern("retrieval8", B, H, T)
    rp, ci = pat.row_ptr.to(DEV), pat.col_idx.to(DEV)
    o1, l1 = ub.block_sparse_attn_fwd(q, k, v, rp, ci)
    o2, l2 = ub.block_sparse_attn_fwd(q, k, v.half(), rp, ci)
    o3, l3 = ub.block_sparse_attn_fwd(q, k, v, rp, ci)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    assert torch.equal(o1, o3) and torch.equal(l1, l3)


@pytest.mark.parametrize("fam", ["window8", "retrieval8"])
def test_benchmark_size_heads(fam):
    B, H, T = 2, 16, 8192
    g = torch.Generator(device=DEV).manual_seed(24)
    q, k, v = [torch.randn(B, H, T, 128, generator=g, device=DEV).bfloat16() for _ in range(3)]
    pat = P.family_pattern(fam, B, H, T)
    o, lse = ub.block_sparse_attn_fwd(q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV),
                                      out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    flat = lambda t: t.reshape(B * H, *t.shape[2:])  # noqa: E731
    for bh in (0, 17, 31):
        sub = lambda t: flat(t)[bh:bh + 1].unsqueeze(0).cpu()  # noqa: E731
        rp = pat.row_ptr.reshape(B * H, -1)[bh:bh + 1].reshape(1, 1, -1)
        ci = pat.col_idx.reshape(B * H, -1)[bh:bh + 1].reshape(1, 1, -1)
        ro, rl = attn_blockwise(sub(q), sub(k), sub(v), rp, ci)
        _check(sub(o), sub(lse), ro, rl, f"{fam} head {bh}")
