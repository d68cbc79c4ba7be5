"""Failure detection on the GPU without a GPU fault: every pipeline wait in the kernel is bounded by
``bsattn_set_timeout_ns``.  The test hook ``bsattn_test_unsignalled_wait`` makes the QK^T-issuing
thread of every CTA first wait on a barrier that nothing signals; with a 10 ms bound that wait runs
out, the CTA raises its abort flag, the other roles leave their loops, the copies and MMAs in flight
are drained (the drain has its own floor of 100 ms), tensor memory is freed and BSATTN_E_TIMEOUT is
left in the error word.

The test checks that the host reads that status and that the CUDA context stays usable: the next
call with the hook off and the normal bound gives bit-identical output to a call made before.
"""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import _lib
from usagi_b200 import patterns as P

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
DEFAULT_TIMEOUT_NS = 2_000_000_000  # the library's default bound


def _inputs():
    B, H, T = 1, 4, 2048
    g = torch.Generator(device=DEV).manual_seed(77)
    q, k, v = [torch.randn(B, H, T, 128, generator=g, device=DEV).half() for _ in range(3)]
    pat = P.retrieval_pattern(B, H, T, 8, seed=3)
    return q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV)


def test_wait_timeout_is_reported_and_context_survives():
    ub.setup(device="cuda:0")
    q, k, v, rp, ci = _inputs()
    o_ref, lse_ref = ub.block_sparse_attn_fwd(q, k, v, rp, ci)
    ub.check_errors(DEV)
    lib = _lib.load()
    try:
        ub.set_timeout_ns(10_000_000)
        lib.bsattn_test_unsignalled_wait(1)
        ub.block_sparse_attn_fwd(q, k, v, rp, ci)
        with pytest.raises(ub.BsattnError) as err:
            ub.check_errors(DEV)
        assert err.value.code == _lib.E_TIMEOUT
    finally:
        lib.bsattn_test_unsignalled_wait(0)
        ub.set_timeout_ns(DEFAULT_TIMEOUT_NS)
    # The error word was cleared by the read above; the context still runs kernels.
    o, lse = ub.block_sparse_attn_fwd(q, k, v, rp, ci)
    ub.check_errors(DEV)
    assert torch.equal(o, o_ref)
    assert torch.equal(lse, lse_ref)
    x = torch.randn(256, 256, device=DEV)
    assert torch.isfinite(x @ x).all()
