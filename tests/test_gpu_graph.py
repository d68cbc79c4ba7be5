"""CUDA graphs and streams on the GPU.  The entry points only enqueue work on the caller's stream
(no allocation of their own, no synchronisation; kernels/v4_leaderboard_0740ms.py:167-179 launched
the same way), so a call can be captured into a CUDA graph and replayed with new inputs copied
into the captured buffers, and calls on two streams, each with its own workspace, can overlap.
Every result must equal the eager call on the same inputs bit for bit.
"""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import patterns as P

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _setup():
    ub.setup(device="cuda:0")
    yield
    ub.check_errors(DEV)


def _randn(shape, seed, dtype=torch.float16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(shape, generator=g, device=DEV).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_graph_replay_matches_eager(dtype):
    B, H, T = 2, 4, 4096
    pat = P.retrieval_pattern(B, H, T, 8)
    rp, ci = pat.row_ptr.to(DEV), pat.col_idx.to(DEV)
    sl = torch.tensor([3000, 4096], dtype=torch.int32, device=DEV)
    plan = ub.make_plan(pat.row_ptr, pat.col_idx, B, H, T, sl.cpu(), device=DEV)
    q, k, v = [_randn((B, H, T, 128), 60 + i, dtype) for i in range(3)]
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), device=DEV)
    ow = torch.empty_like(q)
    lsew = torch.empty((B, H, T), device=DEV)

    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):  # warm-up on the capture stream: its workspace exists before
        ub.block_sparse_attn_fwd(q, k, v, rp, ci, sl, out=o, lse_out=lse, plan=plan)
        ub.block_sparse_attn_fwd_window(q, k, v, sl, window=4, global_blocks=4, out=ow,
                                        lse_out=lsew)
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        ub.block_sparse_attn_fwd(q, k, v, rp, ci, sl, out=o, lse_out=lse, plan=plan)
        ub.block_sparse_attn_fwd_window(q, k, v, sl, window=4, global_blocks=4, out=ow,
                                        lse_out=lsew)
    for rep in range(3):
        nq, nk, nv = [_randn((B, H, T, 128), 70 + 3 * rep + i, dtype) for i in range(3)]
        q.copy_(nq)
        k.copy_(nk)
        v.copy_(nv)
        graph.replay()
        torch.cuda.synchronize()
        eo, el = ub.block_sparse_attn_fwd(nq, nk, nv, rp, ci, sl, plan=plan)
        wo, wl = ub.block_sparse_attn_fwd_window(nq, nk, nv, sl, window=4, global_blocks=4)
        torch.cuda.synchronize()
        assert torch.equal(o, eo) and torch.equal(lse, el), rep
        assert torch.equal(ow, wo) and torch.equal(lsew, wl), rep
    ub.check_errors(DEV)
    with torch.cuda.stream(side):
        ub.check_errors(DEV)
    del graph


def test_two_streams_overlap():
    B, H, T = 2, 8, 8192
    pats = [P.family_pattern(f, B, H, T) for f in ("window8", "retrieval8")]
    inputs = [[_randn((B, H, T, 128), 80 + 3 * j + i) for i in range(3)] for j in range(2)]
    eager = []
    for (q, k, v), pat in zip(inputs, pats):
        eager.append(ub.block_sparse_attn_fwd(q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV)))
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(DEV) for _ in range(2)]
    outs = [None, None]
    for rep in range(2):
        for j, s in enumerate(streams):
            s.wait_stream(torch.cuda.current_stream(DEV))
            with torch.cuda.stream(s):
                q, k, v = inputs[j]
                outs[j] = ub.block_sparse_attn_fwd(q, k, v, pats[j].row_ptr.to(DEV),
                                                   pats[j].col_idx.to(DEV))
        torch.cuda.synchronize()
        for j, s in enumerate(streams):
            with torch.cuda.stream(s):
                ub.check_errors(DEV)
            assert torch.equal(outs[j][0], eager[j][0]) and torch.equal(outs[j][1], eager[j][1])


def test_first_call_on_a_stream_inside_capture_is_refused():
    """The first call on a stream creates and zeroes its error word; inside capture that fill
    would only be recorded, so the call must refuse with a clear error instead."""
    from usagi_b200 import api
    B, H, T = 1, 1, 256
    pat = P.window_pattern(B, H, T, 2)
    rp, ci = pat.row_ptr.to(DEV), pat.col_idx.to(DEV)
    q, k, v = [_randn((B, H, T, 128), 90 + i) for i in range(3)]
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), device=DEV)
    fresh = torch.cuda.Stream(DEV)
    fresh.wait_stream(torch.cuda.current_stream(DEV))
    api._workspaces.pop((DEV.index, fresh.cuda_stream), None)  # as if never used
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="outside graph capture"):
        with torch.cuda.graph(graph, stream=fresh):
            ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=o, lse_out=lse)
    del graph
    # after an eager warm-up on the stream, the same call captures and replays
    with torch.cuda.stream(fresh):
        ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=o, lse_out=lse)
    fresh.synchronize()
    ref = o.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=fresh):
        ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=o, lse_out=lse)
    o.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(o, ref)
