"""Work lists from bsattn_plan (host only, no GPU): every item exactly once, CTAs balanced to within
one item, big items in the kernel's head-grouped order, inactive items (past seq_len) last."""
import ctypes

import pytest
import torch

from usagi_b200 import _lib, api
from usagi_b200 import patterns as P

MAGIC = 0x4E4C5042


def _plan(pat, B, H, T, grid, seq_lens=None):
    lib = _lib.load()
    rp, rps = api._bh_view(pat.row_ptr, B, H, "row_ptr")
    nb = ctypes.c_size_t(0)
    assert lib.bsattn_plan_bytes(B, H, T, grid, ctypes.byref(nb)) == 0
    buf = torch.empty(nb.value // 4, dtype=torch.int32)
    sl = None if seq_lens is None else seq_lens.to(torch.int32).contiguous()
    rc = lib.bsattn_plan(rp.data_ptr(), rps, sl.data_ptr() if sl is not None else None, B, H, T,
                         int(pat.col_idx.shape[-1]), grid, buf.data_ptr(), nb.value)
    assert rc == 0, _lib.strerror(rc)
    return buf


def _sizes(pat, B, H, T, seq_lens=None):
    """Tile count of every item g in the kernel's order (host restatement of load_item)."""
    nqb, BH = T // 128, B * H
    rp = pat.row_ptr.reshape(BH, nqb + 1).to(torch.int64)
    gh = max(1, min(BH, (32 << 20) // (512 * T)))
    per = gh * nqb
    out = []
    for g in range(BH * nqb):
        grp, r = divmod(g, per)
        ghh = min(gh, BH - grp * gh)
        band = r // ghh
        bh, qb = grp * gh + (r - band * ghh), nqb - 1 - band
        sl = T if seq_lens is None else min(int(seq_lens[bh // H]), T)
        out.append(0 if qb * 128 >= sl else max(int(rp[bh, qb + 1] - rp[bh, qb]) - 1, 0) + 1)
    return out


@pytest.mark.parametrize("fam,grid", [("window8", 148), ("prefix4+window4", 148),
                                      ("retrieval8", 148), ("retrieval8", 37), ("window8", 2048)])
def test_plan_is_a_balanced_permutation(fam, grid):
    B, H, T = 2, 16, 8192
    pat = P.family_pattern(fam, B, H, T)
    buf = _plan(pat, B, H, T, grid)
    items = B * H * (T // 128)
    assert buf[:4].tolist() == [MAGIC, grid, items, 0]
    off = buf[4:4 + grid + 1].tolist()
    lst = buf[4 + grid + 1:].tolist()
    assert off[0] == 0 and off[-1] == items and all(a <= b for a, b in zip(off, off[1:]))
    assert sorted(lst) == list(range(items))
    size = _sizes(pat, B, H, T)
    loads = [sum(size[g] for g in lst[off[c]:off[c + 1]]) for c in range(grid)]
    assert max(loads) - min(loads) <= max(size)
    assert max(loads) <= sum(size) / grid + max(size)
    # Each CTA's list is sorted by size, largest first; equal sizes keep the item order.
    for c in range(grid):
        mine = lst[off[c]:off[c + 1]]
        keys = [(-size[g], g) for g in mine]
        assert keys == sorted(keys)


def test_plan_puts_inactive_items_last_and_handles_seq_lens():
    B, H, T = 2, 3, 2048
    pat = P.retrieval_pattern(B, H, T, 8)
    sl = torch.tensor([300, 2048], dtype=torch.int32)
    buf = _plan(pat, B, H, T, 16, sl)
    size = _sizes(pat, B, H, T, sl)
    lst = buf[4 + 17:].tolist()
    off = buf[4:4 + 17].tolist()
    for c in range(16):
        mine = [size[g] for g in lst[off[c]:off[c + 1]]]
        assert mine == sorted(mine, reverse=True)
    assert sum(1 for x in size if x == 0) == 3 * (T // 128 - 3)  # batch 0: 3 live query blocks


def test_plan_argument_errors():
    lib = _lib.load()
    nb = ctypes.c_size_t(0)
    assert lib.bsattn_plan_bytes(1, 1, 100, 4, ctypes.byref(nb)) == _lib.E_SHAPE
    assert lib.bsattn_plan_bytes(1, 1, 256, 3, ctypes.byref(nb)) == _lib.E_SHAPE  # grid > items
    assert lib.bsattn_plan_bytes(1, 1, 256, 0, ctypes.byref(nb)) == _lib.E_SHAPE
    assert lib.bsattn_plan_bytes(1, 1, 256, 2, None) == _lib.E_NULL
    rp = torch.tensor([0, 1, 2], dtype=torch.int32)
    small = torch.empty(4, dtype=torch.int32)
    assert lib.bsattn_plan(rp.data_ptr(), 0, None, 1, 1, 256, 2, 2, small.data_ptr(),
                           16) == _lib.E_WORKSPACE
    assert lib.bsattn_plan(None, 0, None, 1, 1, 256, 2, 2, small.data_ptr(), 16) == _lib.E_NULL


def _window_plan(B, H, T, window, global_blocks, grid, seq_lens=None):
    lib = _lib.load()
    nb = ctypes.c_size_t(0)
    assert lib.bsattn_plan_bytes(B, H, T, grid, ctypes.byref(nb)) == 0
    buf = torch.empty(nb.value // 4, dtype=torch.int32)
    sl = None if seq_lens is None else seq_lens.to(torch.int32).contiguous()
    rc = lib.bsattn_plan_window(sl.data_ptr() if sl is not None else None, B, H, T, window,
                                global_blocks, grid, buf.data_ptr(), nb.value)
    assert rc == 0, _lib.strerror(rc)
    return buf


@pytest.mark.parametrize("window,global_blocks", [(8, 0), (4, 4), (1, 0), (16, 8), (3, 1)])
def test_window_plan_equals_csr_plan(window, global_blocks):
    """Analytic rows and the same rows as CSR give the same work list, entry for entry."""
    B, H, T = 2, 3, 4096
    for sl in (None, torch.tensor([1000, 4096])):
        if global_blocks:
            pat = P.prefix_window_pattern(B, H, T, global_blocks, window)
        else:
            pat = P.window_pattern(B, H, T, window)
        for grid in (148, 37):
            assert torch.equal(_window_plan(B, H, T, window, global_blocks, grid, sl),
                               _plan(pat, B, H, T, grid, sl))


def test_window_plan_argument_errors():
    lib = _lib.load()
    buf = torch.empty(64, dtype=torch.int32)
    assert lib.bsattn_plan_window(None, 1, 1, 256, 0, 0, 2, buf.data_ptr(), 256) == _lib.E_SHAPE
    assert lib.bsattn_plan_window(None, 1, 1, 256, 4, -1, 2, buf.data_ptr(), 256) == _lib.E_SHAPE
    assert lib.bsattn_plan_window(None, 1, 1, 256, 4, 0, 2, None, 256) == _lib.E_NULL
    assert lib.bsattn_plan_window(None, 1, 1, 256, 4, 0, 2, buf.data_ptr(), 8) == _lib.E_WORKSPACE
    assert lib.bsattn_plan_window(None, 1, 1, 256, 4, 0, 2, buf.data_ptr(), 256) == _lib.OK


def _sizes_rows(rp_bh, B, H, T, max_nnz, seq_lens):
    """Tile counts in the kernel's item order for explicit per-head row offsets, including the
    rule that a row whose range does not fit the max_nnz columns counts as its diagonal alone."""
    nqb, BH = T // 128, B * H
    gh = max(1, min(BH, (32 << 20) // (512 * T)))
    per = gh * nqb
    out = []
    for g in range(BH * nqb):
        grp, r = divmod(g, per)
        ghh = min(gh, BH - grp * gh)
        band = r // ghh
        bh, qb = grp * gh + (r - band * ghh), nqb - 1 - band
        sl = T if seq_lens is None else min(int(seq_lens[bh // H]), T)
        if qb * 128 >= sl:
            out.append(0)
            continue
        rs, re = int(rp_bh[bh][qb]), int(rp_bh[bh][qb + 1])
        n_off = max(re - rs - 1, 0)
        if n_off > 0 and (rs < 0 or rs + n_off > max_nnz):
            n_off = 0
        out.append(n_off + 1)
    return out


def test_plan_properties_on_random_rows():
    """Any row lengths, seq_lens and grid: the list is an exact permutation of the items, every
    CTA's items are sorted by tile count (ties in item order), and the snake deal keeps the CTA
    loads within one largest item of each other."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=80, deadline=None, derandomize=True)
    @hyp.given(st.data())
    def check(data):
        B = data.draw(st.integers(1, 3))
        H = data.draw(st.integers(1, 4))
        nqb = data.draw(st.integers(1, 12))
        T, BH = 128 * nqb, B * H
        lens = data.draw(st.lists(st.integers(0, 9), min_size=BH * nqb, max_size=BH * nqb))
        rp_bh = []
        for bh in range(BH):
            offs = [0]
            for i in range(nqb):
                offs.append(offs[-1] + lens[bh * nqb + i])
            rp_bh.append(offs)
        max_nnz = data.draw(st.integers(0, max(o[-1] for o in rp_bh) + 2))
        seq_lens = None
        if data.draw(st.booleans()):
            seq_lens = torch.tensor(data.draw(st.lists(st.integers(0, T + 64), min_size=B,
                                                       max_size=B)), dtype=torch.int32)
        items = BH * nqb
        grid = data.draw(st.integers(1, items))
        lib = _lib.load()
        rp = torch.tensor(rp_bh, dtype=torch.int32).contiguous()
        nb = ctypes.c_size_t(0)
        assert lib.bsattn_plan_bytes(B, H, T, grid, ctypes.byref(nb)) == 0
        buf = torch.empty(nb.value // 4, dtype=torch.int32)
        rc = lib.bsattn_plan(rp.data_ptr(), nqb + 1,
                             seq_lens.data_ptr() if seq_lens is not None else None, B, H, T,
                             max_nnz, grid, buf.data_ptr(), nb.value)
        assert rc == 0, _lib.strerror(rc)
        assert buf[:4].tolist() == [MAGIC, grid, items, 0]
        off = buf[4:4 + grid + 1].tolist()
        lst = buf[4 + grid + 1:].tolist()
        assert off[0] == 0 and off[-1] == items and all(a <= b for a, b in zip(off, off[1:]))
        assert sorted(lst) == list(range(items))
        size = _sizes_rows(rp_bh, B, H, T, max_nnz, seq_lens)
        loads = [sum(size[g] for g in lst[off[c]:off[c + 1]]) for c in range(grid)]
        assert max(loads) - min(loads) <= max(size)
        for c in range(grid):
            keys = [(-size[g], g) for g in lst[off[c]:off[c + 1]]]
            assert keys == sorted(keys)

    check()
