"""CSR family generators: live-block counts, row structure, determinism (CPU)."""
import torch

from usagi_b200 import patterns as P


def rows_of(pat, bh):
    rp = pat.row_ptr.reshape(-1, pat.nqb + 1)[bh]
    ci = pat.col_idx.reshape(-1, pat.col_idx.shape[-1])[bh]
    return [ci[int(rp[i]):int(rp[i + 1])].tolist() for i in range(pat.nqb)]


def test_live_block_counts_match_benchmark_configs():
    assert P.family_pattern("window8", 2, 16, 8192).live_blocks() == 15488
    assert P.family_pattern("prefix4+window4", 2, 16, 8192).live_blocks() == 15488
    assert P.family_pattern("retrieval8", 2, 16, 8192).live_blocks() == 19040
    assert P.window_pattern(1, 2, 1024, 4).live_blocks() == 52


def test_mixed_scaling_pattern_count():
    # B=4, H=32, T=32768: window16 / prefix8+window8 / retrieval(2+16) by bh % 3, seed 1.
    assert P.mixed_pattern(4, 32, 32768).live_blocks() == 529046


def test_rows_sorted_and_end_with_diagonal():
    for name in ["window8", "prefix4+window4", "retrieval8"]:
        pat = P.family_pattern(name, 1, 3, 4096)
        for bh in range(3):
            for i, r in enumerate(rows_of(pat, bh)):
                assert r == sorted(set(r)), (name, bh, i)
                assert r[-1] == i
                assert all(0 <= c <= i for c in r)


def test_retrieval_row_contents():
    pat = P.retrieval_pattern(1, 1, 64 * 128, 8, seed=1)
    rows = rows_of(pat, 0)
    assert rows[0] == [0] and rows[1] == [0, 1]
    for i in range(2, 64):
        r = rows[i]
        assert i in r and i - 1 in r
        assert len(r) == 2 + min(8, i - 1)


def test_retrieval_deterministic_and_per_head():
    a = P.retrieval_pattern(2, 2, 2048, 8, seed=1)
    b = P.retrieval_pattern(2, 2, 2048, 8, seed=1)
    assert torch.equal(a.row_ptr, b.row_ptr) and torch.equal(a.col_idx, b.col_idx)
    assert not torch.equal(a.col_idx[0, 0], a.col_idx[0, 1])


def test_shared_equals_materialized():
    s = P.window_pattern(2, 3, 2048, 8, shared=True)
    m = P.window_pattern(2, 3, 2048, 8, shared=False)
    assert s.row_ptr.stride(0) == 0 and s.row_ptr.stride(1) == 0
    assert torch.equal(s.row_ptr.contiguous(), m.row_ptr)
    assert torch.equal(s.col_idx.contiguous()[..., : m.col_idx.shape[-1]], m.col_idx)


def test_prefix_window_rows():
    r = P.prefix_window_rows(10, 4, 4)
    assert r[0] == [0] and r[3] == [0, 1, 2, 3] and r[4] == [0, 1, 2, 3, 4]
    assert r[9] == [0, 1, 2, 3, 6, 7, 8, 9]


# --- the library's device CSR builder: host-side pieces (closed-form offsets, validation) ---
def _nnz(kind, nqb, prefix=0, window=0, n_random=0):
    import ctypes
    from usagi_b200 import _lib
    v = ctypes.c_int64(-1)
    rc = _lib.load().bsattn_csr_nnz(kind, nqb, prefix, window, n_random, ctypes.byref(v))
    return rc, v.value


def test_device_builder_row_offsets_match_host_builder():
    """row_ptr[i] of the device builder is the column count of the first i rows, i.e. nnz of a
    pattern with i rows; it must equal the host builder's row_ptr for every i."""
    from usagi_b200 import _lib
    n = 70
    cases = [(_lib.CSR_WINDOW, dict(window=8), P.window_pattern(1, 1, n * 128, 8)),
             (_lib.CSR_WINDOW, dict(window=1), P.window_pattern(1, 1, n * 128, 1)),
             (_lib.CSR_PREFIX_WINDOW, dict(prefix=4, window=4), P.prefix_window_pattern(1, 1, n * 128, 4, 4)),
             (_lib.CSR_PREFIX_WINDOW, dict(prefix=8, window=8), P.prefix_window_pattern(1, 1, n * 128, 8, 8)),
             (_lib.CSR_RETRIEVAL, dict(n_random=8), P.retrieval_pattern(1, 1, n * 128, 8)),
             (_lib.CSR_RETRIEVAL, dict(n_random=16), P.retrieval_pattern(1, 1, n * 128, 16))]
    for kind, kw, pat in cases:
        rp = pat.row_ptr.reshape(-1)
        for i in range(1, n + 1):
            rc, v = _nnz(kind, i, **kw)
            assert rc == 0 and v == int(rp[i]), (kind, kw, i, v, int(rp[i]))


def test_device_builder_validation():
    from usagi_b200 import _lib
    lib = _lib.load()
    assert _nnz(7, 8, window=4)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_WINDOW, 0, window=4)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_WINDOW, 8, window=0)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_WINDOW, 8, prefix=2, window=4)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_RETRIEVAL, 8, n_random=65)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_RETRIEVAL, 8, n_random=-1)[0] == _lib.E_SHAPE
    assert lib.bsattn_csr_nnz(_lib.CSR_WINDOW, 8, 0, 4, 0, None) == _lib.E_NULL
    # argument errors are returned before anything touches a device
    assert lib.bsattn_build_csr(_lib.CSR_WINDOW, 8, 0, 4, 0, 1, 1, None, 16, 64, None) == _lib.E_NULL
    assert lib.bsattn_build_csr(_lib.CSR_WINDOW, 8, 0, 4, 0, 1, 1, 16, 16, 3, None) == _lib.E_SHAPE
    assert lib.bsattn_build_csr(_lib.CSR_WINDOW, 8, 0, 4, 0, 1, 0, 16, 16, 64, None) == _lib.E_SHAPE
    # prefix + window past INT_MAX (it would wrap the row arithmetic) is rejected up front
    big = 2 ** 31 - 2
    assert _nnz(_lib.CSR_PREFIX_WINDOW, 8, prefix=2, window=big)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_PREFIX_WINDOW, 8, prefix=big, window=2)[0] == _lib.E_SHAPE
    assert _nnz(_lib.CSR_WINDOW, 8, window=2 ** 24 + 1)[0] == _lib.E_SHAPE
    assert lib.bsattn_build_csr(_lib.CSR_PREFIX_WINDOW, 8, 2, big, 0, 1, 1, 16, 16, 64,
                                None) == _lib.E_SHAPE
    # the largest accepted window still gives the closed-form count (every row is 0 .. i)
    assert _nnz(_lib.CSR_PREFIX_WINDOW, 8, prefix=2 ** 24, window=2 ** 24) == (0, 36)
