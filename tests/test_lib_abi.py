"""The C-ABI library loads and exports every symbol include/bsattn.h declares; argument checks
that run before any CUDA call behave as documented (CPU only, no compute calls)."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from usagi_b200 import _lib, api

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "bsattn.h")).read()
    return sorted(set(re.findall(r"BSATTN_API\s+[\w\s\*]+?\b(bsattn_\w+)\s*\(", src)))


def test_header_declares_abi():
    syms = header_symbols()
    assert set(syms) == set(_lib.SIGNATURES), syms


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    for s in header_symbols():
        assert hasattr(lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.library_path())],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (bsattn_\w+)", out))
    assert set(header_symbols()) <= exported


def test_library_is_sm100a_only_and_driver_free():
    out = subprocess.run(["ldd", str(_lib.library_path())], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "libcudart.so" not in out  # static cudart, driver at run time


def test_version_workspace_strerror():
    lib = _lib.load()
    assert lib.bsattn_version() == 102
    assert lib.bsattn_workspace_bytes() >= 4
    for code in range(0, -12, -1):
        assert _lib.strerror(code) != "unknown error"
    assert _lib.strerror(-99) == "unknown error"


def _call(**kw):
    lib = _lib.load()
    a = dict(q=16, k=16, v=16, o=16, lse=None, rp=16, ci=16, sl=None, B=1, H=1, T=128, D=128,
             rps=0, cis=0, nnz=1, scale=0.0, od=0, ws=16, wsb=256, stream=None)
    a.update(kw)
    return lib.bsattn_fwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["rp"], a["ci"], a["sl"],
                          a["B"], a["H"], a["T"], a["D"], a["rps"], a["cis"], a["nnz"],
                          a["scale"], a["od"], a["ws"], a["wsb"], a["stream"])


def test_argument_validation_before_device():
    assert _call(q=None) == _lib.E_NULL
    assert _call(rp=None) == _lib.E_NULL
    assert _call(T=200) == _lib.E_SHAPE
    assert _call(D=64) == _lib.E_SHAPE
    assert _call(B=0) == _lib.E_SHAPE
    assert _call(nnz=-1) == _lib.E_SHAPE
    assert _call(od=7) == _lib.E_DTYPE
    assert _call(od=4) == _lib.E_DTYPE
    assert _call(q=24) == _lib.E_ALIGN
    assert _call(ws=None) == _lib.E_WORKSPACE
    assert _call(wsb=4) == _lib.E_WORKSPACE


def test_window_entry_validation_before_device():
    lib = _lib.load()

    def call(**kw):
        a = dict(q=16, sl=None, B=1, H=1, T=128, D=128, window=4, glob=0, od=0, plan=None, pg=0,
                 ws=16, wsb=256)
        a.update(kw)
        return lib.bsattn_fwd_window(a["q"], 16, 16, 16, None, a["sl"], a["B"], a["H"], a["T"],
                                     a["D"], a["window"], a["glob"], 0.0, a["od"], a["plan"],
                                     a["pg"], a["ws"], a["wsb"], None)

    assert call(window=0) == _lib.E_SHAPE
    assert call(window=-3) == _lib.E_SHAPE
    assert call(glob=-1) == _lib.E_SHAPE
    assert call(q=None) == _lib.E_NULL
    assert call(T=200) == _lib.E_SHAPE
    assert call(D=64) == _lib.E_SHAPE
    assert call(od=4) == _lib.E_DTYPE
    assert call(q=24) == _lib.E_ALIGN
    assert call(wsb=4) == _lib.E_WORKSPACE
    assert call(plan=16, pg=0) == _lib.E_PLAN
    assert call(plan=18, pg=1) == _lib.E_PLAN


def test_bf16_converter_validation_before_device():
    lib = _lib.load()
    assert lib.bsattn_bf16_to_f16(None, 16, 8, None) == _lib.E_NULL
    assert lib.bsattn_bf16_to_f16(16, 32, 12, None) == _lib.E_SHAPE
    assert lib.bsattn_bf16_to_f16(16, 32, -8, None) == _lib.E_SHAPE
    assert lib.bsattn_bf16_to_f16(24, 32, 8, None) == _lib.E_ALIGN
    assert lib.bsattn_bf16_to_f16(16, 32, 0, None) == _lib.OK


def test_python_api_dtype_rules():
    q = torch.zeros(1, 1, 128, 128, dtype=torch.float16)
    rp = torch.tensor([0, 1], dtype=torch.int32)
    ci = torch.tensor([0], dtype=torch.int32)
    for qq, kk, vv in ((q.bfloat16(), q, q), (q.float(), q.float(), q.float()),
                       (q, q, q.bfloat16())):
        with pytest.raises(TypeError):
            api.block_sparse_attn_fwd(qq, kk, vv, rp, ci)


def test_python_api_refuses_cpu_tensors():
    q = torch.zeros(1, 1, 128, 128, dtype=torch.float16)
    rp = torch.tensor([0, 1], dtype=torch.int32)
    ci = torch.tensor([0], dtype=torch.int32)
    with pytest.raises(ValueError, match="no CPU path"):
        api.block_sparse_attn_fwd(q, q, q, rp, ci)


def test_bh_view_strides():
    B, H = 2, 3
    full = torch.arange(B * H * 5, dtype=torch.int32).reshape(B, H, 5)
    t, s = api._bh_view(full, B, H, "x")
    assert s == 5 and t.data_ptr() == full.data_ptr()
    shared = torch.arange(5, dtype=torch.int32).reshape(1, 1, 5).expand(B, H, 5)
    t, s = api._bh_view(shared, B, H, "x")
    assert s == 0
    t, s = api._bh_view(torch.arange(5, dtype=torch.int64), B, H, "x")
    assert s == 0 and t.dtype == torch.int32
    t, s = api._bh_view(full.reshape(B * H, 5), B, H, "x")
    assert s == 5
    nc = full.transpose(0, 1)  # [H, B, 5] viewed as wrong layout for B,H -> must reject shape
    with pytest.raises(ValueError):
        api._bh_view(nc, B, H, "x")
    with pytest.raises(ValueError):
        api._bh_view(torch.zeros(4, 5, dtype=torch.int32), B, H, "x")


def test_bh_view_noncontiguous_copies():
    B, H = 2, 3
    base = torch.arange(H * B * 5, dtype=torch.int32).reshape(H, B, 5).transpose(0, 1)
    t, s = api._bh_view(base, B, H, "x")
    flat = t.contiguous().reshape(-1) if s else t.reshape(-1)
    assert s == 5
    # head (b, h) must read row_ptr + (b*H + h) * s
    for b in range(B):
        for h in range(H):
            assert torch.equal(flat[(b * H + h) * s:(b * H + h) * s + 5], base[b, h])
