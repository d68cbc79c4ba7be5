"""usagi_b200 -- B200-native (sm_100a) block-sparse causal attention forward.

Drop-in for the ``block_sparse_attn_fwd`` submission API of sissississi-013/usagi
(kernels/v4_leaderboard_0740ms.py:25, :189, :242), backed by a hand-written tcgen05/TMA kernel in
``libbsattn.so`` (C ABI: include/bsattn.h).
"""
from .api import (  # noqa: F401
    VARIANT_MANIFEST,
    BsattnError,
    Plan,
    block_sparse_attn_fwd,
    block_sparse_attn_fwd_into,
    block_sparse_attn_fwd_window,
    make_plan,
    make_window_plan,
    check_errors,
    set_timeout_ns,
    setup,
)
from . import patterns  # noqa: F401

__version__ = "0.1.0"
