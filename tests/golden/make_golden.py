"""Generate tests/golden/*.npz from the reference's own Triton kernels.

Runs ``block_sparse_attn_fwd`` of sissississi-013/usagi (kernels v4, v7 and v1) under
``TRITON_INTERPRET=1`` on CPU tensors -- the reference executing its own code path -- for each
case in ``cases.py`` and stores the reference's outputs (o as bf16 bit patterns, lse fp32).

This script needs a checkout of the reference, named by $USAGI_REFERENCE; the committed fixtures
are what the tests read, so nothing at test time touches the reference.

    USAGI_REFERENCE=<reference checkout> TRITON_INTERPRET=1 python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.environ.get("USAGI_REFERENCE")
if not REF:
    raise SystemExit("set USAGI_REFERENCE to the reference checkout")
KERNELS = {
    "v4": "kernels/v4_leaderboard_0740ms.py",
    "v7": "kernels/v7_blockptr_warpspec.py",
    "v1": "kernels/v1_baseline.py",
}


def load_module(tag):
    path = os.path.join(REF, KERNELS[tag])
    spec = importlib.util.spec_from_file_location(f"usagi_ref_{tag}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    mods = {t: load_module(t) for t in KERNELS}
    meta = {}
    for name in cases.CASES:
        c = cases.case(name)
        B, H, T, D = c["q"].shape
        sl = c["seq_lens"] if c["seq_lens"] is not None else torch.full((B,), T, dtype=torch.int32)
        outs = {}
        for tag, mod in mods.items():
            o, lse = mod.block_sparse_attn_fwd(c["q"], c["k"], c["v"], c["row_ptr"], c["col_idx"], sl)
            outs[tag] = (o.clone(), lse.clone())
        o4, l4 = outs["v4"]
        agree = {}
        for tag in ("v7", "v1"):
            o, l = outs[tag]
            # v1 only writes rows < seq_len (masked store, :435-441) into zero/-inf initialised
            # buffers, so it matches v4 on every element.
            agree[tag] = bool(torch.equal(o.view(torch.int16), o4.view(torch.int16))
                              and torch.equal(l, l4))
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            o_bf16_bits=o4.contiguous().view(torch.int16).numpy(),
            lse=l4.contiguous().numpy(),
            q_sum=np.float64(cases.checksum(c["q"])),
            k_sum=np.float64(cases.checksum(c["k"])),
            v_sum=np.float64(cases.checksum(c["v"])),
        )
        meta[name] = {"shape": [B, H, T, D], "dtype": str(c["q"].dtype), "v7_equal_v4": agree["v7"],
                      "v1_equal_v4": agree["v1"]}
        print(name, meta[name], flush=True)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump({"generator": "reference kernels under TRITON_INTERPRET=1",
                   "triton": __import__("triton").__version__, "torch": torch.__version__,
                   "cases": meta}, f, indent=1)


if __name__ == "__main__":
    main()
