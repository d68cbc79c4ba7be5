"""Generate tests/golden/full_*.npz: the reference's own outputs at the benchmark sizes.

The small fixtures of ``make_golden.py`` pin the oracle at T <= 1024.  These pin the kernel at
the benchmark configurations themselves, on their exact seeded inputs (``cases.full_inputs``):

* the three families at B=2, H=16, T=8192 (q, k, v ~ N(0,1) fp32 from CPU seed 0, drawn in the
  order q, k, v, cast to fp16; retrieval rows from seed 1);
* the scaling mix at B=4, H=32, T=32768 (same draw at its shape; heads cycle through window16,
  prefix8+window8 and retrieval 2+16 by head index).

For each selected (b, h) the reference's ``block_sparse_attn_fwd`` (kernels v4, under
``TRITON_INTERPRET=1`` on CPU tensors) runs on the single-head slice of those inputs with that
head's pattern; heads are independent in the reference (one program per (query block, head),
v4 :31-61), so the slice gives the head's output of the full call.  Stored per head: o as bf16
bit patterns for the selected query blocks (all of them for the family heads), lse, and checksums
of the head's q, k, v slices and CSR rows, which the tests use to detect generator drift.

    USAGI_REFERENCE=<reference checkout> TRITON_INTERPRET=1 python tests/golden/make_golden_full.py [case ...]
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import time

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.environ.get("USAGI_REFERENCE")
V4 = "kernels/v4_leaderboard_0740ms.py"


def load_v4():
    spec = importlib.util.spec_from_file_location("usagi_ref_v4", os.path.join(REF, V4))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_case(mod, name, inputs):
    spec = cases.FULL_CASES[name]
    q, k, v, pat = inputs[spec["config"]][0], inputs[spec["config"]][1], \
        inputs[spec["config"]][2], cases.full_pattern(name, inputs)
    heads = {}
    for (b, h) in spec["heads"]:
        sl = cases.head_slice(q, k, v, pat, b, h)
        T = sl["q"].shape[2]
        # The reference caches its int32 metadata by data_ptr() (v4 :155-164); a new head's
        # tensors can reuse a freed address, so the cache is emptied before every call.
        mod._meta_cache.clear()
        t0 = time.time()
        o, lse = mod.block_sparse_attn_fwd(sl["q"], sl["k"], sl["v"], sl["row_ptr"],
                                           sl["col_idx"], torch.tensor([T], dtype=torch.int32))
        dt = time.time() - t0
        qbs = spec["qblocks"] if spec["qblocks"] is not None else list(range(T // 128))
        rows = torch.cat([torch.arange(qb * 128, qb * 128 + 128) for qb in qbs])
        heads[f"{b}_{h}"] = dict(
            o_bf16_bits=o[0, 0][rows].contiguous().view(torch.int16).numpy(),
            lse=lse[0, 0][rows].contiguous().numpy(),
            qblocks=np.asarray(qbs, dtype=np.int32),
            sums=np.asarray(cases.head_checksums(sl), dtype=np.float64),
        )
        print(f"{name} head ({b},{h}): {dt:.1f} s", flush=True)
    arrays = {}
    for key, d in heads.items():
        for f, a in d.items():
            arrays[f"{key}__{f}"] = a
    np.savez_compressed(os.path.join(HERE, f"full_{name}.npz"), **arrays)
    return {"heads": spec["heads"], "config": spec["config"],
            "qblocks": "all" if spec["qblocks"] is None else spec["qblocks"]}


def main():
    if not REF:
        raise SystemExit("set USAGI_REFERENCE to the reference checkout")
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    names = sys.argv[1:] or list(cases.FULL_CASES)
    mod = load_v4()
    meta_path = os.path.join(HERE, "golden_full_meta.json")
    meta = {}
    if os.path.exists(meta_path):
        with open(meta_path) as f:
            meta = json.load(f).get("cases", {})
    inputs = {}
    for name in names:
        cfg = cases.FULL_CASES[name]["config"]
        if cfg not in inputs:
            inputs.clear()  # the mix inputs take ~3 GB in fp16: keep one configuration at a time
            t0 = time.time()
            inputs[cfg] = cases.full_inputs(cfg)
            print(f"inputs {cfg}: {time.time() - t0:.1f} s", flush=True)
        meta[name] = run_case(mod, name, inputs)
    with open(meta_path, "w") as f:
        json.dump({"generator": "reference kernel v4 under TRITON_INTERPRET=1, single-head slices",
                   "triton": __import__("triton").__version__, "torch": torch.__version__,
                   "cases": meta}, f, indent=1)


if __name__ == "__main__":
    main()
