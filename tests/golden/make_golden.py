# SPDX-License-Identifier: MIT
"""Regenerates tests/golden/*.npz from the reference CPU library (oracle/_ref/libdbs.so,
compiled from beamgrad 2.3.0's own sources by oracle/Makefile).

Each fixture stores one problem's inputs and the reference's outputs (decode trace,
row_lse, dense backward). tests/test_oracle.py checks the C restatement against them,
which also works where the reference tree is absent (the GPU box).

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from _cases import make_problem  # noqa: E402
from oracle import oracle  # noqa: E402
from beamgrad_b200 import _abi as A  # noqa: E402

CASES = {
    # name: make_problem kwargs
    "c1_small": dict(B=2, T=8, K=4, V=100, seed=0, eos=2, alpha=0.6, min_length=4),
    "logits_bf16": dict(B=2, T=6, K=4, V=300, dtype=A.DTYPE_BF16, from_logits=True, seed=1, eos=3, alpha=1.0),
    "logits_f16_constrained": dict(B=2, T=6, K=3, V=257, dtype=A.DTYPE_F16, from_logits=True, seed=2, eos=-1,
                                   ngram=2, rep_penalty=1.5, banned_frac=0.02),
    "ties_extra_eos": dict(B=3, T=7, K=5, V=31, mode="ties", seed=3, eos=4, min_length=2, alpha=0.6,
                           extra_eos=(7, 9), variable_steps=True),
    "neginf_large_k": dict(B=1, T=4, K=33, V=64, mode="neginf", seed=4, eos=1, alpha=1.3),
    "naninf": dict(B=2, T=5, K=4, V=128, mode="naninf", seed=5, eos=0),
}


def reference_outputs(pb: oracle.Problem) -> dict[str, np.ndarray]:
    with oracle.RefDecoder(pb) as d:
        out = d.decode()
        B, T, K, V = pb.shape
        rng = np.random.default_rng(17)
        g = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32),
             "scores": rng.uniform(-1, 1, (B, T, K)).astype(np.float32)}
        logits = pb.x if pb.from_logits else None
        row_lse = out["row_lse"] if pb.from_logits else None
        grad = d.backward(out, g, logits=logits, row_lse=row_lse)
    out.pop("invalid")
    out["grad"] = grad
    out["g_final_scores"] = g["final_scores"]
    out["g_scores"] = g["scores"]
    return out


def main() -> None:
    oracle.build()
    for name, kw in CASES.items():
        pb = make_problem(**kw)
        out = reference_outputs(pb)
        meta = np.array([pb.dtype, int(pb.from_logits), pb.eos, pb.min_length, pb.ngram], np.int32)
        fl = np.array([pb.alpha, pb.rep_penalty], np.float32)
        extra = np.array(pb.extra_eos, np.int32)
        arrays = dict(x=pb.x, meta=meta, fl=fl, extra=extra, **{f"out_{k}": v for k, v in out.items()})
        if pb.steps is not None:
            arrays["steps"] = pb.steps
        if pb.banned is not None:
            arrays["banned"] = pb.banned
        path = Path(__file__).parent / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
