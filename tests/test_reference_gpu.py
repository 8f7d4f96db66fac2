# SPDX-License-Identifier: MIT
"""The reference's own GPU engine (beamgrad 2.3.0 cuda/dbs_cuda.cu, built unmodified for
sm_100a by oracle/Makefile) against this engine and the CPU oracle, through the same C ABI.

The reference engine is the GPU speed bar bench.py times beside this engine; these cases
show that both engines compute the same decode (the reference's device suite checks its
engine against its CPU library the same way, tests/cuda_device_tests.cpp:200-229).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _cases import make_problem, random_case
from beamgrad_b200 import _abi as A
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import _gpu as G

FIELDS = oracle.TRACE_FIELDS + ("row_lse", "invalid")


@pytest.fixture(scope="module")
def ref_lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not oracle.ref_cuda_available():
        pytest.skip("the reference GPU engine was not built (needs the reference sources)")
    lib = oracle.ref_cuda_lib()
    assert lib.dbs_cuda_available() == 1
    return lib


def _same(a: dict, b: dict, ctx: str):
    for f in FIELDS:
        x, y = np.ascontiguousarray(a[f]), np.ascontiguousarray(b[f])
        assert x.shape == y.shape and x.tobytes() == y.tobytes(), f"{ctx}: field {f} differs"


@pytest.mark.parametrize("seed", range(12))
def test_reference_engine_equals_this_engine(ref_lib, seed):
    pb = random_case(3000 + seed, allow_per_example=False)
    ref = G.engine_decode(pb, lib=ref_lib)
    _same(G.engine_decode(pb), ref, f"seed {seed}")
    _same(oracle.oracle_decode(pb), ref, f"seed {seed} (oracle)")


def test_reference_engine_on_c2_rows(ref_lib):
    # BASELINE configs[1] rows (bf16 logits, K = 8, V = 32000, eos 2, alpha 1) for two examples.
    pb = make_problem(2, 16, 8, 32000, dtype=A.DTYPE_BF16, from_logits=True, seed=77, eos=2, alpha=1.0)
    ref = G.engine_decode(pb, lib=ref_lib)
    _same(G.engine_decode(pb), ref, "C2 rows")
