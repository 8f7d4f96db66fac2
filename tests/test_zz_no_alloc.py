# SPDX-License-Identifier: MIT
"""dbs_cuda_decode_no_alloc: the decode for callers that may not allocate device memory.

Some callers (an inference runtime's plugin enqueue, a serving loop with a fixed memory
budget) must not allocate while they run and have no buffer to pass as workspace. This
entry point runs the same decode on a fixed 4 MiB device array owned by the library. These
tests call it through the C ABI and check that its outputs equal those of
dbs_cuda_decode_ex2 (given a workspace of its own) bit for bit, on two calls in a row that
share the array, and that a decode needing more scratch than the array holds is refused.

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from beamgrad_b200 import _abi as A
from _cases import make_problem
from _gpu import DeviceProblem, _out_struct, _outputs, engine_decode, ptr, stream_ptr

pytestmark = pytest.mark.gpu


def no_alloc_decode(pb) -> dict[str, np.ndarray]:
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    o = _outputs(B, T, K)
    args = dp.args()
    opts = pb.options()
    rc = lib.dbs_cuda_decode_no_alloc(ptr(dp.x), pb.dtype, int(pb.from_logits), C.byref(args),
                                      C.byref(opts) if opts is not None else None, C.byref(_out_struct(o)),
                                      ptr(o["row_lse"]), stream_ptr())
    A.check(rc, "decode_no_alloc")
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in o.items()}


def assert_same(got, want):
    for name, w in want.items():
        np.testing.assert_array_equal(got[name].view(np.uint8), w.view(np.uint8), err_msg=name)


def test_two_calls_in_a_row_match_decode_ex2():
    # The first call leaves its state in the shared array; the second, of another shape with
    # n-gram prefixes in the array, must not see it.
    first = make_problem(4, 12, 8, 5003, dtype=A.DTYPE_BF16, from_logits=True, seed=21, eos=2, alpha=1.0)
    second = make_problem(3, 9, 5, 777, dtype=A.DTYPE_F16, from_logits=False, seed=22, eos=4, min_length=2,
                          alpha=0.6, ngram=2, rep_penalty=1.3, extra_eos=(7,))
    for pb in (first, second):
        ws = A.load().dbs_cuda_decode_workspace_size(C.byref(pb.args()))
        assert 0 < ws <= A.NO_ALLOC_SCRATCH_BYTES
        assert_same(no_alloc_decode(pb), engine_decode(pb))


def test_scratch_beyond_the_array_is_refused():
    lib = A.load()
    pb = make_problem(64, 2, 128, 4, seed=1)
    need = lib.dbs_cuda_decode_workspace_size(C.byref(pb.args()))
    assert need > A.NO_ALLOC_SCRATCH_BYTES
    dp = DeviceProblem(pb)
    o = _outputs(*pb.shape[:3])
    rc = lib.dbs_cuda_decode_no_alloc(ptr(dp.x), pb.dtype, 0, C.byref(dp.args()), None, C.byref(_out_struct(o)),
                                      None, stream_ptr())
    assert rc == 2  # DBS_CUDA_STATUS_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert (o["final_scores"] == 12345.0).all()
