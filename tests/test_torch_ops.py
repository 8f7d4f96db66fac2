# SPDX-License-Identifier: MIT
"""torch.ops.beamgrad.* on the engine (beamgrad_b200._C_cuda), the drop-in for beamgrad's
own _C_cuda (python/csrc/cuda_ops.cpp of beamgrad 2.3.0, tested there by
python/tests/test_cuda.py): every output against the CPU oracle bit for bit, argument
errors as ValueError, and no CPU fallback.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _cases import make_problem
from beamgrad_b200 import _abi as A
from beamgrad_b200 import ops
from oracle import oracle

OUT_EX = oracle.TRACE_FIELDS + ("row_lse",)
TORCH_DTYPE = {A.DTYPE_F32: torch.float32, A.DTYPE_F16: torch.float16, A.DTYPE_BF16: torch.bfloat16}


def test_module_registers_cuda_kernels_without_a_device():
    m = ops.load()
    assert m.max_beam_size() == 1024
    assert m.device_available() == torch.cuda.is_available()
    for name in ops.OPERATORS:
        assert torch._C._dispatch_has_kernel_for_dispatch_key(f"beamgrad::{name}", "CUDA"), name


def test_cpu_tensors_have_no_fallback():
    ops.load()
    if torch._C._dispatch_has_kernel_for_dispatch_key("beamgrad::length_penalty", "CPU"):
        pytest.skip("beamgrad's own CPU kernels are registered in this process")
    with pytest.raises(NotImplementedError):
        torch.ops.beamgrad.length_penalty(torch.ones(3, dtype=torch.int32), 1.0)


# ---------------------------------------------------------------------------- GPU


def to_dev(pb: oracle.Problem) -> torch.Tensor:
    x = torch.from_numpy(np.ascontiguousarray(pb.x).copy())
    if pb.dtype != A.DTYPE_F32:
        x = x.view(torch.int16).view(TORCH_DTYPE[pb.dtype])
    return x.cuda()


def same(a: torch.Tensor, b: np.ndarray, what: str):
    a = a.cpu().numpy()
    assert a.shape == b.shape, what
    assert a.tobytes() == np.ascontiguousarray(b).tobytes(), what


def run_decode_ex(pb: oracle.Problem, validate=True):
    steps = torch.from_numpy(pb.steps).cuda() if pb.steps is not None else None
    banned = torch.from_numpy(pb.banned).cuda() if pb.banned is not None else None
    return torch.ops.beamgrad.decode_ex(to_dev(pb), pb.from_logits, steps, pb.eos, pb.min_length, pb.alpha, banned,
                                        pb.ngram, pb.rep_penalty, validate, list(pb.extra_eos))


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(8))
def test_decode_ex_parity(case):
    ops.load()
    dtype = [A.DTYPE_F32, A.DTYPE_F16, A.DTYPE_BF16][case % 3]
    pb = make_problem(3, 6, [1, 4, 8, 16, 33][case % 5], 301 + 37 * case, dtype=dtype, from_logits=case % 2 == 0,
                      seed=70 + case, eos=4, min_length=case % 3, alpha=0.6 * (case % 3), ngram=2 if case == 5 else 0,
                      rep_penalty=1.4 if case == 6 else 1.0, banned_frac=0.02 if case in (3, 6) else 0.0,
                      extra_eos=(9,) if case == 7 else (), variable_steps=case in (2, 7))
    ref = oracle.oracle_decode(pb)
    ours = run_decode_ex(pb)
    for name, t in zip(OUT_EX, ours):
        same(t, ref[name], name)


@pytest.mark.gpu
def test_decode_float32_parity():
    ops.load()
    pb = make_problem(4, 7, 5, 1000, seed=3, eos=2, min_length=2, alpha=1.0)
    ref = oracle.oracle_decode(pb)
    ours = torch.ops.beamgrad.decode(to_dev(pb), None, pb.eos, pb.min_length, pb.alpha, None, 0, 1.0, True)
    assert len(ours) == 9
    for name, t in zip(oracle.TRACE_FIELDS, ours):
        same(t, ref[name], name)


@pytest.mark.gpu
def test_validate_and_argument_errors_are_value_errors():
    ops.load()
    pb = make_problem(3, 4, 2, 64, seed=3, eos=1)
    pb.x[1, 0, 0, 17] = np.nan  # row (b=1, t=0, k=0) is always read
    ref = oracle.oracle_decode(pb)
    assert ref["invalid"].tolist() == [0, 1, 0]
    with pytest.raises(ValueError, match="NaN or \\+inf"):
        run_decode_ex(pb, validate=True)
    run_decode_ex(pb, validate=False)  # no read-back, no error
    x = to_dev(make_problem(2, 3, 2, 16, seed=1))
    with pytest.raises(ValueError):
        torch.ops.beamgrad.decode_ex(x, False, torch.tensor([1, 4], device="cuda"), -1, 0, 0.0, None, 0, 1.0, False, [])
    with pytest.raises(ValueError):
        torch.ops.beamgrad.decode_ex(x, False, None, 16, 0, 0.0, None, 0, 1.0, False, [])
    with pytest.raises(ValueError):
        torch.ops.beamgrad.decode_ex(x, False, None, -1, 0, -1.0, None, 0, 1.0, False, [])
    with pytest.raises(ValueError):
        torch.ops.beamgrad.decode(x.double(), None, -1, 0, 0.0, None, 0, 1.0, False)


@pytest.mark.gpu
def test_decode_step_parity_and_inputs_untouched():
    ops.load()
    B, T, K, V = 3, 5, 4, 200
    pb = make_problem(B, T, K, V, seed=11, eos=3, min_length=1, alpha=0.6, ngram=2, rep_penalty=1.3)
    raw = np.full((B, K), -np.inf, np.float32)
    raw[:, 0] = 0.0
    lengths = np.zeros((B, K), np.int32)
    finished = np.zeros((B, K), np.uint8)
    prefixes = np.full((B, K, T), -1, np.int32)
    for t in range(T):
        step_pb = oracle.Problem(np.ascontiguousarray(pb.x[:, t:t + 1]), eos=pb.eos, min_length=pb.min_length,
                                 alpha=pb.alpha, ngram=pb.ngram, rep_penalty=pb.rep_penalty)
        ref = oracle.oracle_step(step_pb, raw, lengths, finished, prefixes)
        st = [torch.from_numpy(a.copy()).cuda() for a in (raw, lengths, finished, prefixes)]
        before = [s.clone() for s in st]
        out = torch.ops.beamgrad.decode_step(to_dev(step_pb)[:, 0], *st, pb.eos, pb.min_length, pb.alpha, None,
                                             pb.ngram, pb.rep_penalty, True, [])
        for s, s0 in zip(st, before):
            assert torch.equal(s, s0)
        tokens, parents, new_len, scores, new_raw, from_lp, new_fin, final = out
        same(tokens, ref["tokens"][:, 0], "tokens")
        same(parents, ref["parents"][:, 0], "parents")
        same(scores, ref["scores"][:, 0], "scores")
        same(from_lp, ref["from_logprob"][:, 0], "from_logprob")
        same(final, ref["final_scores"], "final_scores")
        same(new_raw, ref["state_raw"], "state raw")
        same(new_len, ref["state_lengths"], "state lengths")
        same(new_fin, ref["state_finished"], "state finished")
        # caller-side prefix bookkeeping: a slot continues its parent's prefix, plus the new token
        newp = np.full_like(prefixes, -1)
        for b in range(B):
            for k in range(K):
                par = ref["parents"][b, 0, k]
                if par >= 0:
                    L = lengths[b, par]
                    newp[b, k, :L] = prefixes[b, par, :L]
                    if ref["from_logprob"][b, 0, k]:
                        newp[b, k, L] = ref["tokens"][b, 0, k]
        prefixes = newp
        raw, lengths, finished = ref["state_raw"], ref["state_lengths"], ref["state_finished"]


@pytest.mark.gpu
@pytest.mark.parametrize("from_logits", [False, True])
def test_backward_operators_parity(from_logits):
    ops.load()
    pb = make_problem(3, 6, 4, 500, dtype=A.DTYPE_BF16 if from_logits else A.DTYPE_F32, from_logits=from_logits,
                      seed=21, eos=2, alpha=0.6, variable_steps=True)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    rng = np.random.default_rng(5)
    g_final = rng.uniform(-1, 1, (B, K)).astype(np.float32)
    g_scores = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
    dev = {k: torch.from_numpy(np.ascontiguousarray(trace[k])).cuda() for k in ("parents", "tokens", "lengths", "from_logprob")}
    steps = torch.from_numpy(pb.steps).cuda()
    gf = torch.from_numpy(g_final).cuda()
    args = (dev["parents"], dev["tokens"], dev["lengths"], dev["from_logprob"], steps, V, pb.alpha)
    if not from_logits:
        dense = torch.ops.beamgrad.final_scores_backward(gf, *args)
        same(dense, oracle.oracle_backward(pb, trace, {"final_scores": g_final}), "final_scores_backward")
        draws = torch.ops.beamgrad.final_scores_path_gradient(gf, *args)
        same(draws, oracle.oracle_path_gradient(pb, trace, g_final), "path gradient")
    logits = to_dev(pb) if from_logits else None
    lse = torch.from_numpy(trace["row_lse"]).cuda() if from_logits else None
    grad = torch.ops.beamgrad.decode_backward(gf, None, torch.from_numpy(g_scores).cuda(), None, *args, logits, lse)
    ref = oracle.oracle_backward(pb, trace, {"final_scores": g_final, "scores": g_scores},
                                 logits=pb.x if from_logits else None, row_lse=trace["row_lse"] if from_logits else None)
    same(grad, ref, "decode_backward")
    # The added operator writes the gradient in the input's dtype: decode_backward(...).to(dtype), bit for bit.
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        cast = torch.ops.beamgrad_b200.decode_backward_as(gf, None, torch.from_numpy(g_scores).cuda(), None, *args,
                                                          logits, lse, dt)
        assert cast.dtype == dt
        assert torch.equal(cast.cpu().view(torch.uint8), torch.from_numpy(ref).to(dt).view(torch.uint8)), dt


@pytest.mark.gpu
def test_length_penalty_parity():
    ops.load()
    lengths = np.arange(-3, 400, dtype=np.int64).reshape(13, 31)
    for alpha in (0.0, 0.6, 1.0, 2.5):
        ours = torch.ops.beamgrad.length_penalty(torch.from_numpy(lengths).cuda(), alpha)
        same(ours, oracle.oracle_length_penalty(np.clip(lengths, 0, None), alpha), f"alpha {alpha}")
