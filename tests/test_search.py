# SPDX-License-Identifier: MIT
"""The device-resident search loop (beamgrad_b200.search) against beamgrad's loop semantics
(python/beamgrad/_search.py:330-467 of beamgrad 2.3.0): the trace and final beams equal the CPU
oracle's decode of the rows the loop consumed, bit for bit, and the sequences equal the loop's own
gather + cat rule; the loop stops where beamgrad's does; a whole search captured in one CUDA
graph replays to the same results on new inputs.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from _cases import make_problem
from beamgrad_b200 import _abi as A
from beamgrad_b200 import search as S
from oracle import oracle

TORCH_DTYPE = {A.DTYPE_F32: torch.float32, A.DTYPE_F16: torch.float16, A.DTYPE_BF16: torch.bfloat16}


def test_cpu_device_rejected():
    with pytest.raises(ValueError):
        S.DeviceSearch(2, 4, 10, 5, device="cpu")
    with pytest.raises(ValueError):
        S.beam_search(lambda st: None, 2, 4, 5, check_every=0)


def sequences_rule(trace: dict, T: int, max_steps: int) -> np.ndarray:
    """beamgrad's per-step sequence update (python/beamgrad/_search.py:450-455), in numpy."""
    tokens, parents, flp = trace["tokens"], trace["parents"], trace["from_logprob"]
    B, _, K = tokens.shape
    seq = np.zeros((B, K, 0), np.int64)
    for t in range(T):
        par = parents[:, t].astype(np.int64)
        src = np.clip(par, 0, None)
        gathered = np.take_along_axis(seq, src[..., None].repeat(t, 2), 1) if t else seq
        emitted = np.where(flp[:, t] != 0, tokens[:, t], -1).astype(np.int64)
        seq = np.concatenate([gathered, emitted[..., None]], 2)
        seq = np.where((par >= 0)[..., None], seq, -1)
    return np.concatenate([seq, np.full((B, K, max_steps - T), -1, np.int64)], 2)


def to_dev(pb) -> torch.Tensor:
    x = torch.from_numpy(np.ascontiguousarray(pb.x).copy())
    if pb.dtype != A.DTYPE_F32:
        x = x.view(torch.int16).view(TORCH_DTYPE[pb.dtype])
    return x.cuda()


def options(pb) -> dict:
    banned = None if pb.banned is None else [int(i) for i in np.nonzero(pb.banned)[0]]
    return dict(from_logits=pb.from_logits, eos_token=pb.eos, extra_eos=tuple(pb.extra_eos),
                min_length=pb.min_length, length_penalty_alpha=pb.alpha, banned_tokens=banned,
                no_repeat_ngram_size=pb.ngram, repetition_penalty=pb.rep_penalty)


def check_against_oracle(pb, res, T_run: int, max_steps: int):
    ref = oracle.oracle_decode(dataclasses.replace(pb, x=np.ascontiguousarray(pb.x[:, :T_run])))
    tr = res.trace
    got = {"final_scores": tr.final_scores, "final_raw_scores": tr.final_raw_scores,
           "final_lengths": tr.final_lengths.int(), "tokens": tr.tokens.int(), "parents": tr.parents.int(),
           "lengths": tr.lengths.int(), "scores": tr.scores, "raw_scores": tr.raw_scores,
           "from_logprob": tr.from_logprob.to(torch.uint8)}
    for f, v in got.items():
        a = v.cpu().numpy()
        assert a.tobytes() == np.ascontiguousarray(ref[f]).tobytes(), f
    if pb.from_logits:
        assert res.row_lse.cpu().numpy().tobytes() == ref["row_lse"].tobytes()
    assert np.array_equal(res.sequences.cpu().numpy(), sequences_rule(ref, T_run, max_steps))


CASES = [
    dict(B=3, T=7, K=4, V=50, dtype=A.DTYPE_F32, eos=2, min_length=2, alpha=0.6),
    dict(B=2, T=6, K=8, V=1000, dtype=A.DTYPE_BF16, from_logits=True, eos=2, alpha=1.0),
    dict(B=2, T=8, K=5, V=40, dtype=A.DTYPE_F16, eos=3, ngram=2, rep_penalty=1.5, banned_frac=0.05),
    dict(B=3, T=6, K=3, V=30, dtype=A.DTYPE_F32, eos=1, extra_eos=(4, 7), alpha=0.3),
    dict(B=2, T=5, K=33, V=300, dtype=A.DTYPE_F32, eos=5),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("check_every", [1, 3])
def test_search_matches_oracle(case, check_every):
    c = dict(CASES[case])
    B, T, K, V = c.pop("B"), c.pop("T"), c.pop("K"), c.pop("V")
    pb = make_problem(B, T, K, V, seed=40 + case, **c)
    x = to_dev(pb)
    seen = []

    def step_fn(st):
        # The state handed to the model: beamgrad's BeamState fields, on the device.
        if st.step > 0:
            assert st.sequences.shape == (B, K, st.step) and st.sequences.dtype == torch.long
            assert st.active.dtype == torch.bool and st.parents.shape == (B, K)
        seen.append(st.step)
        return x[:, st.step].contiguous()

    res = S.beam_search(step_fn, B, K, T, check_every=check_every, validate=False, **options(pb))
    T_run = int(res.trace.steps[0])
    assert seen == list(range(len(seen))) and len(seen) >= T_run
    if check_every == 1:
        assert len(seen) == T_run
    check_against_oracle(pb, res, T_run, T)


@pytest.mark.gpu
@pytest.mark.parametrize("check_every", [1, 4])
def test_search_stops_when_all_beams_finish(check_every):
    """Rows that favour EOS: every beam finishes early; the loop stops where beamgrad's does and
    extra steps (check_every > 1) leave the result unchanged."""
    B, T, K, V, eos = 3, 12, 4, 20, 2
    pb = make_problem(B, T, K, V, seed=7, eos=eos, alpha=0.6)
    pb.x[..., eos] = -0.05  # EOS nearly certain from the first step on
    x = to_dev(pb)
    calls = []

    def step_fn(st):
        calls.append(st.step)
        return x[:, st.step].contiguous()

    res = S.beam_search(step_fn, B, K, T, check_every=check_every, eos_token=eos, length_penalty_alpha=0.6)
    T_run = int(res.trace.steps[0])
    assert T_run < T
    full = oracle.oracle_decode(pb)
    live = np.isfinite(full["raw_scores"]) & (full["tokens"] != eos) & (full["from_logprob"] == 1)
    expect = next(t + 1 for t in range(T) if not live[:, t].any())  # beamgrad stops before step t+1
    assert T_run == expect
    assert len(calls) == T_run if check_every == 1 else len(calls) >= T_run
    check_against_oracle(pb, res, T_run, T)


@pytest.mark.gpu
def test_search_flags_invalid_rows():
    B, T, K, V = 2, 4, 3, 30
    pb = make_problem(B, T, K, V, seed=3, eos=-1)
    pb.x[1, 0, 0, 5] = np.nan
    x = to_dev(pb)
    with pytest.raises(ValueError, match="example 1"):
        S.beam_search(lambda st: x[:, st.step].contiguous(), B, K, T)


@pytest.mark.gpu
def test_whole_search_in_one_cuda_graph():
    """reset + T steps (input copy, search step, prefix advance) captured once; replays on new
    inputs give the eager results bit for bit."""
    B, T, K, V = 4, 10, 8, 2000
    pb = make_problem(B, T, K, V, dtype=A.DTYPE_BF16, from_logits=True, seed=11, eos=2, alpha=1.0)
    pb2 = make_problem(B, T, K, V, dtype=A.DTYPE_BF16, from_logits=True, seed=12, eos=2, alpha=1.0)
    opts = dict(from_logits=True, eos_token=2, length_penalty_alpha=1.0)
    src = to_dev(pb)                       # the model's outputs, at a fixed address
    rows = torch.empty((B, K, V), dtype=torch.bfloat16, device="cuda")
    search = S.DeviceSearch(B, K, V, T, dtype=torch.bfloat16, **opts)

    def run():
        search.reset()
        for t in range(T):
            rows.copy_(src[:, t])          # stands in for the model's step
            search.step(rows)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()                              # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    for p in (pb, pb2):
        src.copy_(to_dev(p))
        g.replay()
        torch.cuda.synchronize()
        res = search.result()
        check_against_oracle(p, res, int(res.trace.steps[0]), T)
