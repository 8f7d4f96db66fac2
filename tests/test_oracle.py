# SPDX-License-Identifier: MIT
"""Pins the CPU oracle (oracle/dbs_oracle.c) to the reference, bit for bit.

* the reference's own known-answer tests (beamgrad 2.3.0 tests/dbs_tests.cpp:128-142
  deterministic ties, :489-507 golden output; tests/internal_tests.cpp:1246-1262 length
  penalty vs pow, :814 exhaustive half conversions);
* committed golden fixtures (tests/golden/, made by tests/golden/make_golden.py from the
  reference library compiled from its sources);
* seeded random cases against that library itself (oracle/_ref/libdbs.so), when it is
  present (it is built wherever the reference sources are).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from _cases import make_problem, random_case
from beamgrad_b200 import _abi as A
from oracle import oracle

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")

FIELDS = oracle.TRACE_FIELDS + ("row_lse",)


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    return a.tobytes() == b.tobytes()


def test_golden_output_known_answer():
    # tests/dbs_tests.cpp:489-507: T=2, K=2, V=3, no EOS; tokens[0][0] == 0 and tokens[1][0] == 1.
    x = np.array([0.0, -1.0, -2.0, -3.0, -4.0, -5.0, -0.5, -0.1, -2.0, -0.2, -0.3, -2.0], np.float32).reshape(1, 2, 2, 3)
    out = oracle.oracle_decode(oracle.Problem(x))
    assert out["tokens"][0, 0, 0] == 0
    assert out["tokens"][0, 1, 0] == 1


def test_deterministic_ties_known_answer():
    # tests/dbs_tests.cpp:128-142: all entries equal -> tokens 0 then 1 (lower index first).
    x = np.full((1, 1, 2, 5), -1.0, np.float32)
    out = oracle.oracle_decode(oracle.Problem(x))
    assert list(out["tokens"][0, 0]) == [0, 1]


def test_length_penalty_close_to_pow():
    # tests/internal_tests.cpp:1246-1256: within one float ulp of pow().
    lengths = np.arange(0, 2001, dtype=np.int32)
    for alpha in (0.1, 0.25, 0.5, 0.6, 0.7, 1.0, 1.3, 2.0, 3.7):
        a = np.float32(alpha)
        got = oracle.oracle_length_penalty(lengths, a)
        base = (5.0 + np.maximum(lengths, 1).astype(np.float64)) / 6.0
        want = np.power(base, np.float64(a)).astype(np.float32)
        diff = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
        assert diff.max() <= 1, alpha


def test_length_penalty_huge_alpha_saturates():
    # tests/internal_tests.cpp:1257-1262.
    lib = oracle.oracle_lib()
    for alpha in (64.5, 1.0e4, 3.0e9, 1.0e30, float(np.finfo(np.float32).max)):
        assert lib.oracle_gnmt_penalty(1, alpha) == 1.0
        assert lib.oracle_gnmt_penalty(100, alpha) == float("inf")


def test_half_conversions_exact():
    # tests/internal_tests.cpp:814: every fp16 / bf16 bit pattern widens exactly.
    lib = oracle.oracle_lib()
    bits = np.arange(0, 65536, dtype=np.uint32)
    f16 = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    bf16 = (bits << 16).view(np.float32)
    for i in range(0, 65536, 97):  # a stride through the whole space keeps this fast
        g16 = np.float32(lib.oracle_half_to_float(int(i), A.DTYPE_F16))
        gbf = np.float32(lib.oracle_half_to_float(int(i), A.DTYPE_BF16))
        if np.isnan(f16[i]):
            assert np.isnan(g16)
        else:
            assert g16.view(np.uint32) == f16[i].view(np.uint32)
        if np.isnan(bf16[i]):
            assert np.isnan(gbf)
        else:
            assert gbf.view(np.uint32) == bf16[i].view(np.uint32)


def _problem_from_fixture(z) -> oracle.Problem:
    dtype, from_logits, eos, min_length, ngram = (int(v) for v in z["meta"])
    alpha, rep = (float(v) for v in z["fl"])
    pb = oracle.Problem(z["x"], dtype=dtype, from_logits=bool(from_logits), eos=eos, min_length=min_length,
                        alpha=alpha, ngram=ngram, rep_penalty=rep, extra_eos=[int(t) for t in z["extra"]])
    if "steps" in z:
        pb.steps = z["steps"]
    if "banned" in z:
        pb.banned = z["banned"]
    return pb


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_golden_fixture(path):
    z = np.load(path)
    pb = _problem_from_fixture(z)
    out = oracle.oracle_decode(pb)
    for f in FIELDS:
        assert same_bits(out[f], z[f"out_{f}"]), f
    g = {"final_scores": z["out_g_final_scores"], "scores": z["out_g_scores"]}
    grad = oracle.oracle_backward(pb, out, g, logits=pb.x if pb.from_logits else None,
                                  row_lse=out["row_lse"] if pb.from_logits else None)
    assert same_bits(grad, z["out_grad"])


@needs_ref
@pytest.mark.parametrize("seed", range(60))
def test_oracle_matches_reference_library(seed):
    pb = random_case(seed, max_kv=60_000, allow_per_example=False)
    ours = oracle.oracle_decode(pb)
    ref = oracle.ref_decode(pb)
    for f in FIELDS:
        assert same_bits(ours[f], ref[f]), f


@needs_ref
@pytest.mark.parametrize("seed", range(20))
def test_oracle_backward_matches_reference_library(seed):
    pb = random_case(1000 + seed, max_kv=20_000, allow_per_example=False)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    rng = np.random.default_rng(seed)
    grads = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32)}
    if seed % 2:
        grads["scores"] = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
        grads["raw_scores"] = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
        grads["final_raw_scores"] = rng.uniform(-1, 1, (B, K)).astype(np.float32)
    logits = pb.x if pb.from_logits else None
    lse = trace["row_lse"] if pb.from_logits else None
    ours = oracle.oracle_backward(pb, trace, grads, logits=logits, row_lse=lse)
    with oracle.RefDecoder(pb) as d:
        ref = d.backward(trace, grads, logits=logits, row_lse=lse)
    assert same_bits(ours, ref)


@needs_ref
@pytest.mark.parametrize("seed", range(16))
def test_selected_weights_match_reference_library(seed):
    """Selected-beam weights (softmax_selected) and their backward term, against the reference
    library's single-example API (dbs_decode -> dbs_result_weights; dbs_backward_dense with
    grad_selected_weights), bit for bit."""
    rng = np.random.default_rng(500 + seed)
    T = int(rng.integers(1, 9))
    K = int(rng.choice([1, 2, 3, 4, 8, 13, 33]))
    V = int(rng.choice([5, 31, 300]))
    eos = int(rng.integers(-1, V))
    alpha = float(rng.choice([0.0, 0.6, 1.0]))
    ml = int(rng.integers(0, 3))
    temp = float(rng.choice([1.0, 0.5, 2.0, 0.01]))
    mode = "ties" if seed % 4 == 3 else ("neginf" if seed % 4 == 2 else "continuous")
    pb = make_problem(1, T, K, V, seed=seed, eos=eos, alpha=alpha, min_length=ml, mode=mode)
    gw = rng.uniform(-1, 1, (T, K)).astype(np.float32)
    gf = rng.uniform(-1, 1, (K,)).astype(np.float32)
    w_ref, g_ref = oracle.ref_selected(pb.x[0], K, eos, alpha, ml, temp, gw, gf)
    trace = oracle.oracle_decode(pb)
    w = oracle.oracle_selected_weights(pb, trace["scores"], temp)
    g = oracle.oracle_backward_selected(pb, trace, {"final_scores": gf[None]}, w, gw[None], temp)
    assert same_bits(w[0], w_ref)
    assert same_bits(g[0], g_ref)


@needs_ref
def test_oracle_c1_config_matches_reference():
    # fp32 log-probs [8, 32, 4, 1000], eos=2, alpha=0.6, min_length=4.
    pb = make_problem(8, 32, 4, 1000, seed=0, eos=2, alpha=0.6, min_length=4)
    ours = oracle.oracle_decode(pb)
    ref = oracle.ref_decode(pb, threads=4)
    for f in FIELDS:
        assert same_bits(ours[f], ref[f]), f


def test_path_gradient_scatters_to_dense():
    pb = make_problem(3, 6, 4, 50, seed=9, eos=3, alpha=0.6)
    trace = oracle.oracle_decode(pb)
    g = np.random.default_rng(0).uniform(-1, 1, (3, 4)).astype(np.float32)
    dense = oracle.oracle_backward(pb, trace, {"final_scores": g})
    draws = oracle.oracle_path_gradient(pb, trace, g)
    scattered = np.zeros_like(dense)
    B, T, K, V = pb.shape
    for b in range(B):
        for t in range(T):
            for k in range(K):
                p, tok = trace["parents"][b, t, k], trace["tokens"][b, t, k]
                if p >= 0 and trace["from_logprob"][b, t, k]:
                    scattered[b, t, p, tok] += draws[b, t, k]
    assert same_bits(scattered, dense)


@needs_ref
@pytest.mark.parametrize("seed", range(4))
def test_reference_pool_apis_agree(seed):
    """The two reference checkers of the relaxed pool (the batch API's pool outputs and the
    single-example API's pool accessors) give the same pool, whose first K entries per step
    are the step's selected beams; the relaxed weights of a step sum to K within tolerance."""
    K, m, temp, tol = 4, 3, 0.5, 1e-4
    pb = make_problem(2, 6, K, 80, seed=300 + seed, eos=2, alpha=0.6, min_length=seed % 3)
    with oracle.RefDecoder(pb, pool_multiplier=m) as ref:
        out = ref.decode()
    assert (out["pool_parents"][:, :, :K] == out["parents"]).all()
    P = K * m
    for b in range(2):
        one = oracle.ref_relaxed(pb.x[b], K, pb.eos, pb.alpha, pb.min_length, m, temp, tol, 60,
                                 np.zeros((6, P), np.float32), np.zeros(K, np.float32))
        for k in ("pool_scores", "pool_raw_scores", "pool_tokens", "pool_parents", "pool_lengths"):
            assert one[k].tobytes() == out[k][b].tobytes(), k
        live = (one["pool_parents"] >= 0).sum(1) > K
        sums = one["relaxed_weights"].sum(1)
        assert np.all(np.abs(sums[live] - K) < 1e-2)
