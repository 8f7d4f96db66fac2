# SPDX-License-Identifier: MIT
"""Parity of the CUDA engine (called through its C ABI) with the CPU oracle, bit for bit.

The cases follow the reference's own device suite (beamgrad 2.3.0
tests/cuda_device_tests.cpp:200-229 randomized parity, :232 step API, :340 NaN flags,
:544-581 the _ex variants) and python/tests/test_cuda.py:26-39.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from _cases import encode, make_problem, random_case
from beamgrad_b200 import _abi as A
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import _gpu as G

FIELDS = oracle.TRACE_FIELDS + ("row_lse", "invalid")


def assert_same(ours: dict, ref: dict, fields=FIELDS, ctx=""):
    """Bit-exact equality of every field (NaN payloads included)."""
    for f in fields:
        a, b = np.ascontiguousarray(ours[f]), np.ascontiguousarray(ref[f])
        assert a.shape == b.shape, (f, ctx)
        if a.tobytes() != b.tobytes():
            ai = a.view(np.uint8).reshape(a.shape + (-1,))
            bi = b.view(np.uint8).reshape(b.shape + (-1,))
            diff = np.argwhere((ai != bi).any(-1))
            idx = tuple(diff[0])
            raise AssertionError(f"{ctx} field {f}: {len(diff)} entries differ, first at {idx}: "
                                 f"engine {a[idx]!r} oracle {b[idx]!r}")


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = A.load()
    assert lib.dbs_cuda_available() == 1


@pytest.mark.parametrize("seed", range(120))
def test_randomized_parity(seed):
    pb = random_case(seed)
    assert_same(G.engine_decode(pb, use_workspace=bool(seed % 2)), oracle.oracle_decode(pb), ctx=f"seed {seed}")


REFERENCE_CASES = [
    # python/tests/test_cuda.py:26-33 (shape [B, T, K, V], options)
    ((1, 4, 2, 128), dict(eos=-1)),
    ((3, 6, 4, 1024), dict(eos=2)),
    ((2, 8, 8, 32000), dict(eos=7, min_length=3, alpha=0.6)),
    ((2, 5, 33, 300), dict(eos=1, alpha=1.0)),
    ((1, 3, 64, 5000), dict(eos=0)),
    ((1, 2, 1024, 7), dict(eos=-1)),
]


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("from_logits", [False, True])
def test_rounding_ties_between_distinct_entries(seed, from_logits):
    """Distinct entries whose raw scores round to one value once the parent score is large.

    Entries of a row are spaced 2^-18 apart near -150 while parent scores reach about -150
    after the first step (ulp 2^-16), so groups of entries with different x tie on raw and
    are ordered by token; the chained decode's per-row records must then either prove
    themselves sufficient or be rescanned.
    """
    rng = np.random.default_rng(900 + seed)
    B, T, K, V = 3, 5, 8, 700
    base = rng.uniform(-160.0, -140.0, size=(B, T, K, 1))
    x = (base + rng.integers(0, 96, size=(B, T, K, V)) * 2.0 ** -18).astype(np.float32)
    if from_logits:
        x = x + np.float32(150.0)
    pb = oracle.Problem(encode(x, A.DTYPE_F32), dtype=A.DTYPE_F32, from_logits=from_logits, eos=3, alpha=0.6)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx=f"seed {seed}")


@pytest.mark.parametrize("case", range(len(REFERENCE_CASES)))
@pytest.mark.parametrize("mode", ["continuous", "ties"])
def test_reference_cuda_cases(case, mode):
    shape, opts = REFERENCE_CASES[case]
    pb = make_problem(*shape, mode=mode, seed=sum(shape), **opts)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb))


@pytest.mark.parametrize("K", [1, 2, 15, 16, 17, 32, 64, 128])
@pytest.mark.parametrize("dtype", [A.DTYPE_F32, A.DTYPE_F16, A.DTYPE_BF16])
@pytest.mark.parametrize("from_logits", [False, True])
def test_beam_boundaries(K, dtype, from_logits):
    pb = make_problem(2, 4, K, 777, dtype=dtype, from_logits=from_logits, seed=K * 7 + dtype, eos=5, alpha=0.6,
                      min_length=2)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx=f"K={K}")


@pytest.mark.parametrize("V", [1, 2, 3, 7, 15, 16, 17, 255, 256, 257, 50257])
def test_ragged_vocab(V):
    for dtype in (A.DTYPE_F32, A.DTYPE_BF16):
        for from_logits in (False, True):
            pb = make_problem(2, 3, 4, V, dtype=dtype, from_logits=from_logits, seed=V, eos=min(1, V - 1))
            assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx=f"V={V} dt={dtype} logits={from_logits}")


def test_c1_config():
    # fp32 log_softmax(3 N(0,1)) [8, 32, 4, 1000], eos=2, alpha=0.6, min_length=4.
    rng = np.random.default_rng(0)
    z = (3.0 * rng.standard_normal((8, 32, 4, 1000))).astype(np.float32)
    from _cases import log_softmax
    pb = oracle.Problem(log_softmax(z), eos=2, alpha=0.6, min_length=4)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb))


def test_constraints_extra_eos_per_example():
    for seed in range(12):
        pb = make_problem(3, 7, 6, 97, seed=seed, eos=4, min_length=3, alpha=0.6, ngram=1 + seed % 3,
                          rep_penalty=1.0 + 0.5 * (seed % 3), banned_frac=0.05, extra_eos=(9, 11),
                          per_example=seed % 2 == 1, variable_steps=seed % 3 == 0, from_logits=seed % 4 == 0,
                          dtype=seed % 3)
        assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx=f"seed {seed}")


@pytest.mark.parametrize("seed", range(6))
def test_heavy_blocking_records_fall_back(seed):
    """1-gram blocking over long prefixes in a small vocabulary removes many of a row's best
    entries at selection time, so row records often cannot prove themselves and the row is
    rescanned with the parent's constraints."""
    K = [2, 4, 8, 16, 17, 40][seed]
    pb = make_problem(2, 14, K, 48 + 3 * seed, seed=500 + seed, eos=5, alpha=0.6, ngram=1,
                      rep_penalty=1.0 + 0.4 * (seed % 2), from_logits=seed % 2 == 1, dtype=seed % 3,
                      mode="ties" if seed % 3 == 2 else "continuous")
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx=f"seed {seed}")


def test_nan_flags_and_never_selected():
    pb = make_problem(4, 5, 3, 64, mode="naninf", seed=3, eos=1)
    ours = G.engine_decode(pb)
    assert_same(ours, oracle.oracle_decode(pb))
    assert ours["invalid"].any()


def test_large_vocab_fp16_logits_streamed():
    # Rows too large for shared memory (fp16 V = 151936) take the streaming path.
    pb = make_problem(2, 3, 8, 151936, dtype=A.DTYPE_F16, from_logits=True, seed=11, eos=-1, ngram=3,
                      rep_penalty=1.2, banned_frac=0.01)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb))


def test_step_api_matches_decode():
    for seed in range(10):
        rng = np.random.default_rng(seed + 1000)
        K = int(rng.choice([1, 3, 4, 16, 17, 64]))
        B, T, V = int(rng.integers(1, 4)), int(rng.integers(1, 7)), int(rng.integers(5, 3000))
        constrained = seed % 2 == 0
        pb = make_problem(B, T, K, V, seed=seed, eos=int(rng.integers(0, V)), alpha=0.6, min_length=2,
                          ngram=2 if constrained else 0, rep_penalty=1.5 if constrained else 1.0,
                          extra_eos=(min(3, V - 1),) if seed % 3 == 0 else (), from_logits=seed % 4 == 1,
                          dtype=seed % 3)
        full = oracle.oracle_decode(pb)
        raw = np.full((B, K), -np.inf, np.float32)
        raw[:, 0] = 0.0
        lengths = np.zeros((B, K), np.int32)
        finished = np.zeros((B, K), np.uint8)
        prefixes = np.full((B, K, T), -1, np.int32)
        for t in range(T):
            step_pb = oracle.Problem(np.ascontiguousarray(pb.x[:, t:t + 1]), dtype=pb.dtype, from_logits=pb.from_logits,
                                     eos=pb.eos, min_length=pb.min_length, alpha=pb.alpha, ngram=pb.ngram,
                                     rep_penalty=pb.rep_penalty, extra_eos=pb.extra_eos)
            ours = G.engine_step(step_pb, raw, lengths, finished, prefixes)
            ref = oracle.oracle_step(step_pb, raw, lengths, finished, prefixes)
            assert_same(ours, ref, fields=("tokens", "parents", "lengths", "scores", "raw_scores", "from_logprob",
                                           "row_lse", "invalid", "final_scores", "state_raw", "state_lengths",
                                           "state_finished"), ctx=f"seed {seed} step {t}")
            for f in ("tokens", "parents", "scores", "raw_scores"):
                assert ours[f][:, 0].tobytes() == full[f][:, t].tobytes(), (seed, t, f)
            # caller-side prefix bookkeeping
            new_pre = np.full_like(prefixes, -1)
            for b in range(B):
                for k in range(K):
                    p = ours["parents"][b, 0, k]
                    if p >= 0:
                        L = lengths[b, p]
                        new_pre[b, k, :L] = prefixes[b, p, :L]
                        if ours["from_logprob"][b, 0, k]:
                            new_pre[b, k, L] = ours["tokens"][b, 0, k]
            prefixes = new_pre
            raw, lengths, finished = ours["state_raw"], ours["state_lengths"], ours["state_finished"]
        assert full["final_scores"].tobytes() == ours["final_scores"].tobytes()


@pytest.mark.parametrize("seed", range(16))
def test_backward_parity(seed):
    pb = random_case(2000 + seed, max_kv=50_000)
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
    ours = G.engine_backward(pb, trace, grads, logits=logits, row_lse=lse, use_workspace=bool(seed % 3))
    ref = oracle.oracle_backward(pb, trace, grads, logits=logits, row_lse=lse)
    assert ours.tobytes() == ref.tobytes()


@pytest.mark.parametrize("K", [65, 256, 1024])
@pytest.mark.parametrize("mode", ["continuous", "ties"])
def test_backward_large_beams_parity(K, mode):
    """Beams above 64 find each parent's children through one sort per step (slot order kept)."""
    pb = make_problem(2, 5, K, 9 if K == 1024 else 61, mode=mode, seed=K, eos=3, alpha=0.6, variable_steps=True)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    rng = np.random.default_rng(K)
    grads = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32),
             "scores": rng.uniform(-1, 1, (B, T, K)).astype(np.float32)}
    ours = G.engine_backward(pb, trace, grads)
    assert ours.tobytes() == oracle.oracle_backward(pb, trace, grads).tobytes()
    draws = G.engine_path_gradient(pb, trace, grads["final_scores"])
    assert draws.tobytes() == oracle.oracle_path_gradient(pb, trace, grads["final_scores"]).tobytes()


def test_backward_time_at_beam_1024(capsys):
    """The per-step parent sums at K = 1024 (one CTA per example walking its steps): timed."""
    import ctypes as C

    pb = make_problem(4, 32, 1024, 9, seed=5, eos=3, alpha=0.6)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    lib = A.load()
    dp = G.DeviceProblem(pb)
    t = {k: G.dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    g = G.dev(np.linspace(-1, 1, B * K, dtype=np.float32).reshape(B, K))
    draws = torch.empty((B, T, K), dtype=torch.float32, device="cuda")
    call = lambda: A.check(lib.dbs_cuda_path_gradient(C.byref(dp.args()), G.ptr(t["parents"]), G.ptr(t["tokens"]),  # noqa: E731
                                                      G.ptr(t["lengths"]), G.ptr(t["from_logprob"]), G.ptr(g),
                                                      G.ptr(draws), G.stream_ptr()), "path_gradient")
    call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        call()
    e1.record()
    torch.cuda.synchronize()
    with capsys.disabled():
        print(f"\nbackward path gradient, B={B} T={T} K={K}: {e0.elapsed_time(e1) / 10 * 1e3:.1f} us per call")
    ref = oracle.oracle_path_gradient(pb, trace, g.cpu().numpy())
    assert draws.cpu().numpy().tobytes() == ref.tobytes()


@pytest.mark.parametrize("seed", range(12))
def test_backward_dense_parity(seed):
    """dbs_cuda_backward_dense == zero-filled float32 backward, cast to the output type, bit for bit."""
    pb = random_case(2100 + seed, max_kv=40_000)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    rng = np.random.default_rng(100 + seed)
    grads = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32)}
    if seed % 2:
        grads["scores"] = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
        grads["final_raw_scores"] = rng.uniform(-1, 1, (B, K)).astype(np.float32)
    logits = pb.x if pb.from_logits else None
    lse = trace["row_lse"] if pb.from_logits else None
    ref = oracle.oracle_backward(pb, trace, grads, logits=logits, row_lse=lse)
    out_type = (A.DTYPE_F32, A.DTYPE_BF16, A.DTYPE_F16)[seed % 3]
    misalign = (0, 1, 3)[(seed // 3) % 3]
    ours = G.engine_backward(pb, trace, grads, logits=logits, row_lse=lse, use_workspace=seed % 4 != 3,
                             dense=out_type, misalign=misalign)
    if out_type == A.DTYPE_F32:
        assert ours.tobytes() == ref.tobytes()
    else:
        want = torch.from_numpy(ref).to(torch.bfloat16 if out_type == A.DTYPE_BF16 else torch.float16)
        assert ours.view(torch.int16).numpy().tobytes() == want.view(torch.int16).numpy().tobytes()


@pytest.mark.parametrize("K", [1, 31, 32, 33])
@pytest.mark.parametrize("from_logits", [False, True])
def test_backward_dense_warp_and_block_paths(K, from_logits):
    """Beams <= 32 take the warp-per-row writer, larger beams the CTA-per-row one."""
    pb = make_problem(3, 5, K, 257, dtype=A.DTYPE_BF16 if from_logits else A.DTYPE_F32, from_logits=from_logits,
                      seed=60 + K, eos=2, alpha=0.6, variable_steps=True)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    rng = np.random.default_rng(K)
    grads = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32),
             "scores": rng.uniform(-1, 1, (B, T, K)).astype(np.float32)}
    logits = pb.x if from_logits else None
    lse = trace["row_lse"] if from_logits else None
    ref = oracle.oracle_backward(pb, trace, grads, logits=logits, row_lse=lse)
    for out_type, tdt in ((A.DTYPE_F32, torch.float32), (A.DTYPE_BF16, torch.bfloat16), (A.DTYPE_F16, torch.float16)):
        ours = G.engine_backward(pb, trace, grads, logits=logits, row_lse=lse, dense=out_type)
        want = torch.from_numpy(ref).to(tdt)
        got = torch.from_numpy(ours) if out_type == A.DTYPE_F32 else ours
        assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), (K, out_type)


def test_backward_dense_rejects_bad_arguments():
    lib = A.load()
    pb = make_problem(2, 3, 4, 50, seed=3)
    trace = oracle.oracle_decode(pb)
    dp = G.DeviceProblem(pb)
    t = {k: G.dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    bi = A.BackwardInputs()
    bi.parents, bi.tokens, bi.lengths, bi.from_logprob = (G.ptr(t[k]) for k in ("parents", "tokens", "lengths",
                                                                                  "from_logprob"))
    grad = torch.empty((2, 3, 4, 50), dtype=torch.float32, device="cuda")
    args = dp.args()
    for gtype in (-1, 3, 7):
        rc = lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), G.ptr(grad), gtype, None, 0, G.stream_ptr())
        assert rc == A.STATUS_INVALID_ARGUMENT
    assert lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), None, A.DTYPE_F32, None, 0,
                                       G.stream_ptr()) == A.STATUS_INVALID_ARGUMENT
    ws_bytes = lib.dbs_cuda_backward_workspace_size(C.byref(args))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    assert lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), G.ptr(grad), A.DTYPE_F32, G.ptr(ws), ws_bytes - 1,
                                       G.stream_ptr()) != A.STATUS_OK
    bi.logits, bi.logits_type = G.ptr(dp.x), A.DTYPE_F32  # logits without row_lse
    assert lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), G.ptr(grad), A.DTYPE_F32, None, 0,
                                       G.stream_ptr()) == A.STATUS_INVALID_ARGUMENT


@pytest.mark.parametrize("seed", range(12))
def test_selected_weights_and_backward_parity(seed):
    """Selected-beam weights and the backward through them (the oracle's restatement is pinned to
    the reference library's single-example API in test_oracle.py), bit for bit."""
    pb = random_case(2300 + seed, max_kv=20_000)
    B, T, K, V = pb.shape
    trace = oracle.oracle_decode(pb)
    temp = (1.0, 0.5, 2.0, 0.01)[seed % 4]
    want_w = oracle.oracle_selected_weights(pb, trace["scores"], temp)
    got_w = G.engine_selected_weights(pb, trace["scores"], temp)
    assert got_w.tobytes() == want_w.tobytes()
    rng = np.random.default_rng(seed)
    gw = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
    grads = {"final_scores": rng.uniform(-1, 1, (B, K)).astype(np.float32)}
    if seed % 2:
        grads["scores"] = rng.uniform(-1, 1, (B, T, K)).astype(np.float32)
    logits = pb.x if pb.from_logits else None
    lse = trace["row_lse"] if pb.from_logits else None
    want = oracle.oracle_backward_selected(pb, trace, grads, want_w, gw, temp, logits=logits, row_lse=lse)
    got = G.engine_backward_selected(pb, trace, grads, want_w, gw, temp, logits=logits, row_lse=lse)
    assert got.tobytes() == want.tobytes()


def test_selected_weights_reject_bad_temperature():
    lib = A.load()
    pb = make_problem(2, 3, 4, 20, seed=1)
    dp = G.DeviceProblem(pb)
    sc = torch.zeros((2, 3, 4), dtype=torch.float32, device="cuda")
    w = torch.empty_like(sc)
    for temp in (0.0, -1.0, float("inf"), float("nan")):
        rc = lib.dbs_cuda_selected_weights(C.byref(dp.args()), G.ptr(sc), temp, G.ptr(w), G.stream_ptr())
        assert rc == A.STATUS_INVALID_ARGUMENT


def test_bounded_waits_time_out_and_context_survives():
    """Failure detection without a GPU fault: the decode kernels' bounded waits (a flag that
    nothing sets, an mbarrier nothing arrives at) give up after a 2 ms limit, record the timeout
    in the error word, and the host reports LAUNCH_FAILED; the next decode is still exact."""
    lib = A.load()
    words = torch.full((4,), 7, dtype=torch.int32, device="cuda")
    rc = lib.dbs_cuda_b200_wait_selftest(2_000_000, G.ptr(words), G.stream_ptr())
    assert rc == A.STATUS_LAUNCH_FAILED
    assert words.cpu().tolist() == [0, 0, 1, 0]  # both waits gave up; error word = timeout
    assert lib.dbs_cuda_b200_wait_selftest(10, G.ptr(words), G.stream_ptr()) == A.STATUS_INVALID_ARGUMENT
    pb = make_problem(2, 5, 4, 300, seed=9, eos=2, alpha=0.6)
    assert_same(G.engine_decode(pb), oracle.oracle_decode(pb), ctx="after the timeout self-test")


def test_path_gradient_parity():
    for seed in range(8):
        pb = random_case(3000 + seed, max_kv=20_000)
        trace = oracle.oracle_decode(pb)
        g = np.random.default_rng(seed).uniform(-1, 1, (pb.shape[0], pb.shape[2])).astype(np.float32)
        assert G.engine_path_gradient(pb, trace, g).tobytes() == oracle.oracle_path_gradient(pb, trace, g).tobytes()


def test_length_penalty_parity():
    lengths = np.concatenate([np.arange(-5, 5000), np.array([2**31 - 1, 123456789])]).astype(np.int32)
    for alpha in (0.0, 0.1, 0.6, 1.0, 1.3, 2.0, 3.7, 64.0, 64.5, 1e4):
        a = np.float32(alpha)
        assert G.engine_length_penalty(lengths, a).tobytes() == oracle.oracle_length_penalty(lengths, a).tobytes()


def test_backtrack_parity():
    pb = make_problem(5, 9, 6, 40, seed=5, eos=3, variable_steps=True)
    trace = oracle.oracle_decode(pb)
    ours = G.engine_backtrack(pb, trace["tokens"], trace["parents"])
    assert np.array_equal(ours, oracle.backtrack(trace["tokens"], trace["parents"], pb.steps))


def test_invalid_per_example_arguments_rejected():
    pb = make_problem(3, 4, 4, 50, seed=1)
    pb.steps = np.array([1, 5, 2], np.int32)  # 5 > T
    with pytest.raises(A.InvalidArgument):
        G.engine_decode(pb)
    pb.steps = None
    pb.beams = np.array([1, 0, 2], np.int32)
    with pytest.raises(A.InvalidArgument):
        G.engine_decode(pb)


def test_invalid_scalar_arguments_rejected():
    lib = A.load()
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = 1, 1, 2000, 10  # beam > DBS_CUDA_MAX_BEAM
    assert lib.dbs_cuda_decode_workspace_size(C.byref(a)) < 0
    a.beam_size, a.reserved0 = 2, 1
    assert lib.dbs_cuda_decode_workspace_size(C.byref(a)) < 0
    a.reserved0 = 0
    a.eos_token = 10
    assert lib.dbs_cuda_decode_workspace_size(C.byref(a)) < 0


def test_undersized_workspace_rejected():
    lib = A.load()
    pb = make_problem(2, 3, 4, 30, seed=2)
    dp = G.DeviceProblem(pb)
    out = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    o = A.DecodeOutputs()
    o.final_scores = G.ptr(out)
    args = dp.args()
    need = lib.dbs_cuda_decode_workspace_size(C.byref(args))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    rc = lib.dbs_cuda_decode_ex2(G.ptr(dp.x), 0, 0, C.byref(args), None, C.byref(o), None, G.ptr(ws), need - 1,
                                 G.stream_ptr())
    assert rc == A.STATUS_INVALID_ARGUMENT


def test_sync_mode_and_repeatability(monkeypatch):
    monkeypatch.setenv("DBS_CUDA_SYNC_CHECK", "1")
    pb = make_problem(3, 6, 8, 2000, dtype=A.DTYPE_BF16, from_logits=True, seed=8, eos=2, alpha=1.0)
    a = G.engine_decode(pb)
    b = G.engine_decode(pb, use_workspace=False)
    assert_same(a, b)
    assert_same(a, oracle.oracle_decode(pb))


def test_runs_on_a_side_stream():
    pb = make_problem(2, 5, 3, 257, seed=5, eos=7)
    ref = oracle.oracle_decode(pb)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ours = G.engine_decode(pb)
    assert_same(ours, ref)


def test_c2_shape_subset_parity():
    # BASELINE configs[1] shape (bf16 logits [64, 128, 8, 32000], eos=2, alpha=1.0) at full size on the
    # device; examples are independent, so two seeded examples are checked against the oracle.
    B, T, K, V = 64, 128, 8, 32000
    g = torch.Generator(device="cuda").manual_seed(123)
    bias = -1.1 * torch.log(torch.randperm(V, generator=g, device="cuda").float() + 1.0)
    x = (torch.randn((B, T, K, V), generator=g, device="cuda") * 2.0 + bias).to(torch.bfloat16)
    host = oracle.Problem(np.zeros((B, T, K, 1), np.uint16), dtype=A.DTYPE_BF16, from_logits=True, eos=2, alpha=1.0)
    host.x = np.lib.stride_tricks.as_strided(host.x, shape=(B, T, K, V), strides=(0, 0, 0, 0))  # shape only
    ours = G.engine_decode(host, dp=G.DeviceProblem(host, x_dev=x))
    for b in (0, 41):
        xb = x[b:b + 1].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        sub = oracle.Problem(xb, dtype=A.DTYPE_BF16, from_logits=True, eos=2, alpha=1.0)
        ref = oracle.oracle_decode(sub)
        assert_same({k: v[b:b + 1] for k, v in ours.items()}, ref, ctx=f"example {b}")
    assert np.isfinite(ours["final_scores"][:, 0]).all()
