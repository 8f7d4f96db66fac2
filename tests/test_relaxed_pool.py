# SPDX-License-Identifier: MIT
"""The relaxed pool on the GPU (dbs_cuda_relaxed_pool, dbs_cuda_backward_pool) against beamgrad's
own CPU library: the pool arrays and the pool-score gradients through the batch API
(dbs_decode_batch_into_ex / dbs_backward_batch_into_ex with relaxed_pool_multiplier), the relaxed
top-K weights and their gradient through the single-example API (dbs_result_relaxed_weights,
dbs_backward_dense's grad_relaxed_weights). Bit-exact."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from beamgrad_b200 import _abi as A
from oracle import oracle
from _cases import make_problem

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

if not oracle.ref_available():
    pytest.skip("beamgrad's CPU library (oracle/_ref) is not built", allow_module_level=True)

import _gpu as G  # noqa: E402

_POOL_KEYS = (("parents", torch.int32), ("tokens", torch.int32), ("lengths", torch.int32),
              ("scores", torch.float32), ("raw_scores", torch.float32), ("from_logprob", torch.uint8))


def engine_pool(pb, trace, P, temperature=0.0, tolerance=0.0, max_iters=0, relaxed=False, dp=None):
    """dbs_cuda_relaxed_pool over the decode `trace` (numpy, as engine_decode returned it)."""
    lib = A.load()
    dp = dp or G.DeviceProblem(pb)
    B, T, K, V = pb.shape
    tr = {k: G.dev(trace[k]) for k in ("parents", "tokens", "lengths", "raw_scores", "from_logprob", "row_lse")}
    ts = A.DecodeOutputs()
    for k in ("parents", "tokens", "lengths", "raw_scores", "from_logprob"):
        setattr(ts, k, G.ptr(tr[k]))
    out = {k: torch.full((B, T, P), 77, dtype=dt, device="cuda") for k, dt in _POOL_KEYS}
    ps = A.PoolOutputs()
    for k, _ in _POOL_KEYS:
        setattr(ps, k, G.ptr(out[k]))
    if relaxed:
        out["relaxed_weights"] = torch.full((B, T, P), 99.0, dtype=torch.float32, device="cuda")
        ps.relaxed_weights = G.ptr(out["relaxed_weights"])
    rc = lib.dbs_cuda_relaxed_pool(G.ptr(dp.x), pb.dtype, int(pb.from_logits), C.byref(dp.args()), C.byref(ts),
                                   G.ptr(tr["row_lse"]), P, temperature, tolerance, max_iters, C.byref(ps),
                                   G.stream_ptr())
    A.check(rc, "relaxed_pool")
    torch.cuda.synchronize()
    return {("pool_" + k if k != "relaxed_weights" else k): v.cpu().numpy() for k, v in out.items()}


def engine_backward_pool(pb, trace, pool, grads, P, temperature=0.0):
    """dbs_cuda_backward_pool into a zeroed float32 [B, T, K, V] gradient."""
    lib = A.load()
    dp = G.DeviceProblem(pb)
    B, T, K, V = pb.shape
    t = {k: G.dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    g = {k: G.dev(np.ascontiguousarray(v, np.float32)) for k, v in grads.items() if v is not None}
    pl = {k: G.dev(pool[k]) for k in pool if k.startswith("pool_") or k == "relaxed_weights"}
    bi = A.BackwardInputs()
    bi.parents, bi.tokens, bi.lengths, bi.from_logprob = (G.ptr(t[k]) for k in ("parents", "tokens", "lengths", "from_logprob"))
    bi.grad_final_scores = G.ptr(g.get("final_scores"))
    bi.grad_final_raw_scores = G.ptr(g.get("final_raw_scores"))
    bi.grad_scores = G.ptr(g.get("scores"))
    bi.grad_raw_scores = G.ptr(g.get("raw_scores"))
    pg = A.PoolGradients()
    pg.pool_size = P
    pg.parents, pg.tokens = G.ptr(pl["pool_parents"]), G.ptr(pl["pool_tokens"])
    pg.lengths, pg.from_logprob = G.ptr(pl["pool_lengths"]), G.ptr(pl["pool_from_logprob"])
    pg.relaxed_weights = G.ptr(pl.get("relaxed_weights"))
    pg.grad_relaxed_weights = G.ptr(g.get("relaxed_weights"))
    pg.grad_pool_scores = G.ptr(g.get("pool_scores"))
    pg.grad_pool_raw_scores = G.ptr(g.get("pool_raw_scores"))
    pg.soft_topk_temperature = temperature
    grad = torch.zeros((B, T, K, V), dtype=torch.float32, device="cuda")
    A.check(lib.dbs_cuda_backward_pool(C.byref(dp.args()), C.byref(bi), C.byref(pg), G.ptr(grad), G.stream_ptr()),
            "backward_pool")
    torch.cuda.synchronize()
    return grad.cpu().numpy()


def _same(got, want, what):
    np.testing.assert_array_equal(got.view(np.uint32) if got.dtype == np.float32 else got,
                                  want.view(np.uint32) if want.dtype == np.float32 else want, err_msg=what)


_POOL_CASES = [
    # (B, T, K, V, multiplier, kwargs)
    (2, 6, 4, 50, 3, dict(eos=2, alpha=0.6)),
    (3, 7, 5, 97, 2, dict(eos=3, alpha=1.0, min_length=3, variable_steps=True)),
    (2, 5, 1, 40, 4, dict(eos=1, alpha=0.0)),
    (2, 4, 3, 5, 4, dict(eos=0, alpha=0.6)),                     # fewer candidates than P early on
    (2, 6, 8, 300, 2, dict(eos=5, alpha=0.8, banned_frac=0.1, mode="ties")),
    (2, 5, 4, 1000, 3, dict(eos=7, alpha=0.6, from_logits=True, dtype=A.DTYPE_BF16)),
    (1, 6, 16, 2000, 4, dict(eos=9, alpha=1.2, dtype=A.DTYPE_F16)),
    (2, 4, 6, 64, 1, dict(eos=-1, alpha=0.6)),                   # no EOS: nothing carried
    (1, 3, 64, 512, 16, dict(eos=4, alpha=0.6)),                 # P = 1024, the largest pool
    (1, 3, 4, 12000, 2, dict(eos=1, alpha=0.6, mode="ties")),    # > 2048 keys reach the bound
    (2, 5, 6, 700, 4, dict(eos=2, alpha=0.6, mode="neginf")),    # -inf entries are not candidates
    (2, 4, 32, 300, 8, dict(eos=3, alpha=0.6)),                  # P = 256, the largest compacted pool
]


@pytest.mark.parametrize("case", range(len(_POOL_CASES)))
def test_pool_matches_reference(case):
    B, T, K, V, m, kw = _POOL_CASES[case]
    pb = make_problem(B, T, K, V, seed=100 + case, **kw)
    with oracle.RefDecoder(pb, pool_multiplier=m) as ref:
        want = ref.decode()
    trace = G.engine_decode(pb)
    got = engine_pool(pb, trace, K * m)
    for k, _ in _POOL_KEYS:
        _same(got["pool_" + k], want["pool_" + k], "pool_" + k)
    # the first K pool entries of a step are its selected beams
    sel = want["pool_parents"][:, :, :K]
    np.testing.assert_array_equal(sel, trace["parents"])


@pytest.mark.parametrize("case", [0, 1, 4, 5, 6])
def test_pool_score_gradients_match_reference(case):
    B, T, K, V, m, kw = _POOL_CASES[case]
    pb = make_problem(B, T, K, V, seed=100 + case, **kw)
    if pb.from_logits:
        pytest.skip("dbs_cuda_backward_pool takes log-probabilities")
    rng = np.random.default_rng(case)
    P = K * m
    grads = {"final_scores": rng.standard_normal((B, K)).astype(np.float32),
             "scores": rng.standard_normal((B, T, K)).astype(np.float32),
             "pool_scores": rng.standard_normal((B, T, P)).astype(np.float32),
             "pool_raw_scores": rng.standard_normal((B, T, P)).astype(np.float32)}
    with oracle.RefDecoder(pb, pool_multiplier=m) as ref:
        trace = ref.decode()
        want = ref.backward(trace, grads, pool=trace)
    got_trace = G.engine_decode(pb)
    pool = engine_pool(pb, got_trace, P)
    got = engine_backward_pool(pb, got_trace, pool, grads, P)
    _same(got, want, "grad_inputs")


@pytest.mark.parametrize("seed,K,V,m,temp", [(0, 4, 60, 3, 0.5), (1, 8, 200, 2, 0.1), (2, 3, 30, 4, 2.0),
                                             (3, 16, 1000, 4, 0.25), (4, 2, 9, 2, 1.0)])
def test_relaxed_weights_and_gradient_match_reference(seed, K, V, m, temp):
    T, B = 6, 2
    pb = make_problem(B, T, K, V, seed=200 + seed, eos=1 + seed, alpha=0.6, min_length=seed % 3)
    P, tol, iters = K * m, 1e-4, 60
    trace = G.engine_decode(pb)
    pool = engine_pool(pb, trace, P, temp, tol, iters, relaxed=True)
    rng = np.random.default_rng(seed)
    g_rel = rng.standard_normal((B, T, P)).astype(np.float32)
    g_fin = rng.standard_normal((B, K)).astype(np.float32)
    got = engine_backward_pool(pb, trace, pool, {"relaxed_weights": g_rel, "final_scores": g_fin}, P, temp)
    for b in range(B):
        want = oracle.ref_relaxed(pb.x[b], K, pb.eos, pb.alpha, pb.min_length, m, temp, tol, iters, g_rel[b], g_fin[b])
        for k in ("pool_scores", "pool_raw_scores", "pool_tokens", "pool_parents", "pool_lengths"):
            _same(pool[k][b], want[k], k)
        _same(pool["relaxed_weights"][b], want["relaxed_weights"], "relaxed_weights")
        _same(got[b], want["grad"], "grad_inputs")


def test_pool_rejects_unsupported_and_bad_arguments():
    lib = A.load()
    pb = make_problem(1, 3, 4, 20, seed=1, eos=2, alpha=0.6)
    trace = G.engine_decode(pb)
    for P, temp in ((3, 0.5), (A.MAX_POOL + 1, 0.5), (8, 0.0), (8, float("nan"))):
        with pytest.raises(RuntimeError):
            engine_pool(pb, trace, P, temp, 1e-4, 10, relaxed=True)
    ng = make_problem(1, 3, 4, 20, seed=1, eos=2, alpha=0.6, ngram=2)
    with pytest.raises(RuntimeError):
        engine_pool(ng, trace, 8)
    dp = G.DeviceProblem(pb)
    pg = A.PoolGradients()
    pg.pool_size = 8
    bi = A.BackwardInputs()
    grad = torch.zeros((1, 3, 4, 20), device="cuda")
    rc = lib.dbs_cuda_backward_pool(C.byref(dp.args()), C.byref(bi), C.byref(pg), G.ptr(grad), G.stream_ptr())
    assert rc == A.STATUS_INVALID_ARGUMENT
