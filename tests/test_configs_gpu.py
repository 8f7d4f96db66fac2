# SPDX-License-Identifier: MIT
"""Parity at the shapes of BASELINE configs[2..4] (C3, C4, C5), bit for bit.

Each test builds the whole config tensor on the device with a seeded generator (the bench's
recipe: N(0, 2) logits plus a Zipf(1.1) bias -1.1 ln(rank) over a seeded permutation of the
vocabulary), decodes all of it through the C ABI, and checks seeded examples against the CPU
oracle. Examples are independent in the reference (docs/algorithm.md:144), so a subset of the
full batch pins the whole decode; the reference's own device suite checks parity the same way
on seeded subsets (tests/cuda_device_tests.cpp:200-229).

* C3: fp16 logits [32, 64, 8, 151936], 1 % banned tokens, repetition penalty 1.2,
  no_repeat_ngram 3, EOS suppressed, alpha 0. Sixty-four steps let 3-gram blocking fire; the
  test checks that it changes the checked examples' decode (so the path really ran).
* C4: bf16 log-probs [256, 256, 4, 50257], steps per example U{16..256}, eos 50256, alpha 0;
  the decode and the dense bf16 input gradient of the mean minimum-risk loss.
* C5: fp32 logits [16, 32, 64, 256000], eos 1, alpha 0.6, the vocabulary split over eight
  lane-interleaved shards decoded on one GPU, and the same input through the single-GPU wide
  decode: both equal on every example, and equal to the oracle on a checked one.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from beamgrad_b200 import _abi as A
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import _gpu as G


def _same(ours: dict, ref: dict, fields, ctx: str):
    for f in fields:
        a = np.ascontiguousarray(ours[f])
        b = np.ascontiguousarray(ref[f])
        assert a.shape == b.shape, (ctx, f)
        if a.tobytes() != b.tobytes():
            diff = np.argwhere((a.view(np.uint8).reshape(a.shape + (-1,)) != b.view(np.uint8).reshape(b.shape + (-1,))).any(-1))
            raise AssertionError(f"{ctx} field {f}: {len(diff)} entries differ, first at {tuple(diff[0])}")


FIELDS = oracle.TRACE_FIELDS + ("row_lse", "invalid")


@pytest.fixture(autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def zipf_bias(g: torch.Generator, V: int) -> torch.Tensor:
    return -1.1 * torch.log(torch.randperm(V, generator=g, device="cuda").float() + 1.0)


def shape_only(B, T, K, V, dtype, **opts) -> oracle.Problem:
    """A Problem that carries the shape and options; its inputs live on the device."""
    pb = oracle.Problem(np.zeros((B, T, K, 1), np.uint16 if dtype != A.DTYPE_F32 else np.float32), dtype=dtype, **opts)
    pb.x = np.lib.stride_tricks.as_strided(pb.x, shape=(B, T, K, V), strides=(0, 0, 0, 0))
    return pb


def host_bits(x: torch.Tensor) -> np.ndarray:
    if x.dtype == torch.float32:
        return x.cpu().numpy()
    return x.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def example(out: dict, b: int) -> dict:
    return {k: v[b:b + 1] for k, v in out.items()}


# ---------------------------------------------------------------------------- C3


def test_c3_shape_parity_with_ngram_blocking():
    B, T, K, V = 32, 64, 8, 151936
    g = torch.Generator(device="cuda").manual_seed(303)
    bias = zipf_bias(g, V)
    banned = torch.zeros(V, dtype=torch.uint8, device="cuda")
    banned[torch.randperm(V, generator=g, device="cuda")[: V // 100]] = 1
    x = torch.empty((B, T, K, V), dtype=torch.float16, device="cuda")
    for b in range(B):
        x[b] = (torch.randn((T, K, V), generator=g, device="cuda") * 2.0 + bias).half()
    opts = dict(from_logits=True, eos=-1, alpha=0.0, ngram=3, rep_penalty=1.2)
    host = shape_only(B, T, K, V, A.DTYPE_F16, **opts)
    host.banned = banned.cpu().numpy()
    ours = G.engine_decode(host, dp=G.DeviceProblem(host, x_dev=x))
    banned_h = host.banned
    for b in (0, 19):
        sub = oracle.Problem(host_bits(x[b:b + 1]), dtype=A.DTYPE_F16, banned=banned_h, **opts)
        ref = oracle.oracle_decode(sub)
        _same(example(ours, b), ref, FIELDS, f"C3 example {b}")
        # The constraints shape this example's decode: without n-gram blocking (or without the
        # repetition penalty) the oracle selects differently.
        for drop in (dict(ngram=0), dict(rep_penalty=1.0)):
            loose = oracle.Problem(sub.x, dtype=A.DTYPE_F16, banned=banned_h, **{**opts, **drop})
            assert oracle.oracle_decode(loose)["tokens"].tobytes() != ref["tokens"].tobytes(), (b, drop)
        assert not np.isin(ref["tokens"][ref["tokens"] >= 0], np.flatnonzero(banned_h)).any()


# ---------------------------------------------------------------------------- C4


def c4_inputs(seed: int):
    B, T, K, V = 256, 256, 4, 50257
    g = torch.Generator(device="cuda").manual_seed(seed)
    bias = zipf_bias(g, V)
    steps = torch.randint(16, T + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    costs = torch.rand((B, K), generator=g, device="cuda")
    x = torch.empty((B, T, K, V), dtype=torch.bfloat16, device="cuda")
    for b in range(B):
        x[b] = torch.log_softmax(torch.randn((T, K, V), generator=g, device="cuda") * 2.0 + bias, -1).to(x.dtype)
    return x, steps, costs


def minimum_risk_grad(final_scores: torch.Tensor, costs: torch.Tensor) -> torch.Tensor:
    """d/d final_scores of the mean over examples of sum_k softmax(final_scores)_k * cost_k over
    live beams (python/beamgrad/losses.py:139-169 of beamgrad 2.3.0, temperature 1)."""
    live = torch.isfinite(final_scores)
    any_live = live.any(-1, keepdim=True)
    logits = torch.where(any_live, torch.where(live, final_scores, float("-inf")), torch.zeros_like(final_scores))
    p = torch.softmax(logits, -1)
    c = torch.where(live, costs, 0.0)
    expected = (p * c).sum(-1, keepdim=True)
    return torch.where(any_live, p * (c - expected) / final_scores.shape[0], 0.0).contiguous()


def test_c4_shape_parity_decode_and_dense_backward():
    B, T, K, V = 256, 256, 4, 50257
    eos = 50256
    x, steps, costs = c4_inputs(404)
    host = shape_only(B, T, K, V, A.DTYPE_BF16, from_logits=False, eos=eos, alpha=0.0)
    host.steps = steps.cpu().numpy()
    dp = G.DeviceProblem(host, x_dev=x)
    ours = G.engine_decode(host, dp=dp)
    assert (ours["final_lengths"].max(-1) <= host.steps).all()

    # The dense bf16 input gradient of the whole batch, written once (dbs_cuda_backward_dense).
    lib = A.load()
    dev = {k: torch.from_numpy(ours[k]).cuda() for k in ("parents", "tokens", "lengths", "from_logprob")}
    g_final = minimum_risk_grad(torch.from_numpy(ours["final_scores"]).cuda(), costs)
    bi = A.BackwardInputs()
    bi.parents, bi.tokens, bi.lengths, bi.from_logprob = (G.ptr(dev[k]) for k in ("parents", "tokens", "lengths", "from_logprob"))
    bi.grad_final_scores = G.ptr(g_final)
    args = dp.args()
    ws_bytes = lib.dbs_cuda_backward_workspace_size(C.byref(args))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    grad = torch.empty((B, T, K, V), dtype=torch.bfloat16, device="cuda")
    A.check(lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), G.ptr(grad), A.DTYPE_BF16, G.ptr(ws), ws_bytes,
                                        G.stream_ptr()), "backward_dense")
    torch.cuda.synchronize()
    nonzero = int((grad != 0).sum())
    assert 0 < nonzero <= B * T * K

    g_host = g_final.cpu().numpy()
    short = int(np.argmin(host.steps))
    for b in (3, short):
        sub = oracle.Problem(host_bits(x[b:b + 1]), dtype=A.DTYPE_BF16, from_logits=False, eos=eos, alpha=0.0)
        sub.steps = host.steps[b:b + 1].copy()
        ref = oracle.oracle_decode(sub)
        _same(example(ours, b), ref, FIELDS, f"C4 example {b}")
        want = oracle.oracle_backward(sub, ref, {"final_scores": g_host[b:b + 1]})
        want_bf16 = torch.from_numpy(want).to(torch.bfloat16).view(torch.int16).numpy()
        got = grad[b:b + 1].view(torch.int16).cpu().numpy()
        assert got.tobytes() == want_bf16.tobytes(), f"C4 example {b}: dense bf16 gradient differs"


# ---------------------------------------------------------------------------- C5


def test_c5_shape_parity_vocab_sharded_over_eight():
    from beamgrad_b200 import vocab_sharding as vs

    B, T, K, V = 16, 32, 64, 256000
    eos, alpha = 1, 0.6
    g = torch.Generator(device="cuda").manual_seed(505)
    bias = zipf_bias(g, V)
    x = torch.empty((B, T, K, V), dtype=torch.float32, device="cuda")
    for b in range(B):
        x[b] = torch.randn((T, K, V), generator=g, device="cuda") * 2.0 + bias
    W = 8
    ds = [vs.ShardDecode(vs.shard_inputs(x, W, r), V, True, W, r, eos_token=eos, length_penalty_alpha=alpha)
          for r in range(W)]
    out = {k: v.cpu().numpy() for k, v in vs.decode_vocab_shards(ds).items()}
    del ds
    torch.cuda.empty_cache()

    # The single-GPU wide decode of the full vocabulary: every example equal to the sharded one.
    host = shape_only(B, T, K, V, A.DTYPE_F32, from_logits=True, eos=eos, alpha=alpha)
    whole = G.engine_decode(host, dp=G.DeviceProblem(host, x_dev=x))
    _same(whole, out, FIELDS, "C5 single GPU vs eight shards")

    b = 6
    sub = oracle.Problem(host_bits(x[b:b + 1]), dtype=A.DTYPE_F32, from_logits=True, eos=eos, alpha=alpha)
    _same(example(out, b), oracle.oracle_decode(sub), FIELDS, f"C5 example {b}")
