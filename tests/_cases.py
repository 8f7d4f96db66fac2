# SPDX-License-Identifier: MIT
"""Seeded problem generators shared by the tests.

Value modes follow the reference's parity generators (beamgrad 2.3.0,
tests/cuda_emulation_tests.cpp:55-77): continuous log-probabilities, heavy ties
(-0.5 * {0..3}), 30% -inf, and sparse NaN / +inf.
"""

from __future__ import annotations

import numpy as np

from beamgrad_b200 import _abi as A
from oracle.oracle import Problem


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bits (NaN kept NaN)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bits_to_f32(bits: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == A.DTYPE_F16:
        return bits.view(np.float16).astype(np.float32)
    if dtype == A.DTYPE_BF16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits


def encode(x: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == A.DTYPE_F16:
        return x.astype(np.float16).view(np.uint16)
    if dtype == A.DTYPE_BF16:
        return f32_to_bf16_bits(x)
    return np.ascontiguousarray(x, np.float32)


def log_softmax(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.float64)
    m = z.max(-1, keepdims=True)
    return (z - m - np.log(np.exp(z - m).sum(-1, keepdims=True))).astype(np.float32)


def values(rng: np.random.Generator, shape, mode: str, logits: bool) -> np.ndarray:
    if mode == "ties":
        return (-0.5 * rng.integers(0, 4, size=shape)).astype(np.float32)
    z = (rng.standard_normal(shape) * 2.0).astype(np.float32)
    x = z if logits else log_softmax(z)
    if mode == "neginf":
        x[rng.random(shape) < 0.3] = -np.inf
    elif mode == "naninf":
        r = rng.random(shape)
        x[r < 0.002] = np.nan
        x[(r >= 0.002) & (r < 0.004)] = np.inf
    return x.astype(np.float32)


def make_problem(B, T, K, V, *, dtype=A.DTYPE_F32, from_logits=False, mode="continuous", seed=0, eos=-1,
                 min_length=0, alpha=0.0, ngram=0, rep_penalty=1.0, variable_steps=False, per_example=False,
                 banned_frac=0.0, extra_eos=()) -> Problem:
    rng = np.random.default_rng(seed)
    x = values(rng, (B, T, K, V), mode, from_logits)
    pb = Problem(encode(x, dtype), dtype=dtype, from_logits=from_logits, eos=eos, min_length=min_length,
                 alpha=alpha, ngram=ngram, rep_penalty=rep_penalty, extra_eos=list(extra_eos))
    if variable_steps:
        pb.steps = rng.integers(1, T + 1, size=B).astype(np.int32)
    if per_example:
        pb.beams = rng.integers(1, K + 1, size=B).astype(np.int32)
        pb.eos_pe = rng.integers(-1, V, size=B).astype(np.int32)
        pb.minlen_pe = rng.integers(0, 4, size=B).astype(np.int32)
    if banned_frac > 0:
        banned = np.zeros(V, np.uint8)
        banned[rng.permutation(V)[: max(1, int(banned_frac * V))]] = 1
        pb.banned = banned
    return pb


def random_case(seed: int, max_kv: int = 200_000, allow_per_example: bool = True) -> Problem:
    """A randomized configuration in the spirit of the reference's device parity suite."""
    rng = np.random.default_rng(seed * 7919 + 1)
    beams = [1, 2, 3, 4, 5, 8, 13, 16, 17, 33, 64]
    vocabs = [2, 7, 31, 256, 1000, 5003, 32000]
    K = int(rng.choice(beams))
    V = int(rng.choice(vocabs))
    if K * V > max_kv:
        V = max(2, max_kv // K)
    B = int(rng.integers(1, 5))
    T = int(rng.integers(1, 9))
    eos = -1 if rng.integers(0, 3) == 0 else int(rng.integers(0, V))
    extra = []
    if eos >= 0 and rng.integers(0, 4) == 0:
        extra = sorted({int(t) for t in rng.integers(0, V, size=int(rng.integers(1, 4)))})
    return make_problem(
        B, T, K, V,
        dtype=int(rng.integers(0, 3)),
        from_logits=bool(rng.integers(0, 2)),
        mode=str(rng.choice(["continuous", "ties", "neginf", "naninf"])),
        seed=seed,
        eos=eos,
        min_length=int(rng.integers(0, 4)),
        alpha=0.0 if rng.integers(0, 2) else 0.3 * float(rng.integers(0, 5)),
        ngram=int(rng.integers(1, 4)) if rng.integers(0, 3) == 0 else 0,
        rep_penalty=1.0 + 0.5 * float(rng.integers(1, 4)) if rng.integers(0, 3) == 0 else 1.0,
        variable_steps=bool(rng.integers(0, 3) == 0),
        per_example=allow_per_example and bool(rng.integers(0, 4) == 0),
        banned_frac=0.01 if rng.integers(0, 3) == 0 else 0.0,
        extra_eos=extra,
    )
