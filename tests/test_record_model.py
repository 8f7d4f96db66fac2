# SPDX-License-Identifier: MIT
"""CPU models of two shortcuts the from-logits chained decode takes (no GPU needed).

1. The record of a staged row (csrc/decode_impl.cuh, prepare_row's all-warps path): the
   filter bound is the R-th largest of the union of each warp's four largest thread maxima
   (chunk c of 16 bytes on thread c mod 256, ragged ends on threads 0..n_ends-1, threads
   owning an EOS token give no maximum), the candidates are the eligible entries at or
   above it (only threads whose own maximum reaches it are looked at), and the record is
   their best LIST by key (x descending, token ascending). The model checks that this record
   equals the row's true best LIST eligible entries whenever the candidates fit the list.
2. The warp selection (select_fast_core): with no carried beams and every scanned candidate
   of one length, the order by key (raw descending, then parent * V + token ascending) is
   the full candidate order (score, raw, parent, token; src/common.hpp:269-276 of beamgrad
   2.3.0), because score = raw * (1 / penalty) never decreases as raw grows.
"""

from __future__ import annotations

import numpy as np
import pytest

THREADS, WARPS, CAND_CAP = 256, 8, 256


def thread_maxima(x: np.ndarray, per: int, head: int, owner_excluded: np.ndarray):
    """Per-thread maxima over the chunk assignment, and each entry's owning thread."""
    V = x.shape[0]
    nvec = (V - head) // per
    tail0 = head + nvec * per
    owner = np.empty(V, np.int64)
    owner[:head] = np.arange(head)
    owner[head:tail0] = (np.arange(nvec * per) // per) % THREADS
    owner[tail0:] = head + np.arange(V - tail0)
    tmax = np.full(THREADS, -np.inf, np.float32)
    np.maximum.at(tmax, owner, x)
    me = tmax.copy()
    me[np.unique(owner[owner_excluded])] = -np.inf
    return tmax, me, owner


def record_by_bound(x, eligible, R, LIST, per, head, is_eos):
    tmax, me, owner = thread_maxima(x, per, head, is_eos)
    top4 = np.sort(me.reshape(WARPS, 32), axis=1)[:, ::-1][:, :4].ravel()
    xb = np.sort(top4)[::-1][R - 1]
    if xb == -np.inf:
        return None
    qualifying = tmax >= xb
    cand = np.nonzero(qualifying[owner] & (x >= xb) & eligible)[0]
    if cand.size > CAND_CAP:
        return None  # the kernel falls back to the list warps' record scan
    order = sorted(cand.tolist(), key=lambda v: (-x[v], v))
    return order[:LIST], cand.size


def true_record(x, eligible, LIST):
    idx = np.nonzero(eligible)[0]
    return sorted(idx.tolist(), key=lambda v: (-x[v], v))[:LIST]


@pytest.mark.parametrize("seed", range(40))
def test_record_from_bound_and_owner_candidates(seed):
    rng = np.random.default_rng(seed)
    V = int(rng.choice([300, 1000, 4099, 32000]))
    per = int(rng.choice([4, 8]))                # fp32 or 16-bit entries per 16-byte chunk
    head = int(rng.integers(0, per))             # ragged head of an unaligned row
    LIST = int(rng.choice([8, 16, 32]))
    banned = rng.random(V) < (0.01 if seed % 2 else 0.0)
    R = LIST + LIST // 2 if banned.any() else LIST
    if R > 32:
        pytest.skip("R above 32 uses the per-warp minimum bound")
    if seed % 3 == 0:
        x = (-0.5 * rng.integers(0, 4, size=V)).astype(np.float32)  # heavy ties
    else:
        bias = -1.1 * np.log(rng.permutation(V).astype(np.float32) + 1.0)
        x = (rng.standard_normal(V).astype(np.float32) * 2.0 + bias).astype(np.float32)
    eos = int(rng.integers(0, V))
    mask_eos = bool(seed % 4 == 1)
    is_eos = np.zeros(V, bool)
    is_eos[eos] = True
    eligible = ~banned & ~(mask_eos & is_eos)
    got = record_by_bound(x, eligible, R, LIST, per, head, is_eos)
    if got is None:
        return  # fallback path: the full record scan (covered by the GPU parity tests)
    rec, n = got
    want = true_record(x, eligible, LIST)
    if n >= LIST:
        assert rec == want
    else:
        # Fewer than LIST eligible entries reached the bound (banned or EOS entries took
        # thread maxima): the kernel rescans without a bound; what it holds is still exact.
        assert rec == want[: len(rec)]


def full_order_key(score, raw, parent, token):
    return (-score, -raw, parent, token)


@pytest.mark.parametrize("seed", range(20))
def test_one_length_key_order_is_the_full_order(seed):
    rng = np.random.default_rng(100 + seed)
    V, K = 32000, 8
    n = 16
    length = int(rng.integers(1, 200))
    alpha = np.float64(rng.choice([0.0, 0.6, 1.0, 2.0]))
    pen = np.float32(((5.0 + max(length, 1)) / 6.0) ** alpha) if alpha != 0 else np.float32(1.0)
    inv = np.float32(np.float32(1.0) / pen)
    # raws drawn from few values so that ties in raw and rounding ties in score both occur
    raws = (np.float32(-3.0) * rng.integers(0, 6, size=n).astype(np.float32) -
            np.float32(1e-3) * rng.integers(0, 3, size=n).astype(np.float32)).astype(np.float32)
    parents = rng.integers(0, K, size=n)
    tokens = rng.permutation(V)[:n]
    idx = parents * V + tokens
    by_key = sorted(range(n), key=lambda i: (-raws[i], idx[i]))
    scores = (raws * inv).astype(np.float32)
    by_full = sorted(range(n), key=lambda i: full_order_key(scores[i], raws[i], parents[i], tokens[i]))
    assert by_key == by_full
