# SPDX-License-Identifier: MIT
"""Vocabulary-sharded decode (beamgrad_b200.vocab_sharding, dbs_cuda_vshard_*): the shard
layout and plan on CPU; on a GPU, every shard count W = 1, 2, 4, 8 run in one process
(decode_vocab_shards) against the CPU oracle's decode of the full vocabulary, bit for bit,
including rows that need a rescan (forced with one-entry shard records)."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from _cases import make_problem
from beamgrad_b200 import _abi as A
from beamgrad_b200 import vocab_sharding as vs
from oracle import oracle

OUT = oracle.TRACE_FIELDS + ("row_lse", "invalid")
TORCH_DTYPE = {A.DTYPE_F32: torch.float32, A.DTYPE_F16: torch.float16, A.DTYPE_BF16: torch.bfloat16}


def test_shards_partition_the_vocabulary_by_lane():
    for V in (1, 7, 255, 256, 257, 1000, 50257):
        for W in (1, 2, 4, 8):
            toks = [vs.shard_tokens(V, W, r) for r in range(W)]
            assert sorted(torch.cat(toks).tolist()) == list(range(V))
            L = 256 // W
            for r, t in enumerate(toks):
                assert len(t) == vs.shard_vocab_size(V, W, r)
                assert bool(((t % 256) // L == r).all())
                assert bool((t[1:] > t[:-1]).all())
    with pytest.raises(ValueError):
        vs.shard_lanes(3)


def _args(B, T, K, V):
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = B, T, K, V
    a.eos_token = -1
    return a


def test_plan_without_a_device():
    lib = A.load()
    for K, V, W, logits in ((4, 1000, 8, True), (64, 256000, 8, True), (16, 50257, 2, False), (1, 5, 4, True)):
        a = _args(3, 5, K, V)
        for r in range(W):
            p = A.VocabShardPlan()
            A.check(lib.dbs_cuda_vshard_plan(C.byref(a), int(logits), W, r, 0, C.byref(p)), "plan")
            L = 256 // W
            assert (p.world_size, p.rank, p.lanes) == (W, r, L)
            assert p.shard_vocab == vs.shard_vocab_size(V, W, r)
            assert p.list_len == (8 if K <= 4 else 2 * K)
            assert p.shard_list_len == (p.list_len if W <= 2 else p.list_len // 2)
            assert p.row_words == 1 + (L // 2 if logits else 0) + p.shard_list_len
            assert p.rows == 3 * 5 * K and p.workspace_bytes > 0
    p = A.VocabShardPlan()
    a = _args(3, 5, 4, 100)
    for world, rank in ((3, 0), (16, 0), (2, 2), (2, -1)):
        assert lib.dbs_cuda_vshard_plan(C.byref(a), 1, world, rank, 0, C.byref(p)) == A.STATUS_INVALID_ARGUMENT
    assert lib.dbs_cuda_vshard_plan(C.byref(a), 1, 2, 0, 3, C.byref(p)) == A.STATUS_OK and p.shard_list_len == 3


def test_wrong_shard_width_is_rejected():
    x = torch.zeros((1, 2, 2, 10))
    with pytest.raises(ValueError, match="holds"):
        vs.ShardDecode(x, 100, True, 2, 0)


# ---------------------------------------------------------------------------- GPU


def full_inputs(pb: oracle.Problem) -> torch.Tensor:
    x = torch.from_numpy(np.ascontiguousarray(pb.x).copy())
    if pb.dtype != A.DTYPE_F32:
        x = x.view(torch.int16).view(TORCH_DTYPE[pb.dtype])
    return x.cuda()


def run_shards(pb: oracle.Problem, W: int, shard_list_len: int = 0):
    x = full_inputs(pb)
    V = pb.shape[3]
    shards = [vs.shard_inputs(x, W, r) for r in range(W)]
    steps = torch.from_numpy(pb.steps).cuda() if pb.steps is not None else None
    banned = torch.from_numpy(pb.banned).cuda() if pb.banned is not None else None
    ds = [vs.ShardDecode(s, V, pb.from_logits, W, r, steps=steps, eos_token=pb.eos, min_length=pb.min_length,
                         length_penalty_alpha=pb.alpha, banned_tokens=banned, no_repeat_ngram_size=pb.ngram,
                         repetition_penalty=pb.rep_penalty, extra_eos=pb.extra_eos, shard_list_len=shard_list_len)
          for r, s in enumerate(shards)]
    out = vs.decode_vocab_shards(ds)
    outs = [d.outputs() for d in ds]
    for o in outs[1:]:
        for name in OUT:
            assert torch.equal(o[name], outs[0][name]), name
    return out, ds[0].rounds


def assert_same(out, ref):
    for name in OUT:
        ours = out[name].cpu().numpy()
        assert ours.shape == ref[name].shape, name
        assert ours.tobytes() == np.ascontiguousarray(ref[name]).tobytes(), name


CASES = [
    # B, T, K, V, dtype, logits, extra
    (3, 6, 4, 1000, A.DTYPE_F32, True, {}),
    (3, 6, 4, 1000, A.DTYPE_F32, False, {}),
    (2, 5, 8, 1531, A.DTYPE_BF16, True, dict(eos=3, min_length=2, alpha=0.6)),
    (2, 5, 16, 700, A.DTYPE_F16, True, dict(eos=5, alpha=1.0, variable_steps=True)),
    (2, 4, 33, 2049, A.DTYPE_BF16, False, dict(eos=1, alpha=0.6)),
    (2, 4, 64, 4099, A.DTYPE_F32, True, dict(eos=1, alpha=0.6)),
    (3, 6, 4, 300, A.DTYPE_F32, True, dict(eos=2, ngram=2, rep_penalty=1.3)),
    (3, 5, 5, 513, A.DTYPE_BF16, True, dict(eos=4, banned_frac=0.05, extra_eos=(9,))),
    (3, 5, 3, 777, A.DTYPE_F32, True, dict(mode="naninf", eos=2)),
    (3, 5, 3, 600, A.DTYPE_F32, False, dict(mode="ties", eos=2)),
    (2, 4, 6, 90, A.DTYPE_F32, True, dict(mode="neginf", eos=1)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("W", [1, 2, 4, 8])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_vocab_sharded_decode_matches_oracle(case, W):
    B, T, K, V, dtype, logits, extra = CASES[case]
    pb = make_problem(B, T, K, V, dtype=dtype, from_logits=logits, seed=500 + case, **extra)
    ref = oracle.oracle_decode(pb)
    out, _ = run_shards(pb, W)
    assert_same(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("W", [2, 8])
@pytest.mark.parametrize("case", [0, 2, 4, 6, 7])
def test_rescans_keep_the_decode_exact(case, W):
    """One-entry shard records leave most rows short: the stalled-row rescans carry the decode."""
    B, T, K, V, dtype, logits, extra = CASES[case]
    pb = make_problem(B, T, K, V, dtype=dtype, from_logits=logits, seed=900 + case, **extra)
    ref = oracle.oracle_decode(pb)
    out, rounds = run_shards(pb, W, shard_list_len=1)
    assert rounds > 0
    assert_same(out, ref)


@pytest.mark.gpu
def test_validate_raises_on_nan_rows():
    pb = make_problem(2, 3, 2, 600, seed=3, eos=1, from_logits=True)
    pb.x[1, 0, 0, 17] = np.nan
    x = full_inputs(pb)
    shards = [vs.shard_inputs(x, 2, r) for r in range(2)]
    with pytest.raises(ValueError, match="NaN"):
        vs.decode_vocab_shards(shards, 600, True, eos_token=1, validate=True)


# ---------------------------------------------------------------------------- gloo ranks (CPU)


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_problem():
    return make_problem(3, 5, 3, 600, from_logits=True, seed=77, eos=2, min_length=2, alpha=0.6,
                        variable_steps=True)


def _gloo_rank(rank: int, world: int, port: int, result_path: str, shard_list_len: int):
    import os
    from pathlib import Path

    import torch.distributed as dist

    from _vshard_emu import EmuEngine

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pb = _gloo_problem()
        V = pb.shape[3]
        x = torch.from_numpy(np.ascontiguousarray(pb.x))
        shard = vs.shard_inputs(x, world, rank)
        d = vs.ShardDecode(shard, V, True, world, rank, steps=torch.from_numpy(pb.steps), eos_token=pb.eos,
                           min_length=pb.min_length, length_penalty_alpha=pb.alpha, shard_list_len=shard_list_len,
                           engine=EmuEngine())
        out = vs.decode_vocab_sharded(d)
        ref = oracle.oracle_decode(pb)
        bad = [n for n in OUT if out[n].numpy().tobytes() != np.ascontiguousarray(ref[n]).tobytes()]
        Path(f"{result_path}.{rank}").write_text(f"rounds={d.rounds} " + ("ok" if not bad else "mismatch " + ",".join(bad)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shard_list_len", [0, 1])
def test_vocab_sharded_protocol_on_gloo_ranks(tmp_path, shard_list_len):
    """Two gloo ranks run decode_vocab_sharded with a CPU model of the stages; the result is
    the oracle's full decode. One-entry shard records force the stalled-row rescans."""
    import torch.multiprocessing as mp
    from pathlib import Path

    world = 2
    result = str(tmp_path / "result")
    mp.start_processes(_gloo_rank, args=(world, _free_port(), result, shard_list_len), nprocs=world,
                       start_method="spawn", join=True)
    texts = [Path(f"{result}.{r}").read_text() for r in range(world)]
    for t in texts:
        assert t.endswith("ok"), texts
    if shard_list_len == 1:
        assert int(texts[0].split()[0].split("=")[1]) > 0, texts


def test_shard_lanes_rebuild_the_row_logsumexp():
    """The oracle's per-shard lane sums, put together lane by lane, give its full-row lse."""
    rng = np.random.default_rng(4)
    lib = oracle.oracle_lib()
    for V in (1, 200, 256, 1000, 1537):
        row = (rng.standard_normal(V) * 3).astype(np.float32)
        row[rng.random(V) < 0.05] = -np.inf
        inv = C.c_int(0)
        ref = lib.oracle_row_lse(row.ctypes.data_as(C.c_void_p), V, C.byref(inv))
        mx = np.float32(row[row < np.inf].max())
        for W in (1, 2, 4, 8):
            lanes = []
            for r in range(W):
                sh = np.ascontiguousarray(row[vs.shard_tokens(V, W, r).numpy()])
                out = np.zeros(256 // W, np.float32)
                lib.oracle_shard_lanes(sh.ctypes.data_as(C.c_void_p), sh.size, W, float(mx),
                                       out.ctypes.data_as(C.c_void_p))
                lanes.append(out)
            lanes = np.ascontiguousarray(np.concatenate(lanes))
            got = lib.oracle_lse_from_lanes(lanes.ctypes.data_as(C.c_void_p), float(mx))
            assert np.float32(got).tobytes() == np.float32(ref).tobytes(), (V, W)


# ---------------------------------------------------------------------------- NCCL ranks (2 GPUs)


def _nccl_rank(rank: int, world: int, port: int, result_path: str, case: int, shard_list_len: int):
    import datetime
    import os
    from pathlib import Path

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        B, T, K, V, dtype, logits, extra = CASES[case]
        pb = make_problem(B, T, K, V, dtype=dtype, from_logits=logits, seed=1300 + case, **extra)
        x = full_inputs(pb)
        steps = torch.from_numpy(pb.steps).cuda() if pb.steps is not None else None
        banned = torch.from_numpy(pb.banned).cuda() if pb.banned is not None else None
        out = vs.decode_vocab_sharded(vs.shard_inputs(x, world, rank), V, logits, steps, eos_token=pb.eos,
                                      min_length=pb.min_length, length_penalty_alpha=pb.alpha, banned_tokens=banned,
                                      no_repeat_ngram_size=pb.ngram, repetition_penalty=pb.rep_penalty,
                                      extra_eos=pb.extra_eos, shard_list_len=shard_list_len)
        ref = oracle.oracle_decode(pb)
        bad = [n for n in OUT if out[n].cpu().numpy().tobytes() != np.ascontiguousarray(ref[n]).tobytes()]
        Path(f"{result_path}.{rank}").write_text("ok" if not bad else "mismatch " + ",".join(bad))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("case,shard_list_len", [(0, 0), (5, 0), (6, 0), (2, 1)])
def test_vocab_sharded_decode_on_two_nccl_ranks(tmp_path, case, shard_list_len):
    """One process per GPU over NCCL: every rank's outputs are the oracle's full decode."""
    import torch.multiprocessing as mp
    from pathlib import Path

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    result = str(tmp_path / "result")
    mp.start_processes(_nccl_rank, args=(world, _free_port(), result, case, shard_list_len), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert Path(f"{result}.{r}").read_text() == "ok", r
