# SPDX-License-Identifier: MIT
"""Batch-sharded decode (beamgrad_b200.sharding): slicing, and the gather of every output
back into example order, on world-size-2 gloo ranks (CPU, with the oracle as the per-rank
decode), plus the engine on one GPU and, with two GPUs, NCCL ranks."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from beamgrad_b200 import sharding  # noqa: E402


def test_shard_ranges_partition_the_batch():
    for batch in (0, 1, 5, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [sharding.shard_range(batch, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def _problem():
    from _cases import make_problem

    return make_problem(5, 6, 3, 90, seed=41, eos=2, alpha=0.6, variable_steps=True)


def _oracle_decode_fn(pb):
    """Per-rank decode on CPU: the oracle on the rank's slice of pb."""
    from oracle import oracle

    def run(x, steps):
        sub = oracle.Problem(np.ascontiguousarray(x.numpy()), dtype=pb.dtype, from_logits=pb.from_logits, eos=pb.eos,
                             min_length=pb.min_length, alpha=pb.alpha,
                             steps=None if steps is None else steps.numpy().astype(np.int32))
        out = oracle.oracle_decode(sub)
        return tuple(torch.from_numpy(np.ascontiguousarray(out[name])) for name in sharding.OUTPUTS)

    return run


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, result_path: str):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle

        pb = _problem()
        a, b = sharding.shard_range(pb.shape[0], rank, world)
        x = torch.from_numpy(np.ascontiguousarray(pb.x[a:b]))
        steps = torch.from_numpy(pb.steps[a:b].copy())
        full = sharding.decode_sharded(x, pb.shape[0], _oracle_decode_fn(pb), steps)
        local = sharding.decode_sharded(x, pb.shape[0], _oracle_decode_fn(pb), steps, gather=False)
        ref = oracle.oracle_decode(pb)
        ok = all(full[n].numpy().tobytes() == np.ascontiguousarray(ref[n]).tobytes() for n in sharding.OUTPUTS)
        ok &= all(local[n].shape[0] == b - a for n in sharding.OUTPUTS)
        Path(result_path + f".{rank}").write_text("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_decode_sharded_gathers_in_example_order_on_gloo(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    result = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(world, _free_port(), result), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert Path(f"{result}.{r}").read_text() == "ok", r


def test_wrong_slice_size_is_rejected():
    pb = _problem()
    x = torch.from_numpy(np.ascontiguousarray(pb.x[:2]))
    with pytest.raises(ValueError, match="expected 5"):
        sharding.decode_sharded(x, 5, _oracle_decode_fn(pb))


@pytest.mark.gpu
def test_engine_decode_fn_on_one_gpu():
    from oracle import oracle

    pb = _problem()
    x = torch.from_numpy(np.ascontiguousarray(pb.x)).cuda()
    steps = torch.from_numpy(pb.steps.copy()).cuda()
    fn = sharding.engine_decode_fn(False, eos_token=pb.eos, length_penalty_alpha=pb.alpha)
    out = sharding.decode_sharded(x, pb.shape[0], fn, steps)
    ref = oracle.oracle_decode(pb)
    for n in sharding.OUTPUTS:
        assert out[n].cpu().numpy().tobytes() == np.ascontiguousarray(ref[n]).tobytes(), n
