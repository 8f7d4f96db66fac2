# SPDX-License-Identifier: MIT
"""Vocabulary-sharded decode: every row's vocabulary split over W ranks (W = 1, 2, 4 or 8).

The result is the decode of the full [B, T, K, V] input (beamgrad's ``decode_ex``, the same
outputs bit for bit) on every rank. Rank r holds the tokens v with ``(v mod 256)`` in
``[r * 256 / W, (r + 1) * 256 / W)``, in increasing v (:func:`shard_tokens`); that keeps
each of the reference's 256 logsumexp lanes on one rank, so lane sums need no exchange.

Per decode the ranks exchange: one all-reduce (MAX) of the row maxima (from logits), one
all-gather of a packed row per input row (flags, lane sums, the shard's best entries), and,
only when an example reaches a row whose merged record cannot prove its selection exact,
an all-gather of the shards' rescanned candidate lists for those rows. Stages run on the
GPU through the C ABI (``dbs_cuda_vshard_*``, include/dbs_cuda_b200.h); this module issues
them and the collectives.

:func:`decode_vocab_sharded` runs on ``torch.distributed`` ranks (one process per GPU);
:func:`decode_vocab_shards` runs every shard in one process, with the exchanges done by
plain tensor operations.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from beamgrad_b200 import _abi as A

LANES = 256
# decode_ex's outputs, in its order, then the per-example NaN/+inf flags.
OUTPUTS = ("final_scores", "final_raw_scores", "final_lengths", "tokens", "parents", "lengths", "scores",
           "raw_scores", "from_logprob", "row_lse")
_DTYPES = {torch.float32: A.DTYPE_F32, torch.float16: A.DTYPE_F16, torch.bfloat16: A.DTYPE_BF16}


def shard_lanes(world: int) -> int:
    """Logsumexp lanes per rank (256 / world)."""
    if world not in (1, 2, 4, 8):
        raise ValueError(f"vocabulary sharding needs 1, 2, 4 or 8 ranks, not {world}")
    return LANES // world


def shard_vocab_size(vocab: int, world: int, rank: int) -> int:
    """Tokens of rank `rank`: L = 256 / world of every full block of 256, and its part of the last."""
    L = shard_lanes(world)
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    full, rest = divmod(vocab, LANES)
    return full * L + min(max(rest - rank * L, 0), L)


def shard_tokens(vocab: int, world: int, rank: int, device=None) -> torch.Tensor:
    """Global token ids of rank `rank`'s shard, in shard order (int64)."""
    L = shard_lanes(world)
    n = shard_vocab_size(vocab, world, rank)
    i = torch.arange(n, dtype=torch.int64, device=device)
    return (i // L) * LANES + rank * L + i % L


def shard_inputs(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """Rank `rank`'s shard of full inputs x [..., V] (a copy)."""
    return x.index_select(-1, shard_tokens(x.shape[-1], world, rank, x.device)).contiguous()


class CudaEngine:
    """The stages on the GPU, through the C ABI."""

    def __init__(self):
        self.lib = A.load()

    def plan(self, args: A.DecodeArgs, from_logits: bool, world: int, rank: int, shard_list_len: int):
        plan = A.VocabShardPlan()
        A.check(self.lib.dbs_cuda_vshard_plan(C.byref(args), int(from_logits), world, rank, shard_list_len,
                                              C.byref(plan)), "vshard plan")
        return plan

    def run(self, stage: str, d: "ShardDecode") -> None:
        stream = torch.cuda.current_stream(d.device).cuda_stream
        A.check(getattr(self.lib, f"dbs_cuda_vshard_{stage}")(C.byref(d.call), stream), f"vshard {stage}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


class ShardDecode:
    """One rank's part of a vocabulary-sharded decode: buffers, outputs and the stage calls."""

    def __init__(self, shard: torch.Tensor, vocab_size: int, from_logits: bool, world: int, rank: int, *,
                 steps: torch.Tensor | None = None, eos_token: int = -1, min_length: int = 0,
                 length_penalty_alpha: float = 0.0, banned_tokens: torch.Tensor | None = None,
                 no_repeat_ngram_size: int = 0, repetition_penalty: float = 1.0, extra_eos: Sequence[int] = (),
                 shard_list_len: int = 0, engine=None):
        if shard.dim() != 4:
            raise ValueError("shard inputs must be [B, T, K, shard_vocab]")
        if shard.dtype not in _DTYPES:
            raise ValueError(f"unsupported input dtype {shard.dtype}")
        self.engine = engine if engine is not None else CudaEngine()
        self.device = shard.device
        self.shard = shard.contiguous()
        B, T, K, Vr = (int(s) for s in shard.shape)
        self.B, self.T, self.K, self.V = B, T, K, int(vocab_size)
        self.world, self.rank, self.from_logits = world, rank, bool(from_logits)
        if Vr != shard_vocab_size(self.V, world, rank):
            raise ValueError(f"rank {rank} of {world} holds {shard_vocab_size(self.V, world, rank)} tokens of "
                             f"{self.V}, not {Vr}")
        dev = self.device
        self.steps = None if steps is None else steps.to(device=dev, dtype=torch.int32).contiguous()
        self.banned = None if banned_tokens is None else banned_tokens.to(device=dev, dtype=torch.uint8).contiguous()
        if self.banned is not None and self.banned.numel() != self.V:
            raise ValueError("banned_tokens must have one entry per token of the full vocabulary")
        a = A.DecodeArgs()
        a.batch_size, a.steps, a.beam_size, a.vocab_size = B, T, K, self.V
        a.eos_token, a.min_length = eos_token, min_length
        a.length_penalty_alpha = length_penalty_alpha
        a.no_repeat_ngram_size = no_repeat_ngram_size
        a.repetition_penalty = repetition_penalty
        a.steps_per_example = _ptr(self.steps)
        a.banned_tokens = _ptr(self.banned)
        self.args = a
        self.options = None
        if extra_eos:
            o = A.SearchOptions()
            o.extra_eos_count = len(extra_eos)
            for i, tok in enumerate(extra_eos):
                o.extra_eos_tokens[i] = int(tok)
            self.options = o
        self.settings = dict(eos_token=eos_token, min_length=min_length, length_penalty_alpha=length_penalty_alpha,
                             no_repeat_ngram_size=no_repeat_ngram_size, repetition_penalty=repetition_penalty,
                             extra_eos=tuple(extra_eos))
        self.plan = self.engine.plan(a, self.from_logits, world, rank, shard_list_len)
        p = self.plan
        rows = B * T * K
        self.row_max = torch.empty(rows, dtype=torch.float32, device=dev)
        self.row_min = torch.empty(rows, dtype=torch.float32, device=dev)
        self.exchange = torch.empty((rows, p.row_words), dtype=torch.int64, device=dev)
        self.exchange_all = torch.empty((world * rows, p.row_words), dtype=torch.int64, device=dev)
        self.resume = torch.zeros(B, dtype=torch.int32, device=dev)
        self.stalled = torch.zeros((B, (K + 31) // 32), dtype=torch.int32, device=dev)
        self.workspace = torch.empty(max(int(p.workspace_bytes), 1), dtype=torch.uint8, device=dev)
        f32, i32, u8 = torch.float32, torch.int32, torch.uint8
        self.out = {
            "final_scores": torch.empty((B, K), dtype=f32, device=dev),
            "final_raw_scores": torch.empty((B, K), dtype=f32, device=dev),
            "final_lengths": torch.empty((B, K), dtype=i32, device=dev),
            "tokens": torch.empty((B, T, K), dtype=i32, device=dev),
            "parents": torch.empty((B, T, K), dtype=i32, device=dev),
            "lengths": torch.empty((B, T, K), dtype=i32, device=dev),
            "scores": torch.empty((B, T, K), dtype=f32, device=dev),
            "raw_scores": torch.empty((B, T, K), dtype=f32, device=dev),
            "from_logprob": torch.empty((B, T, K), dtype=u8, device=dev),
            "row_lse": torch.empty((B, T, K), dtype=f32, device=dev),
            "invalid": torch.empty(B, dtype=u8, device=dev),
        }
        self.rescan_rows = self.rescan_slot = self.rescan = self.rescan_all = None
        self.rounds = 0
        self.timings = None  # {stage: [(start, end) CUDA events]} when set to a dict
        c = A.VocabShardCall()
        c.shard_inputs = _ptr(self.shard)
        c.data_type = _DTYPES[shard.dtype]
        c.from_logits = int(self.from_logits)
        c.world_size, c.rank = world, rank
        c.shard_list_len = shard_list_len
        c.args = C.pointer(self.args)
        c.options = C.pointer(self.options) if self.options is not None else None
        bf = c.buffers
        bf.row_max, bf.row_min = _ptr(self.row_max), _ptr(self.row_min)
        bf.exchange, bf.exchange_all = _ptr(self.exchange), _ptr(self.exchange_all)
        bf.resume, bf.stalled = _ptr(self.resume), _ptr(self.stalled)
        bf.n_rescan = 0
        bf.workspace, bf.workspace_bytes = _ptr(self.workspace), int(self.workspace.numel())
        o = c.outputs
        for name in OUTPUTS[:-1]:
            setattr(o, name, _ptr(self.out[name]))
        o.invalid_input = _ptr(self.out["invalid"])
        c.row_lse = _ptr(self.out["row_lse"])
        self.call = c

    def begin(self) -> None:
        """Starts a decode: no rescanned lists yet (buffers of an earlier decode are reused), then scan."""
        self.call.buffers.n_rescan = 0
        self.rounds = 0
        self.stage("scan")

    def stage(self, name: str) -> None:
        self.timed(name, lambda: self.engine.run(name, self))

    def timed(self, name: str, fn: Callable[[], None]) -> None:
        """fn() (a device stage or a collective on this rank's stream), between two CUDA events
        recorded under `name` when timings are enabled."""
        if self.timings is None:
            fn()
            return
        s = torch.cuda.current_stream(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        fn()
        e1.record(s)
        self.timings.setdefault(name, []).append((e0, e1))

    def stage_ms(self) -> dict[str, float]:
        """Device milliseconds per stage summed over the recorded calls (timings enabled)."""
        torch.cuda.synchronize(self.device)
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in (self.timings or {}).items()}

    def stalled_rows(self) -> list[int]:
        """Rows b * K + k the last select stopped at (examples ascending, then k); waits for the GPU."""
        resume = self.resume.cpu().tolist()
        stalled = self.stalled.cpu()
        rows = []
        for b, t in enumerate(resume):
            if t >= self.T:
                continue
            for w, word in enumerate(stalled[b].tolist()):
                word &= 0xFFFFFFFF
                while word:
                    low = word & -word
                    rows.append(b * self.K + w * 32 + low.bit_length() - 1)
                    word ^= low
        return rows

    def set_rescan(self, rows: list[int]) -> None:
        dev, n, K = self.device, len(rows), self.K
        self.rescan_rows = torch.tensor(rows, dtype=torch.int32, device=dev)
        slot = torch.full((self.B * K,), -1, dtype=torch.int32)
        slot[torch.tensor(rows, dtype=torch.int64)] = torch.arange(n, dtype=torch.int32)
        self.rescan_slot = slot.to(dev)
        self.rescan = torch.empty((n, K), dtype=torch.int64, device=dev)
        self.rescan_all = torch.empty((self.world * n, K), dtype=torch.int64, device=dev)
        bf = self.call.buffers
        bf.rescan_rows, bf.rescan_slot = _ptr(self.rescan_rows), _ptr(self.rescan_slot)
        bf.rescan, bf.rescan_all = _ptr(self.rescan), _ptr(self.rescan_all)
        bf.n_rescan = n
        self.rounds += 1

    def outputs(self) -> dict[str, torch.Tensor]:
        return dict(self.out)


def _check_invalid(d: ShardDecode, validate: bool) -> None:
    if validate and bool(d.out["invalid"].any()):
        raise ValueError("beamgrad_b200 vocab-sharded decode: inputs hold NaN or +inf in rows the search read")


def _gather(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    if dist.get_backend(group) == dist.Backend.NCCL:
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.chunk(dist.get_world_size(group))), inp, group=group)


def _agree(n: int, device, group) -> None:
    """Every rank computed the same stalled rows (they select from the same data)."""
    t = torch.tensor([n, -n], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    hi, lo = int(t[0]), -int(t[1])
    if hi != n or lo != n:
        raise RuntimeError(f"vocab-sharded decode: ranks disagree on the rows to rescan ({lo}..{hi})")


def decode_vocab_sharded(shard: torch.Tensor | ShardDecode, vocab_size: int | None = None, from_logits: bool = False,
                         steps: torch.Tensor | None = None, *, group=None, validate: bool = False, engine=None,
                         **settings) -> dict[str, torch.Tensor]:
    """The decode of the full vocabulary from this rank's shard; all ranks call it together.

    shard: [B, T, K, shard_vocab_size(vocab_size, W, rank)] (see :func:`shard_inputs`), or a
    ShardDecode built for this rank (its buffers are reused; the other arguments are ignored);
    settings: eos_token, min_length, length_penalty_alpha, banned_tokens ([V]),
    no_repeat_ngram_size, repetition_penalty, extra_eos, shard_list_len (0: default).
    Returns decode_ex's outputs (and ``invalid``) for the whole batch, on every rank.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if isinstance(shard, ShardDecode):
        d = shard  # a prepared decode (buffers reused; its inputs may have been refilled)
    else:
        d = ShardDecode(shard, vocab_size, from_logits, world, rank, steps=steps, engine=engine, **settings)
    if world == 1:
        return decode_vocab_shards([d], validate=validate)
    d.begin()
    if d.from_logits:
        d.timed("allreduce_max", lambda: dist.all_reduce(d.row_max, op=dist.ReduceOp.MAX, group=group))
        d.stage("lanes")
    d.timed("allgather", lambda: _gather(d.exchange_all, d.exchange, group))
    d.stage("merge")
    for _ in range(d.B * d.T + 1):
        d.stage("select")
        rows = d.stalled_rows()
        _agree(len(rows), d.resume.device, group)
        if not rows:
            break
        d.set_rescan(rows)
        d.stage("rescan")
        d.timed("allgather_rescan", lambda: _gather(d.rescan_all, d.rescan, group))
    else:
        raise RuntimeError("vocab-sharded decode: selection made no progress")
    _check_invalid(d, validate)
    return d.outputs()


def decode_vocab_shards(shards: Sequence[torch.Tensor] | Sequence[ShardDecode], vocab_size: int | None = None,
                        from_logits: bool = False, steps: torch.Tensor | None = None, *, validate: bool = False,
                        engine=None, **settings) -> dict[str, torch.Tensor]:
    """Every shard of a vocabulary-sharded decode in this process (shards[r] is rank r's); the
    exchanges are tensor operations. Returns rank 0's outputs (every rank's are identical)."""
    if shards and isinstance(shards[0], ShardDecode):
        ds = list(shards)
    else:
        world = len(shards)
        ds = [ShardDecode(s, vocab_size, from_logits, world, r, steps=steps, engine=engine, **settings)
              for r, s in enumerate(shards)]
    for d in ds:
        d.begin()
    if ds[0].from_logits:
        m = ds[0].row_max.clone()
        for d in ds[1:]:
            m = torch.maximum(m, d.row_max.to(m.device))
        for d in ds:
            d.row_max.copy_(m)
            d.stage("lanes")
    allx = torch.cat([d.exchange.to(ds[0].device) for d in ds])
    for d in ds:
        d.exchange_all.copy_(allx)
        d.stage("merge")
    for _ in range(ds[0].B * ds[0].T + 1):
        for d in ds:
            d.stage("select")
        rows = [d.stalled_rows() for d in ds]
        if any(r != rows[0] for r in rows[1:]):
            raise RuntimeError("vocab-sharded decode: shards disagree on the rows to rescan")
        if not rows[0]:
            break
        for d in ds:
            d.set_rescan(rows[0])
            d.stage("rescan")
        alls = torch.cat([d.rescan.to(ds[0].device) for d in ds])
        for d in ds:
            d.rescan_all.copy_(alls)
    else:
        raise RuntimeError("vocab-sharded decode: selection made no progress")
    _check_invalid(ds[0], validate)
    return ds[0].outputs()


def decode_fn(from_logits: bool, **settings) -> Callable[[torch.Tensor, int, torch.Tensor | None], dict]:
    """decode_vocab_sharded with fixed settings (shard, vocab_size, steps) -> outputs."""

    def run(shard: torch.Tensor, vocab_size: int, steps: torch.Tensor | None = None) -> dict:
        return decode_vocab_sharded(shard, vocab_size, from_logits, steps, **settings)

    return run
