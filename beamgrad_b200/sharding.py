# SPDX-License-Identifier: MIT
"""Batch-sharded decode over several GPUs (one process per GPU, ``torch.distributed``).

Examples of a beam search are independent, so a batch is split into contiguous slices, one
per rank; every rank decodes its slice with the engine and, when asked, the per-example
outputs are all-gathered back into the full batch in example order. There is no
collective inside the decode itself.

``decode_fn`` is the per-rank decode: by default the engine's ``decode_ex`` operator
(:func:`engine_decode_fn`); tests substitute a CPU reference to check the slicing and
gathering on ``gloo`` ranks without a GPU.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist

# Per-example outputs of decode_ex, in its output order; all have the batch as dimension 0.
OUTPUTS = ("final_scores", "final_raw_scores", "final_lengths", "tokens", "parents", "lengths", "scores",
           "raw_scores", "from_logprob", "row_lse")


def shard_range(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Examples [start, stop) of `rank` when `batch` examples are split as evenly as possible."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def engine_decode_fn(from_logits: bool, eos_token: int = -1, min_length: int = 0, length_penalty_alpha: float = 0.0,
                     banned_tokens: torch.Tensor | None = None, no_repeat_ngram_size: int = 0,
                     repetition_penalty: float = 1.0, validate: bool = False,
                     extra_eos: Sequence[int] = ()) -> Callable[[torch.Tensor, torch.Tensor | None], tuple]:
    """The engine's decode_ex on one rank's slice (inputs [b, T, K, V] on this rank's GPU)."""
    from beamgrad_b200 import ops

    ops.load()

    def run(x: torch.Tensor, steps: torch.Tensor | None) -> tuple:
        return torch.ops.beamgrad.decode_ex(x, from_logits, steps, eos_token, min_length, length_penalty_alpha,
                                            banned_tokens, no_repeat_ngram_size, repetition_penalty, validate,
                                            list(extra_eos))

    return run


def decode_sharded(local_inputs: torch.Tensor, batch: int, decode_fn: Callable, local_steps: torch.Tensor | None = None,
                   gather: bool = True, group=None) -> dict[str, torch.Tensor]:
    """Decodes this rank's slice and (gather=True) returns every output for the whole batch.

    local_inputs holds examples shard_range(batch, rank, world) of the batch; local_steps
    (optional) their step counts. With gather=False only the local slice's outputs are
    returned. All ranks must call this together (the gather is a collective).
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    start, stop = shard_range(batch, rank, world)
    if local_inputs.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local_inputs.shape[0]} examples, expected {stop - start} "
                         f"(examples [{start}, {stop}) of {batch})")
    outs = dict(zip(OUTPUTS, decode_fn(local_inputs, local_steps)))
    if not gather or world == 1:
        return outs
    sizes = [shard_range(batch, r, world) for r in range(world)]
    most = max(b - a for a, b in sizes)
    full = {}
    for name, t in outs.items():
        # Slices differ by at most one example: pad to the largest, gather, then cut.
        pad = torch.zeros((most - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        buf = torch.cat([t, pad]) if most > t.shape[0] else t.contiguous()
        parts = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf, group=group)
        full[name] = torch.cat([parts[r][: b - a] for r, (a, b) in enumerate(sizes)])
    return full
