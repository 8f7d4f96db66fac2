# SPDX-License-Identifier: MIT
"""A step-by-step beam search whose state never leaves the GPU.

beamgrad's ``beam_search`` (python/beamgrad/_search.py:330-467 of beamgrad 2.3.0) calls the
model once per step and hands the step's ``[B, K, V]`` rows to ``decode_step``. Per step it
clones the state, casts the rows to float32, converts the int64 sequences to int32 prefixes,
reads the validation flags back (a host sync), checks ``active.any()`` (another sync), and
grows the sequences with a gather + cat. :class:`DeviceSearch` runs the same search on this
engine with:

* the beam state (raw scores, lengths, finished) and the trace in preallocated device
  buffers, advanced in place by ``dbs_cuda_decode_step_ex2`` (rows of any input dtype, or
  logits, read as they are: no float32 copy);
* the token prefixes resident on the device, advanced by one ``dbs_cuda_advance_prefixes``
  kernel per step (ping-pong buffers), which also records on the device whether any beam is
  still live after the step;
* no host synchronisation inside :meth:`DeviceSearch.step`: the early stop (all beams
  finished) is read back only every ``check_every`` steps and the invalid-input flags at
  the end, so a fixed-shape loop (model step + search step) can be captured in one CUDA graph.

The results equal beamgrad's search on the same rows: the same trace, final beams and
sequences, trimmed to the steps the reference runs (steps taken after every beam finished only
carry the finished beams forward and are dropped). The surrogate-gradient autograd wrapper of
beamgrad's Python layer is not part of this module; the trace it returns feeds
``torch.ops.beamgrad.decode_backward`` (or ``beamgrad_b200::decode_backward_as``).
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, NamedTuple, Sequence

import torch

from beamgrad_b200 import _abi as A

_DTYPES = {torch.float32: A.DTYPE_F32, torch.float16: A.DTYPE_F16, torch.bfloat16: A.DTYPE_BF16}


class StepState:
    """The beams entering a step (the fields of beamgrad's ``BeamState``,
    python/beamgrad/_search.py:26-48). Fields are computed on first access, on the device
    and without a host sync; ``sequences`` is ``[B, K, step]`` int64."""

    def __init__(self, search: "DeviceSearch"):
        self._s = search
        self.step = search.t

    @property
    def sequences(self) -> torch.Tensor:
        return self._s.prefixes()[..., : self.step].long()

    @property
    def parents(self) -> torch.Tensor:
        s = self._s
        return s._parents[self.step - 1].long() if self.step > 0 else torch.full_like(s._raw, -1, dtype=torch.long)

    @property
    def tokens(self) -> torch.Tensor:
        s = self._s
        return s._tokens[self.step - 1].long() if self.step > 0 else torch.full_like(s._raw, -1, dtype=torch.long)

    @property
    def lengths(self) -> torch.Tensor:
        return self._s._len.long()

    @property
    def scores(self) -> torch.Tensor:
        s = self._s
        return s._scores[self.step - 1].clone() if self.step > 0 else s._raw.clone()

    @property
    def finished(self) -> torch.Tensor:
        return self._s._fin.bool()

    @property
    def active(self) -> torch.Tensor:
        s = self._s
        return torch.isfinite(s._raw) & (s._fin == 0)


class SearchTrace(NamedTuple):
    """The per-step trace, as beamgrad's ``BeamSearchOutput`` (python/beamgrad/_torch.py:99-116)."""

    final_scores: torch.Tensor
    final_raw_scores: torch.Tensor
    final_lengths: torch.Tensor
    tokens: torch.Tensor
    parents: torch.Tensor
    lengths: torch.Tensor
    scores: torch.Tensor
    raw_scores: torch.Tensor
    from_logprob: torch.Tensor
    steps: torch.Tensor


class SearchResult(NamedTuple):
    """Result of :func:`beam_search` (the fields of beamgrad's ``BeamSearchResult``,
    python/beamgrad/_search.py:51-59, without autograd); ``row_lse`` is the per-step
    logsumexp ``[B, T, K]`` when the rows were logits, else None."""

    scores: torch.Tensor
    sequences: torch.Tensor
    lengths: torch.Tensor
    raw_scores: torch.Tensor
    trace: SearchTrace
    step_log_probs: tuple
    row_lse: torch.Tensor | None


class DeviceSearch:
    """State and trace of one step-by-step search on the device.

    ``dtype`` / ``from_logits`` describe the rows each :meth:`step` receives (``[B, K, V]``,
    contiguous, on ``device``). Options are beamgrad's ``BeamOptions`` in native form (EOS
    token or -1, extra EOS tokens, minimum length, GNMT alpha, banned token ids, n-gram size,
    repetition penalty).
    """

    def __init__(self, batch_size: int, beam_size: int, vocab_size: int, max_steps: int, *,
                 dtype: torch.dtype = torch.float32, from_logits: bool = False, eos_token: int = -1,
                 extra_eos: Sequence[int] = (), min_length: int = 0, length_penalty_alpha: float = 0.0,
                 banned_tokens: Sequence[int] | torch.Tensor | None = None, no_repeat_ngram_size: int = 0,
                 repetition_penalty: float = 1.0, device: torch.device | str | None = None):
        if dtype not in _DTYPES:
            raise ValueError(f"rows must be float32, float16 or bfloat16, got {dtype}")
        if batch_size < 1 or beam_size < 1 or beam_size > 1024 or vocab_size < 1 or max_steps < 1:
            raise ValueError("batch_size, vocab_size and max_steps must be positive and beam_size in [1, 1024]")
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if device.type != "cuda":
            raise ValueError("DeviceSearch runs on a CUDA device; there is no CPU path")
        self.lib = A.load()
        self.B, self.K, self.V, self.T = batch_size, beam_size, vocab_size, max_steps
        self.dtype, self.from_logits, self.device = dtype, bool(from_logits), device
        B, K, T = batch_size, beam_size, max_steps
        f32, i32, u8 = torch.float32, torch.int32, torch.uint8
        mk = lambda shape, dt, fill: torch.full(shape, fill, dtype=dt, device=device)  # noqa: E731
        self._raw = mk((B, K), f32, float("-inf"))
        self._raw[:, 0] = 0.0
        self._len = mk((B, K), i32, 0)
        self._fin = mk((B, K), u8, 0)
        self._pre = mk((2, B, K, T), i32, -1)  # ping-pong prefixes
        self._tokens = mk((T, B, K), i32, -1)
        self._parents = mk((T, B, K), i32, -1)
        self._lengths = mk((T, B, K), i32, 0)
        self._scores = mk((T, B, K), f32, float("-inf"))
        self._raws = mk((T, B, K), f32, float("-inf"))
        self._flp = mk((T, B, K), u8, 0)
        self._finals = mk((T, B, K), f32, float("-inf"))  # final scores after each step
        self._invalid = mk((T, B), u8, 0)
        self._live = mk((T,), u8, 0)
        self._lse = mk((T, B, K), f32, 0.0) if self.from_logits else None
        self._banned = None
        if banned_tokens is not None:
            if isinstance(banned_tokens, torch.Tensor) and banned_tokens.dtype == torch.uint8 and \
                    banned_tokens.numel() == vocab_size:
                self._banned = banned_tokens.to(device).contiguous()
            else:
                ids = torch.as_tensor(list(banned_tokens), dtype=torch.long)
                if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= vocab_size):
                    raise ValueError("banned token ids must lie in [0, vocab_size)")
                self._banned = torch.zeros(vocab_size, dtype=u8).index_fill_(0, ids, 1).to(device)
        a = A.DecodeArgs()
        a.batch_size, a.steps, a.beam_size, a.vocab_size = B, 1, K, vocab_size
        a.eos_token, a.min_length = int(eos_token), int(min_length)
        a.length_penalty_alpha = float(length_penalty_alpha)
        a.no_repeat_ngram_size = int(no_repeat_ngram_size)
        a.repetition_penalty = float(repetition_penalty)
        if self._banned is not None:
            a.banned_tokens = self._banned.data_ptr()
        self._args = a
        self._opts = None
        if extra_eos:
            if len(extra_eos) > A.MAX_EXTRA_EOS:
                raise ValueError(f"at most {A.MAX_EXTRA_EOS} extra EOS tokens")
            o = A.SearchOptions()
            o.extra_eos_count = len(extra_eos)
            for i, tok in enumerate(extra_eos):
                o.extra_eos_tokens[i] = int(tok)
            self._opts = o
        ws = self.lib.dbs_cuda_decode_step_workspace_size(C.byref(a), T)
        if ws < 0:
            raise ValueError("the engine rejects these search options")
        self._ws_bytes = int(ws)
        self._ws = torch.empty(max(self._ws_bytes, 1), dtype=u8, device=device)
        st = A.BeamState()
        st.raw_scores, st.lengths, st.finished = self._raw.data_ptr(), self._len.data_ptr(), self._fin.data_ptr()
        st.prefix_stride = T
        self._state = st
        self.t = 0

    def reset(self) -> None:
        """Back to the state before step 0, by device-side fills only (no allocation and no
        host sync, so a CUDA graph may capture it together with the steps)."""
        self._raw.fill_(float("-inf"))
        self._raw[:, 0] = 0.0
        self._len.zero_()
        self._fin.zero_()
        self._live.zero_()
        self._invalid.zero_()
        self.t = 0

    # -- stepping -----------------------------------------------------------------------
    def prefixes(self) -> torch.Tensor:
        """[B, K, max_steps] int32 token prefixes of the current beams (-1 past step t)."""
        return self._pre[self.t % 2]

    def state(self) -> StepState:
        return StepState(self)

    def step(self, rows: torch.Tensor) -> None:
        """One search step over rows [B, K, V] (row k extends beam k). Enqueued on the current
        stream; no host synchronisation."""
        t = self.t
        if t >= self.T:
            raise RuntimeError(f"the search already ran its {self.T} steps")
        if rows.dtype != self.dtype or tuple(rows.shape) != (self.B, self.K, self.V) or rows.device != self.device:
            raise ValueError(f"rows must be a {self.dtype} [{self.B}, {self.K}, {self.V}] tensor on {self.device}")
        rows = rows.contiguous()
        cur, nxt = self._pre[t % 2], self._pre[(t + 1) % 2]
        self._state.prefixes = cur.data_ptr()
        o = A.DecodeOutputs()
        o.tokens, o.parents, o.lengths = self._tokens[t].data_ptr(), self._parents[t].data_ptr(), self._lengths[t].data_ptr()
        o.scores, o.raw_scores, o.from_logprob = self._scores[t].data_ptr(), self._raws[t].data_ptr(), self._flp[t].data_ptr()
        o.final_scores = self._finals[t].data_ptr()
        o.invalid_input = self._invalid[t].data_ptr()
        stream = C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        lse = C.c_void_p(self._lse[t].data_ptr()) if self._lse is not None else None
        A.check(self.lib.dbs_cuda_decode_step_ex2(
            C.c_void_p(rows.data_ptr()), _DTYPES[self.dtype], int(self.from_logits), C.byref(self._args),
            C.byref(self._opts) if self._opts is not None else None, C.byref(self._state), C.byref(o), lse,
            C.c_void_p(self._ws.data_ptr()), self._ws_bytes, stream), "decode_step")
        # The raw scores and lengths of the state after the step are the trace's; the state
        # arrays advanced in place. Prefixes and the live flag follow on the device.
        A.check(self.lib.dbs_cuda_advance_prefixes(
            self.B, self.K, t, self.T, C.c_void_p(self._parents[t].data_ptr()), C.c_void_p(self._tokens[t].data_ptr()),
            C.c_void_p(self._flp[t].data_ptr()), C.c_void_p(cur.data_ptr()), C.c_void_p(nxt.data_ptr()),
            C.c_void_p(self._raw.data_ptr()), C.c_void_p(self._fin.data_ptr()),
            C.c_void_p(self._live[t].data_ptr()), stream), "advance_prefixes")
        self.t = t + 1

    def live_after(self, t: int) -> bool:
        """Whether some beam was live and unfinished after step t (reads one byte: a host sync)."""
        return bool(self._live[t].item())

    def steps_run(self) -> int:
        """The steps beamgrad's loop runs on the same rows: it stops before step t > 0 once no
        beam is live and unfinished (python/beamgrad/_search.py:366-368). One host sync."""
        if self.t == 0:
            return 0
        live = self._live[: self.t - 1].cpu()
        dead = (live == 0).nonzero()
        return int(dead[0, 0]) + 1 if dead.numel() else self.t

    def check_inputs(self, steps: int | None = None) -> None:
        """Raises ValueError like beamgrad's validated decode_step when a row the search read held
        NaN or +inf (python/csrc/cuda_ops.cpp:297-310 of beamgrad 2.3.0)."""
        steps = self.t if steps is None else steps
        bad = self._invalid[:steps].amax(0).cpu()
        for b in range(self.B):
            if int(bad[b]):
                raise ValueError(f"example {b}: log_probs contains NaN or +inf in a row the search reads")

    def result(self, step_log_probs: tuple = ()) -> SearchResult:
        """The search's result over the steps beamgrad's loop runs (:meth:`steps_run`)."""
        T = self.steps_run()
        if T == 0:
            raise RuntimeError("the search has not run a step")
        perm = lambda x: x[:T].permute(1, 0, 2).contiguous()  # noqa: E731  [T, B, K] -> [B, T, K]
        tokens, parents, flp = perm(self._tokens), perm(self._parents), perm(self._flp)
        if T == self.t:
            seq = self._pre[T % 2].long()
        else:
            # Steps after every beam finished overwrote the prefix buffers: follow the parents
            # back from step T-1, with the tokens of carried-forward slots masked to -1 (the
            # prefixes' own rule), in one kernel.
            emitted = torch.where(flp.bool(), tokens, -1).contiguous()
            a = A.DecodeArgs()
            a.batch_size, a.steps, a.beam_size, a.vocab_size = self.B, T, self.K, self.V
            back = torch.empty((self.B, self.K, T), dtype=torch.long, device=self.device)
            A.check(self.lib.dbs_cuda_backtrack(C.byref(a), C.c_void_p(emitted.data_ptr()),
                                                C.c_void_p(parents.data_ptr()), C.c_void_p(back.data_ptr()),
                                                C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)),
                    "backtrack")
            seq = torch.full((self.B, self.K, self.T), -1, dtype=torch.long, device=self.device)
            seq[..., :T] = back
        seq = seq.clone()
        seq[..., T:] = -1
        final_raw = self._raws[T - 1].clone()
        final_len = self._lengths[T - 1].long()
        trace = SearchTrace(
            final_scores=self._finals[T - 1].clone(), final_raw_scores=final_raw, final_lengths=final_len,
            tokens=tokens.long(), parents=parents.long(), lengths=perm(self._lengths).long(),
            scores=perm(self._scores), raw_scores=perm(self._raws), from_logprob=flp.bool(),
            steps=torch.full((self.B,), T, dtype=torch.long, device=self.device))
        lse = perm(self._lse) if self._lse is not None else None
        return SearchResult(scores=trace.final_scores, sequences=seq, lengths=final_len, raw_scores=final_raw,
                            trace=trace, step_log_probs=tuple(step_log_probs[:T]), row_lse=lse)


def beam_search(step_fn: Callable[[StepState], torch.Tensor], batch_size: int, beam_size: int, max_steps: int, *,
                check_every: int = 1, return_log_probs: bool = False, validate: bool = True,
                **options) -> SearchResult:
    """beamgrad's ``beam_search`` loop (python/beamgrad/_search.py:330-467) on the device.

    ``step_fn(state)`` returns the step's rows ``[B, K, V]`` (float32 / float16 / bfloat16
    log-probabilities, or logits with ``from_logits=True``). The dtype and vocabulary are taken
    from the first call. The loop reads the live flag back every ``check_every`` steps (1 =
    beamgrad's behaviour: stop as soon as every beam has finished); larger values sync less
    and may call step_fn up to ``check_every - 1`` times after the last live step, with the
    same result. ``options`` are :class:`DeviceSearch`'s keyword options.
    """
    if check_every < 1:
        raise ValueError("check_every must be >= 1")
    device = options.pop("device", None)
    search = None
    rows_kept = []
    for t in range(max_steps):
        if search is not None and t > 0 and t % check_every == 0 and not search.live_after(t - 1):
            break
        lp = step_fn(search.state() if search is not None else _InitialState(batch_size, beam_size, device))
        if not isinstance(lp, torch.Tensor) or not lp.is_floating_point():
            raise TypeError("step_fn must return a floating-point tensor of log-probabilities")
        if lp.dim() != 3 or lp.shape[0] != batch_size or lp.shape[1] != beam_size:
            raise ValueError(f"step_fn must return [B, K, V] = [{batch_size}, {beam_size}, V] rows, "
                             f"got {tuple(lp.shape)}")
        if search is None:
            if device is not None and torch.device(device) != lp.device:
                raise ValueError(f"step_fn returned rows on {lp.device}, but the search runs on {device}")
            search = DeviceSearch(batch_size, beam_size, lp.shape[2], max_steps, dtype=lp.dtype,
                                  device=lp.device, **options)
        if return_log_probs:
            rows_kept.append(lp)
        search.step(lp.detach())
    result = search.result(tuple(rows_kept))
    if validate:
        search.check_inputs(int(result.trace.steps[0]) if result.trace.steps.numel() else 0)
    return result


class _InitialState:
    """The state entering step 0 (the vocabulary, and so the device buffers, are not known yet)."""

    def __init__(self, B: int, K: int, device):
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.step = 0
        f = lambda v, dt: torch.full((B, K), v, dtype=dt, device=device)  # noqa: E731
        self.sequences = torch.empty((B, K, 0), dtype=torch.long, device=device)
        self.parents = f(-1, torch.long)
        self.tokens = f(-1, torch.long)
        self.lengths = f(0, torch.long)
        raw = f(float("-inf"), torch.float32)
        raw[:, 0] = 0.0
        self.scores = raw
        self.finished = f(False, torch.bool)
        self.active = torch.isfinite(raw)
