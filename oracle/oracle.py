# SPDX-License-Identifier: MIT
"""TEST INFRASTRUCTURE ONLY: ctypes front ends of the two CPU checkers.

* ``liboracle.so`` -- the plain-C restatement of the reference decoder in this
  directory (dbs_oracle.c); takes the engine's own argument structs.
* ``_ref/libdbs.so`` -- beamgrad 2.3.0's CPU library compiled from its sources
  (oracle/Makefile); called through its public C ABI (include/dbs.h:
  dbs_create_ex, dbs_set_extra_eos_tokens, dbs_decode_batch_into_ex,
  dbs_backward_batch_into_ex).
* ``_ref/libdbs_cuda_ref.so`` -- beamgrad 2.3.0's GPU engine (cuda/dbs_cuda.cu) built for
  sm_100a; called through its include/dbs_cuda.h (the reference GPU speed bar).

Only tests/, __graft_entry__.smoke() and bench.py's baseline legs (the CPU
baseline, the reference arm, the reference GPU engine's timing) import this module. Inputs are numpy arrays: float32 values, or the raw
uint16 bits of float16 / bfloat16 values.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libdbs.so"
REF_CUDA_LIB = HERE / "_ref" / "libdbs_cuda_ref.so"

import sys  # noqa: E402

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
from beamgrad_b200 import _abi as A  # noqa: E402  (struct definitions only; no engine call)

_p = C.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_p)


def reference_dir() -> Path | None:
    """The reference source tree (beamgrad 2.3.0): $BEAMGRAD_REF, else a directory named
    ``reference`` beside this repository; None when neither holds the sources."""
    for cand in (os.environ.get("BEAMGRAD_REF"), ROOT.parent / "reference"):
        if cand and (Path(cand) / "src" / "decoder.cpp").exists():
            return Path(cand)
    return None


def build(verbose: bool = False) -> None:
    """Compile liboracle.so and, where the reference sources exist, _ref/libdbs.so and
    _ref/libdbs_cuda_ref.so (the reference's own GPU engine, for sm_100a)."""
    ref = reference_dir()
    cmd = ["make", "-s", "-C", str(HERE), "all"] + ([f"REF={ref}"] if ref is not None else [])
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")
    if verbose:
        print(out.stdout, out.stderr)


@dataclass
class Problem:
    """One decode problem, in the engine's [B, T, K, V] layout."""

    x: np.ndarray                 # float32 values or uint16 bits, shape [B, T, K, V]
    dtype: int = A.DTYPE_F32      # A.DTYPE_*
    from_logits: bool = False
    eos: int = -1
    min_length: int = 0
    alpha: float = 0.0
    ngram: int = 0
    rep_penalty: float = 1.0
    steps: np.ndarray | None = None        # int32 [B]
    beams: np.ndarray | None = None        # int32 [B]
    eos_pe: np.ndarray | None = None       # int32 [B]
    minlen_pe: np.ndarray | None = None    # int32 [B]
    banned: np.ndarray | None = None       # uint8 [V]
    extra_eos: list[int] = field(default_factory=list)

    @property
    def shape(self):
        return tuple(int(s) for s in self.x.shape)

    def args(self) -> A.DecodeArgs:
        B, T, K, V = self.shape
        a = A.DecodeArgs()
        a.batch_size, a.steps, a.beam_size, a.vocab_size = B, T, K, V
        a.eos_token, a.min_length = self.eos, self.min_length
        a.length_penalty_alpha = self.alpha
        a.no_repeat_ngram_size = self.ngram
        a.repetition_penalty = self.rep_penalty
        a.steps_per_example = _ptr(self.steps)
        a.beam_sizes_per_example = _ptr(self.beams)
        a.eos_tokens_per_example = _ptr(self.eos_pe)
        a.min_lengths_per_example = _ptr(self.minlen_pe)
        a.banned_tokens = _ptr(self.banned)
        return a

    def options(self) -> A.SearchOptions | None:
        if not self.extra_eos:
            return None
        o = A.SearchOptions()
        o.extra_eos_count = len(self.extra_eos)
        for i, t in enumerate(self.extra_eos):
            o.extra_eos_tokens[i] = t
        return o


TRACE_FIELDS = ("final_scores", "final_raw_scores", "final_lengths", "tokens", "parents", "lengths", "scores",
                "raw_scores", "from_logprob")


def empty_outputs(B: int, T: int, K: int) -> dict[str, np.ndarray]:
    f32, i32, u8 = np.float32, np.int32, np.uint8
    return {
        "final_scores": np.zeros((B, K), f32),
        "final_raw_scores": np.zeros((B, K), f32),
        "final_lengths": np.zeros((B, K), i32),
        "tokens": np.zeros((B, T, K), i32),
        "parents": np.zeros((B, T, K), i32),
        "lengths": np.zeros((B, T, K), i32),
        "scores": np.zeros((B, T, K), f32),
        "raw_scores": np.zeros((B, T, K), f32),
        "from_logprob": np.zeros((B, T, K), u8),
        "invalid": np.zeros((B,), u8),
        "row_lse": np.zeros((B, T, K), f32),
    }


def _outputs_struct(o: dict[str, np.ndarray]) -> A.DecodeOutputs:
    s = A.DecodeOutputs()
    for name in TRACE_FIELDS:
        setattr(s, name, _ptr(o[name]))
    s.invalid_input = _ptr(o["invalid"])
    return s


# ---------------------------------------------------------------------------
# The C restatement
# ---------------------------------------------------------------------------
_olib = None


def oracle_lib() -> C.CDLL:
    global _olib
    if _olib is None:
        if not ORACLE_LIB.exists():
            build()
        lib = C.CDLL(str(ORACLE_LIB))
        lib.oracle_decode.restype = C.c_int
        lib.oracle_decode.argtypes = [_p, C.c_int, C.c_int, C.POINTER(A.DecodeArgs), C.POINTER(A.SearchOptions),
                                      C.POINTER(A.DecodeOutputs), _p]
        lib.oracle_decode_step.restype = C.c_int
        lib.oracle_decode_step.argtypes = [_p, C.c_int, C.c_int, C.POINTER(A.DecodeArgs), C.POINTER(A.SearchOptions),
                                           C.POINTER(A.BeamState), C.POINTER(A.DecodeOutputs), _p]
        lib.oracle_backward.restype = C.c_int
        lib.oracle_backward.argtypes = [C.POINTER(A.DecodeArgs), C.POINTER(A.BackwardInputs), _p]
        lib.oracle_path_gradient.restype = C.c_int
        lib.oracle_path_gradient.argtypes = [C.POINTER(A.DecodeArgs), _p, _p, _p, _p, _p, _p]
        lib.oracle_length_penalty.restype = None
        lib.oracle_length_penalty.argtypes = [_p, C.c_int64, C.c_float, _p]
        lib.oracle_gnmt_penalty.restype = C.c_float
        lib.oracle_gnmt_penalty.argtypes = [C.c_int, C.c_float]
        lib.oracle_exp_nonpositive.restype = C.c_float
        lib.oracle_exp_nonpositive.argtypes = [C.c_float]
        lib.oracle_row_lse.restype = C.c_float
        lib.oracle_row_lse.argtypes = [_p, C.c_int, C.POINTER(C.c_int)]
        lib.oracle_shard_lanes.restype = None
        lib.oracle_shard_lanes.argtypes = [_p, C.c_int, C.c_int, C.c_float, _p]
        lib.oracle_lse_from_lanes.restype = C.c_float
        lib.oracle_lse_from_lanes.argtypes = [_p, C.c_float]
        lib.oracle_half_to_float.restype = C.c_float
        lib.oracle_half_to_float.argtypes = [C.c_uint16, C.c_int]
        lib.oracle_backward_selected.restype = C.c_int
        lib.oracle_backward_selected.argtypes = [C.POINTER(A.DecodeArgs), C.POINTER(A.BackwardInputs), _p, _p,
                                                 C.c_float, _p]
        lib.oracle_selected_weights.restype = None
        lib.oracle_selected_weights.argtypes = [C.POINTER(A.DecodeArgs), _p, C.c_float, _p]
        _olib = lib
    return _olib


def oracle_decode(pb: Problem) -> dict[str, np.ndarray]:
    B, T, K, V = pb.shape
    out = empty_outputs(B, T, K)
    x = np.ascontiguousarray(pb.x)
    opts = pb.options()
    rc = oracle_lib().oracle_decode(_ptr(x), pb.dtype, int(pb.from_logits), C.byref(pb.args()),
                                    C.byref(opts) if opts is not None else None, C.byref(_outputs_struct(out)),
                                    _ptr(out["row_lse"]))
    if rc != 0:
        raise ValueError(f"oracle_decode: invalid argument ({rc})")
    return out


def oracle_step(pb: Problem, raw: np.ndarray, lengths: np.ndarray, finished: np.ndarray,
                prefixes: np.ndarray | None) -> dict[str, np.ndarray]:
    """One step over pb.x of shape [B, 1, K, V]; returns the step outputs and the new state."""
    B, T, K, V = pb.shape
    assert T == 1
    out = empty_outputs(B, 1, K)
    raw, lengths, finished = raw.copy(), lengths.copy(), finished.copy()
    st = A.BeamState()
    st.raw_scores, st.lengths, st.finished = _ptr(raw), _ptr(lengths), _ptr(finished)
    st.prefixes = _ptr(prefixes)
    st.prefix_stride = 0 if prefixes is None else int(prefixes.shape[-1])
    opts = pb.options()
    x = np.ascontiguousarray(pb.x)
    rc = oracle_lib().oracle_decode_step(_ptr(x), pb.dtype, int(pb.from_logits), C.byref(pb.args()),
                                         C.byref(opts) if opts is not None else None, C.byref(st),
                                         C.byref(_outputs_struct(out)), _ptr(out["row_lse"]))
    if rc != 0:
        raise ValueError(f"oracle_decode_step: invalid argument ({rc})")
    out["state_raw"], out["state_lengths"], out["state_finished"] = raw, lengths, finished
    return out


def oracle_backward(pb: Problem, trace: dict[str, np.ndarray], grads: dict[str, np.ndarray | None],
                    logits: np.ndarray | None = None, row_lse: np.ndarray | None = None) -> np.ndarray:
    B, T, K, V = pb.shape
    grad = np.zeros((B, T, K, V), np.float32)
    bi = A.BackwardInputs()
    bi.parents, bi.tokens = _ptr(trace["parents"]), _ptr(trace["tokens"])
    bi.lengths, bi.from_logprob = _ptr(trace["lengths"]), _ptr(trace["from_logprob"])
    bi.grad_final_scores = _ptr(grads.get("final_scores"))
    bi.grad_final_raw_scores = _ptr(grads.get("final_raw_scores"))
    bi.grad_scores = _ptr(grads.get("scores"))
    bi.grad_raw_scores = _ptr(grads.get("raw_scores"))
    if logits is not None:
        bi.logits = _ptr(logits)
        bi.logits_type = pb.dtype
        bi.row_lse = _ptr(row_lse)
    rc = oracle_lib().oracle_backward(C.byref(pb.args()), C.byref(bi), _ptr(grad))
    if rc != 0:
        raise ValueError("oracle_backward: invalid argument")
    return grad


def _backward_inputs(pb: Problem, trace, grads, logits, row_lse) -> A.BackwardInputs:
    bi = A.BackwardInputs()
    bi.parents, bi.tokens = _ptr(trace["parents"]), _ptr(trace["tokens"])
    bi.lengths, bi.from_logprob = _ptr(trace["lengths"]), _ptr(trace["from_logprob"])
    bi.grad_final_scores = _ptr(grads.get("final_scores"))
    bi.grad_final_raw_scores = _ptr(grads.get("final_raw_scores"))
    bi.grad_scores = _ptr(grads.get("scores"))
    bi.grad_raw_scores = _ptr(grads.get("raw_scores"))
    if logits is not None:
        bi.logits = _ptr(logits)
        bi.logits_type = pb.dtype
        bi.row_lse = _ptr(row_lse)
    return bi


def oracle_selected_weights(pb: Problem, scores: np.ndarray, temperature: float) -> np.ndarray:
    """softmax_selected per step (src/kernels_scalar.cpp:277-302) of the decode's scores [B, T, K]."""
    B, T, K, V = pb.shape
    sc = np.ascontiguousarray(scores, np.float32)
    w = np.empty((B, T, K), np.float32)
    oracle_lib().oracle_selected_weights(C.byref(pb.args()), _ptr(sc), temperature, _ptr(w))
    return w


def oracle_backward_selected(pb: Problem, trace, grads, weights, grad_weights, temperature: float,
                             logits=None, row_lse=None) -> np.ndarray:
    """oracle_backward plus the selected-beam weights term (src/decoder.cpp:599-604)."""
    B, T, K, V = pb.shape
    grad = np.zeros((B, T, K, V), np.float32)
    bi = _backward_inputs(pb, trace, grads, logits, row_lse)
    w = np.ascontiguousarray(weights, np.float32)
    gw = np.ascontiguousarray(grad_weights, np.float32)
    rc = oracle_lib().oracle_backward_selected(C.byref(pb.args()), C.byref(bi), _ptr(w), _ptr(gw), temperature,
                                               _ptr(grad))
    if rc != 0:
        raise ValueError("oracle_backward_selected: invalid argument")
    return grad


def oracle_path_gradient(pb: Problem, trace: dict[str, np.ndarray], g_final: np.ndarray) -> np.ndarray:
    B, T, K, V = pb.shape
    draws = np.zeros((B, T, K), np.float32)
    rc = oracle_lib().oracle_path_gradient(C.byref(pb.args()), _ptr(trace["parents"]), _ptr(trace["tokens"]),
                                           _ptr(trace["lengths"]), _ptr(trace["from_logprob"]), _ptr(g_final),
                                           _ptr(draws))
    if rc != 0:
        raise ValueError("oracle_path_gradient: invalid argument")
    return draws


def oracle_length_penalty(lengths: np.ndarray, alpha: float) -> np.ndarray:
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    out = np.zeros(lengths.shape, np.float32)
    oracle_lib().oracle_length_penalty(_ptr(lengths), lengths.size, alpha, _ptr(out))
    return out


def backtrack(tokens: np.ndarray, parents: np.ndarray, steps: np.ndarray | None) -> np.ndarray:
    """[B, K, T] token sequences (python/beamgrad/_torch.py:582-606 restated in numpy)."""
    B, T, K = tokens.shape
    steps = np.full(B, T) if steps is None else steps
    seq = np.full((B, K, T), -1, np.int64)
    beam = np.tile(np.arange(K), (B, 1))
    for t in range(T - 1, -1, -1):
        decoded = (t < steps)[:, None]
        alive = (beam >= 0) & decoded
        idx = np.clip(beam, 0, None)
        st = np.take_along_axis(tokens[:, t, :], idx, 1)
        sp = np.take_along_axis(parents[:, t, :], idx, 1)
        seq[:, :, t] = np.where(alive, st, -1)
        beam = np.where(decoded, np.where(beam >= 0, sp, -1), beam)
    return seq


# ---------------------------------------------------------------------------
# The reference library (beamgrad 2.3.0 libdbs)
# ---------------------------------------------------------------------------
class _Options(C.Structure):  # DBSOptionsC, include/dbs.h:64-79
    _fields_ = [("beam_size", C.c_int), ("eos_token", C.c_int), ("selected_temperature", C.c_float),
                ("soft_topk_temperature", C.c_float), ("relaxed_pool_multiplier", C.c_int),
                ("vocab_block", C.c_int), ("length_penalty_alpha", C.c_float), ("soft_topk_tolerance", C.c_float),
                ("soft_topk_max_iters", C.c_int), ("min_length", C.c_int), ("validate_inputs", C.c_int),
                ("max_dense_gradient_elements", C.c_int64), ("reserved0", C.c_int), ("reserved1", C.c_int)]


class _Constraints(C.Structure):  # DBSAdvancedConstraintsC, include/dbs.h:139-148
    _fields_ = [("banned_tokens", _p), ("forced_tokens", _p), ("min_length", C.c_int),
                ("repetition_penalty", C.c_float), ("no_repeat_ngram_size", C.c_int), ("token_filter", _p),
                ("token_filter_user_data", _p), ("batch_index", C.c_int)]


class _OutputsC(C.Structure):  # DBSDecodeOutputsC, include/dbs.h:153-163
    _fields_ = [(n, _p) for n in TRACE_FIELDS]


class _OutputsEx(C.Structure):  # DBSDecodeOutputsExC, include/dbs.h:339-349
    _fields_ = [("base", _OutputsC), ("pool_parents", _p), ("pool_tokens", _p), ("pool_lengths", _p),
                ("pool_scores", _p), ("pool_raw_scores", _p), ("pool_from_logprob", _p), ("row_lse", _p),
                ("reserved", _p * 4)]


class _BackwardC(C.Structure):  # DBSBackwardInputsC, include/dbs.h:373-397
    _fields_ = [("batch_size", C.c_int), ("steps", C.c_int), ("vocab_size", C.c_int), ("pool_size", C.c_int),
                ("steps_per_example", _p), ("parents", _p), ("tokens", _p), ("lengths", _p), ("from_logprob", _p),
                ("pool_parents", _p), ("pool_tokens", _p), ("pool_lengths", _p), ("pool_from_logprob", _p),
                ("grad_final_scores", _p), ("grad_final_raw_scores", _p), ("grad_scores", _p),
                ("grad_raw_scores", _p), ("grad_pool_scores", _p), ("grad_pool_raw_scores", _p), ("logits", _p),
                ("logits_type", C.c_int), ("row_lse", _p), ("reserved", _p * 4)]


_rlib = None
_rclib = None


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_cuda_available() -> bool:
    return REF_CUDA_LIB.exists()


def ref_cuda_lib() -> C.CDLL:
    """beamgrad 2.3.0's own GPU engine (cuda/dbs_cuda.cu built for sm_100a by oracle/Makefile),
    with the 17 entry points of its include/dbs_cuda.h typed like this repository's (the
    structs are layout-identical). The reference speed bar and a second parity check."""
    global _rclib
    if _rclib is None:
        if not REF_CUDA_LIB.exists():
            raise FileNotFoundError(f"{REF_CUDA_LIB} was not built (needs the reference sources and nvcc)")
        lib = C.CDLL(str(REF_CUDA_LIB))
        for name, (res, args) in A.SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is not None:
                fn.restype, fn.argtypes = res, args
        _rclib = lib
    return _rclib


def ref_lib() -> C.CDLL:
    global _rlib
    if _rlib is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} was not built (needs the reference sources; oracle/Makefile)")
        lib = C.CDLL(str(REF_LIB))
        lib.dbs_create_ex.restype = C.c_int
        lib.dbs_create_ex.argtypes = [_Options, C.POINTER(_p)]
        lib.dbs_destroy.restype = None
        lib.dbs_destroy.argtypes = [_p]
        lib.dbs_set_extra_eos_tokens.restype = C.c_int
        lib.dbs_set_extra_eos_tokens.argtypes = [_p, _p, C.c_int]
        lib.dbs_decode_batch_into_ex.restype = C.c_int
        lib.dbs_decode_batch_into_ex.argtypes = [_p, _p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _p,
                                                 C.POINTER(_Constraints), C.c_int, C.POINTER(_OutputsEx)]
        lib.dbs_backward_batch_into_ex.restype = C.c_int
        lib.dbs_backward_batch_into_ex.argtypes = [_p, C.POINTER(_BackwardC), C.c_int, _p]
        lib.dbs_last_global_error.restype = C.c_char_p
        lib.dbs_last_global_error.argtypes = []
        # Single-example API (include/dbs.h:215-221, 448-455, 480-515): the only one that
        # returns the selected-beam weights.
        lib.dbs_decode.restype = C.c_int
        lib.dbs_decode.argtypes = [_p, _p, C.c_int, C.c_int, C.POINTER(_p)]
        lib.dbs_result_weights.restype = C.POINTER(C.c_float)
        lib.dbs_result_weights.argtypes = [_p]
        lib.dbs_backward_dense.restype = C.c_int
        lib.dbs_backward_dense.argtypes = [_p, _p, _p, _p, _p, C.POINTER(_p)]
        lib.dbs_backward_grad_log_probs.restype = C.POINTER(C.c_float)
        lib.dbs_backward_grad_log_probs.argtypes = [_p]
        lib.dbs_free_result.restype = None
        lib.dbs_free_result.argtypes = [_p]
        lib.dbs_free_backward.restype = None
        lib.dbs_free_backward.argtypes = [_p]
        lib.dbs_last_error.restype = C.c_char_p
        lib.dbs_last_error.argtypes = [_p]
        _rlib = lib
    return _rlib


class RefDecoder:
    """A libdbs decoder handle configured like `pb` (no per-example beams / EOS / min lengths)."""

    def __init__(self, pb: Problem, pool_multiplier: int = 0):
        if pb.beams is not None or pb.eos_pe is not None or pb.minlen_pe is not None:
            raise ValueError("libdbs has no per-example beam sizes, EOS tokens or minimum lengths")
        lib = ref_lib()
        o = _Options()
        o.beam_size = pb.shape[2]
        o.eos_token = pb.eos
        o.length_penalty_alpha = pb.alpha
        o.min_length = pb.min_length
        o.relaxed_pool_multiplier = pool_multiplier  # P = K * pool_multiplier pool candidates per step
        self.P = pb.shape[2] * pool_multiplier
        o.validate_inputs = 0  # NaN/+inf entries are never selected (the engine reports flags instead)
        h = _p()
        if lib.dbs_create_ex(o, C.byref(h)) != 0:
            raise RuntimeError(lib.dbs_last_global_error().decode())
        self.h = h
        self.pb = pb
        if pb.extra_eos:
            toks = np.array(pb.extra_eos, np.int32)
            if lib.dbs_set_extra_eos_tokens(h, _ptr(toks), len(toks)) != 0:
                raise RuntimeError(lib.dbs_last_global_error().decode())

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        ref_lib().dbs_destroy(self.h)

    def _constraints(self):
        pb = self.pb
        if pb.banned is None and pb.ngram <= 0 and pb.rep_penalty == 1.0:
            return None
        c = _Constraints()
        c.banned_tokens = _ptr(pb.banned)
        c.min_length = -1
        c.repetition_penalty = pb.rep_penalty
        c.no_repeat_ngram_size = pb.ngram
        return c

    def decode(self, threads: int = 1) -> dict[str, np.ndarray]:
        """The decode's outputs; with a pool also pool_parents ... pool_from_logprob [B, T, P]."""
        pb = self.pb
        B, T, K, V = pb.shape
        out = empty_outputs(B, T, K)
        ex = _OutputsEx()
        for n in TRACE_FIELDS:
            setattr(ex.base, n, _ptr(out[n]))
        ex.row_lse = _ptr(out["row_lse"])
        if self.P:
            P = self.P
            for n, dt in (("parents", np.int32), ("tokens", np.int32), ("lengths", np.int32), ("scores", np.float32),
                          ("raw_scores", np.float32), ("from_logprob", np.uint8)):
                out["pool_" + n] = np.full((B, T, P), 77, dt)
                setattr(ex, "pool_" + n, _ptr(out["pool_" + n]))
        c = self._constraints()
        x = np.ascontiguousarray(pb.x)
        rc = ref_lib().dbs_decode_batch_into_ex(self.h, _ptr(x), pb.dtype, int(pb.from_logits), B, T, V,
                                                _ptr(pb.steps), C.byref(c) if c is not None else None, threads,
                                                C.byref(ex))
        if rc != 0:
            raise RuntimeError(ref_lib().dbs_last_global_error().decode())
        return out

    def backward(self, trace, grads, logits=None, row_lse=None, threads: int = 1, pool=None) -> np.ndarray:
        """Dense float32 input gradient; pool: the decode's pool_* arrays, with grads'
        pool_scores / pool_raw_scores gradients [B, T, P]."""
        pb = self.pb
        B, T, K, V = pb.shape
        grad = np.zeros((B, T, K, V), np.float32)
        bi = _BackwardC()
        bi.batch_size, bi.steps, bi.vocab_size, bi.pool_size = B, T, V, 0
        if pool is not None:
            bi.pool_size = self.P
            bi.pool_parents, bi.pool_tokens = _ptr(pool["pool_parents"]), _ptr(pool["pool_tokens"])
            bi.pool_lengths, bi.pool_from_logprob = _ptr(pool["pool_lengths"]), _ptr(pool["pool_from_logprob"])
            bi.grad_pool_scores = _ptr(grads.get("pool_scores"))
            bi.grad_pool_raw_scores = _ptr(grads.get("pool_raw_scores"))
        bi.steps_per_example = _ptr(pb.steps)
        bi.parents, bi.tokens = _ptr(trace["parents"]), _ptr(trace["tokens"])
        bi.lengths, bi.from_logprob = _ptr(trace["lengths"]), _ptr(trace["from_logprob"])
        bi.grad_final_scores = _ptr(grads.get("final_scores"))
        bi.grad_final_raw_scores = _ptr(grads.get("final_raw_scores"))
        bi.grad_scores = _ptr(grads.get("scores"))
        bi.grad_raw_scores = _ptr(grads.get("raw_scores"))
        if logits is not None:
            bi.logits = _ptr(logits)
            bi.logits_type = pb.dtype
            bi.row_lse = _ptr(row_lse)
        rc = ref_lib().dbs_backward_batch_into_ex(self.h, C.byref(bi), threads, _ptr(grad))
        if rc != 0:
            raise RuntimeError(ref_lib().dbs_last_global_error().decode())
        return grad


def ref_decode(pb: Problem, threads: int = 1) -> dict[str, np.ndarray]:
    with RefDecoder(pb) as d:
        return d.decode(threads)


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def ref_selected(x: np.ndarray, beam: int, eos: int, alpha: float, min_length: int, temperature: float,
                 grad_weights: np.ndarray, grad_final: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference library's own selected-beam weights [T, K] and dense input gradient [T, K, V] of
    one float32 log-prob example x [T, K, V] (dbs_decode, dbs_result_weights, dbs_backward_dense with
    grad_selected_weights and grad_final_scores)."""
    lib = ref_lib()
    T, K, V = x.shape
    o = _Options()
    o.beam_size, o.eos_token, o.selected_temperature = beam, eos, temperature
    o.length_penalty_alpha, o.min_length = alpha, min_length
    o.max_dense_gradient_elements = T * K * V + 1
    h = _p()
    if lib.dbs_create_ex(o, C.byref(h)) != 0:
        raise RuntimeError(lib.dbs_last_global_error().decode())
    res, bw = _p(), _p()
    try:
        xc = np.ascontiguousarray(x, np.float32)
        if lib.dbs_decode(h, _ptr(xc), T, V, C.byref(res)) != 0:
            raise RuntimeError(lib.dbs_last_error(h).decode())
        w = np.ctypeslib.as_array(lib.dbs_result_weights(res), shape=(T * K,)).reshape(T, K).copy()
        gw = np.ascontiguousarray(grad_weights, np.float32)
        gf = np.ascontiguousarray(grad_final, np.float32)
        if lib.dbs_backward_dense(h, res, _ptr(gw), None, _ptr(gf), C.byref(bw)) != 0:
            raise RuntimeError(lib.dbs_last_error(h).decode())
        g = np.ctypeslib.as_array(lib.dbs_backward_grad_log_probs(bw), shape=(T * K * V,)).reshape(T, K, V).copy()
    finally:
        if bw:
            lib.dbs_free_backward(bw)
        if res:
            lib.dbs_free_result(res)
        lib.dbs_destroy(h)
    return w, g


def ref_relaxed(x: np.ndarray, beam: int, eos: int, alpha: float, min_length: int, multiplier: int, temperature: float,
                tolerance: float, max_iters: int, grad_relaxed: np.ndarray, grad_final: np.ndarray):
    """The reference library's relaxed pool of one float32 log-prob example x [T, K, V]: the pool
    (tokens, parents, lengths, scores, raw scores [T, P]), its relaxed weights [T, P] and the dense
    input gradient [T, K, V] for grad_relaxed_weights and grad_final_scores (dbs_decode,
    dbs_result_pool_* / dbs_result_relaxed_weights, dbs_backward_dense: include/dbs.h:215-221,
    448-455, 494-501)."""
    lib = ref_lib()
    for name, res_t in (("dbs_result_relaxed_weights", C.POINTER(C.c_float)),
                        ("dbs_result_pool_scores", C.POINTER(C.c_float)),
                        ("dbs_result_pool_raw_scores", C.POINTER(C.c_float)),
                        ("dbs_result_pool_tokens", C.POINTER(C.c_int32)),
                        ("dbs_result_pool_parents", C.POINTER(C.c_int32)),
                        ("dbs_result_pool_lengths", C.POINTER(C.c_int32))):
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res_t, [_p]
    T, K, V = x.shape
    P = K * multiplier
    o = _Options()
    o.beam_size, o.eos_token, o.length_penalty_alpha, o.min_length = beam, eos, alpha, min_length
    o.relaxed_pool_multiplier, o.soft_topk_temperature = multiplier, temperature
    o.soft_topk_tolerance, o.soft_topk_max_iters = tolerance, max_iters
    o.max_dense_gradient_elements = T * K * V + 1
    h = _p()
    if lib.dbs_create_ex(o, C.byref(h)) != 0:
        raise RuntimeError(lib.dbs_last_global_error().decode())
    res, bw = _p(), _p()
    out = {}
    try:
        xc = np.ascontiguousarray(x, np.float32)
        if lib.dbs_decode(h, _ptr(xc), T, V, C.byref(res)) != 0:
            raise RuntimeError(lib.dbs_last_error(h).decode())
        for key, fn in (("relaxed_weights", lib.dbs_result_relaxed_weights), ("pool_scores", lib.dbs_result_pool_scores),
                        ("pool_raw_scores", lib.dbs_result_pool_raw_scores), ("pool_tokens", lib.dbs_result_pool_tokens),
                        ("pool_parents", lib.dbs_result_pool_parents), ("pool_lengths", lib.dbs_result_pool_lengths)):
            out[key] = np.ctypeslib.as_array(fn(res), shape=(T * P,)).reshape(T, P).copy()
        gr = np.ascontiguousarray(grad_relaxed, np.float32)
        gf = np.ascontiguousarray(grad_final, np.float32)
        if lib.dbs_backward_dense(h, res, None, _ptr(gr), _ptr(gf), C.byref(bw)) != 0:
            raise RuntimeError(lib.dbs_last_error(h).decode())
        out["grad"] = np.ctypeslib.as_array(lib.dbs_backward_grad_log_probs(bw), shape=(T * K * V,)).reshape(T, K, V).copy()
    finally:
        if bw:
            lib.dbs_free_backward(bw)
        if res:
            lib.dbs_free_result(res)
        lib.dbs_destroy(h)
    return out
