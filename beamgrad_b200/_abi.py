# SPDX-License-Identifier: MIT
"""ctypes view of the engine's C ABI (include/dbs_cuda.h, include/dbs_cuda_b200.h).

The structs mirror the header field for field (tests/test_abi.py checks every
size and offset against the C compiler's layout of both this header and the
reference's). :func:`load` opens ``libdbs_cuda.so`` from this package and fails
loudly when it is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdbs_cuda.so"

STATUS_OK = 0
STATUS_UNAVAILABLE = 1
STATUS_INVALID_ARGUMENT = 2
STATUS_LAUNCH_FAILED = 3
STATUS_OUT_OF_MEMORY = 4
MAX_BEAM = 1024
MAX_EXTRA_EOS = 16
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

_p = C.c_void_p


class DecodeArgs(C.Structure):
    """DBSCudaDecodeArgs."""

    _fields_ = [
        ("batch_size", C.c_int),
        ("steps", C.c_int),
        ("beam_size", C.c_int),
        ("vocab_size", C.c_int),
        ("eos_token", C.c_int),
        ("min_length", C.c_int),
        ("length_penalty_alpha", C.c_float),
        ("no_repeat_ngram_size", C.c_int),
        ("repetition_penalty", C.c_float),
        ("reserved0", C.c_int),
        ("steps_per_example", _p),
        ("beam_sizes_per_example", _p),
        ("eos_tokens_per_example", _p),
        ("min_lengths_per_example", _p),
        ("banned_tokens", _p),
    ]


class DecodeOutputs(C.Structure):
    """DBSCudaDecodeOutputs."""

    _fields_ = [
        ("final_scores", _p),
        ("final_raw_scores", _p),
        ("final_lengths", _p),
        ("tokens", _p),
        ("parents", _p),
        ("lengths", _p),
        ("scores", _p),
        ("raw_scores", _p),
        ("from_logprob", _p),
        ("invalid_input", _p),
    ]


class BeamState(C.Structure):
    """DBSCudaBeamState."""

    _fields_ = [
        ("raw_scores", _p),
        ("lengths", _p),
        ("finished", _p),
        ("prefixes", _p),
        ("prefix_stride", C.c_int),
        ("reserved0", C.c_int),
    ]


class BackwardInputs(C.Structure):
    """DBSCudaBackwardInputs."""

    _fields_ = [
        ("parents", _p),
        ("tokens", _p),
        ("lengths", _p),
        ("from_logprob", _p),
        ("grad_final_scores", _p),
        ("grad_final_raw_scores", _p),
        ("grad_scores", _p),
        ("grad_raw_scores", _p),
        ("logits", _p),
        ("logits_type", C.c_int),
        ("reserved0", C.c_int),
        ("row_lse", _p),
        ("reserved", _p * 4),
    ]


class SearchOptions(C.Structure):
    """DBSCudaSearchOptions."""

    _fields_ = [
        ("extra_eos_count", C.c_int),
        ("extra_eos_tokens", C.c_int32 * MAX_EXTRA_EOS),
        ("reserved0", C.c_int),
        ("reserved", _p * 4),
    ]


class VocabShardPlan(C.Structure):
    """DBSCudaVocabShardPlan."""

    _fields_ = [
        ("world_size", C.c_int32),
        ("rank", C.c_int32),
        ("shard_vocab", C.c_int32),
        ("lanes", C.c_int32),
        ("list_len", C.c_int32),
        ("shard_list_len", C.c_int32),
        ("row_words", C.c_int32),
        ("reserved0", C.c_int32),
        ("rows", C.c_int64),
        ("workspace_bytes", C.c_int64),
    ]


class VocabShardBuffers(C.Structure):
    """DBSCudaVocabShardBuffers."""

    _fields_ = [
        ("row_max", _p),
        ("row_min", _p),
        ("exchange", _p),
        ("exchange_all", _p),
        ("resume", _p),
        ("stalled", _p),
        ("rescan_rows", _p),
        ("rescan_slot", _p),
        ("rescan", _p),
        ("rescan_all", _p),
        ("n_rescan", C.c_int64),
        ("workspace", _p),
        ("workspace_bytes", C.c_int64),
    ]


class VocabShardCall(C.Structure):
    """DBSCudaVocabShardCall."""

    _fields_ = [
        ("shard_inputs", _p),
        ("data_type", C.c_int32),
        ("from_logits", C.c_int32),
        ("world_size", C.c_int32),
        ("rank", C.c_int32),
        ("shard_list_len", C.c_int32),
        ("reserved0", C.c_int32),
        ("args", C.POINTER(DecodeArgs)),
        ("options", C.POINTER(SearchOptions)),
        ("buffers", VocabShardBuffers),
        ("outputs", DecodeOutputs),
        ("row_lse", _p),
    ]


class PoolOutputs(C.Structure):
    """DBSCudaPoolOutputs."""

    _fields_ = [
        ("parents", _p),
        ("tokens", _p),
        ("lengths", _p),
        ("scores", _p),
        ("raw_scores", _p),
        ("from_logprob", _p),
        ("relaxed_weights", _p),
        ("reserved", _p * 4),
    ]


class PoolGradients(C.Structure):
    """DBSCudaPoolGradients."""

    _fields_ = [
        ("pool_size", C.c_int32),
        ("reserved0", C.c_int32),
        ("parents", _p),
        ("tokens", _p),
        ("lengths", _p),
        ("from_logprob", _p),
        ("relaxed_weights", _p),
        ("grad_relaxed_weights", _p),
        ("grad_pool_scores", _p),
        ("grad_pool_raw_scores", _p),
        ("soft_topk_temperature", C.c_float),
        ("reserved", _p * 4),
    ]


MAX_POOL = 1024  # DBS_CUDA_B200_MAX_POOL

VSHARD_MAX_WORLD = 8

# name -> (restype, argtypes). The 17 reference entry points, then this engine's additions.
SIGNATURES = {
    "dbs_cuda_available": (C.c_int, []),
    "dbs_cuda_status_string": (C.c_char_p, [C.c_int]),
    "dbs_cuda_set_synchronization": (C.c_int, [C.c_int]),
    "dbs_cuda_get_synchronization": (C.c_int, []),
    "dbs_cuda_decode_workspace_size": (C.c_int64, [C.POINTER(DecodeArgs)]),
    "dbs_cuda_backward_workspace_size": (C.c_int64, [C.POINTER(DecodeArgs)]),
    "dbs_cuda_decode_step_workspace_size": (C.c_int64, [C.POINTER(DecodeArgs), C.c_int]),
    "dbs_cuda_decode": (C.c_int, [_p, C.POINTER(DecodeArgs), C.POINTER(DecodeOutputs), _p, C.c_int64, _p]),
    "dbs_cuda_decode_ex": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(DecodeOutputs), _p, _p, C.c_int64, _p],
    ),
    "dbs_cuda_decode_ex2": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(SearchOptions), C.POINTER(DecodeOutputs), _p, _p,
         C.c_int64, _p],
    ),
    "dbs_cuda_decode_step": (
        C.c_int,
        [_p, C.POINTER(DecodeArgs), C.POINTER(BeamState), C.POINTER(DecodeOutputs), _p, C.c_int64, _p],
    ),
    "dbs_cuda_decode_step_ex": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(BeamState), C.POINTER(DecodeOutputs), _p, _p,
         C.c_int64, _p],
    ),
    "dbs_cuda_decode_step_ex2": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(SearchOptions), C.POINTER(BeamState),
         C.POINTER(DecodeOutputs), _p, _p, C.c_int64, _p],
    ),
    "dbs_cuda_backward": (
        C.c_int,
        [C.POINTER(DecodeArgs), _p, _p, _p, _p, _p, _p, _p, C.c_int64, _p],
    ),
    "dbs_cuda_backward_ex": (
        C.c_int,
        [C.POINTER(DecodeArgs), C.POINTER(BackwardInputs), _p, _p, C.c_int64, _p],
    ),
    "dbs_cuda_length_penalty": (C.c_int, [_p, C.c_int64, C.c_float, _p, _p]),
    "dbs_cuda_path_gradient": (C.c_int, [C.POINTER(DecodeArgs), _p, _p, _p, _p, _p, _p, _p]),
    # additions (include/dbs_cuda_b200.h)
    "dbs_cuda_b200_abi_version": (C.c_int, []),
    "dbs_cuda_backtrack": (C.c_int, [C.POINTER(DecodeArgs), _p, _p, _p, _p]),
    "dbs_cuda_advance_prefixes": (
        C.c_int,
        [C.c_int, C.c_int, C.c_int, C.c_int, _p, _p, _p, _p, _p, _p, _p, _p, _p],
    ),
    "dbs_cuda_backward_dense": (
        C.c_int,
        [C.POINTER(DecodeArgs), C.POINTER(BackwardInputs), _p, C.c_int, _p, C.c_int64, _p],
    ),
    "dbs_cuda_selected_weights": (C.c_int, [C.POINTER(DecodeArgs), _p, C.c_float, _p, _p]),
    "dbs_cuda_b200_wait_selftest": (C.c_int, [C.c_int64, _p, _p]),
    "dbs_cuda_backward_selected": (
        C.c_int,
        [C.POINTER(DecodeArgs), C.POINTER(BackwardInputs), _p, _p, C.c_float, _p, C.c_int, _p, C.c_int64, _p],
    ),
    "dbs_cuda_decode_no_alloc": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(SearchOptions), C.POINTER(DecodeOutputs), _p, _p],
    ),
    "dbs_cuda_vshard_plan": (C.c_int, [C.POINTER(DecodeArgs), C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.POINTER(VocabShardPlan)]),
    "dbs_cuda_vshard_scan": (C.c_int, [C.POINTER(VocabShardCall), _p]),
    "dbs_cuda_vshard_lanes": (C.c_int, [C.POINTER(VocabShardCall), _p]),
    "dbs_cuda_vshard_merge": (C.c_int, [C.POINTER(VocabShardCall), _p]),
    "dbs_cuda_vshard_select": (C.c_int, [C.POINTER(VocabShardCall), _p]),
    "dbs_cuda_vshard_rescan": (C.c_int, [C.POINTER(VocabShardCall), _p]),
    "dbs_cuda_relaxed_pool": (
        C.c_int,
        [_p, C.c_int, C.c_int, C.POINTER(DecodeArgs), C.POINTER(DecodeOutputs), _p, C.c_int, C.c_float, C.c_float,
         C.c_int, C.POINTER(PoolOutputs), _p],
    ),
    "dbs_cuda_backward_pool": (
        C.c_int, [C.POINTER(DecodeArgs), C.POINTER(BackwardInputs), C.POINTER(PoolGradients), _p, _p]),
}

VSHARD_SYMBOLS = ("dbs_cuda_vshard_plan", "dbs_cuda_vshard_scan", "dbs_cuda_vshard_lanes", "dbs_cuda_vshard_merge",
                  "dbs_cuda_vshard_select", "dbs_cuda_vshard_rescan")
ADDED_SYMBOLS = ("dbs_cuda_b200_abi_version", "dbs_cuda_backtrack", "dbs_cuda_backward_dense", "dbs_cuda_advance_prefixes",
                 "dbs_cuda_selected_weights", "dbs_cuda_backward_selected", "dbs_cuda_b200_wait_selftest",
                 "dbs_cuda_decode_no_alloc", "dbs_cuda_relaxed_pool", "dbs_cuda_backward_pool") + VSHARD_SYMBOLS
REFERENCE_SYMBOLS = [n for n in SIGNATURES if n not in ADDED_SYMBOLS]

# Size of the fixed device array behind dbs_cuda_decode_no_alloc (DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES).
NO_ALLOC_SCRATCH_BYTES = 4 * 1024 * 1024

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """The engine library, with typed entry points. Raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA engine first (python -m beamgrad_b200.build). "
                "There is no CPU fallback."
            )
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class EngineError(RuntimeError):
    """A status code other than DBS_CUDA_STATUS_OK."""

    def __init__(self, status: int, what: str):
        text = load().dbs_cuda_status_string(status).decode()
        super().__init__(f"beamgrad_b200 {what}: {text} (status {status})")
        self.status = status


class InvalidArgument(EngineError, ValueError):
    pass


def check(status: int, what: str) -> None:
    if status == STATUS_OK:
        return
    if status == STATUS_INVALID_ARGUMENT:
        raise InvalidArgument(status, what)
    raise EngineError(status, what)
