# SPDX-License-Identifier: MIT
"""``torch.ops.beamgrad.*`` on the B200 engine.

:func:`load` makes the seven beamgrad operators callable on CUDA tensors with this engine's
kernels (``beamgrad_b200/_C_cuda``), a drop-in for beamgrad's own ``beamgrad._C_cuda``
(python/csrc/cuda_ops.cpp of beamgrad 2.3.0). The operator schemas are beamgrad's
(python/csrc/cpu_ops.cpp:582-608): when beamgrad's ``_C`` module is importable it defines
them (and its CPU kernels); otherwise they are defined here, with no CPU kernels.

There is no fallback: if the CUDA library or the operator module is not built, load()
raises.
"""

from __future__ import annotations

import importlib

import torch

from beamgrad_b200 import _abi

# beamgrad 2.3.0 python/csrc/cpu_ops.cpp:582-608 (the operator contract, kept identical).
SCHEMAS = (
    "decode(Tensor log_probs, Tensor? steps, int eos_token, int min_length, float length_penalty_alpha, "
    "Tensor? banned_tokens, int no_repeat_ngram_size, float repetition_penalty, bool validate) -> "
    "(Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
    "final_scores_backward(Tensor grad_final, Tensor parents, Tensor tokens, Tensor lengths, "
    "Tensor from_logprob, Tensor? steps, int vocab_size, float length_penalty_alpha) -> Tensor",
    "length_penalty(Tensor lengths, float length_penalty_alpha) -> Tensor",
    "final_scores_path_gradient(Tensor grad_final, Tensor parents, Tensor tokens, Tensor lengths, "
    "Tensor from_logprob, Tensor? steps, int vocab_size, float length_penalty_alpha) -> Tensor",
    "decode_step(Tensor log_probs, Tensor raw_scores, Tensor lengths, Tensor finished, Tensor prefixes, "
    "int eos_token, int min_length, float length_penalty_alpha, Tensor? banned_tokens, int no_repeat_ngram_size, "
    "float repetition_penalty, bool validate, int[] extra_eos=[]) -> "
    "(Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
    "decode_ex(Tensor inputs, bool from_logits, Tensor? steps, int eos_token, int min_length, "
    "float length_penalty_alpha, Tensor? banned_tokens, int no_repeat_ngram_size, float repetition_penalty, "
    "bool validate, int[] extra_eos=[]) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, "
    "Tensor)",
    "decode_backward(Tensor? grad_final_scores, Tensor? grad_final_raw_scores, Tensor? grad_scores, "
    "Tensor? grad_raw_scores, Tensor parents, Tensor tokens, Tensor lengths, Tensor from_logprob, Tensor? steps, "
    "int vocab_size, float length_penalty_alpha, Tensor? logits, Tensor? row_lse) -> Tensor",
)
OPERATORS = tuple(s.split("(", 1)[0] for s in SCHEMAS)

_library = None  # keeps the schema definitions alive when this module made them
_module = None


def _schemas_defined() -> bool:
    try:
        getattr(torch.ops.beamgrad, "decode_ex")
        return True
    except (AttributeError, RuntimeError):
        return False


def load():
    """Registers the CUDA kernels (once) and returns the ``_C_cuda`` module."""
    global _library, _module
    if _module is not None:
        return _module
    _abi.load()  # the engine library, by its soname, before the operator module links to it
    if not _schemas_defined():
        try:
            importlib.import_module("beamgrad._C")  # beamgrad's own schemas and CPU kernels
        except ImportError:
            pass
    if not _schemas_defined():
        _library = torch.library.Library("beamgrad", "DEF")
        for schema in SCHEMAS:
            _library.define(schema)
    try:
        _module = importlib.import_module("beamgrad_b200._C_cuda")
    except ImportError as e:
        raise RuntimeError(
            "beamgrad_b200._C_cuda is not built (python -m beamgrad_b200.build); there is no fallback") from e
    return _module
