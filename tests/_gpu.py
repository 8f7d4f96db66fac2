# SPDX-License-Identifier: MIT
"""Calls the CUDA engine through its C ABI (libdbs_cuda.so) on torch-owned device memory."""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from beamgrad_b200 import _abi as A
from oracle.oracle import Problem

_SENTINEL = {np.float32: np.float32(12345.0), np.int32: np.int32(-777), np.uint8: np.uint8(77)}


def dev(a: np.ndarray | None, device="cuda"):
    if a is None:
        return None
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a.copy()).to(device)


def ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_ptr():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class DeviceProblem:
    """The device copies of a Problem's inputs and the DecodeArgs pointing at them."""

    def __init__(self, pb: Problem, device="cuda", x_dev: torch.Tensor | None = None):
        self.pb = pb
        self.x = x_dev if x_dev is not None else dev(pb.x, device)
        self.steps = dev(pb.steps, device)
        self.beams = dev(pb.beams, device)
        self.eos_pe = dev(pb.eos_pe, device)
        self.minlen_pe = dev(pb.minlen_pe, device)
        self.banned = dev(pb.banned, device)

    def args(self) -> A.DecodeArgs:
        a = self.pb.args()
        a.steps_per_example = ptr(self.steps)
        a.beam_sizes_per_example = ptr(self.beams)
        a.eos_tokens_per_example = ptr(self.eos_pe)
        a.min_lengths_per_example = ptr(self.minlen_pe)
        a.banned_tokens = ptr(self.banned)
        return a


def _outputs(B, T, K, device="cuda"):
    mk = lambda shape, dt, fill: torch.full(shape, fill, dtype=dt, device=device)  # noqa: E731
    return {
        "final_scores": mk((B, K), torch.float32, 12345.0),
        "final_raw_scores": mk((B, K), torch.float32, 12345.0),
        "final_lengths": mk((B, K), torch.int32, -777),
        "tokens": mk((B, T, K), torch.int32, -777),
        "parents": mk((B, T, K), torch.int32, -777),
        "lengths": mk((B, T, K), torch.int32, -777),
        "scores": mk((B, T, K), torch.float32, 12345.0),
        "raw_scores": mk((B, T, K), torch.float32, 12345.0),
        "from_logprob": mk((B, T, K), torch.uint8, 77),
        "invalid": mk((B,), torch.uint8, 77),
        "row_lse": mk((B, T, K), torch.float32, 12345.0),
    }


def _out_struct(o) -> A.DecodeOutputs:
    s = A.DecodeOutputs()
    for name in ("final_scores", "final_raw_scores", "final_lengths", "tokens", "parents", "lengths", "scores",
                 "raw_scores", "from_logprob"):
        setattr(s, name, ptr(o[name]))
    s.invalid_input = ptr(o["invalid"])
    return s


def engine_decode(pb: Problem, use_workspace: bool = True, dp: DeviceProblem | None = None,
                  lib=None) -> dict[str, np.ndarray]:
    """dbs_cuda_decode_ex2 of this repository's engine, or of `lib` (another library with the
    same C ABI, e.g. the reference's own GPU engine)."""
    lib = lib or A.load()
    dp = dp or DeviceProblem(pb)
    B, T, K, V = pb.shape
    o = _outputs(B, T, K)
    args = dp.args()
    opts = pb.options()
    ws = None
    ws_bytes = 0
    if use_workspace:
        ws_bytes = lib.dbs_cuda_decode_workspace_size(C.byref(args))
        assert ws_bytes > 0
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.dbs_cuda_decode_ex2(ptr(dp.x), pb.dtype, int(pb.from_logits), C.byref(args),
                                 C.byref(opts) if opts is not None else None, C.byref(_out_struct(o)),
                                 ptr(o["row_lse"]), ptr(ws), ws_bytes, stream_ptr())
    A.check(rc, "decode")
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in o.items()}


def engine_step(pb: Problem, raw, lengths, finished, prefixes) -> dict[str, np.ndarray]:
    """One dbs_cuda_decode_step_ex2 over pb.x [B, 1, K, V]."""
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    o = _outputs(B, 1, K)
    st_raw, st_len, st_fin = dev(raw), dev(lengths), dev(finished)
    pre = dev(prefixes) if prefixes is not None else None
    st = A.BeamState()
    st.raw_scores, st.lengths, st.finished, st.prefixes = ptr(st_raw), ptr(st_len), ptr(st_fin), ptr(pre)
    st.prefix_stride = 0 if prefixes is None else int(prefixes.shape[-1])
    args = dp.args()
    opts = pb.options()
    ws_bytes = lib.dbs_cuda_decode_step_workspace_size(C.byref(args), st.prefix_stride)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    rc = lib.dbs_cuda_decode_step_ex2(ptr(dp.x), pb.dtype, int(pb.from_logits), C.byref(args),
                                      C.byref(opts) if opts is not None else None, C.byref(st),
                                      C.byref(_out_struct(o)), ptr(o["row_lse"]), ptr(ws), ws_bytes, stream_ptr())
    A.check(rc, "decode_step")
    torch.cuda.synchronize()
    out = {k: v.cpu().numpy() for k, v in o.items()}
    out["state_raw"], out["state_lengths"], out["state_finished"] = st_raw.cpu().numpy(), st_len.cpu().numpy(), st_fin.cpu().numpy()
    return out


def engine_selected_weights(pb: Problem, scores: np.ndarray, temperature: float) -> np.ndarray:
    lib = A.load()
    dp = DeviceProblem(pb)
    sc = dev(np.ascontiguousarray(scores, np.float32))
    w = torch.full(sc.shape, 99.0, dtype=torch.float32, device="cuda")
    A.check(lib.dbs_cuda_selected_weights(C.byref(dp.args()), ptr(sc), temperature, ptr(w), stream_ptr()),
            "selected_weights")
    torch.cuda.synchronize()
    return w.cpu().numpy()


def engine_backward_selected(pb: Problem, trace: dict[str, np.ndarray], grads: dict, weights, grad_weights,
                             temperature: float, logits=None, row_lse=None) -> np.ndarray:
    """dbs_cuda_backward_selected, float32 dense output."""
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    t = {k: dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    g = {k: dev(v) for k, v in grads.items() if v is not None}
    bi = A.BackwardInputs()
    bi.parents, bi.tokens, bi.lengths, bi.from_logprob = (ptr(t[k]) for k in ("parents", "tokens", "lengths", "from_logprob"))
    bi.grad_final_scores = ptr(g.get("final_scores"))
    bi.grad_scores = ptr(g.get("scores"))
    lg = lse = None
    if logits is not None:
        lg, lse = dev(logits), dev(row_lse)
        bi.logits, bi.logits_type, bi.row_lse = ptr(lg), pb.dtype, ptr(lse)
    w, gw = dev(np.ascontiguousarray(weights, np.float32)), dev(np.ascontiguousarray(grad_weights, np.float32))
    grad = torch.full((B, T, K, V), 77.0, dtype=torch.float32, device="cuda")
    args = dp.args()
    ws_bytes = lib.dbs_cuda_backward_workspace_size(C.byref(args))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    rc = lib.dbs_cuda_backward_selected(C.byref(args), C.byref(bi), ptr(w), ptr(gw), temperature, ptr(grad),
                                        A.DTYPE_F32, ptr(ws), ws_bytes, stream_ptr())
    A.check(rc, "backward_selected")
    torch.cuda.synchronize()
    return grad.cpu().numpy()


def engine_backward(pb: Problem, trace: dict[str, np.ndarray], grads: dict, logits=None, row_lse=None,
                    use_workspace: bool = True, dense: int | None = None, misalign: int = 0):
    """dbs_cuda_backward_ex into a zeroed float32 gradient, or (dense = a DTYPE_*)
    dbs_cuda_backward_dense writing the gradient in that type (a torch tensor for 16-bit types)."""
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    t = {k: dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    g = {k: dev(v) for k, v in grads.items() if v is not None}
    bi = A.BackwardInputs()
    bi.parents, bi.tokens, bi.lengths, bi.from_logprob = (ptr(t[k]) for k in ("parents", "tokens", "lengths", "from_logprob"))
    bi.grad_final_scores = ptr(g.get("final_scores"))
    bi.grad_final_raw_scores = ptr(g.get("final_raw_scores"))
    bi.grad_scores = ptr(g.get("scores"))
    bi.grad_raw_scores = ptr(g.get("raw_scores"))
    lg = lse = None
    if logits is not None:
        lg, lse = dev(logits), dev(row_lse)
        bi.logits, bi.logits_type, bi.row_lse = ptr(lg), pb.dtype, ptr(lse)
    args = dp.args()
    ws = None
    ws_bytes = 0
    if use_workspace:
        ws_bytes = lib.dbs_cuda_backward_workspace_size(C.byref(args))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    if dense is None:
        grad = torch.zeros((B, T, K, V), dtype=torch.float32, device="cuda")
        rc = lib.dbs_cuda_backward_ex(C.byref(args), C.byref(bi), ptr(grad), ptr(ws), ws_bytes, stream_ptr())
    else:
        # dbs_cuda_backward_dense overwrites every element: start from a sentinel, optionally
        # at an offset that is not 16-byte aligned (the scalar path).
        tdt = {A.DTYPE_F32: torch.float32, A.DTYPE_F16: torch.float16, A.DTYPE_BF16: torch.bfloat16}[dense]
        store = torch.full((B * T * K * V + misalign,), 77.0, dtype=tdt, device="cuda")
        grad = store[misalign:].view(B, T, K, V)
        rc = lib.dbs_cuda_backward_dense(C.byref(args), C.byref(bi), ptr(grad), dense, ptr(ws), ws_bytes, stream_ptr())
    A.check(rc, "backward")
    torch.cuda.synchronize()
    return grad.cpu().numpy() if dense in (None, A.DTYPE_F32) else grad.cpu()


def engine_path_gradient(pb: Problem, trace, g_final) -> np.ndarray:
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    t = {k: dev(trace[k]) for k in ("parents", "tokens", "lengths", "from_logprob")}
    draws = torch.full((B, T, K), 99.0, dtype=torch.float32, device="cuda")
    gf = dev(g_final)
    rc = lib.dbs_cuda_path_gradient(C.byref(dp.args()), ptr(t["parents"]), ptr(t["tokens"]), ptr(t["lengths"]),
                                    ptr(t["from_logprob"]), ptr(gf), ptr(draws), stream_ptr())
    A.check(rc, "path_gradient")
    torch.cuda.synchronize()
    return draws.cpu().numpy()


def engine_length_penalty(lengths: np.ndarray, alpha: float) -> np.ndarray:
    lib = A.load()
    ln = dev(np.ascontiguousarray(lengths, np.int32))
    out = torch.empty(ln.shape, dtype=torch.float32, device="cuda")
    A.check(lib.dbs_cuda_length_penalty(ptr(ln), ln.numel(), alpha, ptr(out), stream_ptr()), "length_penalty")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def engine_backtrack(pb: Problem, tokens: np.ndarray, parents: np.ndarray) -> np.ndarray:
    lib = A.load()
    dp = DeviceProblem(pb)
    B, T, K, V = pb.shape
    tk, pr = dev(tokens), dev(parents)
    out = torch.empty((B, K, T), dtype=torch.int64, device="cuda")
    A.check(lib.dbs_cuda_backtrack(C.byref(dp.args()), ptr(tk), ptr(pr), ptr(out), stream_ptr()), "backtrack")
    torch.cuda.synchronize()
    return out.cpu().numpy()
