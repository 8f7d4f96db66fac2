# SPDX-License-Identifier: MIT
"""beamgrad 2.3.0's backtrack, search and beam_search on CUDA tensors against the same calls on
CPU tensors (run by tests/test_reference_frontend.py with the ``_frontend_hook`` plugin, so
``beamgrad`` is the reference package and its CUDA operators are this engine's)."""

import torch

import beamgrad
from beamgrad import BeamOptions


def _rows(B, T, K, V, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.log_softmax(torch.randn(B, T, K, V, generator=g) * 2.0, dim=-1)


def test_engine_operators_are_loaded():
    import sys

    assert beamgrad.cuda_available()
    assert "beamgrad_b200" in sys.modules["beamgrad._C_cuda"].__file__


def test_backtrack_matches_cpu():
    x = _rows(3, 9, 4, 300, seed=11)
    options = BeamOptions(beam_size=4, eos_token=5, length_penalty_alpha=0.6)
    steps = [9, 4, 7]
    gpu = beamgrad.decode(x.cuda(), options, steps=steps)
    cpu = beamgrad.decode(x, options, steps=steps)
    assert torch.equal(beamgrad.backtrack(gpu).cpu(), beamgrad.backtrack(cpu))


def test_search_matches_cpu_with_gradients():
    x = _rows(2, 6, 3, 500, seed=12)
    options = BeamOptions(beam_size=3, eos_token=2, length_penalty_alpha=1.0)
    cpu_x = x.clone().requires_grad_(True)
    gpu_x = x.cuda().requires_grad_(True)
    cpu = beamgrad.search(cpu_x, options)
    gpu = beamgrad.search(gpu_x, options)
    assert torch.equal(gpu.scores.detach().cpu(), cpu.scores.detach())
    assert torch.equal(gpu.sequences.cpu(), cpu.sequences)
    w = torch.linspace(-1.0, 1.0, 3)
    (cpu.scores * w).sum().backward()
    (gpu.scores * w.cuda()).sum().backward()
    assert torch.equal(gpu_x.grad.cpu(), cpu_x.grad)


def test_beam_search_over_a_step_function_matches_cpu():
    B, K, V, T = 2, 4, 97, 8
    table = torch.log_softmax(torch.randn(V, V, generator=torch.Generator().manual_seed(13)) * 3.0, dim=-1)

    def run(device):
        w = table.to(device).clone().requires_grad_(True)

        def step(state):
            last = state.tokens.clamp(min=0) if state.step > 0 else torch.zeros(B, K, dtype=torch.long, device=device)
            return w[last]  # [B, K, V]: the next-token distribution after each beam's last token

        out = beamgrad.beam_search(step, BeamOptions(beam_size=K, eos_token=3, length_penalty_alpha=0.6), T,
                                   batch_size=B, device=device)
        out.scores.sum().backward()
        return out, w.grad

    gpu, g_gpu = run("cuda")
    cpu, g_cpu = run("cpu")
    assert torch.equal(gpu.scores.detach().cpu(), cpu.scores.detach())
    assert torch.equal(gpu.sequences.cpu(), cpu.sequences)
    assert torch.equal(g_gpu.cpu(), g_cpu)
