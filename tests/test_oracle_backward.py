"""Pins the gradient reference (oracle/autograd_ref.py) used by the backward's
GPU parity tests: its forward equals the C oracle's (which the golden vectors
pin), and its autograd gradients equal central finite differences."""
import numpy as np
import torch

import cases
import oracle
from oracle import autograd_ref


def _tiny(seed, lens, D=4, HQ=1, HV=2, with_state=True):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    k = r(T, HQ, D)
    k = k / k.norm(dim=-1, keepdim=True)
    return dict(q=r(T, HQ, D), k=k, v=r(T, HV, D),
                state=r(len(lens), HV, D, D) * 0.1 if with_state else None,
                A_log=torch.rand(HV, generator=g, dtype=torch.float64),
                a=r(T, HV), dt_bias=r(HV) * 0.1, b=r(T, HV),
                cu=np.concatenate([[0], np.cumsum(lens)]).tolist())


def test_gradients_match_finite_differences():
    x = _tiny(0, [3, 0, 5])
    names = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
    inputs = tuple(x[n].clone().requires_grad_(True) for n in names)

    def f(q, k, v, state, A_log, a, dt_bias, b):
        return autograd_ref.prefill_forward(q, k, v, state, A_log, a, dt_bias, b, x["cu"], 0.7)

    assert torch.autograd.gradcheck(f, inputs, eps=1e-6, atol=1e-7, rtol=1e-5)


def test_gradients_match_finite_differences_zero_state_and_large_gates():
    # a + dt_bias far on both sides of 0 (both softplus branches), no state
    x = _tiny(1, [6, 2], with_state=False)
    x["a"] = x["a"] * 8.0
    names = ("q", "k", "v", "A_log", "a", "dt_bias", "b")
    inputs = tuple(x[n].clone().requires_grad_(True) for n in names)

    def f(q, k, v, A_log, a, dt_bias, b):
        return autograd_ref.prefill_forward(q, k, v, None, A_log, a, dt_bias, b, x["cu"], None)

    assert torch.autograd.gradcheck(f, inputs, eps=1e-6, atol=1e-7, rtol=1e-5)


def test_forward_matches_c_oracle():
    lens = [5, 70, 1]
    inp = cases.prefill_inputs(seed=11, lens=lens)
    f64 = lambda bits: torch.from_numpy(cases.bits_to_f32(bits).astype(np.float64))  # noqa: E731
    out, final = autograd_ref.prefill_forward(
        f64(inp["q"]), f64(inp["k"]), f64(inp["v"]), torch.from_numpy(inp["state"]).double(),
        torch.from_numpy(inp["A_log"]).double(), f64(inp["a"]),
        torch.from_numpy(inp["dt_bias"]).double(), f64(inp["b"]), inp["cu_seqlens"], None)
    o_ref, f_ref = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                  inp["a"], inp["dt_bias"], inp["b"], inp["cu_seqlens"])
    rel = lambda x, y: float(np.linalg.norm(x - y) / np.linalg.norm(y))  # noqa: E731
    assert rel(out.numpy(), o_ref.astype(np.float64)) < 1e-5
    assert rel(final.numpy(), f_ref.astype(np.float64)) < 1e-5
