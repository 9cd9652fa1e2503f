"""Gradient reference for the prefill backward.  TEST INFRASTRUCTURE ONLY.

The reference project's prefill is forward-only (solution/triton/kernel.py:1),
so there is no reference backward to restate.  The parity anchor is the
gradient of the reference forward itself: `prefill_forward` restates the token
recurrence that the reference's chunked prefill computes
(solution/triton/kernel.py:1762-1802, gates as kernel.py:1712-1722: the
overflow-safe softplus, g = -exp(A_log) softplus(a + dt_bias), beta =
sigmoid(b)) in torch, and torch.autograd differentiates it.  It is pinned in
two ways (tests/test_oracle_backward.py): its forward against the C oracle
(itself pinned to the golden vectors made by the reference's own kernels), and
its gradients against central finite differences (torch.autograd.gradcheck,
float64).  Any head dimension and head counts work, so the finite-difference
check runs on tiny shapes.
"""
from __future__ import annotations

import math

import torch


def softplus_stable(x: torch.Tensor) -> torch.Tensor:
    # kernel.py:1714-1720: x + log(1 + e^-x) for x > 0, else log(1 + e^x)
    return torch.where(x > 0, x + torch.log1p(torch.exp(-x.clamp(min=0))),
                       torch.log1p(torch.exp(x.clamp(max=0))))


def prefill_forward(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """q, k [T,HQ,D]; v [T,HV,D]; a, b [T,HV]; A_log, dt_bias [HV]; state
    [N,HV,D,D] (v rows, k columns) or None; cu_seqlens a list / 1-D tensor of
    N+1 offsets.  v-head h reads q/k head h // (HV // HQ).  Returns
    (out [T,HV,D], final_state [N,HV,D,D]) in the inputs' float dtype."""
    T, HQ, D = q.shape
    HV = v.shape[1]
    ratio = HV // HQ
    cu = [int(x) for x in cu_seqlens]
    N = len(cu) - 1
    if scale is None or float(scale) == 0.0:
        scale = 1.0 / math.sqrt(D)
    g = -torch.exp(A_log)[None, :] * softplus_stable(a + dt_bias[None, :])  # [T,HV]
    beta = torch.sigmoid(b)
    outs, finals = [], []
    for n in range(N):
        S = state[n] if state is not None else q.new_zeros(HV, D, D)
        for t in range(cu[n], cu[n + 1]):
            kt = k[t].repeat_interleave(ratio, 0)  # [HV, D]
            qt = q[t].repeat_interleave(ratio, 0)
            S = S * torch.exp(g[t])[:, None, None]
            delta = beta[t][:, None] * (v[t] - torch.einsum("hvk,hk->hv", S, kt))
            S = S + delta[:, :, None] * kt[:, None, :]
            outs.append(scale * torch.einsum("hvk,hk->hv", S, qt))
        finals.append(S)
    out = torch.stack(outs) if outs else q.new_zeros(0, HV, D)
    return out, torch.stack(finals)


def prefill_grads(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, d_out,
                  d_final=None, dtype=torch.float64):
    """Gradients of sum(out * d_out) + sum(final * d_final) with respect to
    every input, by autograd in `dtype` on the CPU.  Tensors may be of any
    float dtype (bf16 inputs are widened exactly).  Returns a dict with keys
    dq, dk, dv, da, db, dA_log, ddt_bias, d_state (None when state is None)."""
    def leaf(x):
        return None if x is None else x.detach().to("cpu", dtype).clone().requires_grad_(True)

    xs = dict(q=leaf(q), k=leaf(k), v=leaf(v), state=leaf(state), A_log=leaf(A_log), a=leaf(a),
              dt_bias=leaf(dt_bias), b=leaf(b))
    out, final = prefill_forward(xs["q"], xs["k"], xs["v"], xs["state"], xs["A_log"], xs["a"],
                                 xs["dt_bias"], xs["b"], cu_seqlens, scale)
    loss = (out * d_out.detach().to("cpu", dtype)).sum()
    if d_final is not None:
        loss = loss + (final * d_final.detach().to("cpu", dtype)).sum()
    loss.backward()
    names = dict(q="dq", k="dk", v="dv", a="da", b="db", A_log="dA_log", dt_bias="ddt_bias",
                 state="d_state")
    return {names[n]: (None if x is None else x.grad) for n, x in xs.items()}
