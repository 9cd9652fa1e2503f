"""Prefill backward on the GPU against the autograd reference.

The reference is forward-only, so gradients are checked against torch
autograd of the token recurrence in float64 on the CPU
(oracle/autograd_ref.py, pinned by finite differences and by the C oracle's
forward).  Tolerance: relative Frobenius error per gradient tensor below
1e-2 (measured on a B200: 1e-4 to 2.4e-3; the recomputed forward runs its
MMAs on bf16 operands, as the forward does, and the backward reuses its bf16
[P Ainv ; Ainv] images).  The
backward is also deterministic, and the autograd wrapper returns exactly the
direct call's gradients.
"""
import numpy as np
import pytest
import torch

import cases
from gpu_util import prefill_args
from oracle import autograd_ref

pytestmark = pytest.mark.gpu

TOL = 1e-2
NAMES = ("dq", "dk", "dv", "da", "db", "dA_log", "ddt_bias", "d_state")


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _case(seed, lens, with_state, with_dfinal):
    inp = cases.prefill_inputs(seed=seed, lens=lens, with_state=with_state)
    args = prefill_args(inp)
    T, N = sum(lens), len(lens)
    g = torch.Generator().manual_seed(seed + 100)
    d_out = (torch.randn(T, 8, 128, generator=g) * 0.1).bfloat16()
    d_final = torch.randn(N, 8, 128, 128, generator=g) * 0.01 if with_dfinal else None
    return args, d_out, d_final


def _rel(x, ref):
    x, ref = x.double().cpu(), ref.double().cpu()
    return float((x - ref).norm() / max(float(ref.norm()), 1e-30))


@pytest.mark.parametrize("lens,with_state,with_dfinal", [
    ([64], True, True),               # one full chunk
    ([1], False, True),               # one token
    ([100, 37, 200], True, True),     # ragged, tail chunks
    ([130, 0, 64], False, False),     # an empty sequence, no final-state gradient
    ([1000], True, False),            # 16 chunks: error growth along the scan
])
def test_backward_matches_autograd_reference(gdn, lens, with_state, with_dfinal):
    args, d_out, d_final = _case(7 + len(lens) + sum(lens), lens, with_state, with_dfinal)
    got = gdn.prefill.backward(*args, None, d_out.cuda(),
                               None if d_final is None else d_final.cuda())
    q, k, v, state, A_log, a, dt, b, cu = args
    ref = autograd_ref.prefill_grads(q, k, v, state, A_log, a, dt, b, cu.cpu().tolist(), None,
                                     d_out.float(), d_final)
    errs = {}
    for name in NAMES:
        if ref[name] is None:
            continue
        assert torch.isfinite(got[name]).all(), name
        errs[name] = _rel(got[name], ref[name].view_as(got[name]))
    print(lens, {n: f"{e:.2e}" for n, e in errs.items()})
    assert all(e < TOL for e in errs.values()), errs
    if state is None and got["d_state"] is not None:
        # gradient of a zero initial state: compare with the reference given zeros
        z = torch.zeros(len(lens), 8, 128, 128)
        ref0 = autograd_ref.prefill_grads(q, k, v, z, A_log, a, dt, b, cu.cpu().tolist(), None,
                                          d_out.float(), d_final)
        assert _rel(got["d_state"], ref0["d_state"]) < TOL


@pytest.mark.parametrize("lens", [[600, 130]])
def test_backward_with_slow_decay(gdn, lens):
    """A_log in [-5, -2]: the state and its gradient stay large from chunk to
    chunk, so the reverse scan's carried dS (and the chunk-start states the
    recompute saves) are exercised."""
    args, d_out, d_final = _case(17 + sum(lens), lens, True, True)
    q, k, v, state, A_log, a, dt, b, cu = args
    A_log = torch.from_numpy(
        (np.random.default_rng(7).random(8, dtype=np.float32) * 3.0 - 5.0).astype(np.float32)
    ).to(A_log.device)
    args = (q, k, v, state, A_log, a, dt, b, cu)
    got = gdn.prefill.backward(*args, None, d_out.cuda(), d_final.cuda())
    ref = autograd_ref.prefill_grads(q, k, v, state, A_log, a, dt, b, cu.cpu().tolist(), None,
                                     d_out.float(), d_final)
    errs = {name: _rel(got[name], ref[name].view_as(got[name])) for name in NAMES}
    print(lens, {n: f"{e:.2e}" for n, e in errs.items()})
    assert all(e < TOL for e in errs.values()), errs


def test_backward_is_deterministic(gdn):
    args, d_out, d_final = _case(3, [300, 77], True, True)
    g1 = gdn.prefill.backward(*args, None, d_out.cuda(), d_final.cuda())
    g2 = gdn.prefill.backward(*args, None, d_out.cuda(), d_final.cuda())
    for name in NAMES:
        assert torch.equal(g1[name], g2[name]), name


def test_autograd_wrapper_matches_direct_backward(gdn):
    args, d_out, d_final = _case(5, [90, 140], True, True)
    q, k, v, state, A_log, a, dt, b, cu = args
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, state, A_log, a, dt, b)]
    lq, lk, lv, ls, lA, la, ldt, lb = leaves
    out, final = gdn.prefill.run_autograd(lq, lk, lv, ls, lA, la, ldt, lb, cu, None)
    ref_out, ref_final = gdn.prefill.run(q, k, v, state, A_log, a, dt, b, cu, None)
    assert torch.equal(out, ref_out) and torch.equal(final, ref_final)
    loss = (out.float() * d_out.cuda().float()).sum() + (final * d_final.cuda()).sum()
    loss.backward()
    g = gdn.prefill.backward(q, k, v, state, A_log, a, dt, b, cu, None, d_out.cuda(),
                             d_final.cuda())
    for leaf, name in zip(leaves, ("dq", "dk", "dv", "d_state", "dA_log", "da", "ddt_bias", "db")):
        assert leaf.grad is not None and leaf.grad.dtype == leaf.dtype, name
        assert torch.equal(leaf.grad, g[name].to(leaf.dtype).view_as(leaf)), name


def test_backward_is_deterministic_with_many_pairs_per_cluster(gdn):
    """The chunk-gradient kernel is persistent: each cluster of two CTAs walks
    many (chunk, q/k head) pairs, fetching the next pair's operands while the
    current one runs, and the two CTAs exchange their dq / dk halves.  On an
    input with far more pairs than clusters, repeated calls must agree bit for
    bit on every gradient (a missing barrier between two passes of one pair
    shows up here as a few differing chunks)."""
    args, d_out, d_final = _case(4242, [4096, 3000, 2500, 1800, 700, 64, 1, 5000], True, True)
    runs = [gdn.prefill.backward(*args, None, d_out.cuda(), d_final.cuda()) for _ in range(4)]
    for g in runs[1:]:
        for name in NAMES:
            if runs[0][name] is not None:
                assert torch.equal(runs[0][name], g[name]), name


def test_backward_reports_bad_seqlens(gdn):
    args, d_out, _ = _case(9, [64, 64], False, False)
    q, k, v, state, A_log, a, dt, b, cu = args
    bad_cu = torch.tensor([0, 100, 64], dtype=torch.int64, device="cuda")  # decreasing
    T, N = q.shape[0], 2
    f32 = dict(dtype=torch.float32, device="cuda")
    outs = [torch.empty(T, 4, 128, **f32), torch.empty(T, 4, 128, **f32),
            torch.empty(T, 8, 128, **f32), torch.empty(T, 8, **f32), torch.empty(T, 8, **f32),
            torch.empty(8, **f32), torch.empty(8, **f32), None]
    ws = gdn.prefill.alloc_backward_workspace(T, N, "cuda")
    gdn.prefill.backward_into(q, k, v, None, A_log, a, dt, b, bad_cu, None, d_out.cuda(), None,
                              *outs, ws)
    assert gdn._native.read_device_status() == 1


@pytest.mark.parametrize("T", [1, 255, 257, 70_001])
def test_backward_parameter_gradient_reduction(gdn, T):
    """dA_log and ddt_bias are reduced over tokens in two fixed-order stages
    (256 coalesced partial sums, then one pass over them).  At T values whose
    token ranges split unevenly over the 256 blocks (and T < 256, which
    leaves blocks empty) the sums must equal the float64 sums of the
    kernel's own per-token gradients -- ddt_bias = sum_t da_t and dA_log =
    sum_t da_t softplus(x_t) / sigmoid(x_t), x = a + dt_bias, because da_t =
    dg_t (-e^A_log sigmoid(x_t)) and dg_t/dA_log = g_t -- and two calls must
    agree bit for bit.  Small T is also checked against autograd."""
    args, d_out, d_final = _case(1000 + T, [T], T > 1, T > 1)
    g1 = gdn.prefill.backward(*args, None, d_out.cuda(), None if d_final is None else d_final.cuda())
    g2 = gdn.prefill.backward(*args, None, d_out.cuda(), None if d_final is None else d_final.cuda())
    for name in NAMES:
        if g1[name] is not None:
            assert torch.equal(g1[name], g2[name]), name
    q, k, v, state, A_log, a, dt, b, cu = args
    da = g1["da"].double().cpu()                                  # [T, 8]
    x = a.double().cpu() + dt.double().cpu()[None, :]
    sp = torch.where(x > 0, x + torch.log1p(torch.exp(-x)), torch.log1p(torch.exp(x)))
    terms = {"ddt_bias": da, "dA_log": da * sp / torch.sigmoid(x)}
    for name, t in terms.items():
        want = t.sum(0)
        got = g1[name].double().cpu()
        bound = 1e-4 * t.abs().sum(0) + 1e-6
        assert bool(((got - want).abs() <= bound).all()), (name, got, want)
    if T <= 257:
        ref = autograd_ref.prefill_grads(q, k, v, state, A_log, a, dt, b, cu.cpu().tolist(), None,
                                         d_out.float(), d_final)
        for name in ("dA_log", "ddt_bias", "da", "db"):
            assert _rel(g1[name], ref[name].view_as(g1[name])) < TOL, name
