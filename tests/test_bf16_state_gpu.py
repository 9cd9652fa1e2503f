"""Decode with a bf16 state (an opt-in storage format; the reference keeps
fp32 state) on the GPU, through the C ABI.

  * Given a state whose values are bf16-representable, the output equals the
    fp32-state kernel's bit for bit and the stored state equals that
    kernel's new state rounded to nearest even;
  * T tokens equal T single-token calls (the state is rounded after each);
  * against the fp32 oracle on the widened state: output |d| <= 2e-3 +
    1e-2 |ref|, state relative Frobenius <= 4e-3 (one bf16 rounding);
  * the pool form equals the dense form on the gathered states.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import bf16_dev, f32_dev, out_err, rel_fro

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _vec(inp):
    return (bf16_dev(inp["q"]), bf16_dev(inp["k"]), bf16_dev(inp["v"]), f32_dev(inp["A_log"]),
            bf16_dev(inp["a"]), f32_dev(inp["dt_bias"]), bf16_dev(inp["b"]))


@pytest.mark.parametrize("B", [1, 16, 257])
def test_bf16_state_matches_fp32_kernel_rounded(gdn, B):
    inp = cases.decode_inputs(seed=400 + B, B=B, with_state=True)
    q, k, v, A_log, a, dt, b = _vec(inp)
    st16 = f32_dev(inp["state"]).bfloat16().contiguous()
    o_ref, s_ref = gdn.decode.run(q, k, v, st16.float(), A_log, a, dt, b, None)
    o = gdn.decode.run_bf16_state(q, k, v, st16, A_log, a, dt, b, None)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(st16, s_ref.bfloat16())


def test_bf16_state_tokens_equal_single_steps(gdn):
    B, T = 9, 3
    inp = cases.decode_mtp_inputs(seed=410, B=B, T=T, with_state=True)
    q, k, v, A_log, a, dt, b = _vec(inp)
    st_a = f32_dev(inp["state"]).bfloat16().contiguous()
    st_b = st_a.clone()
    o = gdn.decode.run_bf16_state(q, k, v, st_a, A_log, a, dt, b, None)
    for t in range(T):
        sl = slice(t, t + 1)
        ot = gdn.decode.run_bf16_state(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                       v[:, sl].contiguous(), st_b, A_log, a[:, sl].contiguous(),
                                       dt, b[:, sl].contiguous(), None)
        assert torch.equal(o[:, t], ot[:, 0])
    torch.cuda.synchronize()
    assert torch.equal(st_a, st_b)


def test_bf16_state_against_oracle(gdn):
    inp = cases.decode_inputs(seed=420, B=12, with_state=True)
    q, k, v, A_log, a, dt, b = _vec(inp)
    st16 = f32_dev(inp["state"]).bfloat16().contiguous()
    wide = st16.float().cpu().numpy()
    o = gdn.decode.run_bf16_state(q, k, v, st16, A_log, a, dt, b, None)
    ro, rs = oracle.decode(inp["q"], inp["k"], inp["v"], wide, inp["A_log"], inp["a"],
                           inp["dt_bias"], inp["b"])
    torch.cuda.synchronize()
    assert out_err(o, ro) <= 1.0
    assert rel_fro(st16.float().cpu().numpy(), rs) <= 4e-3


def test_bf16_state_pool_equals_dense(gdn):
    P, B = 10, 6
    rng = np.random.default_rng(7)
    slots = torch.tensor(rng.permutation(P)[:B], dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    pool = (torch.randn(P, 8, 128, 128, generator=g, device="cuda") * 0.02).bfloat16()
    inp = cases.decode_inputs(seed=430, B=B, with_state=False)
    q, k, v, A_log, a, dt, b = _vec(inp)
    dense = pool[slots.long()].clone()
    before = pool.clone()
    o_ref = gdn.decode.run_bf16_state(q, k, v, dense, A_log, a, dt, b, None)
    o = gdn.decode.run_bf16_state(q, k, v, pool, A_log, a, dt, b, None, slots=slots)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(pool[slots.long()], dense)
    untouched = torch.ones(P, dtype=torch.bool, device="cuda")
    untouched[slots.long()] = False
    assert torch.equal(pool[untouched], before[untouched])
