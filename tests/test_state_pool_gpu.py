"""Paged state pool (decode and prefill against state_pool[slots]) on the GPU,
through the C ABI.  Each call must give bit for bit what the dense entry
point gives on the gathered states, write the new states back only to the
given slots, and report a slot outside the pool through device status 3."""
import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import bf16_dev, f32_dev, out_err, prefill_args, rel_fro

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _pool(P, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(P, 8, 128, 128, generator=g, device="cuda") * 0.02


def _slots(P, n, seed):
    rng = np.random.default_rng(seed)
    return torch.tensor(rng.permutation(P)[:n], dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("B,T", [(12, 1), (7, 3), (1, 1)])
def test_decode_pool_equals_dense_decode(gdn, B, T):
    P = 20
    pool = _pool(P, 1 + B)
    slots = _slots(P, B, 2 + B)
    inp = cases.decode_mtp_inputs(seed=3 + B, B=B, T=T, with_state=False)
    q, k, v = bf16_dev(inp["q"]), bf16_dev(inp["k"]), bf16_dev(inp["v"])
    A_log, dt = f32_dev(inp["A_log"]), f32_dev(inp["dt_bias"])
    a, b = bf16_dev(inp["a"]), bf16_dev(inp["b"])
    before = pool.clone()
    gathered = pool[slots.long()].clone()
    if T == 1:
        o_ref, s_ref = gdn.decode.run(q, k, v, gathered, A_log, a, dt, b, None)
    else:
        o_ref, s_ref = gdn.decode.run_mtp(q, k, v, gathered, A_log, a, dt, b, None)
    o = gdn.decode.run_pool(q, k, v, pool, slots, A_log, a, dt, b, None)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref.view(B, T, 8, 128))
    assert torch.equal(pool[slots.long()], s_ref)
    untouched = torch.ones(P, dtype=torch.bool, device="cuda")
    untouched[slots.long()] = False
    assert torch.equal(pool[untouched], before[untouched])


@pytest.mark.parametrize("lens", [[70, 130, 257], [2000, 1100]])  # single-pass, segmented
def test_prefill_pool_equals_dense_prefill(gdn, lens):
    P = 9
    N = len(lens)
    pool = _pool(P, 10 + N)
    slots = _slots(P, N, 11 + N)
    inp = cases.prefill_inputs(seed=sum(lens), lens=lens, with_state=False)
    q, k, v, _, A_log, a, dt, b, cu = prefill_args(inp)
    before = pool.clone()
    h0 = pool[slots.long()].clone()
    o_ref, s_ref = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    o = gdn.prefill.run_pool(q, k, v, pool, slots, A_log, a, dt, b, cu, None)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(pool[slots.long()], s_ref)
    untouched = torch.ones(P, dtype=torch.bool, device="cuda")
    untouched[slots.long()] = False
    assert torch.equal(pool[untouched], before[untouched])
    # and directly against the fp32 recurrence, from the states the slots held
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], h0.cpu().numpy(), inp["A_log"],
                            inp["a"], inp["dt_bias"], inp["b"], inp["cu_seqlens"])
    assert out_err(o, ro) <= 1.0
    assert rel_fro(pool[slots.long()].cpu().numpy(), rs) < 5e-3


def test_bad_slot_sets_device_status(gdn):
    P, B = 4, 2
    pool = _pool(P, 99)
    inp = cases.decode_inputs(seed=98, B=B, with_state=False)
    q, k, v = bf16_dev(inp["q"]), bf16_dev(inp["k"]), bf16_dev(inp["v"])
    A_log, dt = f32_dev(inp["A_log"]), f32_dev(inp["dt_bias"])
    a, b = bf16_dev(inp["a"]), bf16_dev(inp["b"])
    before = pool.clone()
    slots = torch.tensor([1, 7], dtype=torch.int32, device="cuda")  # 7 is outside the pool
    gdn.decode.run_pool(q, k, v, pool, slots, A_log, a, dt, b, None)
    assert gdn._native.read_device_status() == 3
    # the valid request was still served, nothing else in the pool changed
    assert not torch.equal(pool[1], before[1])
    assert torch.equal(pool[[0, 2, 3]], before[[0, 2, 3]])
    # prefill with a bad slot writes nothing
    pinp = cases.prefill_inputs(seed=97, lens=[40, 30], with_state=False)
    pq, pk, pv, _, pA, pa, pdt, pb, cu = prefill_args(pinp)
    before = pool.clone()
    gdn.prefill.run_pool(pq, pk, pv, pool, torch.tensor([0, -1], dtype=torch.int32, device="cuda"),
                         pA, pa, pdt, pb, cu, None)
    assert gdn._native.read_device_status() == 3
    assert torch.equal(pool, before)


def test_multi_token_pool_with_bad_slot(gdn):
    """Multi-token pool decode (the streaming kernel, T <= 16) with one slot
    outside the pool: status 3, the other requests served exactly as the
    dense call on their gathered states, nothing else in the pool touched."""
    P, B, T = 40, 37, 3
    pool = _pool(P, 123)
    slots = _slots(P, B, 124)
    slots[5] = P + 3  # outside the pool
    inp = cases.decode_mtp_inputs(seed=125, B=B, T=T, with_state=False)
    q, k, v = bf16_dev(inp["q"]), bf16_dev(inp["k"]), bf16_dev(inp["v"])
    A_log, dt = f32_dev(inp["A_log"]), f32_dev(inp["dt_bias"])
    a, b = bf16_dev(inp["a"]), bf16_dev(inp["b"])
    before = pool.clone()
    good = torch.ones(B, dtype=torch.bool, device="cuda")
    good[5] = False
    gslots = slots[good].long()
    o_ref, s_ref = gdn.decode.run_mtp(q[good], k[good], v[good], pool[gslots].clone(), A_log,
                                      a[good], dt, b[good], None)
    o = gdn.decode.run_pool(q, k, v, pool, slots, A_log, a, dt, b, None)
    assert gdn._native.read_device_status() == 3
    assert torch.equal(o[good], o_ref)
    assert torch.equal(pool[gslots], s_ref)
    untouched = torch.ones(P, dtype=torch.bool, device="cuda")
    untouched[gslots] = False
    assert torch.equal(pool[untouched], before[untouched])
