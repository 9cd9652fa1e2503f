"""GDN decode (qk4_v8_d128_k_last): drop-in for the reference decode solution.

`run` keeps the reference signature, argument meaning, defaults and error
behaviour of `run` in gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py
(lines 100-146 of the reference project): value-returning, a fresh
`new_state` buffer (the input state is not modified), `scale` None or 0 ->
1/sqrt(128), `state` None -> zero state, shape asserts on q/k/v.  The work is
one launch of the sm_100a kernel in libgdn_b200.so on the current stream.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _native

HQ = 4
HV = 8
D = 128


def _scale(scale) -> float:
    # kernel.py:112-115
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(D)
    return float(scale)


def _check_inputs(q, k, v, a, b):
    # kernel.py:117-120
    assert q.shape[1:] == (1, HQ, D)
    assert k.shape[1:] == (1, HQ, D)
    assert v.shape[1:] == (1, HV, D)
    assert q.shape[0] == v.shape[0]
    B = q.shape[0]
    for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"GDN decode expects bf16 {name}, got {t.dtype}")
        if not t.is_cuda:
            raise ValueError(f"GDN decode expects CUDA tensors ({name} is on {t.device})")
    assert a.numel() == B * HV and b.numel() == B * HV, "a, b must be [B,1,8]"


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.float().contiguous()


def decode_into(q, k, v, state, A_log, a, dt_bias, b, scale, out, new_state,
                stream: Optional[int] = None) -> None:
    """Destination-passing form: writes `out` [B,1,8,128] bf16 and
    `new_state` [B,8,128,128] fp32 (may be `state` itself for an in-place
    update).  All tensors must be contiguous CUDA tensors."""
    B = q.shape[0]
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    st = _native.lib.gdn_decode_qk4_v8_d128_k_last(
        q.data_ptr(), k.data_ptr(), v.data_ptr(),
        None if state is None else state.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
        _scale(scale), B, out.data_ptr(), new_state.data_ptr(), stream)
    _native.check(st, "gdn_decode_qk4_v8_d128_k_last")


@torch.no_grad()
def run(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: Optional[torch.Tensor],
        A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, b: torch.Tensor,
        scale: Optional[float]):
    """Returns (output [B,1,8,128] bf16, new_state [B,8,128,128] fp32)."""
    _check_inputs(q, k, v, a, b)
    B = q.shape[0]
    if state is not None:
        assert state.shape == (B, HV, D, D) and state.dtype == torch.float32
        state = state.contiguous()
    output = torch.empty(B, 1, HV, D, dtype=q.dtype, device=q.device)
    new_state = torch.empty(B, HV, D, D, dtype=torch.float32, device=q.device)
    decode_into(q.contiguous(), k.contiguous(), v.contiguous(), state, _f32(A_log),
                a.contiguous(), _f32(dt_bias), b.contiguous(), scale, output, new_state)
    return output, new_state


@torch.no_grad()
def run_inplace(q, k, v, state, A_log, a, dt_bias, b, scale):
    """Same step with the state updated in place (serving form: the state
    pool stays resident and is not copied).  Returns output [B,1,8,128]."""
    _check_inputs(q, k, v, a, b)
    B = q.shape[0]
    assert state.shape == (B, HV, D, D) and state.dtype == torch.float32 and state.is_contiguous()
    output = torch.empty(B, 1, HV, D, dtype=q.dtype, device=q.device)
    decode_into(q.contiguous(), k.contiguous(), v.contiguous(), state, _f32(A_log),
                a.contiguous(), _f32(dt_bias), b.contiguous(), scale, output, state)
    return output


# ---------------------------------------------------------------------------
# multi-token decode (speculative verify / MTP); no counterpart in the reference
# ---------------------------------------------------------------------------
MTP_MAX_TOKENS = 64


def _check_mtp_inputs(q, k, v, a, b):
    assert q.dim() == 4 and q.shape[2:] == (HQ, D), "q must be [B,T,4,128]"
    B, T = q.shape[0], q.shape[1]
    assert k.shape == (B, T, HQ, D), "k must be [B,T,4,128]"
    assert v.shape == (B, T, HV, D), "v must be [B,T,8,128]"
    assert a.numel() == B * T * HV and b.numel() == B * T * HV, "a, b must be [B,T,8]"
    assert 1 <= T <= MTP_MAX_TOKENS, f"1 <= T <= {MTP_MAX_TOKENS}"
    for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"GDN decode expects bf16 {name}, got {t.dtype}")
        if not t.is_cuda:
            raise ValueError(f"GDN decode expects CUDA tensors ({name} is on {t.device})")


def decode_mtp_into(q, k, v, state, A_log, a, dt_bias, b, scale, out, new_state,
                    intermediate: Optional[torch.Tensor] = None,
                    stream: Optional[int] = None) -> None:
    """Destination-passing multi-token decode: T tokens per request applied
    in order (identical to T single-token steps).  Writes `out` [B,T,8,128]
    bf16, `new_state` [B,8,128,128] fp32 (may be `state`) and, if given,
    `intermediate` [B,T,8,128,128] fp32 = the state after each token."""
    B, T = q.shape[0], q.shape[1]
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    st = _native.lib.gdn_decode_mtp_qk4_v8_d128_k_last(
        q.data_ptr(), k.data_ptr(), v.data_ptr(),
        None if state is None else state.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
        _scale(scale), B, T, out.data_ptr(), new_state.data_ptr(),
        None if intermediate is None else intermediate.data_ptr(), stream)
    _native.check(st, "gdn_decode_mtp_qk4_v8_d128_k_last")


@torch.no_grad()
def run_mtp(q, k, v, state, A_log, a, dt_bias, b, scale, return_intermediate: bool = False):
    """Multi-token decode, value-returning like `run`: q, k [B,T,4,128],
    v [B,T,8,128], a, b [B,T,8] bf16; state [B,8,128,128] fp32 or None.
    Returns (output [B,T,8,128] bf16, new_state [B,8,128,128] fp32) and, with
    return_intermediate, the states after each token [B,T,8,128,128] fp32
    (what a speculative decoder keeps to roll back rejected tokens)."""
    _check_mtp_inputs(q, k, v, a, b)
    B, T = q.shape[0], q.shape[1]
    if state is not None:
        assert state.shape == (B, HV, D, D) and state.dtype == torch.float32
        state = state.contiguous()
    output = torch.empty(B, T, HV, D, dtype=q.dtype, device=q.device)
    new_state = torch.empty(B, HV, D, D, dtype=torch.float32, device=q.device)
    inter = (torch.empty(B, T, HV, D, D, dtype=torch.float32, device=q.device)
             if return_intermediate else None)
    decode_mtp_into(q.contiguous(), k.contiguous(), v.contiguous(), state, _f32(A_log),
                    a.contiguous(), _f32(dt_bias), b.contiguous(), scale, output, new_state, inter)
    return (output, new_state, inter) if return_intermediate else (output, new_state)


# ---------------------------------------------------------------------------
# decode against a paged state pool; no counterpart in the reference
# ---------------------------------------------------------------------------
@torch.no_grad()
def run_pool(q, k, v, state_pool, slots, A_log, a, dt_bias, b, scale,
             stream: Optional[int] = None):
    """Decode with the states in a pool: request i's state is
    state_pool[slots[i]] ([P,8,128,128] fp32, updated in place).  q, k, v,
    a, b as in `run` ([B,1,...]) or `run_mtp` ([B,T,...]); slots: [B] int32
    CUDA tensor of distinct slots.  Returns output [B,T,8,128] bf16.  A slot
    outside the pool is reported through the device status (code 3)."""
    if q.shape[1] == 1 and q.dim() == 4:
        _check_inputs(q, k, v, a, b)
    else:
        _check_mtp_inputs(q, k, v, a, b)
    B, T = q.shape[0], q.shape[1]
    assert state_pool.dim() == 4 and state_pool.shape[1:] == (HV, D, D)
    assert state_pool.dtype == torch.float32 and state_pool.is_contiguous()
    assert slots.dtype == torch.int32 and slots.numel() == B and slots.is_cuda
    output = torch.empty(B, T, HV, D, dtype=q.dtype, device=q.device)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    st = _native.lib.gdn_decode_pool_qk4_v8_d128_k_last(
        q.contiguous().data_ptr(), k.contiguous().data_ptr(), v.contiguous().data_ptr(),
        state_pool.data_ptr(), state_pool.shape[0], slots.contiguous().data_ptr(),
        _f32(A_log).data_ptr(), a.contiguous().data_ptr(), _f32(dt_bias).data_ptr(),
        b.contiguous().data_ptr(), _scale(scale), B, T, output.data_ptr(), stream)
    _native.check(st, "gdn_decode_pool_qk4_v8_d128_k_last")
    return output


# ---------------------------------------------------------------------------
# bf16 state storage; no counterpart in the reference (fp32 state only)
# ---------------------------------------------------------------------------
@torch.no_grad()
def run_bf16_state(q, k, v, state_bf16, A_log, a, dt_bias, b, scale,
                   slots: Optional[torch.Tensor] = None, stream: Optional[int] = None):
    """Decode with the state stored in bf16 and updated in place: computed
    in fp32 like `run`, the new state rounded to nearest even (after every
    token when T > 1).  q, k, v, a, b as in `run` ([B,1,...]) or `run_mtp`
    ([B,T,...]); state_bf16 [B,8,128,128] bf16, or a pool [P,8,128,128]
    addressed by `slots` ([B] int32).  Returns output [B,T,8,128] bf16."""
    if q.shape[1] == 1 and q.dim() == 4:
        _check_inputs(q, k, v, a, b)
    else:
        _check_mtp_inputs(q, k, v, a, b)
    B, T = q.shape[0], q.shape[1]
    assert state_bf16.dtype == torch.bfloat16 and state_bf16.is_contiguous()
    assert state_bf16.dim() == 4 and state_bf16.shape[1:] == (HV, D, D)
    if slots is None:
        assert state_bf16.shape[0] == B
    else:
        assert slots.dtype == torch.int32 and slots.numel() == B and slots.is_cuda
    output = torch.empty(B, T, HV, D, dtype=q.dtype, device=q.device)
    decode_bf16_state_into(q.contiguous(), k.contiguous(), v.contiguous(), state_bf16,
                           _f32(A_log), a.contiguous(), _f32(dt_bias), b.contiguous(), scale,
                           output, None if slots is None else slots.contiguous(), stream)
    return output


def decode_bf16_state_into(q, k, v, state_bf16, A_log, a, dt_bias, b, scale, out,
                           slots: Optional[torch.Tensor] = None,
                           stream: Optional[int] = None) -> None:
    """Destination-passing form of run_bf16_state (contiguous CUDA tensors,
    fp32 A_log / dt_bias; state updated in place)."""
    B, T = q.shape[0], q.shape[1]
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    st = _native.lib.gdn_decode_bf16_state_qk4_v8_d128_k_last(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), state_bf16.data_ptr(),
        0 if slots is None else state_bf16.shape[0],
        None if slots is None else slots.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), _scale(scale), B, T,
        out.data_ptr(), stream)
    _native.check(st, "gdn_decode_bf16_state_qk4_v8_d128_k_last")
