"""GDN prefill (qk4_v8_d128_k_last): drop-in for the reference prefill solution.

`run` keeps the signature, argument meaning, defaults and error behaviour of
`run` in solution/triton/kernel.py (lines 1762-1802 of the reference project):
value-returning (output [T,8,128] bf16, final_state [N,8,128,128] fp32),
`scale` None or 0 -> 1/sqrt(128), `state` None -> zero initial state, and the
input checks of `_validate_inputs` (kernel.py:1635-1667), including the
`cu_seqlens[-1] == T` assert, which reads one value back from the device as
the reference does.  `prefill_into` is the destination-passing form with no
host synchronisation at all (the same check then runs on the device).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _native

NUM_Q_HEADS = 4
NUM_K_HEADS = 4
NUM_V_HEADS = 8
HEAD_SIZE = 128
CHUNK_SIZE = 64


def _validate_inputs(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, check_total=True):
    # kernel.py:1635-1667
    assert q.is_cuda and k.is_cuda and v.is_cuda
    assert A_log.is_cuda and a.is_cuda and dt_bias.is_cuda and b.is_cuda and cu_seqlens.is_cuda
    assert q.dtype == torch.bfloat16
    assert k.dtype == torch.bfloat16
    assert v.dtype == torch.bfloat16
    assert A_log.dtype == torch.float32
    assert dt_bias.dtype == torch.float32
    assert a.dtype == torch.bfloat16
    assert b.dtype == torch.bfloat16
    if state is not None:
        assert state.is_cuda and state.dtype == torch.float32
    assert q.shape[1:] == (NUM_Q_HEADS, HEAD_SIZE)
    assert k.shape[1:] == (NUM_K_HEADS, HEAD_SIZE)
    assert v.shape[1:] == (NUM_V_HEADS, HEAD_SIZE)
    assert A_log.shape == (NUM_V_HEADS,)
    assert dt_bias.shape == (NUM_V_HEADS,)
    assert a.shape == (q.shape[0], NUM_V_HEADS)
    assert b.shape == (q.shape[0], NUM_V_HEADS)
    assert cu_seqlens.dtype == torch.int64
    if check_total:
        assert int(cu_seqlens[-1].item()) == q.shape[0]
    if state is not None:
        assert state.shape == (cu_seqlens.numel() - 1, NUM_V_HEADS, HEAD_SIZE, HEAD_SIZE)


def workspace_bytes(total_tokens: int, num_seqs: int) -> int:
    return int(_native.lib.gdn_prefill_workspace_bytes(total_tokens, num_seqs))


def alloc_workspace(total_tokens: int, num_seqs: int, device) -> torch.Tensor:
    """A workspace buffer for `prefill_into` (1024-byte aligned: the caching
    allocator returns 512-byte aligned blocks, so 1 KiB of slack is added and
    `workspace_view` picks the aligned start)."""
    return torch.empty(workspace_bytes(total_tokens, num_seqs) + 1024, dtype=torch.uint8,
                       device=device)


def _aligned_ptr(ws: torch.Tensor):
    p = ws.data_ptr()
    off = (-p) % 1024
    return p + off, ws.numel() - off


def prefill_into(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, out, final_state,
                 workspace: torch.Tensor, stream: Optional[int] = None,
                 events: Optional[Sequence] = None) -> None:
    """Destination-passing prefill: writes `out` [T,8,128] bf16 and
    `final_state` [N,8,128,128] fp32 (which may be `state`).  No host sync.
    `events` (torch.cuda.Event objects, optional): events[i] is recorded on
    the stream right after the call's i-th kernel launch (metadata, chunk
    preparation, scan; with the segmented evaluation also the composition and
    the second scan pass), for per-kernel timing."""
    T = q.shape[0]
    N = cu_seqlens.numel() - 1
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(HEAD_SIZE)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    wptr, wbytes = _aligned_ptr(workspace)
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), None if state is None else state.data_ptr(),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
            cu_seqlens.data_ptr(), N, T, float(scale), out.data_ptr(), final_state.data_ptr(),
            wptr, wbytes)
    if events:
        for e in events:
            if e.cuda_event == 0:  # torch creates the CUDA event on its first record
                e.record()
        handles = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        st = _native.lib.gdn_prefill_qk4_v8_d128_k_last_events(*args, handles, len(events), stream)
        _native.check(st, "gdn_prefill_qk4_v8_d128_k_last_events")
    else:
        st = _native.lib.gdn_prefill_qk4_v8_d128_k_last(*args, stream)
        _native.check(st, "gdn_prefill_qk4_v8_d128_k_last")


@torch.no_grad()
def run(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: Optional[torch.Tensor],
        A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, b: torch.Tensor,
        cu_seqlens: torch.Tensor, scale: Optional[float]):
    _validate_inputs(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens)
    T = q.shape[0]
    N = cu_seqlens.numel() - 1
    out = torch.empty(T, NUM_V_HEADS, HEAD_SIZE, dtype=torch.bfloat16, device=q.device)
    final_state = torch.empty(N, NUM_V_HEADS, HEAD_SIZE, HEAD_SIZE, dtype=torch.float32,
                              device=q.device)
    ws = alloc_workspace(T, N, q.device)
    prefill_into(q.contiguous(), k.contiguous(), v.contiguous(),
                 None if state is None else state.contiguous(), A_log.contiguous(),
                 a.contiguous(), dt_bias.contiguous(), b.contiguous(), cu_seqlens.contiguous(),
                 scale, out, final_state, ws)
    return out, final_state


def prefill_pool_into(q, k, v, state_pool, slots, A_log, a, dt_bias, b, cu_seqlens, scale, out,
                      workspace: torch.Tensor, stream: Optional[int] = None) -> None:
    """Destination-passing prefill against a paged state pool: sequence n
    starts from state_pool[slots[n]] and its final state is written back
    there.  No host sync; a slot outside the pool is reported through the
    device status (code 3) and nothing is written.  No counterpart in the
    reference."""
    T = q.shape[0]
    N = cu_seqlens.numel() - 1
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(HEAD_SIZE)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    wptr, wbytes = _aligned_ptr(workspace)
    st = _native.lib.gdn_prefill_pool_qk4_v8_d128_k_last(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), state_pool.data_ptr(), state_pool.shape[0],
        slots.data_ptr(), A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
        cu_seqlens.data_ptr(), N, T, float(scale), out.data_ptr(), wptr, wbytes, stream)
    _native.check(st, "gdn_prefill_pool_qk4_v8_d128_k_last")


@torch.no_grad()
def run_pool(q, k, v, state_pool, slots, A_log, a, dt_bias, b, cu_seqlens, scale):
    """Prefill with the states in a pool ([P,8,128,128] fp32, updated in
    place at the given slots; slots: [N] int32 CUDA tensor of distinct slots).
    Returns the output [T,8,128] bf16."""
    _validate_inputs(q, k, v, None, A_log, a, dt_bias, b, cu_seqlens)
    assert state_pool.dim() == 4 and state_pool.shape[1:] == (NUM_V_HEADS, HEAD_SIZE, HEAD_SIZE)
    assert state_pool.dtype == torch.float32 and state_pool.is_contiguous()
    N = cu_seqlens.numel() - 1
    assert slots.dtype == torch.int32 and slots.numel() == N and slots.is_cuda
    T = q.shape[0]
    out = torch.empty(T, NUM_V_HEADS, HEAD_SIZE, dtype=torch.bfloat16, device=q.device)
    ws = alloc_workspace(T, N, q.device)
    prefill_pool_into(q.contiguous(), k.contiguous(), v.contiguous(), state_pool,
                      slots.contiguous(), A_log.contiguous(), a.contiguous(), dt_bias.contiguous(),
                      b.contiguous(), cu_seqlens.contiguous(), scale, out, ws)
    return out


# ---------------------------------------------------------------------------
# backward (no counterpart in the reference, whose prefill is forward-only:
# solution/triton/kernel.py:1)
# ---------------------------------------------------------------------------
def backward_workspace_bytes(total_tokens: int, num_seqs: int) -> int:
    return int(_native.lib.gdn_prefill_backward_workspace_bytes(total_tokens, num_seqs))


def alloc_backward_workspace(total_tokens: int, num_seqs: int, device) -> torch.Tensor:
    """Workspace for `backward_into` (1 KiB of slack for the 1024-byte
    alignment, as `alloc_workspace`)."""
    return torch.empty(backward_workspace_bytes(total_tokens, num_seqs) + 1024,
                       dtype=torch.uint8, device=device)


def backward_into(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, d_out, d_final_state,
                  dq, dk, dv, da, db, dA_log, ddt_bias, d_state, workspace: torch.Tensor,
                  stream: Optional[int] = None) -> None:
    """Destination-passing backward: fp32 gradients dq, dk [T,4,128], dv
    [T,8,128], da, db [T,8], dA_log, ddt_bias [8] and (unless None) d_state
    [N,8,128,128], from d_out [T,8,128] bf16 and d_final_state (None: zero).
    The inputs are the forward's; the call recomputes what it needs.  No host
    sync."""
    T = q.shape[0]
    N = cu_seqlens.numel() - 1
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(HEAD_SIZE)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    wptr, wbytes = _aligned_ptr(workspace)

    def p(x):
        return None if x is None else x.data_ptr()

    st = _native.lib.gdn_prefill_backward_qk4_v8_d128_k_last(
        p(q), p(k), p(v), p(state), p(A_log), p(a), p(dt_bias), p(b), p(cu_seqlens), N, T,
        float(scale), p(d_out), p(d_final_state), p(dq), p(dk), p(dv), p(da), p(db), p(dA_log),
        p(ddt_bias), p(d_state), wptr, wbytes, stream)
    _native.check(st, "gdn_prefill_backward_qk4_v8_d128_k_last")


@torch.no_grad()
def backward(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, d_out,
             d_final_state=None, need_d_state: bool = True):
    """Gradients of `run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
    scale)` given d_out ([T,8,128]) and d_final_state ([N,8,128,128] or None).
    Returns a dict of fp32 tensors: dq, dk [T,4,128]; dv [T,8,128]; da, db
    [T,8]; dA_log, ddt_bias [8]; d_state [N,8,128,128] (None unless
    need_d_state)."""
    _validate_inputs(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens)
    T = q.shape[0]
    N = cu_seqlens.numel() - 1
    assert d_out.shape == (T, NUM_V_HEADS, HEAD_SIZE)
    if d_final_state is not None:
        assert d_final_state.shape == (N, NUM_V_HEADS, HEAD_SIZE, HEAD_SIZE)
    dev = q.device
    f32 = dict(dtype=torch.float32, device=dev)
    g = dict(dq=torch.empty(T, NUM_Q_HEADS, HEAD_SIZE, **f32),
             dk=torch.empty(T, NUM_K_HEADS, HEAD_SIZE, **f32),
             dv=torch.empty(T, NUM_V_HEADS, HEAD_SIZE, **f32),
             da=torch.empty(T, NUM_V_HEADS, **f32), db=torch.empty(T, NUM_V_HEADS, **f32),
             dA_log=torch.empty(NUM_V_HEADS, **f32), ddt_bias=torch.empty(NUM_V_HEADS, **f32),
             d_state=(torch.empty(N, NUM_V_HEADS, HEAD_SIZE, HEAD_SIZE, **f32)
                      if need_d_state else None))
    ws = alloc_backward_workspace(T, N, dev)
    backward_into(q.contiguous(), k.contiguous(), v.contiguous(),
                  None if state is None else state.contiguous().float(),
                  A_log.contiguous().float(), a.contiguous(), dt_bias.contiguous().float(),
                  b.contiguous(), cu_seqlens.contiguous(), scale,
                  d_out.to(torch.bfloat16).contiguous(),
                  None if d_final_state is None else d_final_state.float().contiguous(),
                  g["dq"], g["dk"], g["dv"], g["da"], g["db"], g["dA_log"], g["ddt_bias"],
                  g["d_state"], ws)
    return g


class _PrefillFunction(torch.autograd.Function):
    """out, final_state = run(...), differentiable in q, k, v, a, b, A_log,
    dt_bias and state (the backward recomputes the forward's chunk states)."""

    @staticmethod
    def forward(ctx, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale):
        out, final_state = run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
        ctx.save_for_backward(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens)
        ctx.scale = scale
        return out, final_state

    @staticmethod
    def backward(ctx, d_out, d_final):
        q, k, v, state, A_log, a, dt_bias, b, cu_seqlens = ctx.saved_tensors
        if d_out is None:
            d_out = torch.zeros(q.shape[0], NUM_V_HEADS, HEAD_SIZE, dtype=torch.bfloat16,
                                device=q.device)
        g = backward(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, ctx.scale, d_out,
                     d_final, need_d_state=state is not None and ctx.needs_input_grad[3])
        return (g["dq"], g["dk"], g["dv"], g["d_state"], g["dA_log"], g["da"], g["ddt_bias"],
                g["db"], None, None)


def run_autograd(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale):
    """`run` with gradients: the same arguments and results, recorded for
    torch.autograd (grads come back in each input's dtype).  No counterpart
    in the reference."""
    return _PrefillFunction.apply(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
