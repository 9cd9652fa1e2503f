"""Helpers shared by the GPU tests: numpy fixtures <-> CUDA tensors, metrics."""
from __future__ import annotations

import numpy as np
import torch


def bf16_dev(bits: np.ndarray, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16).to(device)


def f32_dev(x, device="cuda"):
    if x is None:
        return None
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device)


def bf16_host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def decode_args(inp, device="cuda"):
    return (bf16_dev(inp["q"], device), bf16_dev(inp["k"], device), bf16_dev(inp["v"], device),
            f32_dev(inp["state"], device), f32_dev(inp["A_log"], device),
            bf16_dev(inp["a"], device), f32_dev(inp["dt_bias"], device),
            bf16_dev(inp["b"], device))


def prefill_args(inp, device="cuda"):
    return (bf16_dev(inp["q"], device), bf16_dev(inp["k"], device), bf16_dev(inp["v"], device),
            f32_dev(inp["state"], device), f32_dev(inp["A_log"], device),
            bf16_dev(inp["a"], device), f32_dev(inp["dt_bias"], device),
            bf16_dev(inp["b"], device),
            torch.from_numpy(np.ascontiguousarray(inp["cu_seqlens"], np.int64)).to(device))


def rel_fro(x: np.ndarray, ref: np.ndarray) -> float:
    return float(np.linalg.norm((x - ref).ravel()) / max(np.linalg.norm(ref.ravel()), 1e-30))


def out_err(o_gpu_bf16: torch.Tensor, o_ref_f32: np.ndarray) -> float:
    """max |o_gpu - o_ref| - 1e-2 |o_ref| scaled: returns the largest violation
    ratio of |d| <= atol + rtol*|ref| with atol=2e-3, rtol=1e-2 (<=1 passes)."""
    o = o_gpu_bf16.float().cpu().numpy().reshape(o_ref_f32.shape)
    d = np.abs(o - o_ref_f32)
    return float((d / (2e-3 + 1e-2 * np.abs(o_ref_f32))).max()) if d.size else 0.0


def device_prefill_inputs(lengths, with_state: bool, seed: int, device="cuda"):
    """Benchmark-distribution prefill inputs drawn on the GPU (torch
    generator; q/k L2-normalised randn, v randn, a/b randn, initial states
    randn*0.02, A_log ~ U(0, 2.7), dt_bias ~ N(0, 0.1)) for sizes where
    numpy generation would take minutes.  Returns (device args in `run`
    order, host dict of the same inputs in the oracle's formats)."""
    import torch.nn.functional as F
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    lengths = np.asarray(lengths, np.int64)
    T, N = int(lengths.sum()), len(lengths)
    cu = np.zeros(N + 1, np.int64)
    cu[1:] = np.cumsum(lengths)
    q = F.normalize(torch.randn(T, 4, 128, generator=g, device=device), dim=-1).bfloat16()
    k = F.normalize(torch.randn(T, 4, 128, generator=g, device=device), dim=-1).bfloat16()
    v = torch.randn(T, 8, 128, generator=g, device=device).bfloat16()
    a = torch.randn(T, 8, generator=g, device=device).bfloat16()
    b = torch.randn(T, 8, generator=g, device=device).bfloat16()
    A_log = (torch.rand(8, generator=g, device=device) * 2.7).float()
    dt = (torch.randn(8, generator=g, device=device) * 0.1).float()
    h0 = (torch.randn(N, 8, 128, 128, generator=g, device=device) * 0.02) if with_state else None
    cu_d = torch.from_numpy(cu).to(device)
    host = dict(q=bf16_host_bits(q), k=bf16_host_bits(k), v=bf16_host_bits(v),
                a=bf16_host_bits(a), b=bf16_host_bits(b), A_log=A_log.cpu().numpy(),
                dt_bias=dt.cpu().numpy(), state=None if h0 is None else h0.cpu().numpy(),
                cu_seqlens=cu)
    return (q, k, v, h0, A_log, a, dt, b, cu_d), host


def out_err_np(o: np.ndarray, o_ref: np.ndarray) -> float:
    """out_err on host arrays (o already widened from bf16)."""
    d = np.abs(o - o_ref)
    return float((d / (2e-3 + 1e-2 * np.abs(o_ref))).max()) if d.size else 0.0
