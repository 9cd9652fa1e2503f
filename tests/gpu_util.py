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
