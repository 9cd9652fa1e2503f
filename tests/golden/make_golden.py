"""Generate golden vectors by running the reference's own Triton kernels.

Run in the build container (needs the reference checkout; not on GPU boxes):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref <reference checkout>

The reference solutions are loaded from the checkout, unmodified for decode
(gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py).  For prefill
(solution/triton/kernel.py) three in-memory adjustments are applied so the
file runs on CPU under the Triton 3.6 interpreter; nothing is written back:
  1. `i_t.to(tl.int64)` (kernel.py:1154) -> `tl.cast(i_t, tl.int64)`: the
     interpreter's loop variable is a plain Python int;
  2. every `tl.dot` upcasts its operands to fp32 with ieee precision: the
     interpreter's bf16 dot is wrong (errors ~1e11).  bf16 x bf16 products are
     exact in fp32 and every bf16 rounding point of the reference (w, u, h,
     v_new, the output's A) is kept;
  3. `_validate_inputs` (kernel.py:1635-1667) is bypassed: it asserts CUDA
     tensors.  The shape/dtype contract it checks is enforced by the inputs
     built here.
One interpreter behaviour is corrected for both kernels: the Triton 3.6
interpreter converts fp32 -> bf16 by truncation when `.to()` is given no
rounding mode, whereas compiled Triton on NVIDIA GPUs rounds to nearest even
(cvt.rn).  `_rne_convert_float` below restores round-to-nearest-even for that
one conversion so the fixtures carry the GPU kernels' rounding, not the
interpreter's.
Inputs come from tests/golden/cases.py (numpy PCG64, regenerable); each
fixture stores their sha256, the reference outputs (bf16 bits of `out`) and a
digest of the returned state plus two full state slices.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import linecache
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

sys.path.insert(0, str(Path(__file__).resolve().parent))
import cases  # noqa: E402

DECODE_REL = "gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py"
PREFILL_REL = "solution/triton/kernel.py"


def _install_rne_bf16():
    import triton.language as tl
    import triton.runtime.interpreter as interp

    orig = interp._convert_float

    def _rne_convert_float(inp, input_dtype, output_dtype, rounding_mode):
        if (input_dtype == tl.float32 and output_dtype == tl.bfloat16
                and rounding_mode in (None, "rtne")):
            u = np.frombuffer(inp.tobytes(), dtype=np.uint32).astype(np.uint64)
            out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            nan = (u & 0x7FFFFFFF) > 0x7F800000
            out[nan] = ((u[nan] >> 16) | 0x0040).astype(np.uint16)
            return out.reshape(inp.shape)
        return orig(inp, input_dtype, output_dtype, rounding_mode)

    interp._convert_float = _rne_convert_float


def _load_decode(ref: Path):
    spec = importlib.util.spec_from_file_location("ref_gdn_decode", ref / DECODE_REL)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _load_prefill(ref: Path):
    src = (ref / PREFILL_REL).read_text()
    old = "i_t_int64 = i_t.to(tl.int64)"
    assert src.count(old) == 1
    src = src.replace(old, "i_t_int64 = tl.cast(i_t, tl.int64)")
    src = src.replace("tl.dot(", "_fp32dot(")
    shim = (
        "\n@triton.jit\n"
        "def _fp32dot(x, y, allow_tf32=True):\n"
        "    return tl.dot(x.to(tl.float32), y.to(tl.float32), input_precision=\"ieee\")\n\n"
    )
    anchor = "SUPPORTS_AUTOTUNE_CACHE ="
    assert src.count(anchor) == 1
    src = src.replace(anchor, shim + anchor)
    fname = "<ref_gdn_prefill_interp>"
    linecache.cache[fname] = (len(src), None, src.splitlines(True), fname)
    mod = types.ModuleType("ref_gdn_prefill")
    mod.__file__ = fname
    exec(compile(src, fname, "exec"), mod.__dict__)
    mod._validate_inputs = lambda *args, **kwargs: None
    return mod


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(cases.bits_to_f32(bits)).to(torch.bfloat16)


def _out_bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _pack(name, kind, params, inp, out, state_out, ref_sha):
    S = state_out.numpy().astype(np.float32)
    dig = cases.state_digest(S)
    n_last = S.shape[0] - 1
    rec = {
        "kind": np.array(kind),
        "ref_sha256": np.array(ref_sha),
        "out_bits": _out_bits(out),
        "state_rowsum": dig["rowsum"],
        "state_proj": dig["proj"],
        "state_slice_first": S[0, 0],
        "state_slice_last": S[n_last, cases.HV - 1],
        "scale": np.array(params.get("scale", 0.0) or 0.0, np.float64),
    }
    for key, val in inp.items():
        rec["sha_" + key] = np.array("none" if val is None else cases.sha(val))
    for key, val in params.items():
        if key != "scale":
            rec["param_" + key] = np.array(val)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, type=Path, help="reference checkout")
    ap.add_argument("--out", type=Path, default=Path(__file__).resolve().parent)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    torch.set_grad_enabled(False)
    _install_rne_bf16()

    dec = _load_decode(args.ref)
    pre = _load_prefill(args.ref)
    dsha = hashlib.sha256((args.ref / DECODE_REL).read_bytes()).hexdigest()
    psha = hashlib.sha256((args.ref / PREFILL_REL).read_bytes()).hexdigest()

    for name, p in cases.DECODE_CASES.items():
        if args.only and args.only != name:
            continue
        gen = {k: v for k, v in p.items() if k != "scale"}
        inp = cases.decode_inputs(**gen)
        st = None if inp["state"] is None else torch.from_numpy(inp["state"])
        out, new_state = dec.run(
            _bf16(inp["q"]), _bf16(inp["k"]), _bf16(inp["v"]), st,
            torch.from_numpy(inp["A_log"]), _bf16(inp["a"]),
            torch.from_numpy(inp["dt_bias"]), _bf16(inp["b"]), p.get("scale"))
        rec = _pack(name, "decode", p, inp, out, new_state, dsha)
        np.savez_compressed(args.out / f"{name}.npz", **rec)
        print("wrote", name, out.shape)

    for name, p in cases.PREFILL_CASES.items():
        if args.only and args.only != name:
            continue
        gen = {k: v for k, v in p.items() if k != "scale"}
        inp = cases.prefill_inputs(**gen)
        st = None if inp["state"] is None else torch.from_numpy(inp["state"])
        out, final = pre.run(
            _bf16(inp["q"]), _bf16(inp["k"]), _bf16(inp["v"]), st,
            torch.from_numpy(inp["A_log"]), _bf16(inp["a"]),
            torch.from_numpy(inp["dt_bias"]), _bf16(inp["b"]),
            torch.from_numpy(inp["cu_seqlens"]), p.get("scale"))
        rec = _pack(name, "prefill", p, inp, out, final, psha)
        np.savez_compressed(args.out / f"{name}.npz", **rec)
        print("wrote", name, out.shape)


if __name__ == "__main__":
    main()
