"""Helpers to load golden fixtures and compare results against them."""
from __future__ import annotations

from pathlib import Path

import numpy as np

import cases

GOLDEN = Path(__file__).resolve().parent / "golden"


def names(kind: str | None = None):
    out = []
    for p in sorted(GOLDEN.glob("*.npz")):
        if kind is None or p.stem.startswith(kind):
            out.append(p.stem)
    return out


def load(name: str):
    """Returns (kind, inputs, scale, fixture) with inputs regenerated from the
    case's seed and checked against the sha256 stored in the fixture."""
    z = np.load(GOLDEN / f"{name}.npz")
    kind = str(z["kind"])
    params = {k[len("param_"):]: z[k].tolist() for k in z.files if k.startswith("param_")}
    scale = float(z["scale"]) or None
    inp = cases.decode_inputs(**params) if kind == "decode" else cases.prefill_inputs(**params)
    for key, val in inp.items():
        want = str(z["sha_" + key])
        got = "none" if val is None else cases.sha(val)
        assert want == got, f"{name}: regenerated input {key} differs from the fixture's"
    return kind, inp, scale, z


def compare(z, out_f32: np.ndarray, state: np.ndarray):
    """Returns (max |out - golden| after rounding out to bf16, max |golden out|,
    relative error of the state digest (projection), relative error of the two
    stored full state slices)."""
    gold_o = cases.bits_to_f32(z["out_bits"])
    ob = cases.bits_to_f32(cases.to_bf16_bits(out_f32)).reshape(gold_o.shape)
    e_out = float(np.abs(ob - gold_o).max()) if gold_o.size else 0.0
    d = cases.state_digest(state)
    e_proj = float(np.linalg.norm(d["proj"] - z["state_proj"]) / max(np.linalg.norm(z["state_proj"]), 1e-30))
    n_last = state.shape[0] - 1
    e_sl = 0.0
    for got, want in ((state[0, 0], z["state_slice_first"]), (state[n_last, cases.HV - 1], z["state_slice_last"])):
        e_sl = max(e_sl, float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)))
    return e_out, float(np.abs(gold_o).max()) if gold_o.size else 0.0, e_proj, e_sl
