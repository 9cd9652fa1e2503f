"""A bounded device wait that runs out.

Every mbarrier wait in the prefill and backward kernels polls for a bounded
number of SM cycles; when the budget runs out the kernel records device
status 2, skips the rest of its work, frees its TMEM and returns, so the
CUDA context stays usable and the host learns of it through
gdn_b200_read_device_status.  The index-checked debug build lets a probe
lower the budget and wait on an mbarrier that nothing arrives on (no copy
or MMA in flight, so giving up leaves nothing behind):
gdn_b200_debug_wait_timeout_probe (include/gdn_b200_debug.h).  The test
runs in a fresh process on libgdn_b200_debug.so; it asserts that every
thread's wait gave up, that the CTA reached its end after freeing its TMEM,
that the device status reads 2 once (and is then cleared), and that a
following prefill on the same context is correct and leaves the status at 0.
"""
import ctypes
import importlib
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_bounded_wait_runs_out_and_reports_status_2():
    sys.path.insert(0, str(ROOT / "track-c-gdn_b200"))
    try:
        import build as native_build
    finally:
        sys.path.pop(0)
    lib = native_build.build(debug=True)
    env = dict(os.environ, GDN_B200_LIBRARY=str(lib))
    res = subprocess.run([sys.executable, __file__], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "probe ok" in res.stdout, res.stdout[-2000:]


def _probe_main():
    import torch

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases
    import oracle
    from gpu_util import out_err, prefill_args, rel_fro

    gdn = importlib.import_module("track-c-gdn_b200")
    assert gdn._native.LIB_PATH.name == "libgdn_b200_debug.so", gdn._native.LIB_PATH
    lib = gdn._native.lib
    probe = lib.gdn_b200_debug_wait_timeout_probe
    probe.restype = ctypes.c_int
    probe.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    assert gdn._native.read_device_status(stream) == 0
    result = (ctypes.c_int * 4)()
    st = probe(1 << 20, result, ctypes.c_void_p(stream))  # ~0.5 ms at full clock
    assert st == 0, lib.gdn_b200_status_string(st)
    wait_ok, broken, reached_end, gave_up = list(result)
    assert wait_ok == 0 and broken == 1 and reached_end == 1 and gave_up == 128, list(result)
    assert gdn._native.read_device_status(stream) == 2
    assert gdn._native.read_device_status(stream) == 0  # read-and-clear
    # the budget is restored and the context is usable: a normal prefill
    inp = cases.prefill_inputs(seed=404, lens=[17, 200, 64], with_state=True)
    o, s = gdn.prefill.run(*prefill_args(inp), None)
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                            inp["dt_bias"], inp["b"], inp["cu_seqlens"])
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < 5e-3
    assert gdn._native.read_device_status(stream) == 0
    print("probe ok")


if __name__ == "__main__":
    _probe_main()
