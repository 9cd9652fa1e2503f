"""The debug build (libgdn_b200_debug.so, compiled with -DGDN_DEBUG_CHECKS)
runs the prefill, multi-token decode and state-pool GPU tests in a fresh
process.  Its device-side index checks (work-item sequence, token and chunk
ranges against the call's sizes, segment slots, the prep chunk table) record
device status 4 on a violation instead of trapping; those tests assert a
clean device status after every case, so any violation fails them."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_gpu_suites_pass_on_the_index_checked_build():
    sys.path.insert(0, str(ROOT / "track-c-gdn_b200"))
    try:
        import build as native_build
    finally:
        sys.path.pop(0)
    lib = native_build.build(debug=True)
    env = dict(os.environ, GDN_B200_LIBRARY=str(lib))
    files = ["tests/test_prefill_gpu.py", "tests/test_decode_mtp_gpu.py",
             "tests/test_state_pool_gpu.py", "tests/test_bf16_state_gpu.py"]
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", *files],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]
