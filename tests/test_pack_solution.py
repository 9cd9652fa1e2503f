"""Solution packaging: pack a definition into the solution record, extract it
into an empty directory, build the extracted copy with nvcc (cross-compiles
for sm_100a without a GPU) and check the library it produces exports every
declared entry point, and that the packed kernel.py binds `run`."""
import ctypes
import importlib
import json
import subprocess
import sys

import pytest

pack = importlib.import_module("track-c-gdn_b200.pack")


@pytest.mark.parametrize("definition", sorted(pack.DEFINITIONS))
def test_pack_record_fields(definition):
    sol = pack.pack_solution(definition)
    assert sol["definition"] == definition
    assert sol["spec"]["entry_point"] == "kernel.py::run"
    assert sol["spec"]["destination_passing_style"] is False
    assert sol["spec"]["target_hardware"] == ["cuda"]
    paths = [s["path"] for s in sol["sources"]]
    assert paths[0] == "kernel.py"
    assert "include/gdn_b200.h" in paths
    assert any(p.endswith("csrc/gdn_b200.cu") for p in paths)
    json.dumps(sol)  # serialisable


def test_extract_rejects_unsafe_paths(tmp_path):
    with pytest.raises(ValueError):
        pack.extract_solution({"sources": [{"path": "../x.py", "content": ""}]}, tmp_path)


def test_extracted_solution_builds_and_exports(tmp_path):
    sol = pack.pack_solution("gdn_prefill_qk4_v8_d128_k_last")
    root = pack.extract_solution(json.loads(json.dumps(sol)), tmp_path / "sol")
    build = root / pack.PACKAGE / "build.py"
    res = subprocess.run([sys.executable, str(build)], capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-2000:]
    lib = ctypes.CDLL(str(root / pack.PACKAGE / "libgdn_b200.so"))
    for name in ("gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last",
                 "gdn_prefill_workspace_bytes", "gdn_decode_mtp_qk4_v8_d128_k_last"):
        assert hasattr(lib, name)
    # the packed entry point binds run (its import builds, then loads the package)
    code = ("import importlib.util, sys; "
            f"s = importlib.util.spec_from_file_location('k', r'{root / 'kernel.py'}'); "
            "m = importlib.util.module_from_spec(s); s.loader.exec_module(m); "
            "import inspect; print(list(inspect.signature(m.run).parameters))")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=900, cwd=tmp_path)
    assert res.returncode == 0, res.stderr[-2000:]
    assert "cu_seqlens" in res.stdout
