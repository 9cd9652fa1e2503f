"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gdn_b200.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = header_functions()
    for n in ("gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last",
              "gdn_decode_mtp_qk4_v8_d128_k_last", "gdn_prefill_kernel_launches",
              "gdn_decode_pool_qk4_v8_d128_k_last", "gdn_prefill_pool_qk4_v8_d128_k_last",
              "gdn_prefill_workspace_bytes", "gdn_b200_status_string",
              "gdn_prefill_backward_qk4_v8_d128_k_last",
              "gdn_prefill_backward_workspace_bytes", "gdn_prefill_backward_kernel_launches",
              "gdn_b200_abi_version", "gdn_b200_read_device_status",
              "gdn_prefill_qk4_v8_d128_k_last_events"):
        assert n in names


def test_library_exports_every_declared_symbol(gdn):
    lib = ctypes.CDLL(str(gdn._native.LIB_PATH))
    for name in header_functions():
        assert hasattr(lib, name), f"libgdn_b200.so does not export {name}"
    # and the Python binding covers each of them
    assert set(header_functions()) == set(gdn._native.SIGNATURES)


def test_debug_entry_points_only_in_the_debug_build(gdn):
    """include/gdn_b200_debug.h declares what libgdn_b200_debug.so alone exports."""
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "gdn_b200_debug.h").read_text(), flags=re.S)
    names = sorted(set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", text)))
    assert names == ["gdn_b200_debug_wait_timeout_probe"]
    release = ctypes.CDLL(str(gdn._native.LIB_PATH))
    debug_path = gdn._native.LIB_PATH.with_name("libgdn_b200_debug.so")
    if not debug_path.exists():
        pytest.skip("debug build not present")
    debug = ctypes.CDLL(str(debug_path))
    for n in names:
        assert hasattr(debug, n) and not hasattr(release, n), n
    for n in header_functions():
        assert hasattr(debug, n), n


def test_status_strings(gdn):
    lib = gdn._native.lib
    assert lib.gdn_b200_abi_version() == 1
    for code in range(8):
        assert lib.gdn_b200_status_string(code)
    assert lib.gdn_b200_status_string(0) == b"ok"


def test_workspace_size_monotone(gdn):
    ws = gdn.prefill.workspace_bytes
    assert ws(0, 1) > 0
    # single-pass evaluation (many or short sequences): the 16 KiB [PA;Ainv]
    # image per (chunk, v-head) dominates, ~2 KiB per token
    assert ws(4096, 32) < ws(8192, 32) < ws(8192, 64)
    assert 2048 * 8192 < ws(8192, 16) < 2048 * 8192 * 1.3   # 128 chunks < 12 x 16: single pass
    # segmented evaluation (few long sequences) adds three fp32 states
    # (512 KiB each) per segment: T = 4096, N = 1 -> segments of 4 chunks,
    # at most 1 + ceil(65 / 4) = 18 of them
    seg_states = 3 * 18 * 8 * 128 * 128 * 4
    assert 2048 * 4096 + seg_states < ws(4096, 1) < (2048 * 4096 + seg_states) * 1.1
    assert ws(4096, 1) < ws(8192, 1)


def test_prefill_launch_count_follows_segment_policy(gdn):
    n = gdn._native.prefill_kernel_launches
    assert n(0, 0) == 0
    assert n(4096, 1) == 5        # one long sequence: segmented (3 passes + compose)
    assert n(16384, 4) == 5
    assert n(269, 1) == 3         # 5 chunks: too short to segment
    assert n(44450, 32) == 3      # more than 16 sequences: single pass
    assert n(11 * 64 * 2, 2) == 3  # fewer than 12 chunks per sequence on average
    assert n(12 * 64 * 2, 2) == 5


def test_argument_validation_without_device(gdn):
    lib = gdn._native.lib
    P = ctypes.c_void_p
    ok = P(0x10000)
    # decode: NULL pointers, negative batch, misalignment
    assert lib.gdn_decode_qk4_v8_d128_k_last(None, ok, ok, None, ok, ok, ok, ok, 0.0, 4, ok, ok, None) == 1
    assert lib.gdn_decode_qk4_v8_d128_k_last(ok, ok, ok, None, ok, ok, ok, ok, 0.0, -1, ok, ok, None) == 2
    assert lib.gdn_decode_qk4_v8_d128_k_last(ok, ok, ok, None, ok, ok, ok, ok, 0.0, 0, ok, ok, None) == 0
    assert lib.gdn_decode_qk4_v8_d128_k_last(P(0x10004), ok, ok, None, ok, ok, ok, ok, 0.0, 4, ok, ok, None) == 3
    # decode: new_state partially overlapping state
    assert lib.gdn_decode_qk4_v8_d128_k_last(ok, ok, ok, P(0x100000), ok, ok, ok, ok, 0.0, 4, ok,
                                             P(0x100000 + 4096), None) == 7
    # prefill: workspace too small / misaligned, NULL cu_seqlens
    args = [ok, ok, ok, None, ok, ok, ok, ok, ok, 2, 128, 0.0, ok, ok]
    assert lib.gdn_prefill_qk4_v8_d128_k_last(*args, ok, 16, None) == 4
    assert lib.gdn_prefill_qk4_v8_d128_k_last(*args, P(0x10010), 1 << 30, None) == 4
    bad = list(args)
    bad[8] = None
    assert lib.gdn_prefill_qk4_v8_d128_k_last(*bad, ok, 1 << 30, None) == 1
    assert lib.gdn_prefill_qk4_v8_d128_k_last(*args[:9], -1, 128, *args[11:], ok, 1 << 30, None) == 2


def test_pool_entry_points_argument_validation_without_device(gdn):
    lib = gdn._native.lib
    P = ctypes.c_void_p
    ok = P(0x10000)
    dec = lib.gdn_decode_pool_qk4_v8_d128_k_last
    # (q, k, v, pool, pool_slots, slots, A_log, a, dt_bias, b, scale, B, T, out, stream)
    assert dec(ok, ok, ok, ok, 0, ok, ok, ok, ok, ok, 0.0, 4, 1, ok, None) == 2   # empty pool
    assert dec(ok, ok, ok, ok, 8, ok, ok, ok, ok, ok, 0.0, 4, 0, ok, None) == 2   # T = 0
    assert dec(ok, ok, ok, ok, 8, None, ok, ok, ok, ok, 0.0, 4, 1, ok, None) == 1  # no slots
    assert dec(ok, ok, ok, P(0x10008), 8, ok, ok, ok, ok, ok, 0.0, 4, 1, ok, None) == 3
    assert dec(ok, ok, ok, ok, 8, ok, ok, ok, ok, ok, 0.0, 0, 1, ok, None) == 0
    pre = lib.gdn_prefill_pool_qk4_v8_d128_k_last
    args = [ok, ok, ok, ok, 8, ok, ok, ok, ok, ok, ok, 2, 128, 0.0, ok]
    assert pre(*args, ok, 16, None) == 4                       # workspace too small
    bad = list(args)
    bad[5] = None
    assert pre(*bad, ok, 1 << 30, None) == 1                   # no slots
    bad = list(args)
    bad[4] = 0
    assert pre(*bad, ok, 1 << 30, None) == 2                   # empty pool


def test_mtp_decode_argument_validation_without_device(gdn):
    lib = gdn._native.lib
    P = ctypes.c_void_p
    ok = P(0x10000)
    f = lib.gdn_decode_mtp_qk4_v8_d128_k_last
    base = [ok, ok, ok, None, ok, ok, ok, ok, 0.0]
    # token count outside 1..64, negative batch
    assert f(*base, 4, 0, ok, ok, None, None) == 2
    assert f(*base, 4, 65, ok, ok, None, None) == 2
    assert f(*base, -1, 2, ok, ok, None, None) == 2
    assert f(*base, 0, 2, ok, ok, None, None) == 0
    # NULL output, misaligned intermediate states
    assert f(*base, 4, 2, None, ok, None, None) == 1
    assert f(*base, 4, 2, ok, ok, P(0x20008), None) == 3
    # intermediate states overlapping the state, or the new state
    st = P(0x1000000)
    assert f(ok, ok, ok, st, ok, ok, ok, ok, 0.0, 4, 2, ok, P(0x9000000),
             P(0x1000000 + 1024), None) == 7
    assert f(*base, 4, 2, ok, P(0x9000000), P(0x9000000 + 4096), None) == 7


def test_backward_argument_validation_without_device(gdn):
    lib = gdn._native.lib
    P = ctypes.c_void_p
    ok = P(0x10000)
    f = lib.gdn_prefill_backward_qk4_v8_d128_k_last
    T, N = 128, 2
    need = lib.gdn_prefill_backward_workspace_bytes(T, N)
    assert need > lib.gdn_prefill_workspace_bytes(T, N)
    # (q, k, v, state, A_log, a, dt_bias, b, cu, N, T, scale, d_out, d_final,
    #  dq, dk, dv, da, db, dA_log, ddt_bias, d_state, ws, ws_bytes, stream)
    fwd = [ok, ok, ok, None, ok, ok, ok, ok, ok, N, T, 0.0, ok, None]
    outs = [ok, ok, ok, ok, ok, ok, ok, None]
    assert f(*fwd, *outs, ok, 16, None) == 4                    # workspace too small
    assert f(*fwd, *outs, P(0x10200), need, None) == 4          # workspace misaligned
    bad = list(outs)
    bad[0] = None
    assert f(*fwd, *bad, ok, need, None) == 1                   # no dq
    bad = list(outs)
    bad[5] = None
    assert f(*fwd, *bad, ok, need, None) == 1                   # no dA_log
    bad = list(fwd)
    bad[12] = P(0x10008)
    assert f(*bad, *outs, ok, need, None) == 3                  # misaligned d_out
    bad = list(fwd)
    bad[9], bad[10] = -1, T
    assert f(*bad, *outs, ok, need, None) == 2                  # negative N
    bad = list(fwd)
    bad[9], bad[10] = 0, 0
    assert f(*bad, *outs, ok, need, None) == 0                  # nothing to do
    # d_state overlapping the initial state
    st = P(0x1000000)
    bad = list(fwd)
    bad[3] = st
    aliasing = list(outs)
    aliasing[7] = P(0x1000000 + 4096)
    assert f(*bad, *aliasing, ok, need, None) == 7
    assert lib.gdn_prefill_backward_kernel_launches() == 7


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_reported_not_crashed(gdn):
    lib = gdn._native.lib
    ok = ctypes.c_void_p(0x10000)
    st = lib.gdn_decode_qk4_v8_d128_k_last(ok, ok, ok, None, ok, ok, ok, ok, 0.0, 4, ok,
                                           ctypes.c_void_p(0x20000000), None)
    assert st == 6  # GDN_ERR_DEVICE


def test_reference_signatures_preserved(gdn):
    import inspect
    assert list(inspect.signature(gdn.decode.run).parameters) == [
        "q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale"]
    assert list(inspect.signature(gdn.prefill.run).parameters) == [
        "q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale"]
