"""B200-native Gated DeltaNet kernel pair for the geometry qk4_v8_d128_k_last.

The directory name is not a Python identifier; import it with
`importlib.import_module("track-c-gdn_b200")` (the repository root on
sys.path).  Public API:

  decode.run(q, k, v, state, A_log, a, dt_bias, b, scale)            -> (out, new_state)
  decode.run_inplace(...)                                            -> out
  prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> (out, final_state)
  prefill.prefill_into(...), decode.decode_into(...)                 destination-passing forms
  shard.*                                                            multi-GPU partitioning

All compute runs in libgdn_b200.so (hand-written sm_100a CUDA); importing the
package fails if that library is missing.
"""
from . import _native  # noqa: F401  (raises if libgdn_b200.so is missing)
from . import decode, prefill  # noqa: F401

__all__ = ["decode", "prefill"]
