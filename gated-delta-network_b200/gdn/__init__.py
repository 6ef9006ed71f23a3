"""B200-native Gated DeltaNet operator pair (qk4_v8_d128, k-last fp32 state).

Drop-in entry points with the reference's signatures:

* ``gdn.decode.run(q, k, v, state, A_log, a, dt_bias, b, scale)`` -> (output, new_state)
  (reference/gdn_decode_ref.py:12)
* ``gdn.decode.kernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)``
  (destination passing; solutions/gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:85)
* ``gdn.prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)`` -> (output, new_state)
  (reference/gdn_prefill_ref.py:12)
* ``gdn.prefill.kernel(..., cu_seqlens, scale, output, new_state)``
  (destination passing; solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:1049)

All compute runs in hand-written sm_100a CUDA behind the C ABI of
``include/gdn_b200.h`` (libgdn_b200.so); there is no CPU or Triton fallback.
"""
from . import decode, prefill  # noqa: F401
from ._lib import GDNError  # noqa: F401

__all__ = ["decode", "prefill", "GDNError"]
